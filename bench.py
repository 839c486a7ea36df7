"""Benchmark of the temporal-attention training step (TGAT 2-layer).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl fast|reference] [--config 5|2|...]

Default workload: config 5, the north star's scaling configuration (TGAT
2-layer, recent 10x10, 16,700 nodes / 191 M edges, 413-d node and 186-d edge
features, bf16 projections with fp32 softmax / LayerNorm / loss / Adam).  One
step = one chronological global batch of 4,000 positive edges + 4,000
negatives, split evenly over the N ranks (strong scaling): temporal sampling
(the global batch advances every rank's time pointers), feature gather + time
encoding, Q/K/V projections, edge softmax + aggregate, w_out/LayerNorm, edge
predictor, BCE, backward, gradient all-reduce, Adam (reference
train.py:307-393).  `--config 2` is the fp32 uniform 10x10 line (600 + 600
per GPU, weak scaling).

`value`   positive training edges/s with graph, features and batch lists
          resident in HBM (device-timed, max over ranks).
`e2e`     the same through the product's public training API with host
          buffers: numpy roots/timestamps of every step go through pinned
          staging into the captured step (GraphTrainer.step_host_pipelined),
          H2D inside the timed region, and every step's loss is read back.
`--impl reference` times the reference's CPU path of the same step: the
          reference sampler built from its own source (oracle/_ref, all host
          threads) + the fp32 CPU restatement of layers.py/modules.py
          (oracle/ref_math.py over the parameter tree of oracle/ref_model.py)
          + torch.optim.Adam.  It imports nothing from fast_b200 that loads
          the product's library.
"""
import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "TGAT 2-layer training edges/sec"
UNIT = "edges/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="fast", choices=["fast", "reference"])
    ap.add_argument("--config", type=int, default=5)
    ap.add_argument("--data", default=None,
                    help="dataset directory in the reference's format (edges.csv + ext_full.npz) instead of the "
                         "config's synthetic graph; feature widths and the model still come from --config")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="budget of the cpu_baseline sample")
    ap.add_argument("--cpu-edges", type=int, default=4_000_000,
                    help="config 5 on the CPU: edges of a smaller graph drawn like config 5's (its fp32 edge "
                         "table is 142 GB)")
    ap.add_argument("--cpu-batch-frac", type=float, default=0.25,
                    help="config 5 on the CPU: each step trains on this fraction of the global batch")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-steps", type=int, default=5)
    ap.add_argument("--breakdown-steps", type=int, default=10,
                    help="steps of the per-phase device-time breakdown (sampling, forward+backward, all-reduce, "
                         "Adam), each phase a graph of its own; 0 skips it")
    ap.add_argument("--eager", action="store_true", help="launch kernels step by step instead of a CUDA graph")
    ap.add_argument("--batch", type=int, default=None,
                    help="positive edges per step instead of the config's (one GPU at --batch 500 runs the per-rank "
                         "workload of config 5 on 8 GPUs)")
    ap.add_argument("--edges", type=int, default=None,
                    help="a smaller graph of N edges drawn like the config's (same nodes, endpoint and time "
                         "distributions, so each node's edges lie further apart in time)")
    ap.add_argument("--suite", default=None, choices=["kernels", "bf16"],
                    help="kernels: time each hot kernel alone at config-5 block sizes against the HBM roofline "
                         "(one JSON line per kernel instead of the training-step line)")
    ap.add_argument("--suite-scale", type=float, default=1.0,
                    help="--suite kernels: fraction of the config-5 block sizes (small cases for ncu captures)")
    ap.add_argument("--suite-table-rows", type=int, default=None,
                    help="--suite bf16: rows of the edge-feature table the gather indexes at random "
                         "(default 4 M x --suite-scale)")
    ap.add_argument("--cuda-profiler-range", action="store_true",
                    help="bracket the timed steps with cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    ap.add_argument("--path", default="fused", choices=["fused", "autograd"],
                    help="training step as FusedStep kernels (fused) or the GeneralModel module under autograd")
    ap.add_argument("--gemm", default="tc", choices=["tc", "ffma"],
                    help="projection GEMMs on the tcgen05 tensor cores (tc, 3xTF32) or the CUDA cores (ffma)")
    return ap.parse_args()


# ----------------------------------------------------------------------------- helpers
# DRAM bytes over algorithmic bytes of the wrappers that can be the dominant kernel, from one ncu capture of
# the same step on a 4 M-edge graph drawn like config 5's (profiles/ncu_dram_traffic_bwd_dkv_dq_gather_edges4m.md); the traffic of
# a full-size launch is the ratio times its algorithmic bytes
NCU_TRAFFIC = {"gemm_group:bwd_dkv_dq": 1834.6 / 1873.3, "gather_time_encode": 1081.9 / 1966.7}
NCU_TRAFFIC_SRC = "profiles/ncu_dram_traffic_bwd_dkv_dq_gather_edges4m.md"


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return dict(hbm=float(p["hbm_gbs"]), tf=float(p["bf16_tflops"]), tf_sus=float(p["bf16_tflops_sustained"]),
                    src="measured")
    return dict(hbm=6650.0, tf=1590.0, tf_sus=1400.0, src="fallback")


class NvmlClockSampler:
    """SM clock and clock-event reasons read through NVML every 2 ms on a
    background thread while the timed region runs (it lasts well under a
    second, too short for nvidia-smi's sampling period).  Reads only."""

    BITS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, gpu_index):
        import pynvml
        self.nv = pynvml
        pynvml.nvmlInit()
        self.h = pynvml.nvmlDeviceGetHandleByIndex(gpu_index)
        self.samples, self.stop_flag, self.thread = [], False, None
        get = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            getattr(pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
        self.reasons_of = lambda: get(self.h)

    def _loop(self):
        nv = self.nv
        while not self.stop_flag:
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM), self.reasons_of()))
            except Exception:   # noqa: BLE001 - a failed read skips one sample
                pass
            time.sleep(0.002)

    def start(self):
        import threading
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def stop(self):
        self.stop_flag = True
        self.thread.join(timeout=5)
        if not self.samples:
            return None
        mx = self.nv.nvmlDeviceGetMaxClockInfo(self.h, self.nv.NVML_CLOCK_SM)
        reasons = sorted({k for _, r in self.samples for k, b in self.BITS.items() if r & b})
        return {"sm_mhz": float(np.median([c for c, _ in self.samples])), "sm_max_mhz": float(mx),
                "reasons": reasons, "samples": len(self.samples), "source": "nvml, 2 ms"}


def clock_sampler(gpu_index):
    try:
        return NvmlClockSampler(gpu_index)
    except Exception:           # noqa: BLE001 - no NVML: fall back to nvidia-smi
        return ClockSampler(gpu_index)


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", "fb_clocks_%d_%d.csv" % (os.getpid(), gpu_index))

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.Q,
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


class _RowsModulo:
    """An edge-feature table of `rows` rows standing in for a larger one:
    edge id e reads row e mod rows (rows drawn like the full table's, gathered
    at the same random positions of a table far larger than the caches)."""

    def __init__(self, table):
        self.t = table
        self.shape = (None, table.shape[1])

    def __getitem__(self, idx):
        return self.t[idx % self.t.shape[0]]


def cpu_reference_step_fn(cfg, graph, edge_feats_cpu, node_feats_cpu, threads, B):
    """Closures running one reference-CPU training step on a batch index and
    resetting the sampler (epoch start); returns (step, reset, kind).  The
    sampler is the reference's own (oracle/_ref, built from its source) when
    present; the model is ref_math (layers.py/modules.py, DGL path) over the
    parameter tree of oracle/ref_model.py, trained with torch.optim.Adam.
    Nothing here loads the product's library."""
    import torch
    from oracle import ref_math
    from oracle.ref_model import GeneralModel
    from oracle.sampler import OracleSampler, load_reference
    torch.set_num_threads(threads)
    sp, mp, gp, tp = cpu_model_params(cfg)
    ref = load_reference()
    kind = "reference" if ref is not None else "port"
    S = ref.ParallelSampler if ref is not None else OracleSampler
    sampler = S(graph.indptr, graph.indices, graph.eid, graph.ts_csr, threads, 1, sp["layer"], sp["neighbor"],
                sp["strategy"] == "recent", False, 1, 0.0)
    torch.manual_seed(0)
    model = GeneralModel(0 if node_feats_cpu is None else node_feats_cpu.shape[1], edge_feats_cpu.shape[1],
                         sp, mp, gp, tp)
    opt = torch.optim.Adam(model.parameters(), lr=tp["lr"])
    rng = np.random.default_rng(1)
    stats = dict(edges=0, steps=0)

    def step(i, stride=None):
        """Training step on chronological batch i: positive edges
        [i * stride, i * stride + B) (stride defaults to B)."""
        b0 = i * (stride or B)
        src, dst, t = graph.src[b0:b0 + B], graph.dst[b0:b0 + B], graph.ts[b0:b0 + B]
        roots = np.concatenate([src, dst, rng.integers(0, graph.n_nodes, B).astype(np.int32)])
        rts = np.concatenate([t, t, t]).astype(np.float32)
        sampler.sample(roots, rts, [])
        blocks = sampler.get_ret()
        stats["edges"] += sum(len(b.row()) for b in blocks)
        stats["steps"] += 1
        opt.zero_grad()
        pp, pn = ref_math.model_forward(model, blocks, node_feats_cpu, edge_feats_cpu)
        loss = ref_math.bce_loss(pp, pn)
        loss.backward()
        opt.step()
        return loss.item()

    return step, sampler.reset, kind, stats


def cpu_model_params(cfg):
    """sample/memory/gnn/train parameters of the config's reference model
    (config/TGAT.yml with the CLI overrides of train.py:98), as
    fast_b200.data.model_params gives them; restated here so that the CPU arm
    imports nothing from the product."""
    layers = len(cfg.fanout)
    sample = dict(layer=layers, neighbor=list(cfg.fanout), strategy=cfg.strategy, prop_time=False, history=1,
                  duration=0)
    memory = dict(type="none", dim_out=0)
    gnn = dict(arch="transformer_attention", layer=layers, att_head=2, dim_time=100, dim_out=100)
    train = dict(lr=0.0001, dropout=0.1, att_dropout=0.1)
    return sample, memory, gnn, train


SCHEDULE_NOTE = ("warm-up = the epoch's first W batches; timed = K batches spread evenly over the rest of the "
                 "epoch, chronological; sampler reset before each pass")


def epoch_schedule(n_batches, warmup, steps):
    """Batch indices of a run: the first `warmup` batches of the epoch, then
    `steps` batches spread evenly over the rest of it, in chronological order.
    Sampled neighbourhoods grow as the epoch advances (the first batches have
    almost no history), so the timed steps cover the whole epoch instead of
    its first few batches."""
    warm = list(range(min(warmup, n_batches)))
    lo = len(warm)
    span = max(n_batches - lo, 1)
    timed = [min(lo + int((j + 0.5) * span / steps), n_batches - 1) for j in range(steps)]
    return warm, timed


def cpu_plan(args, cfg):
    """What the CPU arm runs for a config: (graph edges, table rows, fraction
    of the global batch per step, note).  Configs 1-4 run at full size.
    Config 5's fp32 tables (142 GB of edge features) exceed the host, so its
    CPU arm samples a 20 M-edge graph drawn like config 5's (same 16,700 nodes,
    endpoint and time distributions; every fan-out still fills), gathers edge
    features from a 4 M-row table at the edge id modulo 4 M, and trains each
    step on the first quarter of the chronological global batch."""
    if not cfg.sharded or args.data:
        return cfg.edges, cfg.edges, 1.0, "full graph"
    n = min(cfg.edges, max(args.cpu_edges * 5, 1))
    rows = min(n, args.cpu_edges)
    return n, rows, args.cpu_batch_frac, (
        "%d-edge graph drawn like %s (same nodes, endpoint and time distributions), edge features from a %d-row "
        "fp32 table at edge id mod %d, each step %.0f%% of the global batch" %
        (n, cfg.name, rows, rows, 100 * args.cpu_batch_frac))


def cpu_workload(cfg, data=None, n_edges=None, table_rows=None):
    import torch
    from fast_b200.data import make_graph
    if data:
        from fast_b200.dataio import load_graph
        graph = load_graph(data)
    else:
        graph = make_graph(cfg, n_edges=n_edges)
    g = torch.Generator()
    g.manual_seed(7)
    rows = table_rows or len(graph.src)
    ef = torch.randn(rows, cfg.d_edge, generator=g) if cfg.d_edge else None
    if ef is not None and rows < len(graph.src):
        ef = _RowsModulo(ef)
    nf = torch.randn(cfg.nodes, cfg.d_node, generator=g) if cfg.d_node else None
    return graph, ef, nf


def bench_config(args, cfg, world, B, gB):
    """The `config` object of both arms' lines (the workload, not the arm)."""
    bf16 = cfg.dtype == "bf16"
    return {"workload": cfg.name, "global_batch": gB, "local_batch": B, "fanout": list(cfg.fanout),
            "strategy": cfg.strategy, "nodes": cfg.nodes, "edges": cfg.edges, "d_node": cfg.d_node,
            "d_edge": cfg.d_edge, "parallelism": "dp%d" % world, "batches": SCHEDULE_NOTE,
            "l2": "inputs larger than L2 (%.1f GB edge-feature table gathered at random rows)" %
                  (cfg.edges * ((cfg.d_edge + 7) // 8 * 16 if bf16 else cfg.d_edge * 4) / 1e9)}


def batch_sizes(cfg, world):
    """(per-rank batch, global batch) of a step."""
    if cfg.sharded:
        # one global batch split across the ranks (config 5: 4,000 + 4,000 on 1/2/4/8 GPUs)
        if cfg.batch % world:
            raise SystemExit("%s: its global batch of %d does not split over %d ranks" % (cfg.name, cfg.batch, world))
        return cfg.batch // world, cfg.batch
    return cfg.batch, cfg.batch * world


# ----------------------------------------------------------------------------- reference arm
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    world = args.gpus
    from fast_b200.data import CONFIGS
    cfg = CONFIGS[args.config]
    cfg_line = cfg
    if args.data:
        _, cfg_line = workload_graph(args, cfg, device=False)
    elif args.edges or args.batch:
        import dataclasses
        cfg_line = dataclasses.replace(cfg, edges=args.edges or cfg.edges, batch=args.batch or cfg.batch)
    B, gB = batch_sizes(cfg_line, world)
    threads = len(os.sched_getaffinity(0))
    n_edges, rows, frac, note = cpu_plan(args, cfg_line)
    graph, ef, nf = cpu_workload(cfg_line, args.data, n_edges=n_edges, table_rows=rows)
    cB = max(1, int(round(gB * frac)))
    step, reset, kind, stats = cpu_reference_step_fn(cfg_line, graph, ef, nf, threads, cB)
    warm, timed = epoch_schedule(graph.train_end // gB, args.warmup, args.steps)
    reset()
    for i in warm:
        step(i, gB)
    stats.update(edges=0, steps=0)
    t0 = time.perf_counter()
    for i in timed:
        step(i, gB)
    dt = time.perf_counter() - t0
    value = args.steps * cB / dt
    sample = ("%d batches of %d+%d roots (%s), spread over one epoch after %d warm-up batches; %.0f sampled edges "
              "per step" % (args.steps, cB, 2 * cB, note, len(warm), stats["edges"] / max(stats["steps"], 1)))
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * dt / args.steps,
        "higher_is_better": True, "scaling": "strong" if cfg_line.sharded else "weak", "vs_baseline": None,
        "dtype": "f32", "data": data_label(args, cfg_line),
        "config": bench_config(args, cfg_line, world, B, gB),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- fast arm
def run_fast(args):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    from fast_b200 import ops
    from fast_b200.data import CONFIGS, make_features, make_features_bf16, model_params
    ops.USE_TC = args.gemm == "tc"
    from fast_b200.train import GraphTrainer, Trainer
    cfg = CONFIGS[args.config]
    graph, cfg = workload_graph(args, cfg, device=True)
    bf16 = cfg.dtype == "bf16"
    if bf16:
        # bf16 tables, rows padded to 8 columns, generated on the device
        nf, ef = make_features_bf16(cfg, cfg.edges, dev)
    else:
        nf, ef = make_features(cfg, cfg.edges, dev)
    sp, mp, gp, tp = model_params(cfg)
    fused = args.path == "fused"
    prec = dict(precision="bf16", feat_dims=(cfg.d_node, cfg.d_edge)) if bf16 else {}
    B, gB = batch_sizes(cfg, world)
    if args.eager:
        tr = Trainer(graph, nf, ef, sp, mp, gp, tp, dev, rank=rank, world=world, fused=fused, **prec)
    else:
        tr = GraphTrainer(graph, nf, ef, sp, mp, gp, tp, dev, batch=B, rank=rank, world=world,
                          fused=fused, **prec)
    n_batches = graph.train_end // gB
    warm, timed = epoch_schedule(n_batches, args.warmup, args.steps)

    # memory models also take the id of the batch's first edge (its mails carry that batch's edge features)
    e0_kw = (lambda b0: dict(e0=b0)) if getattr(tr, "mailbox", None) is not None else (lambda b0: {})

    def dev_step(i):
        b0, b1 = i * gB, (i + 1) * gB
        if args.eager:
            groots, gts = tr.batch_roots(b0, b1)
            roots, rts = tr.local_of(groots, gts)
            return tr.step_device(roots, rts, groots, gts, **e0_kw(b0))
        tr.load_device_roots(b0, b1)
        return tr.step_device()

    tr.reset_epoch()
    for i in warm:
        dev_step(i)
    torch.cuda.synchronize()
    clock = clock_sampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clock.start()
    l0 = ops.LAUNCHES[0]
    if not args.eager:
        # kernels per replayed step = kernels of one eager launch of the same body
        tr.load_device_roots(timed[0] * gB, (timed[0] + 1) * gB)
        tr._eager_step()
        torch.cuda.synchronize()
        per_step = ops.LAUNCHES[0] - l0 + tr.sampler_kernels_per_step()
        l0 = ops.LAUNCHES[0]
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.cuda_profiler_range:
        torch.cuda.cudart().cudaProfilerStart()
    ev0.record()
    for i in timed:
        loss = dev_step(i)
    ev1.record()
    torch.cuda.synchronize()
    if args.cuda_profiler_range:
        torch.cuda.cudart().cudaProfilerStop()
    clocks = clock.stop()
    ms = ev0.elapsed_time(ev1)
    if args.eager:
        launches = ops.LAUNCHES[0] - l0 + args.steps * tr.sampler_kernels_per_step()
    else:
        launches = per_step * args.steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.barrier()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    value = args.steps * gB / (ms / 1000.0)

    # end-to-end through the product's training API with host buffers, over
    # the same batches from a fresh epoch.  The batches' edge lists come to
    # the host before the timed region, as a user's data loader would hold
    # them; each step's roots and times are built, staged and copied inside it.
    rng = np.random.default_rng(5)
    host_edges = {i: tuple(_host(a[i * gB:(i + 1) * gB]) for a in (graph.src, graph.dst, graph.ts)) for i in timed}
    lo = tr.rank * B
    sel = np.concatenate([np.arange(lo, lo + B), gB + np.arange(lo, lo + B), 2 * gB + np.arange(lo, lo + B)])
    tr.reset_epoch()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    # pipelined when the trainer offers it: step i's loss is read back while
    # step i + 1 runs (every step still copies its inputs in and its loss out)
    host_step = getattr(tr, "step_host_pipelined", tr.step_host)
    t0 = time.perf_counter()
    for i in timed:
        src_np, dst_np, t_np = host_edges[i]
        # the global batch [src | dst | neg] (same rng seed on every rank), then this rank's slice
        groots = np.concatenate([src_np, dst_np, rng.integers(0, graph.n_nodes, gB).astype(np.int32)])
        gts = np.concatenate([t_np, t_np, t_np]).astype(np.float32)
        host_step(groots[sel], gts[sel], groots, gts, **e0_kw(i * gB))
    if hasattr(tr, "finish_pipelined"):
        tr.finish_pipelined()
    torch.cuda.synchronize()
    e2e_s = torch.tensor([time.perf_counter() - t0], device=dev)
    if world > 1:
        dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
    e2e_value = args.steps * gB / float(e2e_s.item())

    # per-kernel device times for the roofline: the kernels launched one by one
    # (outside the graph) with CUDA events around each,
    # at the blocks' true sizes (host-read dims), so bytes and flops are the
    # algorithmic ones of each launch
    ops.TIMER = ops.KernelTimer(reps=10)
    tr.reset_epoch()
    args.profile_steps = max(1, min(args.profile_steps, len(timed)))
    prof = [timed[(2 * j + 1) * len(timed) // (2 * args.profile_steps)] for j in range(args.profile_steps)]
    sampled = []
    for i in prof:
        groots, gts = tr.batch_roots(i * gB, (i + 1) * gB)
        roots, rts = tr.local_of(groots, gts)
        Trainer.step_device(tr, roots, rts, groots, gts, **e0_kw(i * gB))
        sampled.append(sum(int(d[1]) for d in tr.sampler.dims()))
    kern = ops.TIMER.summary()
    ops.TIMER = None
    t_samp = torch.tensor([float(np.mean(sampled))], device=dev)
    if world > 1:
        dist.all_reduce(t_samp)

    # per-phase device time of the step (max over ranks), from graphs of each phase
    breakdown = None
    if args.breakdown_steps > 0 and not args.eager and hasattr(tr, "phase_times"):
        tr.reset_epoch()

        def load(j):
            b = timed[j % len(timed)]
            tr.load_device_roots(b * gB, (b + 1) * gB)

        ph = tr.phase_times(min(args.breakdown_steps, len(timed)), load)
        keys = sorted(ph)
        t_ph = torch.tensor([ph[k] for k in keys], device=dev)
        if world > 1:
            dist.all_reduce(t_ph, op=dist.ReduceOp.MAX)
        breakdown = {k: round(float(v), 4) for k, v in zip(keys, t_ph.tolist())}
        breakdown["sum_of_phases"] = round(sum(v for k, v in breakdown.items() if k != "sample_local_only"), 4)
        breakdown["step_in_one_graph"] = round(ms / args.steps, 4)
        breakdown["note"] = ("ms per step, max over ranks; each phase replayed alone as its own graph (all-reduce "
                             "launched eagerly), so the sum exceeds the one-graph step by the overlap and the "
                             "launch gaps the single graph removes; sample_local_only = the sampler on this rank's "
                             "roots without the global batch's pointer updates")

    if world > 1 and hasattr(tr, "release"):
        tr.release()                       # graphs holding NCCL calls go before the process group
    if rank != 0:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0
    pk = peaks()
    kernels = {}
    for name, r in kern.items():
        per_ms = r["ms"] / r["launches"]
        gbs = r["bytes"] / (r["ms"] / 1000.0) / 1e9 if r["ms"] > 0 else 0.0
        tfs = r["flops"] / (r["ms"] / 1000.0) / 1e12 if r["ms"] > 0 else 0.0
        kernels[name] = {"launches_per_step": r["launches"] / args.profile_steps,
                         "ms_per_step": r["ms"] / args.profile_steps, "us_per_launch": 1000 * per_ms,
                         "GB/s": round(gbs, 1), "TFLOP/s": round(tfs, 2),
                         "hbm_frac": round(gbs / pk["hbm"], 4)}
    # the sampler entry times a whole sample() call (several kernels), not one kernel
    top = max(((k, v) for k, v in kern.items() if k != "sampler"), key=lambda kv: kv[1]["ms"])
    name, r = top
    # the binding roof: a contraction whose algorithmic bytes take longer at the copy bandwidth than its
    # flops at the tensor peak (flops per byte below the machine balance) is bounded by HBM
    tensor_bound = (r["flops"] > 0 and name.startswith("gemm") and
                    r["flops"] / (pk["tf"] * 1e12) >= r["bytes"] / (pk["hbm"] * 1e9))
    if tensor_bound:
        ach = r["flops"] / (r["ms"] / 1000.0) / 1e12
        roof = {"kernel": name, "bound": "tensor", "achieved": round(ach, 3), "peak": pk["tf"], "unit": "TFLOP/s",
                "frac": round(ach / pk["tf"], 5), "traffic": None,
                "peak_source": "%s bf16 burst (MEASURED_PEAKS.json)" % pk["src"],
                "note": ("bf16 operands, fp32 accumulation (tcgen05 kind::f16)" if bf16 else
                         ("fp32-accurate products as three TF32 tcgen05 MMAs each (achieved counts 2MNK, "
                          "not the 3x tensor work)" if args.gemm == "tc" else "fp32 products on the CUDA cores")
                         + "; the bf16 tensor peak is the only measured compute denominator")}
    else:
        ach = r["bytes"] / (r["ms"] / 1000.0) / 1e9
        roof = {"kernel": name, "bound": "hbm", "achieved": round(ach, 1), "peak": pk["hbm"], "unit": "GB/s",
                "frac": round(ach / pk["hbm"], 4), "traffic": None,
                "peak_source": "%s copy bandwidth (MEASURED_PEAKS.json)" % pk["src"]}
        if r["flops"] > 0:
            tfs = r["flops"] / (r["ms"] / 1000.0) / 1e12
            roof["note"] = ("a contraction below the machine balance (%.0f flop/B against %.0f): its algorithmic "
                            "bytes at the copy bandwidth take longer than its flops at the bf16 peak; tensor: "
                            "%.1f TFLOP/s, %.3f of %s" % (r["flops"] / r["bytes"], pk["tf"] * 1e3 / pk["hbm"], tfs,
                                                          tfs / pk["tf"], pk["tf"]))
    if bf16 and name in NCU_TRAFFIC:
        roof["traffic"] = int(NCU_TRAFFIC[name] * r["bytes"] / r["launches"])
        roof["traffic_unit"] = "bytes per launch"
        roof["traffic_source"] = ("dram__bytes_read.sum + dram__bytes_write.sum over the algorithmic bytes of the "
                                  "same launches (%s), times this launch's algorithmic bytes" % NCU_TRAFFIC_SRC)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong" if cfg.sharded else "weak",
        "vs_baseline": None, "dtype": "bf16" if bf16 else "f32", "data": data_label(args, cfg),
        "config": bench_config(args, cfg, world, B, gB),
        "impl_config": {"launch": "eager" if args.eager else "cuda_graph", "gemm": args.gemm, "step": args.path,
                        "precision": ("bf16 projections (w_q, w_k, w_v, w_out and their gradient products on "
                                      "bf16 operands, fp32 accumulation); attention, softmax, LayerNorm, loss and "
                                      "Adam in fp32" if bf16 else "fp32")},
        # every rank copies its own roots and times (3B x 8 bytes) and, with several ranks, the global
        # batch's (3gB x 8 bytes, for the time pointers), and reads back one fp32 loss
        "e2e": {"value": e2e_value, "unit": UNIT,
                "h2d_bytes_per_step": world * 3 * B * 8 + (world * 3 * gB * 8 if world > 1 else 0),
                "d2h_bytes_per_step": world * 4},
        "workload_stats": {"sampled_edges_per_step": round(float(t_samp.item()), 1),
                           "note": "edges of every layer's block summed over the ranks, mean of the profiled "
                                   "steps (the same timed batches)"},
        "step_breakdown_ms": breakdown,
        "gpu_launches": int(launches),
        "roofline": roof,
        "kernels": kernels,
        "clocks": clocks,
        "last_loss": float(loss),
    }
    if world == 1 and not args.no_cpu_baseline and getattr(tr, "mailbox", None) is None:
        line["cpu_baseline"] = cpu_baseline(args, cfg, args.cpu_seconds)
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def cpu_baseline(args, cfg, budget_s):
    """The reference CPU path (as --impl reference) on the GPU run's batch
    schedule (1 GPU), stopped after ~budget_s; a stop before the end keeps
    the earlier, smaller batches, which favours the CPU."""
    threads = len(os.sched_getaffinity(0))
    n_edges, rows, frac, note = cpu_plan(args, cfg)
    graph, ef, nf = cpu_workload(cfg, args.data, n_edges=n_edges, table_rows=rows)
    _, gB = batch_sizes(cfg, 1)
    cB = max(1, int(round(gB * frac)))
    warm, timed = epoch_schedule(graph.train_end // gB, args.warmup, args.steps)
    step, reset, kind, stats = cpu_reference_step_fn(cfg, graph, ef, nf, threads, cB)
    reset()
    for i in warm:
        step(i, gB)
    stats.update(edges=0, steps=0)
    n, t0 = 0, time.perf_counter()
    for i in timed:
        step(i, gB)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    el = time.perf_counter() - t0
    return {"value": n * cB / el, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": "%d of the %d timed batches (%d+%d roots each; %s; spread over one epoch), %.1f s, %.0f "
                      "sampled edges per step" % (n, len(timed), cB, 2 * cB, note, el,
                                                  stats["edges"] / max(stats["steps"], 1))}


# ----------------------------------------------------------------------------- kernel roofline suite
def run_kernel_suite(args):
    """Each HBM-bound kernel of the step, alone, at the block sizes of config 5
    (hop 2: 132 k destinations x fan-out 10 = 1.32 M edges; D = 100, 2 heads,
    172-d edge features, 100-d time encoding).  Algorithmic bytes per launch
    count every tensor the kernel must read or write once; time is the mean
    of 10 back-to-back launches between CUDA events, inputs larger than L2."""
    import torch
    from fast_b200 import ops
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    pk = peaks()
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    Nd, fan, D, H, de, dt_ = int(132_000 * args.suite_scale), 10, 100, 2, 172, 100
    E = Nd * fan
    rows_tab = int(4_000_000 * args.suite_scale)
    table = torch.randn(rows_tab, de, device=dev, generator=g)
    eid = torch.randint(0, rows_tab, (E,), device=dev, generator=g, dtype=torch.int32)
    dts = torch.rand(E, device=dev, generator=g) * 1e5
    w = (1.0 / 10 ** torch.linspace(0, 9, dt_, device=dev)).contiguous()
    b = torch.zeros(dt_, device=dev)
    rptr = torch.arange(0, E + 1, fan, device=dev, dtype=torch.int32)
    q = torch.randn(Nd, D, device=dev, generator=g) * 0.5
    kv = torch.randn(E, 2 * D, device=dev, generator=g) * 0.5
    dagg = torch.randn(Nd, D, device=dev, generator=g)
    z = torch.randn(E, D, device=dev, generator=g)
    gamma, beta = torch.ones(D, device=dev), torch.zeros(D, device=dev)
    dA = torch.randn(E, dt_, device=dev, generator=g)
    out = []

    def timed(name, nbytes, flops, fn, shape):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clock = clock_sampler(0)
        clock.start()
        s0.record()
        for _ in range(10):
            fn()
        s1.record()
        torch.cuda.synchronize()
        clocks = clock.stop()
        us = s0.elapsed_time(s1) * 100.0          # per launch, microseconds
        line = {"suite": "kernels", "kernel": name, "shape": shape, "us_per_launch": round(us, 2),
                "bytes_per_launch": int(nbytes), "clocks": clocks}
        if flops:
            tfs = flops / us / 1e6
            if args.gemm == "tc":
                line.update({"bound": "tensor (tcgen05, three TF32 MMAs per fp32 product)", "TFLOP_s": round(tfs, 2),
                             "peak_TFLOP_s": pk["tf"], "frac": round(tfs / pk["tf"], 4),
                             "peak_source": "%s bf16 burst (the only measured tensor peak)" % pk["src"],
                             "tensor_work_TFLOP_s": round(3 * tfs, 2)})
            else:
                line.update({"bound": "FFMA (fp32 CUDA cores)", "TFLOP_s": round(tfs, 2)})
        else:
            gbs = nbytes / us / 1e3
            line.update({"bound": "hbm", "achieved_GB_s": round(gbs, 1), "peak_GB_s": pk["hbm"],
                         "frac": round(gbs / pk["hbm"], 3), "peak_source": "%s copy bandwidth" % pk["src"]})
        out.append(line)
        print(json.dumps(line), flush=True)

    A = torch.empty(E, de + dt_, device=dev)
    timed("k_gather_time_encode", E * (de * 4 + 4 + 4 + (de + dt_) * 4), 0,
          lambda: ops.gather_time_encode(E, f=table, f_idx=eid, dt=dts, w=w, b=b, out=A),
          "E=%d rows of [f(%d) | cos(%d)]" % (E, de, dt_))
    att_b = 4 * (Nd * D + 2 * E * D + (Nd + 1) + Nd * D + E * H)
    timed("k_attn_fwd (bulk-copy path)", att_b, 0,
          lambda: ops.attn_fwd(q, kv[:, :D], kv[:, D:], rptr, H, 0.2, 0.1, 1, 2),
          "Nd=%d, E=%d, D=%d, H=%d, dropout 0.1" % (Nd, E, D, H))
    agg, att = ops.attn_fwd(q, kv[:, :D], kv[:, D:], rptr, H, 0.2, 0.1, 1, 2)
    dkv = torch.empty(E, 2 * D, device=dev)
    bwd_b = 4 * (2 * Nd * D + 2 * E * D + E * H + (Nd + 1) + 2 * E * D + Nd * D)
    timed("k_attn_bwd (bulk-copy path)", bwd_b, 0,
          lambda: ops.attn_bwd(q, kv[:, :D], kv[:, D:], rptr, att, dagg, H, 0.2, 0.1, 1, 2, dkv=dkv),
          "Nd=%d, E=%d, D=%d, H=%d, dropout 0.1" % (Nd, E, D, H))
    y = torch.empty_like(z)
    o = torch.empty_like(z)
    timed("k_tail_fwd", E * D * 4 * 3 + 8 * D, 0,
          lambda: ops.layer_tail_fwd(z, gamma, beta, drop_p=0.1, seed=5, y=y, out=o),
          "rows=%d, D=%d, dropout 0.1" % (E, D))
    dg, dbb = torch.zeros(D, device=dev), torch.zeros(D, device=dev)
    dz = torch.empty_like(z)
    timed("k_tail_bwd", E * D * 4 * 3 + 12 * D, 0,
          lambda: ops.layer_tail_bwd(z, y, gamma, dg, dbb, drop_p=0.1, dz=dz),
          "rows=%d, D=%d" % (E, D))
    dw_, db_ = torch.zeros(dt_, device=dev), torch.zeros(dt_, device=dev)
    timed("k_te_bwd", E * (dt_ + 1) * 4, 0,
          lambda: ops.time_encode_bwd(dA, dts, w, b, dw_, db_),
          "rows=%d, dtime=%d" % (E, dt_))
    W_kv = torch.randn(2 * D, de + dt_, device=dev, generator=g) * 0.05
    b_kv = torch.zeros(2 * D, device=dev)
    KV = torch.empty(E, 2 * D, device=dev)
    timed("k_gemm_group (K|V projection, NT)", 0, 2 * E * 2 * D * (de + dt_),
          lambda: ops.gemm_group([dict(kind=ops.NT, A=A, B=W_kv, bias=b_kv, out=KV)]),
          "M=%d, N=%d, K=%d" % (E, 2 * D, de + dt_))
    gW = torch.zeros(2 * D, de + dt_, device=dev)
    gb = torch.zeros(2 * D, device=dev)
    timed("k_gemm_group (K|V weight + bias gradient, TN)", 0, 2 * E * 2 * D * (de + dt_ + 1),
          lambda: ops.gemm_group([dict(kind=ops.TN, A=dkv, B=A, out=gW, accumulate=True, db=gb)]),
          "M=%d, N=%d, K=%d+1" % (E, 2 * D, de + dt_))
    dAt = torch.empty(E, dt_, device=dev)
    timed("k_gemm_group (time-encoding input gradient, NN)", 0, 2 * E * dt_ * 2 * D,
          lambda: ops.gemm_group([dict(kind=ops.NN, A=dkv, B=W_kv[:, de:], out=dAt)]),
          "M=%d, N=%d, K=%d" % (E, dt_, 2 * D))
    return 0


def run_bf16_suite(args):
    """The bf16 precision mode's kernels alone at config 5's hop-2 sizes (132 k
    destinations x fan-out 10 = 1.32 M edges; node features 413-d from a
    16,700-row table, edge features 186-d from a 4 M-row table, both bf16 with
    rows padded to 8 columns; 100-d time encoding; D = 100).  The K|V
    projection rows are [h (416) | f (192) | cos (100)] = 708 bf16 columns."""
    import torch
    from fast_b200 import ops
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    pk = peaks()
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    Nd, fan, D, dn, de, dt_ = int(132_000 * args.suite_scale), 10, 100, 413, 186, 100
    E = Nd * fan
    rows_tab = args.suite_table_rows or int(4_000_000 * args.suite_scale)
    ntab = torch.zeros(16_700, ops.pad8(dn), device=dev, dtype=torch.bfloat16)
    ntab[:, :dn] = torch.randn(16_700, dn, device=dev, generator=g)
    etab = torch.zeros(rows_tab, ops.pad8(de), device=dev, dtype=torch.bfloat16)
    etab[:, :de] = torch.randn(rows_tab, de, device=dev, generator=g)
    nid = torch.randint(0, 16_700, (E,), device=dev, generator=g, dtype=torch.int32)
    eid = torch.randint(0, rows_tab, (E,), device=dev, generator=g, dtype=torch.int32)
    dts = torch.rand(E, device=dev, generator=g) * 1e5
    w = (1.0 / 10 ** torch.linspace(0, 9, dt_, device=dev)).contiguous()
    b = torch.zeros(dt_, device=dev)
    (h_at, f_at, t_at), K = ops.bf16_layout(dn, de, dt_)
    X = torch.empty(E, ops.pad8(K), device=dev, dtype=torch.bfloat16)
    out = []

    def timed(name, nbytes, flops, fn, shape):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clock = clock_sampler(0)
        clock.start()
        s0.record()
        for _ in range(10):
            fn()
        s1.record()
        torch.cuda.synchronize()
        clocks = clock.stop()
        us = s0.elapsed_time(s1) * 100.0
        line = {"suite": "bf16", "kernel": name, "shape": shape, "us_per_launch": round(us, 2),
                "bytes_per_launch": int(nbytes), "clocks": clocks}
        gbs = nbytes / us / 1e3
        line.update({"achieved_GB_s": round(gbs, 1), "hbm_frac": round(gbs / pk["hbm"], 3)})
        if flops:
            tfs = flops / us / 1e6
            line.update({"TFLOP_s": round(tfs, 2), "peak_TFLOP_s": pk["tf"], "tensor_frac": round(tfs / pk["tf"], 4)})
        line["peak_source"] = "%s (copy bandwidth, bf16 dense burst)" % pk["src"]
        out.append(line)
        print(json.dumps(line), flush=True)

    timed("k_gather_time_encode_bf16", E * (2 * K + 2 * 416 + 2 * 192 + 12), 0,
          lambda: ops.gather_time_encode_bf16(E, h=ntab, h_idx=nid, f=etab, f_idx=eid, dt=dts, w=w, b=b, out=X,
                                              dn=dn, de=de),
          "E=%d rows of [h(%d) | f(%d) | cos(%d)] bf16" % (E, dn, de, dt_))
    Wb = torch.zeros(2 * D, ops.pad8(K), device=dev, dtype=torch.bfloat16)
    Wb[:, :K] = torch.randn(2 * D, K, device=dev, generator=g) * 0.05
    bkv = torch.zeros(2 * D, device=dev)
    KV = torch.empty(E, 2 * D, device=dev, dtype=torch.bfloat16)      # K|V stored as bf16, as in the step
    timed("k_bf_group (K|V projection, NT, bf16 output)", E * (2 * K + 2 * 2 * D), 2 * E * 2 * D * K,
          lambda: ops.gemm_bf16_group([dict(kind=ops.NT, A=X[:, :K], B=Wb[:, :K], bias=bkv, out=KV)]),
          "M=%d, N=%d, K=%d" % (E, 2 * D, K))
    dkv = (torch.randn(E, 2 * D, device=dev, generator=g)).to(torch.bfloat16)
    gW = torch.zeros(2 * D, dn + de + dt_, device=dev)
    gb = torch.zeros(2 * D, device=dev)
    tn = [dict(kind=ops.TN, A=dkv, B=X[:, :K], out=gW, accumulate=True, db=gb,
               segs=[(h_at, dn, 0), (f_at, de, dn), (t_at, dt_, dn + de)])]
    timed("k_bf_group (K|V weight + bias gradient, TN over the row's 3 segments)", E * (2 * K + 2 * 2 * D),
          2 * E * 2 * D * (dn + de + dt_ + 1),
          lambda: ops.gemm_bf16_group(tn), "M=%d, N=%d, K=%d+%d+%d+1" % (E, 2 * D, dn, de, dt_))
    # layer 0 of the step: the projection rows gathered inside the GEMM from the tables (node rows by node
    # id, edge rows by edge id) plus the time-encoding block, which alone is written
    T, _ = ops.gather_time_encode_bf16(E, dt=dts, w=w, b=b, device=dev)
    timed("k_gather_time_encode_bf16 (time encoding only)", E * (2 * 104 + 4), 0,
          lambda: ops.gather_time_encode_bf16(E, dt=dts, w=w, b=b, out=T),
          "E=%d rows of cos(%d) bf16" % (E, dt_))
    gat = ops.RowGather([(ntab, dn, nid, 448), (etab, de, eid, 192), (T, dt_, None, 128)])
    Wg = torch.zeros(2 * D, gat.K, device=dev, dtype=torch.bfloat16)
    for at, src_at, d in ((0, h_at, dn), (448, f_at, de), (640, t_at, dt_)):
        Wg[:, at:at + d] = Wb[:, src_at:src_at + d]
    timed("k_bf_group (K|V projection, NT, rows gathered from the tables)",
          gat.read_bytes(E) + 2 * 2 * D * gat.K + 2 * E * 2 * D, 2 * E * 2 * D * gat.K,
          lambda: ops.gemm_bf16_group([dict(kind=ops.NT, gather=gat, M=E, B=Wg, bias=bkv, out=KV)]),
          "M=%d, N=%d, K=%d (448 + 192 + 128)" % (E, 2 * D, gat.K))
    tng = [dict(kind=ops.TN, A=dkv, gather=gat, out=gW, accumulate=True, db=gb,
                segs=[(0, dn, 0), (448, de, dn), (640, dt_, dn + de)])]
    timed("k_bf_group (K|V weight + bias gradient, TN, rows gathered from the tables)",
          2 * E * 2 * D + gat.read_bytes(E) + 4 * 2 * D * (dn + de + dt_),
          2 * E * 2 * D * (dn + de + dt_ + 1), lambda: ops.gemm_bf16_group(tng),
          "M=%d, N=%d, K=%d+%d+%d+1" % (E, 2 * D, dn, de, dt_))
    # layer 0 of the step with the node product: the gather writes [f | cos] rows only, and the weight
    # gradient reads the node block from the table by source node (cp.async row copies)
    XF = torch.empty(E, ops.pad8(ops.pad8(de) + dt_), device=dev, dtype=torch.bfloat16)
    timed("k_gather_time_encode_bf16 ([f | cos] rows, node block left out)", E * (2 * XF.shape[1] + 2 * 192 + 12), 0,
          lambda: ops.gather_time_encode_bf16(E, f=etab, f_idx=eid, dt=dts, w=w, b=b, out=XF, de=de),
          "E=%d rows of [f(%d) | cos(%d)] bf16" % (E, de, dt_))
    gnr = ops.RowGather([(ntab, dn, nid, 448), (XF, ops.pad8(de) + dt_, None, 320)])
    tnr = [dict(kind=ops.TN, A=dkv, gather=gnr, out=gW, accumulate=True, db=gb,
                segs=[(0, dn, 0), (448, de, dn), (448 + ops.pad8(de), dt_, dn + de)])]
    timed("k_bf_group (K|V weight + bias gradient, TN, node rows by index + [f | cos] rows)",
          2 * E * 2 * D + gnr.read_bytes(E) + 4 * 2 * D * (dn + de + dt_),
          2 * E * 2 * D * (dn + de + dt_ + 1), lambda: ops.gemm_bf16_group(tnr),
          "M=%d, N=%d, K=%d+%d+%d+1" % (E, 2 * D, dn, de, dt_))
    # the weight gradient over the [f | cos] rows alone (the node block's gradient taken another way)
    tnf = [dict(kind=ops.TN, A=dkv, B=XF[:, :ops.pad8(de) + dt_], out=gW[:, dn:], accumulate=True, db=gb,
                segs=[(0, de, 0), (ops.pad8(de), dt_, de)])]
    timed("k_bf_group (K|V weight + bias gradient, TN over [f | cos] rows only)",
          2 * E * 2 * D + 2 * E * (ops.pad8(de) + dt_) + 4 * 2 * D * (de + dt_),
          2 * E * 2 * D * (de + dt_ + 1), lambda: ops.gemm_bf16_group(tnf),
          "M=%d, N=%d, K=%d+%d+1" % (E, 2 * D, de, dt_))
    # the same TN operand with the node block materialised: both segments read row by row by TMA
    XH = torch.empty(E, 448, device=dev, dtype=torch.bfloat16)
    XH[:, :416] = ntab[nid.long()]
    gtm = ops.RowGather([(XH, dn, None, 448), (XF, ops.pad8(de) + dt_, None, 320)])
    tnm = [dict(tnr[0], gather=gtm)]
    timed("k_bf_group (K|V weight + bias gradient, TN, [node rows | [f | cos] rows] both read row by row)",
          2 * E * 2 * D + gtm.read_bytes(E) + 4 * 2 * D * (dn + de + dt_),
          2 * E * 2 * D * (dn + de + dt_ + 1), lambda: ops.gemm_bf16_group(tnm),
          "M=%d, N=%d, K=%d+%d+%d+1" % (E, 2 * D, dn, de, dt_))
    del XH
    dAt = torch.empty(E, ops.pad8(dt_), device=dev, dtype=torch.bfloat16)[:, :dt_]   # bf16, as in the step
    timed("k_bf_group (time-encoding input gradient, NN, bf16 output)", E * (2 * 2 * D + 2 * dt_),
          2 * E * dt_ * 2 * D,
          lambda: ops.gemm_bf16_group([dict(kind=ops.NN, A=dkv, B=Wb[:, t_at:t_at + dt_], out=dAt)]),
          "M=%d, N=%d, K=%d" % (E, dt_, 2 * D))
    # the time-encoding backward on that gradient: its cost depends on how
    # many arguments w dt + b pass 2^22 (the double-precision reduction)
    dw_, db_ = torch.zeros(dt_, device=dev), torch.zeros(dt_, device=dev)
    for hi in (1e5, 4e6, 2e8):
        dth = torch.rand(E, device=dev, generator=g) * hi
        far = float(((dth[:, None] * w[None, :]).abs() >= 2.0 ** 22).float().mean())
        timed("k_te_bwd_vec (bf16 gradient, dt uniform below %.0e)" % hi, E * (2 * dt_ + 4), 0,
              lambda: ops.time_encode_bwd(dAt, dth, w, b, dw_, db_),
              "rows=%d, dtime=%d, %.1f%% of arguments past 2^22" % (E, dt_, 100 * far))
    q = torch.randn(Nd, D, device=dev, generator=g) * 0.5
    kvf = torch.randn(E, 2 * D, device=dev, generator=g) * 0.5
    rptr = torch.arange(0, E + 1, fan, device=dev, dtype=torch.int32)
    agg, att = ops.attn_fwd(q, kvf[:, :D], kvf[:, D:], rptr, 2, 0.2, 0.1, 1, 2)
    dagg = torch.randn(Nd, D, device=dev, generator=g)
    timed("k_attn_bwd (bulk-copy path, bf16 dK|dV)",
          4 * (2 * Nd * D + 2 * E * D + E * 2 + (Nd + 1) + Nd * D) + 2 * 2 * E * D, 0,
          lambda: ops.attn_bwd_bf16kv(q, kvf[:, :D], kvf[:, D:], rptr, att, dagg, 2, 0.2, 0.1, 1, 2),
          "Nd=%d, E=%d, D=%d, H=2, dropout 0.1" % (Nd, E, D))
    # the step's attention: bf16 K|V rows in, bf16 dK|dV out
    kvb = kvf.to(torch.bfloat16)
    timed("k_attn_fwd (bulk-copy path, bf16 K|V rows)", 4 * (Nd * D + (Nd + 1) + Nd * D + E * 2) + 2 * 2 * E * D,
          0, lambda: ops.attn_fwd_kvbf16(q, kvb, rptr, 2, 0.2, 0.1, 1, 2),
          "Nd=%d, E=%d, D=%d, H=2, dropout 0.1" % (Nd, E, D))
    timed("k_attn_bwd (bulk-copy path, bf16 K|V rows and dK|dV)",
          4 * (2 * Nd * D + E * 2 + (Nd + 1) + Nd * D) + 2 * 4 * E * D, 0,
          lambda: ops.attn_bwd_kvbf16(q, kvb, rptr, att, dagg, 2, 0.2, 0.1, 1, 2),
          "Nd=%d, E=%d, D=%d, H=2, dropout 0.1" % (Nd, E, D))
    return 0


def data_label(args, cfg):
    if args.data:
        return "dataset %s read from edges.csv + ext_full.npz; seeded random features" % cfg.name
    if args.edges:
        return "synthetic (seeded, %s shapes; a %d-edge graph drawn like the config's)" % (cfg.name, cfg.edges)
    return "synthetic (seeded, %s shapes)" % cfg.name


def workload_graph(args, cfg, device=True):
    """The config's synthetic graph, or the dataset of --data (the config then
    takes that graph's node and edge counts).  device: build the bf16 configs'
    graphs on the current GPU (config 5: 191 M edges in seconds)."""
    import dataclasses
    from fast_b200.data import make_graph, make_graph_device
    if args.batch:
        cfg = dataclasses.replace(cfg, batch=args.batch)
    if not args.data:
        n = args.edges or cfg.edges
        cfg = dataclasses.replace(cfg, edges=n)
        if device and cfg.dtype == "bf16":
            import torch
            return make_graph_device(cfg, torch.device("cuda", torch.cuda.current_device())), cfg
        return make_graph(cfg, n_edges=n), cfg
    from fast_b200.dataio import load_graph
    g = load_graph(args.data)
    return g, dataclasses.replace(cfg, name=os.path.basename(os.path.normpath(args.data)), nodes=g.n_nodes,
                                  edges=len(g.src))


def _host(a):
    """A numpy copy of an edge-list slice (numpy array or device tensor)."""
    return a.cpu().numpy() if hasattr(a, "cpu") else np.asarray(a)


def main():
    args = parse()
    if args.warmup < 3:
        args.warmup = 3
    if args.gemm == "ffma":
        os.environ["FB_GEMM"] = "ffma"          # read by fb_gemm_group at every call
    if args.suite == "kernels":
        return run_kernel_suite(args)
    if args.suite == "bf16":
        return run_bf16_suite(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_fast(args)


if __name__ == "__main__":
    sys.exit(main())
