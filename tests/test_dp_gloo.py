"""CPU, two gloo ranks: the data-parallel logic of fast_b200.train.

* Each rank takes a contiguous slice of the chronological batch, samples it,
  runs the model and calls average_gradients (one all-reduce of a flat
  bucket); the result must equal the mean over slices of the per-slice
  gradients computed in one process.
* Failure detection without a GPU: a rank that raises before the collective
  makes its peer's all-reduce end with an error under a short process-group
  timeout, instead of hanging.
* The node-memory exchange of data-parallel TGN (gather_global_order): every
  rank's [src_r | dst_r | neg_r] rows come back in the global batch's order
  [src | dst | neg], on every rank, for id, time and memory-row tensors.
* APAN's neighbour delivery (gather_neighbor_block_global): the ranks' blocks
  for their positive roots, padded to a shared capacity, become the block
  one process sampling the global positive roots lists -- edge nodes and
  each edge's global root row in the same order, and the edge count.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _setup():
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from conftest import small_graph
    from fast_b200.model import GeneralModel
    g = small_graph(n_nodes=120, n_edges=6000, seed=4, int_ts=False, t_max=1e4, zipf=1.0)
    torch.manual_seed(0)
    ef = torch.randn(6000, 24)
    sp = dict(layer=2, neighbor=[6, 4], strategy="recent", prop_time=False, history=1, duration=0)
    gp = dict(arch="transformer_attention", layer=2, att_head=2, dim_time=100, dim_out=100)
    tp = dict(lr=1e-3, dropout=0.0, att_dropout=0.0)
    model = GeneralModel(0, 24, sp, dict(type="none", dim_out=0), gp, tp)
    return g, ef, model


def _slice_grads(g, ef, model, lo, hi, neg_seed):
    from oracle import ref_math
    from oracle.sampler import OracleSampler
    s = OracleSampler(g["indptr"], g["indices"], g["eid"], g["ts"], 1, 1, 2, [6, 4], True, False, 1, 0.0)
    neg = np.random.default_rng(neg_seed).integers(0, 120, hi - lo).astype(np.int32)
    roots = np.concatenate([g["src"][lo:hi], g["dst"][lo:hi], neg])
    rts = np.concatenate([g["t"][lo:hi]] * 3).astype(np.float32)
    s.sample(roots, rts)
    model.zero_grad()
    pp, pn = ref_math.model_forward(model, s.get_ret(), None, ef)
    ref_math.bce_loss(pp, pn).backward()


def _worker(rank, world, port, outdir, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    try:
        from fast_b200.train import average_gradients, slice_for_rank
        g, ef, model = _setup()
        lo, hi = slice_for_rank(3000, 3000 + 80, rank, world)
        _slice_grads(g, ef, model, lo, hi, neg_seed=100 + rank)
        if rank == fail_rank:
            raise RuntimeError("injected failure on rank %d" % rank)
        average_gradients(list(model.parameters()), world)
        torch.save({n: p.grad for n, p in model.named_parameters()}, os.path.join(outdir, "grads%d.pt" % rank))
        status = "ok"
    except RuntimeError as e:
        status = "error: " + str(e)[:200]
    with open(os.path.join(outdir, "status%d.txt" % rank), "w") as f:
        f.write(status)
    try:
        dist.destroy_process_group()
    except Exception:
        pass


def test_dp_average_equals_mean_of_slices(tmp_path):
    mp.spawn(_worker, args=(2, _port(), str(tmp_path), -1), nprocs=2, join=True)
    sys.path.insert(0, ROOT)
    from fast_b200.train import slice_for_rank
    for r in range(2):
        assert (tmp_path / ("status%d.txt" % r)).read_text() == "ok"
    g, ef, model = _setup()
    ref = None
    for r in range(2):
        lo, hi = slice_for_rank(3000, 3080, r, 2)
        _slice_grads(g, ef, model, lo, hi, neg_seed=100 + r)
        gr = {n: p.grad.clone() / 2 for n, p in model.named_parameters()}
        ref = gr if ref is None else {n: ref[n] + gr[n] for n in ref}
    for r in range(2):
        got = torch.load(str(tmp_path / ("grads%d.pt" % r)))
        for n in ref:
            torch.testing.assert_close(got[n], ref[n], rtol=1e-5, atol=1e-7)


def test_dp_failed_rank_is_detected(tmp_path):
    mp.spawn(_worker, args=(2, _port(), str(tmp_path), 1), nprocs=2, join=True)
    assert (tmp_path / "status1.txt").read_text().startswith("error: injected failure")
    s0 = (tmp_path / "status0.txt").read_text()
    assert s0.startswith("error"), s0      # the peer's all-reduce ended with an error, it did not hang


def _gather_worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        sys.path.insert(0, ROOT)
        from fast_b200.train import gather_global_order
        gB = 12
        roots = torch.arange(3 * gB, dtype=torch.int32) * 7 + 1        # a global [src | dst | neg] list
        ts = roots.float() / 3
        h = torch.stack([roots.float(), -roots.float()], 1)
        per = gB // world
        pick = lambda a: torch.cat([a[s * gB + rank * per:s * gB + (rank + 1) * per] for s in range(3)])  # noqa: E731
        outs = [gather_global_order(pick(t), world)[0] for t in (roots, ts, h)]
        ok = all(torch.equal(o, t) for o, t in zip(outs, (roots, ts, h)))
        # a second call reusing the buffers
        o2, _ = gather_global_order(pick(roots), world, out=torch.empty_like(roots), perm=None)
        ok = ok and torch.equal(o2, roots)
        status = "ok" if ok else "mismatch"
    except Exception as e:
        status = "error: " + str(e)[:200]
    with open(os.path.join(outdir, "gather%d.txt" % rank), "w") as f:
        f.write(status)
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_memory_exchange_restores_global_order(tmp_path, world):
    mp.spawn(_gather_worker, args=(world, _port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        assert (tmp_path / ("gather%d.txt" % r)).read_text() == "ok"


def _neighbor_worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        sys.path.insert(0, ROOT)
        from fast_b200.train import gather_neighbor_block_global
        gB, fan = 12, 4
        Br = gB // world
        g = torch.Generator().manual_seed(3)
        deg = torch.randint(0, fan + 1, (2 * gB,), generator=g)       # edges of each global positive root
        # the single-process block: edges in root order [src | dst]
        g_rows = torch.repeat_interleave(torch.arange(2 * gB), deg).to(torch.int32)
        g_nodes = torch.randint(0, 1000, (g_rows.numel(),), generator=g, dtype=torch.int32)
        starts = torch.cumsum(deg, 0) - deg
        # this rank's block: its src roots then its dst roots, local rows
        mine = [s * gB + rank * Br + t for s in range(2) for t in range(Br)]
        nodes, rows, rptr = [], [], [0]
        for j, gr in enumerate(mine):
            a, n = int(starts[gr]), int(deg[gr])
            nodes.append(g_nodes[a:a + n])
            rows.append(torch.full((n,), j, dtype=torch.int32))
            rptr.append(rptr[-1] + n)
        cap = 2 * Br * fan
        E = rptr[-1]
        ne = torch.full((cap,), -7, dtype=torch.int32)
        ro = torch.full((cap,), -9, dtype=torch.int32)
        ne[:E] = torch.cat(nodes)
        ro[:E] = torch.cat(rows)
        out_n, out_r, cnt = gather_neighbor_block_global(ne, ro, torch.tensor(rptr, dtype=torch.int32), Br, world)
        Et = g_rows.numel()
        ok = int(cnt[0]) == Et and torch.equal(out_n[:Et], g_nodes) and torch.equal(out_r[:Et], g_rows)
        status = "ok" if ok else "mismatch"
    except Exception as e:
        status = "error: " + str(e)[:200]
    with open(os.path.join(outdir, "nbr%d.txt" % rank), "w") as f:
        f.write(status)
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_neighbor_block_exchange_restores_global_order(tmp_path, world):
    mp.spawn(_neighbor_worker, args=(world, _port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        assert (tmp_path / ("nbr%d.txt" % r)).read_text() == "ok"
