"""Seeded synthetic temporal graphs with the shapes of the benchmark configs.

The reference trains on LASTFM / WIKITALK / GDELT-style datasets that are not
available offline; these generators stand in for them with the same node and
edge counts, feature widths and endpoint distributions.  The graph layout
follows the reference preprocessing contract (fast_util/preprocess/gen_graph.py):
  * edge id = chronological row index, timestamps float32 and non-decreasing;
  * CSR keyed by the source node only (no reverse edges, gen_graph.py:35-42);
  * every node's adjacency list sorted by timestamp (gen_graph.py:57-76) --
    here by a stable sort of the chronological edge list on the source id;
  * 70/15/15 chronological train/val/test split (txt2csv.py:44-49).
"""
import dataclasses

import numpy as np
import torch


@dataclasses.dataclass
class WorkloadConfig:
    name: str
    nodes: int
    edges: int
    src: tuple
    dst: tuple
    t_max: float
    t_int: bool
    d_node: int
    d_edge: int
    feat: str               # 'normal' | 'zeros'
    model: str              # reference config file stem
    strategy: str           # 'recent' | 'uniform'
    fanout: tuple
    batch: int
    dtype: str = "fp32"
    sharded: bool = False   # the global batch is `batch`, split across the ranks (else `batch` per rank)


CONFIGS = {
    1: WorkloadConfig("tgat1_lastfm_like", 2_000, 1_300_000, ("zipf", 1.1), ("uniform",), 1.4e8, True, 100, 100,
                      "zeros", "TGAT-1", "recent", (10,), 600),
    2: WorkloadConfig("tgat2_wikitalk_like", 1_140_000, 7_830_000, ("powerlaw", 2.1), ("uniform",), 2e8, False,
                      0, 172, "normal", "TGAT", "uniform", (10, 10), 600),
    3: WorkloadConfig("tgn1_synthetic", 10_000, 1_500_000, ("uniform",), ("uniform",), 2e8, False, 0, 172,
                      "normal", "TGN-1", "recent", (10,), 600),
    4: WorkloadConfig("apan1_synthetic", 50_000, 3_000_000, ("zipf", 1.2), ("zipf", 1.2), 2e8, False, 0, 100,
                      "normal", "APAN-1", "recent", (10,), 600),
    5: WorkloadConfig("tgat2_gdelt_like", 16_700, 191_000_000, ("zipf", 1.05), ("zipf", 1.05), 2e8, False, 413, 186,
                      "normal", "TGAT", "recent", (10, 10), 4000, "bf16", True),
}


def _zipf_ids(rng, n_nodes, s, count):
    """Ids with P(rank k) ~ k^-s over a finite support, ranks shuffled onto ids."""
    w = np.arange(1, n_nodes + 1, dtype=np.float64) ** (-s)
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    ranks = np.searchsorted(cdf, rng.random(count), side="right")
    ranks = np.minimum(ranks, n_nodes - 1)
    perm = rng.permutation(n_nodes).astype(np.int32)
    return perm[ranks]


def endpoints(rng, n_nodes, count, spec):
    kind = spec[0]
    if kind == "uniform":
        return rng.integers(0, n_nodes, count, dtype=np.int64).astype(np.int32)
    if kind == "zipf":
        return _zipf_ids(rng, n_nodes, spec[1], count)
    if kind == "powerlaw":
        # out-degree tail exponent alpha <=> rank-frequency exponent 1/(alpha-1)
        return _zipf_ids(rng, n_nodes, 1.0 / (spec[1] - 1.0), count)
    raise ValueError(kind)


@dataclasses.dataclass
class TemporalGraph:
    """The chronological edge list and its CSR, as numpy arrays or (a graph
    built on the device) as device tensors."""
    src: np.ndarray
    dst: np.ndarray
    ts: np.ndarray          # float32, chronological
    indptr: np.ndarray      # int32 [N+1]
    indices: np.ndarray     # int32 [E]
    eid: np.ndarray         # int32 [E]
    ts_csr: np.ndarray      # float32 [E]
    n_nodes: int
    train_end: int
    val_end: int


def make_graph(cfg, seed=42, n_edges=None):
    """Builds the CSR of `cfg` (optionally only its first n_edges edges)."""
    rng = np.random.default_rng(seed)
    E = cfg.edges if n_edges is None else int(n_edges)
    N = cfg.nodes
    src = endpoints(rng, N, E, cfg.src)
    dst = endpoints(rng, N, E, cfg.dst)
    if cfg.t_int:
        ts = np.sort(rng.integers(0, int(cfg.t_max) + 1, E)).astype(np.float32)
    else:
        ts = np.sort(rng.random(E) * cfg.t_max).astype(np.float32)
    order = np.argsort(src, kind="stable")
    indptr = np.zeros(N + 1, dtype=np.int64)
    np.add.at(indptr, src.astype(np.int64) + 1, 1)
    indptr = np.cumsum(indptr).astype(np.int32)
    return TemporalGraph(src=src, dst=dst, ts=ts, indptr=indptr, indices=dst[order].astype(np.int32),
                         eid=order.astype(np.int32), ts_csr=ts[order], n_nodes=N,
                         train_end=int(E * 0.70), val_end=int(E * 0.85))


def _zipf_ids_device(gen, n_nodes, s, count, device, chunk=1 << 25):
    """_zipf_ids on the device: inverse CDF of P(rank k) ~ k^-s by a search of
    uniform draws, ranks shuffled onto ids."""
    w = torch.arange(1, n_nodes + 1, device=device, dtype=torch.float64) ** (-s)
    cdf = torch.cumsum(w, 0)
    cdf /= cdf[-1].clone()
    perm = torch.randperm(n_nodes, device=device, generator=gen).to(torch.int32)
    out = torch.empty(count, device=device, dtype=torch.int32)
    for c0 in range(0, count, chunk):
        c1 = min(count, c0 + chunk)
        u = torch.rand(c1 - c0, device=device, dtype=torch.float64, generator=gen)
        ranks = torch.searchsorted(cdf, u, right=True).clamp_(max=n_nodes - 1)
        out[c0:c1] = perm[ranks]
    return out


def make_graph_device(cfg, device, seed=42, n_edges=None):
    """make_graph's construction on the device, for graphs too large to build
    on the host in seconds (config 5: 191 M edges): Zipf endpoints, sorted
    float32 timestamps, the CSR by a stable sort of the chronological edge
    list on the source id.  Every array (the CSR and the chronological src,
    dst and ts) stays a device tensor: at 191 M edges a host copy per rank
    would cost 2.3 GB of host memory for each process.  Draws come from
    torch's device generator, so the graph differs from make_graph's for the
    same seed."""
    E = cfg.edges if n_edges is None else int(n_edges)
    N = cfg.nodes
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)

    def ends(spec):
        if spec[0] == "uniform":
            return torch.randint(0, N, (E,), device=device, dtype=torch.int32, generator=gen)
        if spec[0] == "zipf":
            return _zipf_ids_device(gen, N, spec[1], E, device)
        if spec[0] == "powerlaw":
            return _zipf_ids_device(gen, N, 1.0 / (spec[1] - 1.0), E, device)
        raise ValueError(spec[0])

    src = ends(cfg.src)
    dst = ends(cfg.dst)
    ts = torch.rand(E, device=device, generator=gen, dtype=torch.float32) * cfg.t_max
    if cfg.t_int:
        ts = ts.floor_()
    ts = torch.sort(ts).values
    _, order = torch.sort(src, stable=True)
    counts = torch.bincount(src, minlength=N)
    indptr = torch.zeros(N + 1, device=device, dtype=torch.int64)
    indptr[1:] = torch.cumsum(counts, 0)
    indices = dst[order]
    ts_csr = ts[order]
    eid = order.to(torch.int32)
    del order
    return TemporalGraph(src=src, dst=dst, ts=ts,
                         indptr=indptr.to(torch.int32), indices=indices, eid=eid, ts_csr=ts_csr, n_nodes=N,
                         train_end=int(E * 0.70), val_end=int(E * 0.85))


def make_features_bf16(cfg, n_edges, device, seed=7):
    """(node_feats, edge_feats) as bf16 device tables with rows padded with
    zeros to a multiple of 8 columns (the bf16 projection mode's layout),
    seeded N(0, 1) values from fb_fill_normal_bf16 (None where the width is 0)."""
    from .capi import call, ptr, stream_ptr

    def mk(rows, cols, salt):
        if cols == 0:
            return None
        ld = (cols + 7) // 8 * 8
        t = torch.empty(rows, ld, device=device, dtype=torch.bfloat16)
        if cfg.feat == "zeros":
            t.zero_()
        else:
            call("fb_fill_normal_bf16", ptr(t), rows, cols, ld, seed * 1000003 + salt, stream_ptr())
        return t

    return mk(cfg.nodes, cfg.d_node, 1), mk(n_edges, cfg.d_edge, 2)


def make_features(cfg, n_edges, device, seed=7, dtype=torch.float32):
    """(node_feats, edge_feats) tensors on `device` (None where the width is 0)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def mk(rows, cols):
        if cols == 0:
            return None
        if cfg.feat == "zeros":
            return torch.zeros(rows, cols, device=device, dtype=dtype)
        return torch.randn(rows, cols, device=device, dtype=dtype, generator=g)

    return mk(cfg.nodes, cfg.d_node), mk(n_edges, cfg.d_edge)


def model_params(cfg):
    """(sample_param, memory_param, gnn_param, train_param) of the reference
    config file cfg.model (config/*.yml), with the CLI overrides of train.py:98."""
    layers = len(cfg.fanout)
    sample = dict(layer=layers, neighbor=list(cfg.fanout), strategy=cfg.strategy, prop_time=False, history=1,
                  duration=0)
    memory = dict(type="none", dim_out=0)
    gnn = dict(arch="transformer_attention", layer=layers, att_head=2, dim_time=100, dim_out=100)
    train = dict(lr=0.0001, dropout=0.1, att_dropout=0.1)
    if cfg.model.startswith("TGN"):
        memory = dict(type="node", dim_time=100, deliver_to="self", mail_combine="last", memory_update="gru",
                      mailbox_size=1, combine_node_feature=True, dim_out=100)
        train = dict(lr=0.0001, dropout=0.2, att_dropout=0.2)
    elif cfg.model.startswith("APAN"):
        # config/APAN-1.yml: sampling without negatives, transformer memory, identity GNN
        sample["no_neg"] = True
        memory = dict(type="node", dim_time=100, deliver_to="neighbors", mail_combine="last",
                      memory_update="transformer", attention_head=2, mailbox_size=10, combine_node_feature=False,
                      dim_out=100)
        gnn = dict(arch="identity")
        train = dict(lr=0.0001, dropout=0.1, att_dropout=0.1)
    return sample, memory, gnn, train
