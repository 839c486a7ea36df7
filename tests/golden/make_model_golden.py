"""Writes tests/golden/model_golden.npz by running the REFERENCE model code.

Run in the build container, where the reference tree is readable:

    python tests/golden/make_model_golden.py

It imports the reference's own layers.py / modules.py / fast_util (read in
place, never copied) and runs one forward + backward of GeneralModel on the
CPU with dropout off, on blocks from the reference sampler built from source
(oracle/_ref).  Three things the reference needs and this container lacks are
stood in for:
  * dgl (not vendored by the reference, README.md:13): a block object with
    srcdata/dstdata/edata and the two operators the DGL path uses,
    ops.edge_softmax (softmax over each destination's in-edges) and
    update_all(copy_u|copy_edge, sum) (sum of messages into destinations),
    written here from DGL's documented semantics;
  * fastAgg: an empty module -- with fast_esm = fast_agg = 0 the reference
    never calls it;
  * torch.device('cuda:0') inside layers.py: mapped to the CPU.
The feature gather follows prepare_input (utils.py:126-196) directly.
"""
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))
from oracle.paths import REF_ROOT as REF  # noqa: E402

from conftest import small_graph  # noqa: E402
from oracle.sampler import load_reference  # noqa: E402


# ---------------------------------------------------------------- stand-in for dgl
class _Frame(dict):
    pass


class FakeBlock:
    def __init__(self, src, dst, num_src_nodes, num_dst_nodes):
        self._src = torch.as_tensor(np.asarray(src)).long()
        self._dst = torch.as_tensor(np.asarray(dst)).long()
        self._ns, self._nd = int(num_src_nodes), int(num_dst_nodes)
        self.srcdata, self.dstdata, self.edata = _Frame(), _Frame(), _Frame()

    def edges(self):
        return self._src, self._dst

    def num_src_nodes(self):
        return self._ns

    def num_dst_nodes(self):
        return self._nd

    def num_edges(self):
        return int(self._src.numel())

    def to(self, *a, **k):
        return self

    def update_all(self, msg, red):
        kind, field, _ = msg
        vals = self.srcdata[field][self._src] if kind == "u" else self.edata[field]
        out = torch.zeros((self._nd,) + tuple(vals.shape[1:]), dtype=vals.dtype)
        self.dstdata[red[2]] = out.index_add(0, self._dst, vals)


def _edge_softmax(block, x):
    dst = block.edges()[1]
    H = x.shape[1]
    mx = torch.full((block.num_dst_nodes(), H), -float("inf"), dtype=x.dtype)
    mx = mx.scatter_reduce(0, dst.unsqueeze(1).expand(-1, H), x, "amax", include_self=True)
    ex = torch.exp(x - mx[dst].detach())
    s = torch.zeros((block.num_dst_nodes(), H), dtype=x.dtype).index_add(0, dst, ex)
    return ex / s[dst]


def install_fakes():
    dgl = types.ModuleType("dgl")
    dgl.create_block = lambda e, num_src_nodes, num_dst_nodes, **k: FakeBlock(e[0], e[1], num_src_nodes,
                                                                              num_dst_nodes)
    dgl.ops = types.SimpleNamespace(edge_softmax=_edge_softmax)
    dgl.function = types.SimpleNamespace(copy_u=lambda f, o: ("u", f, o), copy_edge=lambda f, o: ("e", f, o),
                                         sum=lambda m, o: ("sum", m, o))
    sys.modules["dgl"] = dgl
    sys.modules["fastAgg"] = types.ModuleType("fastAgg")
    ts = types.ModuleType("torch_scatter")
    ts.scatter = None
    sys.modules["torch_scatter"] = ts


class _TorchOnCpu:
    """torch, except that device('cuda:0') means the CPU."""

    def __getattr__(self, k):
        if k == "device":
            return lambda *a, **kw: torch.device("cpu")
        return getattr(torch, k)


# ---------------------------------------------------------------- case
def run_case(out, name, layers, fanout, dn, de, seed):
    import layers as ref_layers
    import modules as ref_modules
    from fast_util.efficientGOP import fm
    ref_layers.torch = _TorchOnCpu()
    fm.fastESMFlag = fm.fastAggFlag = fm.CSR_OUT = 0
    fm.fastKQV = fm.fastTIME = fm.fastDrop = 0
    g = small_graph(n_nodes=150, n_edges=4000, seed=seed, int_ts=False, t_max=2e4, zipf=1.0)
    torch.manual_seed(seed)
    nf = torch.randn(150, dn) if dn else None
    ef = torch.randn(4000, de) if de else None
    sp = dict(layer=layers, neighbor=list(fanout), strategy="recent", prop_time=False, history=1, duration=0)
    mp = dict(type="none", dim_out=0)
    gp = dict(arch="transformer_attention", layer=layers, att_head=2, dim_time=100, dim_out=100)
    tp = dict(lr=1e-4, dropout=0.0, att_dropout=0.0)
    model = ref_modules.GeneralModel(dn, de, sp, mp, gp, tp)
    ref = load_reference()
    s = ref.ParallelSampler(g["indptr"], g["indices"], g["eid"], g["ts"], 1, 1, layers, list(fanout), True, False,
                            1, 0.0)
    rng = np.random.default_rng(seed)
    B, b0 = 40, 2500
    roots = np.concatenate([g["src"][b0:b0 + B], g["dst"][b0:b0 + B], rng.integers(0, 150, B).astype(np.int32)])
    rts = np.concatenate([g["t"][b0:b0 + B]] * 3).astype(np.float32)
    s.sample(roots, rts, [])
    ret = s.get_ret()
    mfgs = []
    for r in ret:        # utils.py:67-87 (to_dgl_blocks)
        b = FakeBlock(r.col(), r.row(), r.dim_in(), r.dim_out())
        b.srcdata["ID"] = torch.from_numpy(r.nodes())
        b.edata["dt"] = torch.from_numpy(r.dts())[b.num_dst_nodes():]
        b.srcdata["ts"] = torch.from_numpy(r.ts())
        b.edata["ID"] = torch.from_numpy(r.eid())
        mfgs.append([b])
    mfgs.reverse()
    if nf is not None:   # utils.py:126-196 (prepare_input)
        for b in mfgs[0]:
            b.srcdata["h"] = nf[b.srcdata["ID"].long()].float()
    if ef is not None:
        for mfg in mfgs:
            for b in mfg:
                if b.num_src_nodes() > b.num_dst_nodes():
                    b.edata["f"] = ef[b.edata["ID"].long()].float()
    pred_pos, pred_neg = model(mfgs)
    crit = torch.nn.BCEWithLogitsLoss()
    loss = crit(pred_pos, torch.ones_like(pred_pos)) + crit(pred_neg, torch.zeros_like(pred_neg))
    loss.backward()
    p = name + "/"
    out[p + "params"] = np.array([layers, dn, de] + list(fanout), np.int64)
    for k, v in model.state_dict().items():
        out[p + "param/" + k] = v.numpy()
    for n, prm in model.named_parameters():
        if prm.grad is not None:
            out[p + "grad/" + n] = prm.grad.numpy()
    if nf is not None:
        out[p + "node_feats"] = nf.numpy()
    if ef is not None:
        out[p + "edge_feats"] = ef.numpy()
    for i, r in enumerate(ret):
        for k in ("row", "col", "eid", "ts", "dts", "nodes"):
            out[p + "block%d/%s" % (i, k)] = getattr(r, k)()
        out[p + "block%d/dims" % i] = np.array([r.dim_in(), r.dim_out()], np.int64)
    out[p + "roots"] = roots
    out[p + "rts"] = rts
    out[p + "pred_pos"] = pred_pos.detach().numpy()
    out[p + "pred_neg"] = pred_neg.detach().numpy()
    out[p + "loss"] = np.array([float(loss)], np.float32)
    out[p + "graph/indptr"] = g["indptr"]
    out[p + "graph/indices"] = g["indices"]
    out[p + "graph/eid"] = g["eid"]
    out[p + "graph/ts"] = g["ts"]


def main():
    if not os.path.isdir(REF):
        raise SystemExit("reference tree not found")
    install_fakes()
    sys.path.insert(0, REF)
    out = {}
    run_case(out, "tgat2_edge", 2, (8, 5), 0, 40, 11)
    run_case(out, "tgat1_node_edge", 1, (10,), 32, 24, 12)
    run_case(out, "tgat2_node_edge", 2, (6, 4), 16, 20, 13)
    path = os.path.join(HERE, "model_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, len(out), "arrays")


if __name__ == "__main__":
    main()
