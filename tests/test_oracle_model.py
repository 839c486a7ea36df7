"""CPU: the model-math oracle (oracle/ref_math.py) pinned against outputs of
the reference's own layers.py / modules.py, recorded by
tests/golden/make_model_golden.py (one forward + backward of GeneralModel,
dropout off, blocks from the reference sampler built from source).

Both sides are fp32 CPU PyTorch; the tolerance is the north-star bound,
rtol 1e-5 / atol 1e-6, on predictions, loss and every parameter gradient.
"""
import os

import numpy as np
import pytest
import torch

from oracle import ref_math
from oracle.sampler import OracleBlock, OracleSampler

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "model_golden.npz")
RTOL, ATOL = 1e-5, 1e-6


def load_case(gold, name):
    g = {k.split("/", 1)[1]: gold[k] for k in gold.files if k.startswith(name + "/")}
    return g


def build(g):
    from fast_b200.model import GeneralModel
    layers, dn, de = (int(x) for x in g["params"][:3])
    fanout = [int(x) for x in g["params"][3:]]
    sp = dict(layer=layers, neighbor=fanout, strategy="recent", prop_time=False, history=1, duration=0)
    gp = dict(arch="transformer_attention", layer=layers, att_head=2, dim_time=100, dim_out=100)
    tp = dict(lr=1e-4, dropout=0.0, att_dropout=0.0)
    m = GeneralModel(dn, de, sp, dict(type="none", dim_out=0), gp, tp)
    sd = {k.split("/", 1)[1]: torch.from_numpy(v) for k, v in g.items() if k.startswith("param/")}
    m.load_state_dict(sd)
    nf = torch.from_numpy(g["node_feats"]) if "node_feats" in g else None
    ef = torch.from_numpy(g["edge_feats"]) if "edge_feats" in g else None
    return m, nf, ef, layers, fanout


def golden_blocks(g, layers):
    blocks = []
    for i in range(layers):
        arr = {k: g["block%d/%s" % (i, k)] for k in ("row", "col", "eid", "ts", "dts", "nodes")}
        din, dout = (int(x) for x in g["block%d/dims" % i])
        blocks.append(OracleBlock(arr["row"], arr["col"], arr["eid"], arr["ts"], arr["dts"], arr["nodes"],
                                  np.zeros(0, np.int32), np.zeros(0, np.int32), np.zeros(0, np.int32), din, dout))
    return blocks


@pytest.mark.parametrize("case", ["tgat2_edge", "tgat1_node_edge", "tgat2_node_edge"])
def test_ref_math_matches_reference_layers(case):
    gold = np.load(GOLDEN)
    g = load_case(gold, case)
    m, nf, ef, layers, fanout = build(g)
    # the oracle sampler reproduces the reference blocks
    s = OracleSampler(g["graph/indptr"], g["graph/indices"], g["graph/eid"], g["graph/ts"], 1, 1, layers, fanout,
                      True, False, 1, 0.0)
    s.sample(g["roots"], g["rts"])
    for i, b in enumerate(s.get_ret()):
        for k in ("row", "col", "eid", "ts", "dts", "nodes"):
            np.testing.assert_array_equal(getattr(b, k)(), g["block%d/%s" % (i, k)])
    pp, pn = ref_math.model_forward(m, golden_blocks(g, layers), nf, ef)
    loss = ref_math.bce_loss(pp, pn)
    loss.backward()
    torch.testing.assert_close(pp.detach(), torch.from_numpy(g["pred_pos"]), rtol=RTOL, atol=ATOL)
    torch.testing.assert_close(pn.detach(), torch.from_numpy(g["pred_neg"]), rtol=RTOL, atol=ATOL)
    torch.testing.assert_close(loss.detach().reshape(1), torch.from_numpy(g["loss"]), rtol=RTOL, atol=ATOL)
    n_grads = 0
    for n, p in m.named_parameters():
        key = "grad/" + n
        if key in g:
            torch.testing.assert_close(p.grad, torch.from_numpy(g[key]), rtol=RTOL, atol=ATOL,
                                       msg=lambda msg: "%s: %s" % (n, msg))
            n_grads += 1
    assert n_grads >= 10
