"""GPU: a whole training step (sample -> gather/time-encode -> Q/K/V ->
softmax/aggregate -> w_out/LayerNorm -> edge predictor -> BCE -> backward)
on the device path against the CPU oracle (reference sampler restatement +
fp32 restatement of layers.py/modules.py) with identical parameters.
Dropout is off so the two paths compute the same function.

Tolerance: rtol 1e-5 / atol 1e-6 on predictions, loss and every parameter
gradient, except the time-encoding frequency gradient, a sum of E terms
each scaled by dt, which is held to the fp32 summation bound of that sum.
"""
import copy

import numpy as np
import pytest
import torch

from conftest import small_graph
from oracle import ref_math
from oracle.sampler import OracleSampler

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-5, 1e-6

CASES = {
    # name: (layers, fanout, strategy-recent, d_node, d_edge)
    "tgat2_edge_feats": (2, [10, 10], 0, 172),
    "tgat1_node_and_edge": (1, [10], 100, 100),
    "tgat2_node_and_edge": (2, [6, 4], 64, 48),
}


def _grads(model):
    return {n: (p.grad.detach().cpu().clone() if p.grad is not None else None) for n, p in model.named_parameters()}


@pytest.mark.parametrize("case", sorted(CASES))
def test_train_step_matches_oracle(cuda, case):
    from fast_b200.ext import sampler_core
    from fast_b200.model import DeviceBlock, GeneralModel
    layers, fanout, dn, de = CASES[case]
    n_nodes, n_edges = 300, 30000
    g = small_graph(n_nodes=n_nodes, n_edges=n_edges, seed=21, int_ts=False, t_max=2e4, zipf=1.0)
    torch.manual_seed(1)
    nf = torch.randn(n_nodes, dn) if dn else None
    ef = torch.randn(n_edges, de) if de else None
    sp = dict(layer=layers, neighbor=fanout, strategy="recent", prop_time=False, history=1, duration=0)
    gnn = dict(arch="transformer_attention", layer=layers, att_head=2, dim_time=100, dim_out=100)
    tr = dict(lr=1e-4, dropout=0.0, att_dropout=0.0)
    m_cpu = GeneralModel(dn, de, sp, dict(type="none", dim_out=0), gnn, tr)
    m_gpu = copy.deepcopy(m_cpu).to(cuda)
    crit = torch.nn.BCEWithLogitsLoss()
    dev = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    smp = sampler_core.ParallelSampler(dev(g["indptr"]), dev(g["indices"]), dev(g["eid"]), dev(g["ts"]), 1, 1,
                                       layers, fanout, True, False, 1, 0.0)
    ora = OracleSampler(g["indptr"], g["indices"], g["eid"], g["ts"], 1, 1, layers, fanout, True, False, 1, 0.0)
    nf_d = nf.to(cuda) if nf is not None else None
    ef_d = ef.to(cuda) if ef is not None else None
    rng = np.random.default_rng(0)
    B = 200
    worst = {}
    for bt, b0 in enumerate(range(5000, 5000 + 3 * B, B)):
        src, dst, t = g["src"][b0:b0 + B], g["dst"][b0:b0 + B], g["t"][b0:b0 + B]
        roots = np.concatenate([src, dst, rng.integers(0, n_nodes, B).astype(np.int32)])
        rts = np.concatenate([t, t, t]).astype(np.float32)
        smp.sample_device(dev(roots), dev(rts))
        blocks = [DeviceBlock(v, d) for v, d in zip(smp.block_views(), smp.dims())]
        ora.sample(roots, rts)
        m_gpu.zero_grad()
        pp, pn = m_gpu(blocks, nf_d, ef_d)
        loss_g = crit(pp, torch.ones_like(pp)) + crit(pn, torch.zeros_like(pn))
        loss_g.backward()
        m_cpu.zero_grad()
        rp, rn = ref_math.model_forward(m_cpu, ora.get_ret(), nf, ef)
        loss_c = ref_math.bce_loss(rp, rn)
        loss_c.backward()
        torch.testing.assert_close(pp.detach().cpu(), rp.detach(), rtol=RTOL, atol=ATOL)
        torch.testing.assert_close(pn.detach().cpu(), rn.detach(), rtol=RTOL, atol=ATOL)
        torch.testing.assert_close(loss_g.detach().cpu(), loss_c.detach(), rtol=RTOL, atol=ATOL)
        gg, gc = _grads(m_gpu), _grads(m_cpu)
        for name in gc:
            a, b = gg[name], gc[name]
            if b is None:
                assert a is None or torch.count_nonzero(a) == 0, name
                continue
            err = (a - b).abs()
            worst[name] = max(worst.get(name, 0.0), float((err / (ATOL + RTOL * b.abs())).max()))
            if name.endswith("time_enc.w.weight"):
                # sum over edges of -sin(w dt + b) * dt * g: fp32 summation bound
                bound = b.abs() * 0 + float(b.abs().max()) * 1e-4 + ATOL
                assert bool((err <= bound + RTOL * b.abs()).all()), (name, float(err.max()))
            else:
                torch.testing.assert_close(a, b, rtol=RTOL, atol=ATOL, msg=lambda m: "%s: %s" % (name, m))
        with torch.no_grad():
            for p in m_cpu.parameters():
                p.add_(torch.randn_like(p) * 1e-3)
            for pc, pg in zip(m_cpu.parameters(), m_gpu.parameters()):
                pg.copy_(pc)
    print("worst err/tol ratio per parameter (%s):" % case,
          {k: round(v, 3) for k, v in sorted(worst.items(), key=lambda kv: -kv[1])[:6]})
