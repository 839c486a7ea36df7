"""GPU: the CUDA-graph trainer (capacity-sized static blocks, sizes read on
the device, whole step replayed) trains exactly like the eager trainer
(host-sized blocks): same losses and parameters step after step, with uniform
sampling and attention dropout on, both keyed by device-side counters that
every replay advances.  Plain SGD keeps the comparison tight: Adam turns
1e-7 differences in near-zero gradients (summation order differs between
host-sized and capacity-sized launches) into +-lr parameter steps.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _graph(seed=3):
    from fast_b200.data import WorkloadConfig, make_graph
    cfg = WorkloadConfig("small", 400, 40000, ("zipf", 1.1), ("uniform",), 1e5, False, 0, 48, "normal", "TGAT",
                         "uniform", (8, 6), 64)
    return cfg, make_graph(cfg, seed=seed)


def test_graph_replay_matches_eager(cuda):
    from fast_b200.train import GraphTrainer, Trainer
    cfg, g = _graph()
    ef = torch.randn(cfg.edges, cfg.d_edge, generator=torch.Generator().manual_seed(1)).to(cuda)
    sp = dict(layer=2, neighbor=[8, 6], strategy="uniform", prop_time=False, history=1, duration=0)
    mp = dict(type="none", dim_out=0)
    gp = dict(arch="transformer_attention", layer=2, att_head=2, dim_time=100, dim_out=100)
    tp = dict(lr=1e-3, dropout=0.0, att_dropout=0.2)
    eager = Trainer(g, None, ef, sp, mp, dict(gp), tp, cuda, seed=5, sampler_seed=77)
    eager.opt = torch.optim.SGD(eager.model.parameters(), lr=tp["lr"])
    graph = GraphTrainer(g, None, ef, sp, mp, dict(gp), tp, cuda, batch=cfg.batch, seed=5, sampler_seed=77,
                         optimizer="sgd")
    B = cfg.batch
    starts = [10000 + i * B for i in range(8)]
    # warm-up / capture: the graph trainer runs three eager steps on batch 0
    graph.load_device_roots(starts[0], starts[0] + B)
    roots0, ts0 = graph.roots_buf.clone(), graph.ts_buf.clone()
    graph.capture()
    for _ in range(3):
        eager.step_device(roots0, ts0)
    for b0 in starts[1:]:
        graph.load_device_roots(b0, b0 + B)
        roots, ts = graph.roots_buf.clone(), graph.ts_buf.clone()
        lg = float(graph.step_device())
        le = float(eager.step_device(roots, ts))
        assert abs(lg - le) <= 1e-5 * abs(le) + 1e-6, (lg, le)
    for (n, pe), pg in zip(eager.model.named_parameters(), graph.model.parameters()):
        torch.testing.assert_close(pg, pe, rtol=1e-4, atol=1e-6, msg=lambda m: "%s: %s" % (n, m))
