"""GPU: the CUDA-graph trainer (capacity-sized static blocks, sizes read on
the device, whole step replayed).

* A replayed step is bit for bit the same step run eagerly on the same
  static blocks, step after step, with uniform sampling and attention dropout
  on (both keyed by device-side counters that every replay advances).
* Against the eager trainer (host-sized blocks) it trains the same: equal
  losses and parameters within fp32 rounding over several steps.  The graph
  here spans a short time range, because TGAT's time encoding cos(w*dt + b)
  with dt ~ 1e5 turns a 1e-8 change in w into a different phase, and the
  two paths round some sums (torch's LayerNorm backward over capacity rows)
  in a different order.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(cuda, t_max, strategy="uniform", att_dropout=0.2):
    from fast_b200.data import WorkloadConfig, make_graph
    cfg = WorkloadConfig("small", 400, 40000, ("zipf", 1.1), ("uniform",), t_max, False, 0, 48, "normal", "TGAT",
                         strategy, (8, 6), 64)
    g = make_graph(cfg, seed=3)
    ef = torch.randn(cfg.edges, cfg.d_edge, generator=torch.Generator().manual_seed(1)).to(cuda)
    sp = dict(layer=2, neighbor=[8, 6], strategy=strategy, prop_time=False, history=1, duration=0)
    mp = dict(type="none", dim_out=0)
    gp = dict(arch="transformer_attention", layer=2, att_head=2, dim_time=100, dim_out=100)
    tp = dict(lr=1e-3, dropout=0.0, att_dropout=att_dropout)
    return cfg, g, ef, sp, mp, gp, tp


@pytest.mark.parametrize("mode", ["fused", "module", "fused_bf16"])
def test_graph_replay_is_the_static_eager_step(cuda, mode):
    from fast_b200.train import GraphTrainer
    cfg, g, ef, sp, mp, gp, tp = _setup(cuda, 1e5)
    fused = mode != "module"
    if fused:
        tp["dropout"] = 0.1            # keyed by the model's device counter, replay-safe
    prec = "bf16" if mode == "fused_bf16" else "fp32"
    mk = lambda: GraphTrainer(g, None, ef, dict(sp), mp, dict(gp), tp, cuda, batch=cfg.batch, seed=5,  # noqa: E731
                              sampler_seed=77, optimizer="sgd", fused=fused, precision=prec)
    graph, static = mk(), mk()
    B = cfg.batch
    starts = [10000 + i * B for i in range(7)]
    graph.load_device_roots(starts[0], starts[0] + B)
    r0, t0 = graph.roots_buf.clone(), graph.ts_buf.clone()
    graph.capture()                      # three eager warm-up steps on batch 0, then capture
    for _ in range(3):
        static.roots_buf.copy_(r0)
        static.ts_buf.copy_(t0)
        static._eager_step()
    for b0 in starts[1:]:
        graph.load_device_roots(b0, b0 + B)
        static.roots_buf.copy_(graph.roots_buf)
        static.ts_buf.copy_(graph.ts_buf)
        lg = float(graph.step_device())
        static._eager_step()
        assert lg == float(static.loss_buf)
    for (n, pg), ps in zip(graph.model.named_parameters(), static.model.parameters()):
        assert torch.equal(pg, ps), n


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("strategy", ["recent", "uniform"])
def test_graph_trainer_matches_eager_trainer(cuda, strategy, fused):
    """The graph trainer (capacity-sized blocks, counts on the device) trains
    like the eager one (exact-sized blocks), loss for loss.  The two round
    differently -- the products of capacity- and exact-sized blocks split their
    sums differently -- so the ReLU inputs are moved off the kink (biases of
    w_out and of the predictor's two projections + 4): a pre-activation within
    rounding of 0 would otherwise switch a whole gradient term between them."""
    from fast_b200.train import GraphTrainer, Trainer
    cfg, g, ef, sp, mp, gp, tp = _setup(cuda, 2e3, strategy)
    if fused:
        tp["dropout"] = 0.1            # same Philox-keyed tail dropout on both paths
    eager = Trainer(g, None, ef, dict(sp), mp, dict(gp), tp, cuda, seed=5, sampler_seed=77, fused=fused)
    eager.opt = torch.optim.SGD(eager.model.parameters(), lr=tp["lr"])
    graph = GraphTrainer(g, None, ef, dict(sp), mp, dict(gp), tp, cuda, batch=cfg.batch, seed=5, sampler_seed=77,
                         optimizer="sgd", fused=fused)
    with torch.no_grad():
        for tr in (eager, graph):
            for name, p in tr.model.named_parameters():
                if name.endswith(("w_out.bias", "src_fc.bias", "dst_fc.bias")):
                    p += 4.0
    B = cfg.batch
    starts = [10000 + i * B for i in range(7)]
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


def test_pipelined_host_steps_equal_synchronous_ones(cuda):
    """step_host_pipelined (inputs through two pinned slots, each loss read one
    call later) trains exactly like step_host, loss for loss."""
    import numpy as np
    from fast_b200.train import GraphTrainer
    cfg, g, ef, sp, mp, gp, tp = _setup(cuda, 2e3)
    mk = lambda: GraphTrainer(g, None, ef, dict(sp), mp, dict(gp), tp, cuda, batch=cfg.batch, seed=5,  # noqa: E731
                              sampler_seed=77, optimizer="adam")
    sync, pipe = mk(), mk()
    B = cfg.batch
    rng = np.random.default_rng(3)
    batches = []
    for i in range(6):
        b0 = 10000 + i * B
        t = g.ts[b0:b0 + B]
        roots = np.concatenate([g.src[b0:b0 + B], g.dst[b0:b0 + B], rng.integers(0, g.n_nodes, B).astype(np.int32)])
        batches.append((roots.astype(np.int32), np.concatenate([t, t, t]).astype(np.float32)))
    want = [sync.step_host(r, t) for r, t in batches]
    got = [pipe.step_host_pipelined(r, t) for r, t in batches]
    assert got[0] is None
    got = got[1:] + [pipe.finish_pipelined()]
    assert got == want
    assert pipe.finish_pipelined() is None
