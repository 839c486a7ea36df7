"""GPU: TGN node memory on the device (fb_mem_gather, the GRU gate kernels and
grouped GEMMs, fb_mailbox_update_self, fb_memory_update) trained through
FusedStep, against the reference's own four-step TGN-1 run recorded by
tests/golden/make_memory_golden.py.

Step 0 (identical inputs): loss, predictions' gradients and the memory /
mailbox tables meet the parity criterion against an fp64 run of the oracle
(oracle/memory_math.py, pinned to the same fixture by test_oracle_memory).
Every step: loss, gradients and tables within rtol 2e-4 / atol 2e-5 of the
reference (two fp32 trajectories separate by rounding after an SGD step);
memory and mail timestamps are exact.  The CUDA-graph replay of a memory
step equals the same step run eagerly on the same static blocks, bit for bit.
The same for APAN-1 (fb_mail_slots_gather, the slot attention on the shared
attention kernels, fb_add_layernorm_*, fb_mailbox_update_neighbors), whose
next-slot table is also exact.
"""
import os

import numpy as np
import pytest
import torch

from conftest import parity

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "memory_golden.npz")


def _golden(case="tgn1"):
    gold = np.load(GOLDEN)
    return {k.split("/", 1)[1]: gold[k] for k in gold.files if k.startswith(case + "/")}


def _graph(g):
    from fast_b200.data import TemporalGraph
    E = g["graph/src"].shape[0]
    return TemporalGraph(src=g["graph/src"], dst=g["graph/dst"], ts=g["graph/t"], indptr=g["graph/indptr"],
                         indices=g["graph/indices"], eid=g["graph/eid"], ts_csr=g["graph/ts"],
                         n_nodes=int(g["params"][0]), train_end=E, val_end=E)


def _params(g):
    N, de, steps, B, B0, DM, DT = (int(x) for x in g["params"])
    sp = dict(layer=1, neighbor=[10], strategy="recent", prop_time=False, history=1, duration=0)
    mp = dict(type="node", dim_time=DT, deliver_to="self", mail_combine="last", memory_update="gru",
              mailbox_size=1, combine_node_feature=True, dim_out=DM)
    gp = dict(arch="transformer_attention", layer=1, att_head=2, dim_time=DT, dim_out=DM)
    tp = dict(lr=float(g["lr"][0]), dropout=0.0, att_dropout=0.0)
    return sp, mp, gp, tp, steps, B


def _load_params(model, g):
    sd = {k.split("/", 1)[1]: torch.from_numpy(v) for k, v in g.items() if k.startswith("param0/")}
    model.load_state_dict(sd)


def _close(got, ref32, name):
    torch.testing.assert_close(got.detach().float().cpu(), torch.as_tensor(ref32), rtol=2e-4, atol=2e-5,
                               msg=lambda m: "%s: %s" % (name, m))


def _oracle_step0(g):
    """fp64 oracle run of step 0: loss, grads, tables after the writes."""
    from oracle import memory_math, ref_math
    from oracle.sampler import OracleSampler
    from fast_b200.memory import MemoryModel
    sp, mp, gp, tp, steps, B = _params(g)
    N, de = int(g["params"][0]), int(g["params"][1])
    m = MemoryModel(0, de, sp, mp, gp, tp)
    _load_params(m, g)
    m = m.double()
    st = memory_math.MemoryState(N, mp["dim_out"], de, dtype=torch.float64)
    s = OracleSampler(g["graph/indptr"], g["graph/indices"], g["graph/eid"], g["graph/ts"], 1, 1, 1, [10], True,
                      False, 1, 0.0)
    roots, rts = g["step0/roots"], g["step0/rts"]
    s.sample(roots, rts)
    ef = torch.from_numpy(g["edge_feats"])
    pos, neg, h = memory_math.model_forward(m, st, s.get_ret()[0], ef)
    loss = ref_math.bce_loss(pos, neg)
    loss.backward()
    b0 = int(g["step0/e0"][0])
    memory_math.update_mailbox_self(st, roots, rts, h, ef[b0:b0 + len(roots) // 3])
    memory_math.update_memory(st, roots, rts, h)
    return loss.detach(), {n: p.grad for n, p in m.named_parameters()}, st


def test_tgn_training_matches_reference(cuda):
    from fast_b200.train import Trainer
    g = _golden()
    sp, mp, gp, tp, steps, B = _params(g)
    ef = torch.from_numpy(g["edge_feats"]).to(cuda)
    tr = Trainer(_graph(g), None, ef, sp, mp, gp, tp, cuda, fused=True)
    _load_params(tr.model, g)
    tr.opt = torch.optim.SGD(tr.model.parameters(), lr=tp["lr"])
    loss64, grads64, st64 = _oracle_step0(g)
    mb = tr.mailbox
    for step in range(steps):
        q = "step%d/" % step
        roots = torch.from_numpy(g[q + "roots"]).to(cuda)
        rts = torch.from_numpy(g[q + "rts"]).to(cuda)
        loss = tr.step_device(roots, rts, e0=int(g[q + "e0"][0]))
        _close(loss.reshape(1), g[q + "loss"], q + "loss")
        for n_, p in tr.model.named_parameters():
            key = q + "grad/" + n_
            if key in g:
                _close(p.grad, g[key], key)
                if step == 0:
                    parity(p.grad, grads64[n_], torch.from_numpy(g[key]), key)
        for name in ("node_memory", "mailbox"):
            _close(getattr(mb, name), g[q + name], q + name)
        assert torch.equal(mb.node_memory_ts.cpu(), torch.from_numpy(g[q + "node_memory_ts"])), step
        assert torch.equal(mb.mailbox_ts.cpu(), torch.from_numpy(g[q + "mailbox_ts"])), step
        if step == 0:
            parity(loss.reshape(1), loss64.reshape(1), torch.from_numpy(g[q + "loss"]), "step0 loss")
            parity(mb.node_memory, st64.node_memory, torch.from_numpy(g[q + "node_memory"]), "step0 memory")
            parity(mb.mailbox, st64.mailbox, torch.from_numpy(g[q + "mailbox"]), "step0 mailbox")


def test_tgn_graph_replay_is_the_static_eager_step(cuda):
    from fast_b200.train import GraphTrainer
    g = _golden()
    sp, mp, gp, tp, steps, B = _params(g)
    ef = torch.from_numpy(g["edge_feats"]).to(cuda)
    mk = lambda: GraphTrainer(_graph(g), None, ef, dict(sp), mp, dict(gp), tp, cuda, batch=B,  # noqa: E731
                              optimizer="sgd")
    graph, static = mk(), mk()
    _load_params(graph.model, g)
    _load_params(static.model, g)
    roots0 = torch.from_numpy(g["step0/roots"]).to(cuda)
    rts0 = torch.from_numpy(g["step0/rts"]).to(cuda)
    for tr in (graph, static):
        tr.roots_buf.copy_(roots0)
        tr.ts_buf.copy_(rts0)
        tr.e0_buf.fill_(int(g["step0/e0"][0]))
    graph.capture()                          # three eager warm-up steps on step 0's batch, then capture
    for _ in range(3):
        static._eager_step()
    for step in range(1, steps):
        q = "step%d/" % step
        roots = torch.from_numpy(g[q + "roots"]).to(cuda)
        rts = torch.from_numpy(g[q + "rts"]).to(cuda)
        e0 = int(g[q + "e0"][0])
        lg = float(graph.step_device(roots, rts, e0=e0))
        static.roots_buf.copy_(roots)
        static.ts_buf.copy_(rts)
        static.e0_buf.fill_(e0)
        static._eager_step()
        assert lg == float(static.loss_buf), step
        for name in ("node_memory", "node_memory_ts", "mailbox", "mailbox_ts"):
            assert torch.equal(getattr(graph.mailbox, name), getattr(static.mailbox, name)), (step, name)
    for (n, pg), ps in zip(graph.model.named_parameters(), static.model.parameters()):
        assert torch.equal(pg, ps), n


def _apan_params(g):
    N, de, steps, B, B0, DM, DT, S = (int(x) for x in g["params"])
    sp = dict(layer=1, neighbor=[10], strategy="recent", prop_time=False, history=1, duration=0, no_neg=True)
    mp = dict(type="node", dim_time=DT, deliver_to="neighbors", mail_combine="last", memory_update="transformer",
              attention_head=2, mailbox_size=S, combine_node_feature=False, dim_out=DM)
    gp = dict(arch="identity")
    tp = dict(lr=float(g["lr"][0]), dropout=0.0, att_dropout=0.0)
    return sp, mp, gp, tp, steps, B


def test_apan_training_matches_reference(cuda):
    from fast_b200.train import Trainer
    g = _golden("apan1")
    sp, mp, gp, tp, steps, B = _apan_params(g)
    ef = torch.from_numpy(g["edge_feats"]).to(cuda)
    tr = Trainer(_graph(g), None, ef, sp, mp, dict(gp), tp, cuda, fused=True)
    _load_params(tr.model, g)
    tr.opt = torch.optim.SGD(tr.model.parameters(), lr=tp["lr"])
    mb = tr.mailbox
    for step in range(steps):
        q = "step%d/" % step
        roots = torch.from_numpy(g[q + "roots"]).to(cuda)
        rts = torch.from_numpy(g[q + "rts"]).to(cuda)
        loss = tr.step_device(roots, rts, e0=int(g[q + "e0"][0]))
        _close(loss.reshape(1), g[q + "loss"], q + "loss")
        _close(tr.engine.last_memory, g[q + "updated_memory"], q + "updated_memory")
        for n_, p in tr.model.named_parameters():
            key = q + "grad/" + n_
            if key in g:
                _close(p.grad, g[key], key)
        for name in ("node_memory", "mailbox"):
            _close(getattr(mb, name), g[q + name], q + name)
        assert torch.equal(mb.node_memory_ts.cpu(), torch.from_numpy(g[q + "node_memory_ts"])), step
        assert torch.equal(mb.mailbox_ts.cpu(), torch.from_numpy(g[q + "mailbox_ts"])), step
        assert torch.equal(mb.next_mail_pos.cpu().long(), torch.from_numpy(g[q + "next_mail_pos"]).long()), step


def test_apan_graph_replay_is_the_static_eager_step(cuda):
    from fast_b200.train import GraphTrainer
    g = _golden("apan1")
    sp, mp, gp, tp, steps, B = _apan_params(g)
    ef = torch.from_numpy(g["edge_feats"]).to(cuda)
    mk = lambda: GraphTrainer(_graph(g), None, ef, dict(sp), mp, dict(gp), tp, cuda, batch=B,  # noqa: E731
                              optimizer="sgd")
    graph, static = mk(), mk()
    _load_params(graph.model, g)
    _load_params(static.model, g)
    for tr in (graph, static):
        tr.roots_buf.copy_(torch.from_numpy(g["step0/roots"]).to(cuda))
        tr.ts_buf.copy_(torch.from_numpy(g["step0/rts"]).to(cuda))
        tr.e0_buf.fill_(int(g["step0/e0"][0]))
    graph.capture()
    for _ in range(3):
        static._eager_step()
    for step in range(1, steps):
        q = "step%d/" % step
        roots = torch.from_numpy(g[q + "roots"]).to(cuda)
        rts = torch.from_numpy(g[q + "rts"]).to(cuda)
        e0 = int(g[q + "e0"][0])
        lg = float(graph.step_device(roots, rts, e0=e0))
        static.roots_buf.copy_(roots)
        static.ts_buf.copy_(rts)
        static.e0_buf.fill_(e0)
        static._eager_step()
        assert lg == float(static.loss_buf), step
        for name in ("node_memory", "node_memory_ts", "mailbox", "mailbox_ts", "next_mail_pos"):
            assert torch.equal(getattr(graph.mailbox, name), getattr(static.mailbox, name)), (step, name)
