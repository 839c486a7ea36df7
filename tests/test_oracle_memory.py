"""CPU: the TGN node-memory oracle (oracle/memory_math.py) pinned against the
reference's own memorys.py / modules.py, recorded by
tests/golden/make_memory_golden.py: four consecutive TGN-1 training steps
(GRU updater, mailbox of one, deliver_to 'self') with SGD, dropout off,
blocks from the reference sampler built from source.

The APAN-1 case (transformer updater over a mailbox of 10, delivery to the
sampled neighbours, identity LayerNorm layer, no_neg sampling) is checked
the same way; its next-slot table matches exactly.

The oracle sampler reproduces each step's block bit for bit.  Step 0 (same
inputs on both sides): losses, predictions, the updated memory, every
gradient and the memory / mailbox tables after the writes meet the parity
criterion against an fp64 run of the oracle (rtol 1e-5 / atol 1e-6, or as
accurate as the reference's fp32 values).  Later steps check the state
carried across batches: after an SGD step the two fp32 trajectories
(oracle, reference) separate by rounding, so every step is also compared
directly with the reference at rtol 2e-4 / atol 2e-5.  Memory and
mail timestamps are copies of input times and match exactly throughout.
"""
import os

import numpy as np
import torch

from conftest import parity
from oracle import memory_math, ref_math
from oracle.sampler import OracleSampler

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "memory_golden.npz")


def load(case="tgn1"):
    gold = np.load(GOLDEN)
    return {k.split("/", 1)[1]: gold[k] for k in gold.files if k.startswith(case + "/")}


def build_model(g, dtype=torch.float32):
    from fast_b200.memory import MemoryModel
    N, de, steps, B, B0, DM, DT = (int(x) for x in g["params"])
    sp = dict(layer=1, neighbor=[10], strategy="recent", prop_time=False, history=1, duration=0)
    mp = dict(type="node", dim_time=DT, deliver_to="self", mail_combine="last", memory_update="gru",
              mailbox_size=1, combine_node_feature=True, dim_out=DM)
    gp = dict(arch="transformer_attention", layer=1, att_head=2, dim_time=DT, dim_out=DM)
    tp = dict(lr=float(g["lr"][0]), dropout=0.0, att_dropout=0.0)
    m = MemoryModel(0, de, sp, mp, gp, tp)
    m.load_state_dict({k.split("/", 1)[1]: torch.from_numpy(v) for k, v in g.items() if k.startswith("param0/")})
    return m.to(dtype), dict(N=N, de=de, steps=steps, B=B, B0=B0, DM=DM, DT=DT)


def check(step, got, ref64, ref32, name):
    """Every step: close to the reference's value (a bug shared by the fp32
    and fp64 oracle runs cannot pass); step 0 also the parity criterion."""
    torch.testing.assert_close(got.float(), ref32, rtol=2e-4, atol=2e-5, msg=lambda m: "%s: %s" % (name, m))
    if step == 0:
        parity(got, ref64, ref32, name)


def test_memory_oracle_matches_reference():
    """fp32 and fp64 oracle runs step in lockstep; each fp32 quantity must be
    as accurate against the fp64 run as the reference's own fp32 value."""
    g = load()
    m32, c = build_model(g)
    m64, _ = build_model(g, torch.float64)
    ef = torch.from_numpy(g["edge_feats"])
    st32 = memory_math.MemoryState(c["N"], c["DM"], c["de"])
    st64 = memory_math.MemoryState(c["N"], c["DM"], c["de"], dtype=torch.float64)
    lr = float(g["lr"][0])
    opts = [torch.optim.SGD(m32.parameters(), lr=lr), torch.optim.SGD(m64.parameters(), lr=lr)]
    s = OracleSampler(g["graph/indptr"], g["graph/indices"], g["graph/eid"], g["graph/ts"], 1, 1, 1, [10], True,
                      False, 1, 0.0)
    for step in range(c["steps"]):
        q = "step%d/" % step
        roots, rts = g[q + "roots"], g[q + "rts"]
        s.sample(roots, rts)
        blk = s.get_ret()[0]
        for k in ("row", "col", "eid", "ts", "dts", "nodes"):
            assert np.array_equal(getattr(blk, k)(), g[q + "block/" + k]), (step, k)
        outs = []
        for m, st, opt in ((m32, st32, opts[0]), (m64, st64, opts[1])):
            opt.zero_grad()
            pos, neg, h = memory_math.model_forward(m, st, blk, ef)
            loss = ref_math.bce_loss(pos, neg)
            loss.backward()
            outs.append(dict(loss=loss.reshape(1).detach(), pred_pos=pos.detach(), pred_neg=neg.detach(),
                             updated_memory=h.detach()))
        grads64 = dict(m64.named_parameters())
        pairs = [(outs[0][k], outs[1][k], q + k) for k in ("loss", "pred_pos", "pred_neg", "updated_memory")]
        pairs += [(prm.grad, grads64[n_].grad, q + "grad/" + n_) for n_, prm in m32.named_parameters()
                  if q + "grad/" + n_ in g]
        for got, ref64, key in pairs:
            check(step, got, ref64, torch.from_numpy(g[key]), key)
        b0 = int(g[q + "e0"][0])
        for m, st, opt, o in ((m32, st32, opts[0], outs[0]), (m64, st64, opts[1], outs[1])):
            opt.step()
            memory_math.update_mailbox_self(st, roots, rts, o["updated_memory"], ef[b0:b0 + len(roots) // 3])
            memory_math.update_memory(st, roots, rts, o["updated_memory"])
        for name in ("node_memory", "mailbox"):
            check(step, getattr(st32, name), getattr(st64, name), torch.from_numpy(g[q + name]), q + name)
        assert torch.equal(st32.node_memory_ts, torch.from_numpy(g[q + "node_memory_ts"])), step
        assert torch.equal(st32.mailbox_ts, torch.from_numpy(g[q + "mailbox_ts"])), step


def build_apan(g, dtype=torch.float32):
    from fast_b200.memory import MemoryModel
    N, de, steps, B, B0, DM, DT, S = (int(x) for x in g["params"])
    sp = dict(layer=1, neighbor=[10], strategy="recent", prop_time=False, history=1, duration=0, no_neg=True)
    mp = dict(type="node", dim_time=DT, deliver_to="neighbors", mail_combine="last", memory_update="transformer",
              attention_head=2, mailbox_size=S, combine_node_feature=False, dim_out=DM)
    tp = dict(lr=float(g["lr"][0]), dropout=0.0, att_dropout=0.0)
    m = MemoryModel(0, de, sp, mp, dict(arch="identity"), tp)
    m.load_state_dict({k.split("/", 1)[1]: torch.from_numpy(v) for k, v in g.items() if k.startswith("param0/")})
    return m.to(dtype), dict(N=N, de=de, steps=steps, B=B, B0=B0, DM=DM, DT=DT, S=S)


def test_apan_oracle_matches_reference():
    g = load("apan1")
    m32, c = build_apan(g)
    m64, _ = build_apan(g, torch.float64)
    ef = torch.from_numpy(g["edge_feats"])
    st32 = memory_math.MemoryState(c["N"], c["DM"], c["de"], c["S"])
    st64 = memory_math.MemoryState(c["N"], c["DM"], c["de"], c["S"], dtype=torch.float64)
    lr = float(g["lr"][0])
    opts = [torch.optim.SGD(m32.parameters(), lr=lr), torch.optim.SGD(m64.parameters(), lr=lr)]
    s = OracleSampler(g["graph/indptr"], g["graph/indices"], g["graph/eid"], g["graph/ts"], 1, 1, 1, [10], True,
                      False, 1, 0.0)
    for step in range(c["steps"]):
        q = "step%d/" % step
        roots, rts = g[q + "roots"], g[q + "rts"]
        n = len(roots) // 3
        s.sample(roots[:2 * n], rts[:2 * n])            # no_neg: the positive roots only
        blk = s.get_ret()[0]
        for k in ("row", "col", "eid", "ts", "dts", "nodes"):
            assert np.array_equal(getattr(blk, k)(), g[q + "block/" + k]), (step, k)
        outs = []
        for m, st, opt in ((m32, st32, opts[0]), (m64, st64, opts[1])):
            opt.zero_grad()
            pos, neg, h = memory_math.apan_forward(m, st, roots, rts)
            loss = ref_math.bce_loss(pos, neg)
            loss.backward()
            outs.append(dict(loss=loss.reshape(1).detach(), updated_memory=h.detach()))
        grads64 = dict(m64.named_parameters())
        pairs = [(outs[0][k], outs[1][k], q + k) for k in ("loss", "updated_memory")]
        pairs += [(prm.grad, grads64[n_].grad, q + "grad/" + n_) for n_, prm in m32.named_parameters()
                  if q + "grad/" + n_ in g]
        for got, ref64, key in pairs:
            check(step, got, ref64, torch.from_numpy(g[key]), key)
        b0 = int(g[q + "e0"][0])
        for m, st, opt, o in ((m32, st32, opts[0], outs[0]), (m64, st64, opts[1], outs[1])):
            opt.step()
            memory_math.update_mailbox_neighbors(st, roots, rts, o["updated_memory"], ef[b0:b0 + n], blk.nodes(),
                                                 blk.row())
            memory_math.update_memory(st, roots, rts, o["updated_memory"])
        for name in ("node_memory", "mailbox"):
            check(step, getattr(st32, name), getattr(st64, name), torch.from_numpy(g[q + name]), q + name)
        assert torch.equal(st32.node_memory_ts, torch.from_numpy(g[q + "node_memory_ts"])), step
        assert torch.equal(st32.mailbox_ts, torch.from_numpy(g[q + "mailbox_ts"])), step
        assert torch.equal(st32.next_mail_pos, torch.from_numpy(g[q + "next_mail_pos"]).long()), step
