"""Writes tests/golden/memory_golden.npz by running the REFERENCE TGN code.

Run in the build container, where the reference tree is readable:

    python tests/golden/make_memory_golden.py

It imports the reference's own modules.py / memorys.py / layers.py (read in
place, never copied) and trains a TGN-1 model (config/TGN-1.yml: GRU memory
updater, mailbox of one, deliver_to 'self', 'last' combine, one attention
layer) for four consecutive batches on the CPU, as train.py:315-391 does:
sample (reference sampler built from source, oracle/_ref) -> prep_input_mails
-> forward -> BCE loss -> backward -> SGD step -> update_mailbox ->
update_memory.  Dropout is off and SGD replaces Adam so that every recorded
quantity is a smooth function of the inputs; timestamps span [0, 50], since
cos(w dt + b) at dt ~ 1e4 turns the last-bit differences of two fp32
gradient computations into visibly different steps.  PyTorch runs on one
thread: update_memory assigns rows with repeated node ids
(node_memory[nid] = memory), which keeps the last occurrence only when the
CPU kernel runs sequentially.  Stand-ins for what this
container lacks are those of make_model_golden.py, plus Tensor.cuda() as the
identity (memorys.py moves gathered rows to the GPU) and an unused
torch_scatter (only the 'mean' combine calls it).
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))
from oracle.paths import REF_ROOT as REF  # noqa: E402
sys.path.insert(0, HERE)

from conftest import small_graph  # noqa: E402
from make_model_golden import FakeBlock, _TorchOnCpu, install_fakes  # noqa: E402
from oracle.sampler import load_reference  # noqa: E402

STEPS, B, B0 = 4, 40, 2000
LR = 0.05
DM, DT = 48, 20          # memory / output width and time-encoding width (the config's 100 / 100, scaled down)


def run_case(out, name, de, seed):
    import layers as ref_layers
    import memorys as ref_mem
    import modules as ref_modules
    from fast_util.efficientGOP import fm
    ref_layers.torch = _TorchOnCpu()
    fm.fastESMFlag = fm.fastAggFlag = fm.CSR_OUT = 0
    fm.fastKQV = fm.fastTIME = fm.fastDrop = 0
    torch.Tensor.cuda = lambda self, *a, **k: self
    N = 120
    g = small_graph(n_nodes=N, n_edges=4000, seed=seed, int_ts=False, t_max=50.0, zipf=1.0)
    torch.manual_seed(seed)
    ef = torch.randn(4000, de)
    sp = dict(layer=1, neighbor=[10], strategy="recent", prop_time=False, history=1, duration=0)
    mp = dict(type="node", dim_time=DT, deliver_to="self", mail_combine="last", memory_update="gru",
              mailbox_size=1, combine_node_feature=True, dim_out=DM)
    gp = dict(arch="transformer_attention", layer=1, att_head=2, dim_time=DT, dim_out=DM)
    tp = dict(lr=LR, dropout=0.0, att_dropout=0.0)
    model = ref_modules.GeneralModel(0, de, sp, mp, gp, tp)
    mailbox = ref_mem.MailBox(mp, N, de)
    opt = torch.optim.SGD(model.parameters(), lr=LR)
    crit = torch.nn.BCEWithLogitsLoss()
    p = name + "/"
    for k, v in model.state_dict().items():
        out[p + "param0/" + k] = v.numpy().copy()
    ref = load_reference()
    s = ref.ParallelSampler(g["indptr"], g["indices"], g["eid"], g["ts"], 1, 1, 1, [10], True, False, 1, 0.0)
    rng = np.random.default_rng(seed)
    for step in range(STEPS):
        b0 = B0 + step * B
        roots = np.concatenate([g["src"][b0:b0 + B], g["dst"][b0:b0 + B], rng.integers(0, N, B).astype(np.int32)])
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
        for mfg in mfgs:     # utils.py:126-196 (prepare_input), edge features only
            for b in mfg:
                if b.num_src_nodes() > b.num_dst_nodes():
                    b.edata["f"] = ef[b.edata["ID"].long()].float()
        mailbox.prep_input_mails(mfgs[0])
        opt.zero_grad()
        pred_pos, pred_neg = model(mfgs)
        loss = crit(pred_pos, torch.ones_like(pred_pos)) + crit(pred_neg, torch.zeros_like(pred_neg))
        loss.backward()
        q = p + "step%d/" % step
        out[q + "loss"] = np.array([float(loss.detach())], np.float32)
        out[q + "pred_pos"] = pred_pos.detach().numpy()
        out[q + "pred_neg"] = pred_neg.detach().numpy()
        out[q + "updated_memory"] = model.memory_updater.last_updated_memory.numpy().copy()
        if step in (0, STEPS - 1):
            for n_, prm in model.named_parameters():
                if prm.grad is not None:
                    out[q + "grad/" + n_] = prm.grad.numpy().copy()
        opt.step()
        mem_edge_feats = ef[b0:b0 + B]        # train.py:386: the batch's own edges
        mailbox.update_mailbox(model.memory_updater.last_updated_nid, model.memory_updater.last_updated_memory,
                               roots, rts, mem_edge_feats, None)
        mailbox.update_memory(model.memory_updater.last_updated_nid, model.memory_updater.last_updated_memory,
                              roots, model.memory_updater.last_updated_ts)
        out[q + "roots"] = roots
        out[q + "rts"] = rts
        out[q + "e0"] = np.array([b0], np.int64)
        out[q + "node_memory"] = mailbox.node_memory.numpy().copy()
        out[q + "node_memory_ts"] = mailbox.node_memory_ts.numpy().copy()
        out[q + "mailbox"] = mailbox.mailbox.numpy().copy()
        out[q + "mailbox_ts"] = mailbox.mailbox_ts.numpy().copy()
        for k in ("row", "col", "eid", "ts", "dts", "nodes"):
            out[q + "block/" + k] = getattr(ret[0], k)()
    out[p + "params"] = np.array([N, de, STEPS, B, B0, DM, DT], np.int64)
    out[p + "edge_feats"] = ef.numpy()
    out[p + "lr"] = np.array([LR], np.float32)
    out[p + "graph/indptr"] = g["indptr"]
    out[p + "graph/indices"] = g["indices"]
    out[p + "graph/eid"] = g["eid"]
    out[p + "graph/ts"] = g["ts"]
    out[p + "graph/src"] = g["src"]
    out[p + "graph/dst"] = g["dst"]
    out[p + "graph/t"] = g["t"]


def run_apan(out, name, de, seed, S=10):
    """APAN-1 (config/APAN-1.yml): transformer memory updater over a mailbox of
    S slots, delivery to the sampled neighbours, identity GNN, no_neg sampling
    (train.py:323-325; the model runs on node_to_dgl_blocks of all roots,
    utils.py:115-124; the reversed sampled block delivers the mails,
    train.py:387-389).  modules.py:57 calls every layer as layer(block, l, h)
    but IdentityNormLayer.forward takes the block alone (layers.py:248), so
    the reference raises there; the layer is called here with the block."""
    import layers as ref_layers
    import memorys as ref_mem
    import modules as ref_modules
    from fast_util.efficientGOP import fm
    ref_layers.torch = _TorchOnCpu()
    fm.fastESMFlag = fm.fastAggFlag = fm.CSR_OUT = 0
    fm.fastKQV = fm.fastTIME = fm.fastDrop = 0
    torch.Tensor.cuda = lambda self, *a, **k: self
    ref_layers.IdentityNormLayer.forward = lambda self, b, *unused: self.norm(b.srcdata["h"])
    N = 120
    g = small_graph(n_nodes=N, n_edges=4000, seed=seed, int_ts=False, t_max=50.0, zipf=1.0)
    torch.manual_seed(seed)
    ef = torch.randn(4000, de)
    sp = dict(layer=1, neighbor=[10], strategy="recent", prop_time=False, history=1, duration=0, no_neg=True)
    mp = dict(type="node", dim_time=DT, deliver_to="neighbors", mail_combine="last", memory_update="transformer",
              attention_head=2, mailbox_size=S, combine_node_feature=False, dim_out=DM)
    gp = dict(arch="identity")
    tp = dict(lr=LR, dropout=0.0, att_dropout=0.0)
    model = ref_modules.GeneralModel(0, de, sp, mp, gp, tp)
    mailbox = ref_mem.MailBox(mp, N, de)
    opt = torch.optim.SGD(model.parameters(), lr=LR)
    crit = torch.nn.BCEWithLogitsLoss()
    p = name + "/"
    for k, v in model.state_dict().items():
        out[p + "param0/" + k] = v.numpy().copy()
    ref = load_reference()
    s = ref.ParallelSampler(g["indptr"], g["indices"], g["eid"], g["ts"], 1, 1, 1, [10], True, False, 1, 0.0)
    rng = np.random.default_rng(seed)
    for step in range(STEPS):
        b0 = B0 + step * B
        roots = np.concatenate([g["src"][b0:b0 + B], g["dst"][b0:b0 + B], rng.integers(0, N, B).astype(np.int32)])
        rts = np.concatenate([g["t"][b0:b0 + B]] * 3).astype(np.float32)
        s.sample(roots[:2 * B], rts[:2 * B], [])
        r = s.get_ret()[0]
        nb = FakeBlock([], [], len(roots), len(roots))            # node_to_dgl_blocks
        nb.srcdata["ID"] = torch.from_numpy(roots)
        nb.srcdata["ts"] = torch.from_numpy(rts)
        mfgs = [[nb]]
        mailbox.prep_input_mails(mfgs[0])
        opt.zero_grad()
        pred_pos, pred_neg = model(mfgs)
        loss = crit(pred_pos, torch.ones_like(pred_pos)) + crit(pred_neg, torch.zeros_like(pred_neg))
        loss.backward()
        q = p + "step%d/" % step
        out[q + "loss"] = np.array([float(loss.detach())], np.float32)
        out[q + "updated_memory"] = model.memory_updater.last_updated_memory.numpy().copy()
        if step in (0, STEPS - 1):
            for n_, prm in model.named_parameters():
                if prm.grad is not None:
                    out[q + "grad/" + n_] = prm.grad.numpy().copy()
        opt.step()
        rb = FakeBlock(r.row(), r.col(), r.dim_out(), r.dim_in())  # to_dgl_blocks(..., reverse=True)
        rb.dstdata["ID"] = torch.from_numpy(r.nodes())
        rb.dstdata["ts"] = torch.from_numpy(r.ts())
        rb.edata["ID"] = torch.from_numpy(r.eid())
        mailbox.update_mailbox(model.memory_updater.last_updated_nid, model.memory_updater.last_updated_memory,
                               roots, rts, ef[b0:b0 + B], rb)
        mailbox.update_memory(model.memory_updater.last_updated_nid, model.memory_updater.last_updated_memory,
                              roots, model.memory_updater.last_updated_ts)
        out[q + "roots"] = roots
        out[q + "rts"] = rts
        out[q + "e0"] = np.array([b0], np.int64)
        out[q + "node_memory"] = mailbox.node_memory.numpy().copy()
        out[q + "node_memory_ts"] = mailbox.node_memory_ts.numpy().copy()
        out[q + "mailbox"] = mailbox.mailbox.numpy().copy()
        out[q + "mailbox_ts"] = mailbox.mailbox_ts.numpy().copy()
        out[q + "next_mail_pos"] = mailbox.next_mail_pos.numpy().copy()
        for k in ("row", "col", "eid", "ts", "dts", "nodes"):
            out[q + "block/" + k] = getattr(r, k)()
    out[p + "params"] = np.array([N, de, STEPS, B, B0, DM, DT, S], np.int64)
    out[p + "edge_feats"] = ef.numpy()
    out[p + "lr"] = np.array([LR], np.float32)
    for k in ("indptr", "indices", "eid", "ts", "src", "dst", "t"):
        out[p + "graph/" + k] = g[k]


def main():
    if not os.path.isdir(REF):
        raise SystemExit("reference tree not found")
    torch.set_num_threads(1)
    install_fakes()
    sys.path.insert(0, REF)
    out = {}
    run_case(out, "tgn1", 24, 21)
    run_apan(out, "apan1", 24, 22)
    path = os.path.join(HERE, "memory_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, len(out), "arrays")


if __name__ == "__main__":
    main()
