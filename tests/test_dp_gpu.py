"""GPU, two NCCL ranks (skipped with fewer than two GPUs): data-parallel
training with the CUDA-graph trainer equals single-process training on the
global batch.

Each rank replays its captured step on a contiguous slice of every global
batch, with the global negative list drawn from a generator seeded alike on
every rank.  It samples its slice with fb_sampler_sample_shard: every layer's
time-pointer update uses the global batch's roots of that layer (the roots
for layer 0, the nodes of the global batch's previous-layer block after
that), so with recent sampling every block of every layer holds exactly the
single process's picks.  Gradients are averaged with one NCCL all-reduce of
the flat gradient buffer, so losses and parameters agree to fp32 rounding,
for one and for two recent layers.

TGN-1 (GRU node memory, mails to the roots themselves) and APAN-1
(transformer memory, mails to the sampled neighbours) the same way: every
rank keeps the whole memory and, after each step, writes all ranks' updated
rows (and, for APAN, all ranks' sampled blocks) in the global batch's order,
so the memory and mailbox tables, their timestamps and slot pointers, the
losses and the parameters agree with one process training on the global
batch.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _setup(dev, layers=1, strategy="recent"):
    sys.path.insert(0, ROOT)
    from fast_b200.data import WorkloadConfig, make_graph
    cfg = WorkloadConfig("small", 400, 40000, ("zipf", 1.1), ("uniform",), 2e3, False, 0, 48, "normal", "TGAT",
                         strategy, (8,) * layers, 64)
    g = make_graph(cfg, seed=3)
    ef = torch.randn(cfg.edges, cfg.d_edge, generator=torch.Generator().manual_seed(1)).to(dev)
    sp = dict(layer=layers, neighbor=[8] * layers, strategy=strategy, prop_time=False, history=1, duration=0)
    mp_ = dict(type="none", dim_out=0)
    gp = dict(arch="transformer_attention", layer=layers, att_head=2, dim_time=100, dim_out=100)
    tp = dict(lr=1e-3, dropout=0.0, att_dropout=0.0)
    return cfg, g, ef, sp, mp_, gp, tp


STEPS = [10000 + 128 * i for i in range(5)]


def _run(tr, gB):
    losses = []
    for b0 in STEPS:
        tr.load_device_roots(b0, b0 + gB)
        losses.append(float(tr.step_device()))
    return losses


def _worker(rank, world, port, outdir, layers=1):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from fast_b200.train import GraphTrainer
        cfg, g, ef, sp, mp_, gp, tp = _setup(dev, layers)
        gB = 128
        tr = GraphTrainer(g, None, ef, sp, mp_, dict(gp), tp, dev, batch=gB // world, rank=rank, world=world,
                          seed=5, sampler_seed=77, optimizer="sgd")
        losses = _run(tr, gB)
        t = torch.tensor(losses, device=dev)
        dist.all_reduce(t)
        params = torch.cat([p.detach().reshape(-1) for p in tr.model.parameters()]).cpu()
        tr.g_main = tr.g_opt = None          # release graphs before tearing down NCCL
        torch.cuda.synchronize()
        if rank == 0:
            np.save(os.path.join(outdir, "dp_loss.npy"), (t / world).cpu().numpy())
            np.save(os.path.join(outdir, "dp_params.npy"), params.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("layers", [1, 2])
def test_dp_two_ranks_equal_single_process(tmp_path, layers):
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(2, _port(), str(tmp_path), layers), nprocs=2, join=True)
    from fast_b200.train import GraphTrainer
    dev = torch.device("cuda", 0)
    cfg, g, ef, sp, mp_, gp, tp = _setup(dev, layers)
    tr = GraphTrainer(g, None, ef, sp, mp_, dict(gp), tp, dev, batch=128, seed=5, sampler_seed=77, optimizer="sgd")
    single = np.array(_run(tr, 128))
    params = torch.cat([p.detach().reshape(-1) for p in tr.model.parameters()]).cpu().numpy()
    dp = np.load(tmp_path / "dp_loss.npy")
    dp_params = np.load(tmp_path / "dp_params.npy")
    np.testing.assert_allclose(dp, single, rtol=1e-5, atol=1e-6)
    # The time encodings' frequencies are checked in norm: their gradient
    # sum_e -sin(w dt + b) dt g cancels heavily (fp32 is good to eps * sum|terms|
    # only), and two ranks' partial sums round differently from one sum, so a
    # few of its elements move by more than 1e-4 relative while the vector
    # agrees to 1e-5 in L2.
    names = [n for n, _ in tr.model.named_parameters()]
    sizes = [p.numel() for p in tr.model.parameters()]
    at = np.cumsum([0] + sizes)
    freq = np.zeros(len(params), dtype=bool)
    for n, a, b in zip(names, at[:-1], at[1:]):
        if n.endswith("time_enc.w.weight"):
            freq[a:b] = True
    np.testing.assert_allclose(dp_params[~freq], params[~freq], rtol=1e-4, atol=1e-6)
    rel = np.linalg.norm(dp_params[freq] - params[freq]) / np.linalg.norm(params[freq])
    assert rel <= 1e-5, rel


def _worker_uniform(rank, world, port, outdir):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from fast_b200.train import GraphTrainer
        cfg, g, ef, sp, mp_, gp, tp = _setup(dev, 2, "uniform")
        gB = 128
        tr = GraphTrainer(g, None, ef, sp, mp_, dict(gp), tp, dev, batch=gB // world, rank=rank, world=world,
                          seed=5, sampler_seed=77, optimizer="sgd")
        losses = _run(tr, gB)
        params = torch.cat([p.detach().reshape(-1) for p in tr.model.parameters()]).cpu()
        tr.release()                         # graphs go before the process group
        np.save(os.path.join(outdir, "uniform_params_%d.npy" % rank), params.numpy())
        np.save(os.path.join(outdir, "uniform_loss_%d.npy" % rank), np.array(losses))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_dp_uniform_two_layers_ranks_stay_equal(tmp_path):
    """Two uniform layers, sharded: the upper layer takes no time-pointer
    update, so no global block is kept for it; each rank draws its own slice's
    neighbours.  The ranks train on one averaged gradient, so their parameters
    stay bit-identical, and every step's loss is finite."""
    import torch.multiprocessing as mp
    mp.spawn(_worker_uniform, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    p0, p1 = (np.load(tmp_path / ("uniform_params_%d.npy" % r)) for r in (0, 1))
    assert np.array_equal(p0, p1)
    for r in (0, 1):
        assert np.isfinite(np.load(tmp_path / ("uniform_loss_%d.npy" % r))).all()


def _setup_tgn(dev, model="tgn"):
    cfg, g, ef, sp, mp_, gp, tp = _setup(dev)
    if model == "apan":
        sp = dict(sp, no_neg=True)
        mp_ = dict(type="node", dim_time=100, deliver_to="neighbors", mail_combine="last",
                   memory_update="transformer", attention_head=2, mailbox_size=10, combine_node_feature=False,
                   dim_out=100)
        gp = dict(arch="identity")
        return cfg, g, ef, sp, mp_, gp, tp
    mp_ = dict(type="node", dim_time=100, deliver_to="self", mail_combine="last", memory_update="gru",
               mailbox_size=1, combine_node_feature=True, dim_out=100)
    return cfg, g, ef, sp, mp_, gp, tp


_TABLES = ("node_memory", "node_memory_ts", "mailbox", "mailbox_ts", "next_mail_pos")


def _tgn_state(tr):
    mb = tr.mailbox
    return dict(params=torch.cat([p.detach().reshape(-1) for p in tr.model.parameters()]).cpu().numpy(),
                **{k: getattr(mb, k).detach().cpu().numpy() for k in _TABLES})


def _tgn_worker(rank, world, port, outdir, model="tgn"):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from fast_b200.train import GraphTrainer
        cfg, g, ef, sp, mp_, gp, tp = _setup_tgn(dev, model)
        gB = 128
        tr = GraphTrainer(g, None, ef, sp, mp_, dict(gp), tp, dev, batch=gB // world, rank=rank, world=world,
                          seed=5, sampler_seed=77, optimizer="sgd")
        losses = _run(tr, gB)
        t = torch.tensor(losses, device=dev)
        dist.all_reduce(t)
        st = _tgn_state(tr)
        tr.g_main = tr.g_opt = None          # release graphs before tearing down NCCL
        torch.cuda.synchronize()
        np.savez(os.path.join(outdir, "%s_rank%d.npz" % (model, rank)), loss=(t / world).cpu().numpy(), **st)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("model", ["tgn", "apan"])
def test_dp_memory_two_ranks_equal_single_process(tmp_path, model):
    """TGN (mails to the roots) and APAN (mails to the sampled neighbours)."""
    import torch.multiprocessing as mp
    mp.spawn(_tgn_worker, args=(2, _port(), str(tmp_path), model), nprocs=2, join=True)
    from fast_b200.train import GraphTrainer
    dev = torch.device("cuda", 0)
    cfg, g, ef, sp, mp_, gp, tp = _setup_tgn(dev, model)
    tr = GraphTrainer(g, None, ef, sp, mp_, dict(gp), tp, dev, batch=128, seed=5, sampler_seed=77, optimizer="sgd")
    single = np.array(_run(tr, 128))
    ref = _tgn_state(tr)
    r0, r1 = (np.load(tmp_path / ("%s_rank%d.npz" % (model, r))) for r in range(2))
    np.testing.assert_allclose(r0["loss"], single, rtol=1e-5, atol=1e-6)
    for k in ("node_memory_ts", "mailbox_ts", "next_mail_pos"):
        assert np.array_equal(r0[k], ref[k]) and np.array_equal(r1[k], ref[k]), k
    for k in ("node_memory", "mailbox", "params"):
        assert np.array_equal(r0[k], r1[k]), k           # the replicas stay identical
        np.testing.assert_allclose(r0[k], ref[k], rtol=1e-4, atol=1e-5, err_msg=k)
