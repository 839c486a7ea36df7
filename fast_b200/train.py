"""Device-resident training loop for the temporal-attention hot path.

One training step follows train.py:307-393 of the reference: roots =
[src | dst | negatives] of a chronological batch, temporal sampling, feature
gather + time encoding, forward, BCE loss, backward, Adam.  Everything stays
in HBM; the only host round trip per step is reading the sampled block
sizes (and, in the end-to-end mode, the batch upload and the loss readback).

Data parallelism: each rank takes a contiguous slice of every chronological
batch, gradients are averaged with one NCCL all-reduce over a single flat
bucket.  Equal slices make the averaged gradient the gradient of the global
batch loss (mean_pos + mean_neg, train.py:373-374).  A memory model keeps
the whole node memory on every rank; after each step all_gathers bring every
rank's updated memory rows (and, for APAN's delivery to sampled neighbours,
every rank's sampled block), and every rank writes them in the global
batch's order, as one process would.
"""
import numpy as np
import torch
import torch.distributed as dist

from . import ops
from .engine import FlatAdam, FusedStep
from .memory import MailBox, MemoryModel
from .model import DeviceBlock, GeneralModel, StaticBlock
from .ext import sampler_core


def slice_for_rank(b0, b1, rank, world):
    """Contiguous slice of the global chronological batch [b0, b1) owned by `rank`."""
    per = (b1 - b0) // world
    lo = b0 + rank * per
    return lo, lo + per


def average_gradients(params, world, flat=None):
    """Averages the gradients of `params` over the process group with ONE
    all-reduce of a flat bucket (the model is ~0.2 M parameters, so one bucket
    is latency-optimal).  Returns the bucket for reuse."""
    grads = [p.grad for p in params if p.grad is not None]
    n = sum(g.numel() for g in grads)
    if flat is None or flat.numel() != n or flat.device != grads[0].device:
        flat = torch.empty(n, device=grads[0].device, dtype=grads[0].dtype)
    torch.cat([g.reshape(-1) for g in grads], out=flat)
    dist.all_reduce(flat)
    flat.div_(world)
    off = 0
    for g in grads:
        g.copy_(flat[off:off + g.numel()].view_as(g))
        off += g.numel()
    return flat


def average_flat(flat, world, async_op=False):
    """Mean of a flat gradient buffer over the process group, in place: one
    all-reduce with NCCL's average (no separate division launch), or sum and
    divide where the backend has no average (gloo)."""
    if dist.get_backend() == "nccl":
        return dist.all_reduce(flat, op=dist.ReduceOp.AVG, async_op=async_op)
    work = dist.all_reduce(flat, async_op=async_op)
    if async_op:
        work.wait()
    flat.div_(world)
    return None


def gather_global_order(local, world, out=None, perm=None):
    """All ranks' rows of a per-rank list [src_r | dst_r | neg_r] (3 equal
    sections of this rank's slice), returned in the global batch's order
    [src | dst | neg] -- the order one process training on the whole batch
    sees.  One all_gather (NCCL on GPUs, gloo on CPUs), then a permutation.
    out / perm: buffers of a previous call with the same shape, reused."""
    R = local.shape[0]
    Br = R // 3
    gathered = torch.empty((world * R,) + tuple(local.shape[1:]), device=local.device, dtype=local.dtype)
    if dist.get_backend() == "nccl":
        dist.all_gather_into_tensor(gathered, local.contiguous())
    else:
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local.contiguous())
        torch.cat(parts, out=gathered)
    if perm is None:
        # global position s*(world*Br) + r*Br + i <- gathered position r*R + s*Br + i
        perm = torch.arange(world * R, device=local.device).view(world, 3, Br).transpose(0, 1).reshape(-1)
    if out is None:
        out = torch.empty_like(gathered)
    torch.index_select(gathered, 0, perm, out=out)
    return out, perm


def _all_gather(t, world):
    out = torch.empty((world,) + tuple(t.shape), device=t.device, dtype=t.dtype)
    if dist.get_backend() == "nccl":
        dist.all_gather_into_tensor(out, t.contiguous())
    else:
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t.contiguous())
        torch.stack(parts, out=out)
    return out


def gather_neighbor_block_global(edge_nodes, row, rptr, Br, world):
    """APAN's mail delivery to sampled neighbours on several ranks: every
    rank's block for its positive roots [src_r | dst_r] (2 Br roots; its
    edges' nodes and root rows padded to the same capacity on every rank,
    rptr the CSR over those roots), listed as the block one process sampling
    the global positive roots [src | dst] would list it -- the edges of the
    src roots rank by rank, then those of the dst roots, each root's edges in
    sampler order, and each row the root's index in the global list.
    Returns (edge nodes, rows, edge count as a device int32 [1]); entries past
    the count are left unset.  All counts stay on the device."""
    cap = edge_nodes.shape[0]
    dev = edge_nodes.device
    gB = Br * world
    cnt = torch.stack([rptr[Br] - rptr[0], rptr[2 * Br] - rptr[Br]]).to(torch.int64)
    g_cnt = _all_gather(cnt, world)                       # [W, 2]: edges of the rank's src / dst roots
    g_nodes = _all_gather(edge_nodes, world)              # [W, cap]
    g_row = _all_gather(row, world).to(torch.int64)       # [W, cap] local root index
    sec = g_cnt.sum(0)                                    # edges of all src roots, of all dst roots
    pre = torch.cumsum(g_cnt, 0) - g_cnt                  # edges of the same section on lower ranks
    e = torch.arange(cap, device=dev).view(1, cap)
    c0, c1 = g_cnt[:, 0:1], g_cnt[:, 1:2]
    in_dst = e >= c0
    pos = torch.where(in_dst, sec[0] + pre[:, 1:2] + (e - c0), pre[:, 0:1] + e)
    pos = torch.where(e < c0 + c1, pos, torch.full_like(pos, world * cap))     # padding -> a spare slot
    r = torch.arange(world, device=dev).view(world, 1)
    grow = (g_row // Br) * gB + r * Br + g_row % Br
    nodes_out = torch.empty(world * cap + 1, device=dev, dtype=edge_nodes.dtype)
    row_out = torch.empty(world * cap + 1, device=dev, dtype=row.dtype)
    nodes_out.scatter_(0, pos.reshape(-1), g_nodes.reshape(-1))
    row_out.scatter_(0, pos.reshape(-1), grow.to(row.dtype).reshape(-1))
    return nodes_out[:-1], row_out[:-1], sec.sum().to(torch.int32).view(1)


class _GlobalBlock:
    """The neighbour-delivery view of the global batch's block (nodes, row,
    edge count) that MailBox.update reads."""

    def __init__(self, nodes, row, n_edges_dev):
        self.nodes, self.row, self.n_edges_dev = nodes, row, n_edges_dev
        self.n_edges = row.shape[0]


def _bf16_table(t, width):
    """A feature table as bf16 rows padded with zeros to a multiple of 8
    columns (kept as is when it already is one)."""
    if t is None or t.dtype == torch.bfloat16:
        return t
    out = torch.zeros(t.shape[0], ops.pad8(width), device=t.device, dtype=torch.bfloat16)
    out[:, :width] = t[:, :width]
    return out


class Trainer:
    """Eager trainer: host-sized blocks (the sampled sizes are read back each
    step).  fused=True runs forward + backward through FusedStep (no
    autograd); fused=False through the GeneralModel module under autograd."""

    def __init__(self, graph, node_feats, edge_feats, sample_param, memory_param, gnn_param, train_param,
                 device, rank=0, world=1, seed=42, sampler_seed=1234, fused=False, precision="fp32",
                 feat_dims=None):
        """precision 'bf16' (fused only) runs the projections on bf16 operands:
        the feature tables are then bf16 with rows padded with zeros to a
        multiple of 8 columns (fp32 tables are converted once here), and
        feat_dims = (dn, de) gives their true widths when they arrive padded."""
        self.device = torch.device(device)
        self.rank, self.world = rank, world
        self.graph = graph
        self.sample_param = sample_param
        torch.manual_seed(seed)
        if feat_dims is not None:
            dn, de = feat_dims
        else:
            dn = 0 if node_feats is None else node_feats.shape[1]
            de = 0 if edge_feats is None else edge_feats.shape[1]
        if precision == "bf16":
            if not fused:
                raise NotImplementedError("the bf16 projection mode runs through FusedStep")
            node_feats = _bf16_table(node_feats, dn)
            edge_feats = _bf16_table(edge_feats, de)
        self.node_feats, self.edge_feats = node_feats, edge_feats
        self.mailbox = None
        if memory_param.get("type", "none") != "none":
            if not fused:
                raise NotImplementedError("node memory trains through FusedStep")
            self.model = MemoryModel(dn, de, sample_param, memory_param, gnn_param, train_param).to(self.device)
            self.mailbox = MailBox(memory_param, graph.n_nodes, de, self.device)
        else:
            self.model = GeneralModel(dn, de, sample_param, memory_param, gnn_param, train_param).to(self.device)
        # id of the batch's first edge (the mailbox reads that batch's edge features)
        self.e0_buf = torch.zeros(1, dtype=torch.int64, device=self.device)
        if world > 1:
            for p in self.model.parameters():   # identical start on every rank
                dist.broadcast(p.data, 0)
        # FusedStep re-seats the parameters in flat buffers: build it before an optimizer sees them
        self.engine = FusedStep(self.model, precision=precision) if fused else None
        self.loss_buf = torch.zeros((), device=self.device)
        self.opt = FlatAdam(self.engine, train_param["lr"]) if fused else \
            torch.optim.Adam(self.model.parameters(), lr=train_param["lr"])
        self.crit = torch.nn.BCEWithLogitsLoss()
        dv = self.device
        # numpy arrays, or device tensors of a graph built on the device
        self.indptr = torch.as_tensor(graph.indptr).to(dv)
        self.indices = torch.as_tensor(graph.indices).to(dv)
        self.eid = torch.as_tensor(graph.eid).to(dv)
        self.ts_csr = torch.as_tensor(graph.ts_csr).to(dv)
        self.src = torch.as_tensor(graph.src).to(dv)
        self.dst = torch.as_tensor(graph.dst).to(dv)
        self.ts = torch.as_tensor(graph.ts).to(dv)
        self.sampler = sampler_core.ParallelSampler(
            self.indptr, self.indices, self.eid, self.ts_csr, 1, 1, sample_param["layer"],
            list(sample_param["neighbor"]), sample_param["strategy"] == "recent", sample_param["prop_time"],
            sample_param["history"], float(sample_param["duration"]), sampler_seed)
        self.neg_gen = torch.Generator(device=dv)
        self.neg_gen.manual_seed(seed + 17)
        self._views = None
        self._flat = None

    def sampler_kernels_per_step(self):
        """Kernels one sample() call launches: a pointer update per layer that
        uses the stateful pointers, then count / scan / write per block."""
        sp = self.sample_param
        n, first = 0, True
        for _ in range(sp["layer"]):
            use_ptr = first or sp["strategy"] == "recent" or (sp["prop_time"] and sp["history"] == 1)
            first = False
            n += (1 if use_ptr else 0) + 3 * sp["history"]
        if self.world > 1:
            # sharded sampling: the global batch's block of every layer whose nodes advance a later layer's
            # pointers (count / scan / write each)
            n += 3 * sum(1 for l in range(1, sp["layer"])
                         if sp["strategy"] == "recent" or (sp["prop_time"] and sp["history"] == 1))
        return n + 1   # the call-counter bump

    def reset_epoch(self):
        self.sampler.reset()
        if self.mailbox is not None:
            self.mailbox.reset()

    # -- inputs ---------------------------------------------------------------
    def local_slice(self, b0, b1):
        """Contiguous slice of the global batch [b0, b1) owned by this rank."""
        return slice_for_rank(b0, b1, self.rank, self.world)

    def batch_roots(self, b0, b1):
        """Roots [src | dst | neg] and times of the global batch [b0, b1)
        (train.py:182-183).  The negatives come from a generator seeded
        identically on every rank, so all ranks hold the same global list."""
        neg = torch.randint(0, self.graph.n_nodes, (b1 - b0,), device=self.device, generator=self.neg_gen,
                            dtype=torch.int32)
        t = self.ts[b0:b1]
        return torch.cat([self.src[b0:b1], self.dst[b0:b1], neg]), torch.cat([t, t, t])

    def local_of(self, roots, ts):
        """This rank's roots [src_r | dst_r | neg_r] of a global [src | dst | neg] list."""
        if self.world == 1:
            return roots, ts
        g = roots.shape[0] // 3
        per = g // self.world
        lo = self.rank * per
        pick = lambda a: torch.cat([a[lo:lo + per], a[g + lo:g + lo + per], a[2 * g + lo:2 * g + lo + per]])
        return pick(roots), pick(ts)

    def device_roots(self, b0, b1):
        """This rank's roots and times of the global batch [b0, b1)."""
        return self.local_of(*self.batch_roots(b0, b1))

    # -- step -----------------------------------------------------------------
    def blocks(self):
        dims = self.sampler.dims()
        views = self.sampler.block_views()
        return [DeviceBlock(v, d) for v, d in zip(views, dims)]

    def _allreduce_grads(self):
        if self.engine is not None:          # the gradients already live in one flat buffer
            average_flat(self.engine.flat, self.world)
        else:
            self._flat = average_gradients(list(self.model.parameters()), self.world, self._flat)

    def _update_memory(self, blocks, roots, root_ts):
        """Mailbox then memory writes of the batch (train.py:385-391), from the
        updated memory the step computed before the optimizer ran (its first
        rows are the roots'), and for delivery to neighbours the block sampled
        for the positive roots."""
        if self.mailbox is None:
            return
        R = roots.shape[0]
        h = self.engine.last_memory[:R]
        block = blocks[0]
        if self.world > 1:
            # every rank keeps the whole memory: all ranks' updates, applied
            # in the global batch's order, keep the replicas equal to the
            # tables of one process training on the global batch
            if self.mailbox.deliver_to == "neighbors":
                block = self._neighbor_block(block, R // 3)
            roots, root_ts, h = self._memory_exchange(roots, root_ts, h)
            if self.mailbox.deliver_to == "neighbors":
                block = _GlobalBlock(torch.cat([roots[:2 * (R // 3) * self.world], block[0]]), block[1], block[2])
        self.mailbox.update(roots, root_ts, h, self.edge_feats, self.e0_buf, block=block)

    def _neighbor_block(self, blk, Br):
        """This rank's block for its positive roots, padded to the capacity
        every rank shares, gathered into the global order."""
        cap = 2 * Br * int(self.sample_param["neighbor"][0])
        n2 = 2 * Br
        E = blk.row.shape[0]
        if E >= cap:                               # capacity-sized block (no root has more than fanout edges)
            nodes_e, row = blk.nodes[n2:n2 + cap], blk.row[:cap]
        else:                                      # host-sized block: pad to the capacity
            nodes_e = torch.zeros(cap, device=blk.row.device, dtype=blk.nodes.dtype)
            row = torch.zeros(cap, device=blk.row.device, dtype=blk.row.dtype)
            nodes_e[:E] = blk.nodes[n2:n2 + E]
            row[:E] = blk.row
        return gather_neighbor_block_global(nodes_e, row, blk.rptr, Br, self.world)

    def _memory_exchange(self, roots, root_ts, h):
        """All ranks' (roots, times, updated memory) in the global order."""
        bufs = getattr(self, "_xbufs", None)
        if bufs is None or bufs[0][0].numel() != self.world * roots.shape[0]:
            bufs = [(None, None)] * 3
        res = []
        for i, t in enumerate((roots, root_ts, h)):
            out, perm = gather_global_order(t, self.world, out=bufs[i][0], perm=bufs[i][1])
            res.append((out, perm))
        self._xbufs = res
        return res[0][0], res[1][0], res[2][0]

    def _sample_roots(self, roots, root_ts):
        """The roots the sampler sees: with no_neg (APAN, train.py:323-325) only
        the positive [src | dst] ones."""
        if self.sample_param.get("no_neg"):
            k = roots.shape[0] // 3 * 2
            return roots[:k], root_ts[:k]
        return roots, root_ts

    def _train_on(self, blocks, roots=None, root_ts=None):
        if self.engine is not None:
            self.engine.step(blocks, self.node_feats, self.edge_feats, self.loss_buf, mailbox=self.mailbox,
                             roots=roots, root_ts=root_ts)
            loss = self.loss_buf
        else:
            self.opt.zero_grad(set_to_none=False)
            pred_pos, pred_neg = self.model(blocks, self.node_feats, self.edge_feats)
            loss = self.crit(pred_pos, torch.ones_like(pred_pos)) + self.crit(pred_neg, torch.zeros_like(pred_neg))
            loss.backward()
        if self.world > 1:
            self._allreduce_grads()
        self.opt.step()
        if self.mailbox is not None:
            self._update_memory(blocks, roots, root_ts)
        return loss.detach()

    def _set_e0(self, e0):
        if e0 is not None:
            self.e0_buf.fill_(int(e0))
        elif self.mailbox is not None:
            raise ValueError("a memory model's step needs e0, the id of the batch's first edge")

    def step_device(self, roots, root_ts, global_roots=None, global_ts=None, e0=None):
        """One training step on device-resident roots; returns the loss tensor.
        With several ranks, the global batch's roots first advance the time
        pointers, as one process training on the whole batch would.  Memory
        models also take e0, the id of the batch's first (positive) edge."""
        self._set_e0(e0)
        sr, st = self._sample_roots(roots, root_ts)
        if self.world > 1 and global_roots is not None:
            gr, gt = self._sample_roots(global_roots, global_ts)
            ops.timed("sampler", lambda: self.sampler.sample_shard(sr, st, gr, gt))
        else:
            ops.timed("sampler", lambda: self.sampler.sample_device(sr, st))
        return self._train_on(self.blocks(), roots, root_ts)

    def step_host(self, roots_np, ts_np, global_roots_np=None, global_ts_np=None, e0=None):
        """End-to-end step through the reference-facing API: host roots in, host loss out."""
        self._set_e0(e0)
        sr, st = self._sample_roots(roots_np, ts_np)
        if self.world > 1 and global_roots_np is not None:
            dv = self.device
            gr, gt = self._sample_roots(global_roots_np, global_ts_np)
            self.sampler.sample_shard(torch.from_numpy(np.ascontiguousarray(sr)).to(dv),
                                      torch.from_numpy(np.ascontiguousarray(st)).to(dv),
                                      torch.from_numpy(np.ascontiguousarray(gr)).to(dv),
                                      torch.from_numpy(np.ascontiguousarray(gt)).to(dv))
        else:
            self.sampler.sample(sr, st, [])
        if self.mailbox is None:
            return float(self._train_on(self.blocks()))
        dev = self.device
        return float(self._train_on(self.blocks(), torch.from_numpy(roots_np).to(dev), torch.from_numpy(ts_np).to(dev)))


def batch_ranges(train_end, batch):
    return [(b, min(b + batch, train_end)) for b in range(0, train_end, batch) if min(b + batch, train_end) - b == batch]


class GraphTrainer(Trainer):
    """Trainer whose whole step -- sampling, gather + time encoding,
    projections, attention, layer tails, loss, backward and Adam -- is
    captured once in a CUDA graph and replayed.  Blocks are StaticBlocks
    (capacity-sized, sizes on the device), so no step reads anything back to
    the host.  With several ranks the step is two graphs around one NCCL
    all-reduce of the flat gradient bucket."""

    def __init__(self, graph, node_feats, edge_feats, sample_param, memory_param, gnn_param, train_param,
                 device, batch, rank=0, world=1, seed=42, sampler_seed=1234, optimizer="adam", fused=True,
                 precision="fp32", feat_dims=None):
        super().__init__(graph, node_feats, edge_feats, sample_param, memory_param, gnn_param, train_param,
                         device, rank=rank, world=world, seed=seed, sampler_seed=sampler_seed, fused=fused,
                         precision=precision, feat_dims=feat_dims)
        self.B = batch
        self.R0 = 3 * batch
        dv = self.device
        # every gradient is a view of one flat buffer: one memset clears them,
        # and the data-parallel all-reduce runs on the buffer itself
        self._params = [p for p in self.model.parameters()]
        if self.engine is not None:
            self._flat = self.engine.flat
        else:
            self._flat = torch.zeros(sum(p.numel() for p in self._params), device=dv)
            off = 0
            for p in self._params:
                p.grad = self._flat[off:off + p.numel()].view_as(p)
                off += p.numel()
        if optimizer == "adam":
            self.opt = FlatAdam(self.engine, train_param["lr"]) if self.engine is not None else \
                torch.optim.Adam(self._params, lr=train_param["lr"], capturable=True, fused=True)
        else:
            self.opt = torch.optim.SGD(self._params, lr=train_param["lr"])
        self.roots_buf = torch.zeros(self.R0, dtype=torch.int32, device=dv)
        self.ts_buf = torch.zeros(self.R0, dtype=torch.float32, device=dv)
        # the global batch's roots (every rank's), for the time-pointer update
        self.groots_buf = torch.zeros(self.R0 * world, dtype=torch.int32, device=dv) if world > 1 else None
        self.gts_buf = torch.zeros(self.R0 * world, dtype=torch.float32, device=dv) if world > 1 else None
        self.h_groots = torch.zeros(self.R0 * world, dtype=torch.int32).pin_memory() if world > 1 else None
        self.h_gts = torch.zeros(self.R0 * world, dtype=torch.float32).pin_memory() if world > 1 else None
        self.h_roots = torch.zeros(self.R0, dtype=torch.int32).pin_memory()
        self.h_ts = torch.zeros(self.R0, dtype=torch.float32).pin_memory()
        # two pinned staging slots for step_host_pipelined
        self._slots = [dict(roots=torch.zeros(self.R0, dtype=torch.int32).pin_memory(),
                            ts=torch.zeros(self.R0, dtype=torch.float32).pin_memory(),
                            groots=torch.zeros(self.R0 * world, dtype=torch.int32).pin_memory() if world > 1 else None,
                            gts=torch.zeros(self.R0 * world, dtype=torch.float32).pin_memory() if world > 1 else None,
                            loss=None, done=None) for _ in range(2)]
        self._slot = 0
        self._pending = None
        self.g_main = self.g_opt = None

    # the body of one step on the static input buffers
    def _sample(self):
        sr, st = self._sample_roots(self.roots_buf, self.ts_buf)
        if self.world > 1:
            gr, gt = self._sample_roots(self.groots_buf, self.gts_buf)
            self.sampler.sample_shard(sr, st, gr, gt)
        else:
            self.sampler.sample_device(sr, st)
        views = self.sampler.block_views()
        self._blocks = [StaticBlock(views[0], n_roots=sr.shape[0])] + [StaticBlock(v) for v in views[1:]]

    def _compute(self, overlap=False):
        """Forward + backward on the sampled blocks.  overlap (several ranks,
        FusedStep): each gradient bucket is all-reduced (NCCL average,
        asynchronously) as soon as the backward has written it, while the
        layers below run their backward; _apply waits for them."""
        blocks = self._blocks
        if self.engine is not None:
            hook = None
            self._works = []
            if overlap:
                def hook(i):
                    lo, hi = self.engine.grad_buckets[i]
                    self._works.append(average_flat(self._flat[lo:hi], self.world, async_op=True))
            self.engine.step(blocks, self.node_feats, self.edge_feats, self.loss_buf, mailbox=self.mailbox,
                             roots=self.roots_buf, root_ts=self.ts_buf, grad_hook=hook)
            return
        self._flat.zero_()
        pred_pos, pred_neg = self.model(blocks, self.node_feats, self.edge_feats)
        loss = self.crit(pred_pos, torch.ones_like(pred_pos)) + self.crit(pred_neg, torch.zeros_like(pred_neg))
        loss.backward()
        self.loss_buf.copy_(loss.detach())

    def _fwd_bwd(self):
        self._sample()
        self._compute()

    def _reduce(self):
        """The data-parallel gradient average (after an overlapped backward:
        waits for its bucket all-reduces)."""
        works = getattr(self, "_works", None)
        if works:
            for w in works:
                if w is not None:
                    w.wait()
            self._works = []
        else:
            average_flat(self._flat, self.world)

    def _apply(self):
        self.opt.step()
        if self.mailbox is not None and self.world == 1:
            self._update_memory(self._blocks, self.roots_buf, self.ts_buf)

    def _memory_ranks(self):
        """Several ranks: the memory exchange (NCCL) and writes, after the
        optimizer graph and outside every captured graph."""
        if self.mailbox is not None and self.world > 1:
            self._update_memory(self._blocks, self.roots_buf, self.ts_buf)

    def _overlap(self):
        """Bucketed all-reduce inside the backward: several ranks on NCCL with
        the fused engine (FB_NCCL_IN_GRAPH=0 keeps the all-reduce outside the
        captured graph, between two graphs)."""
        import os
        return (self.world > 1 and self.engine is not None and dist.get_backend() == "nccl"
                and os.environ.get("FB_NCCL_IN_GRAPH", "1") != "0")

    def _eager_step(self):
        self._sample()
        self._compute(overlap=self._overlap())
        if self.world > 1:
            self._reduce()
        self._apply()
        self._memory_ranks()

    def capture(self, warmup=3):
        """Warm up on a side stream (allocator, lazy kernel loads, Adam state,
        NCCL communicators), then capture.  The warm-up steps are real
        training steps on whatever is in the input buffers.  The whole step
        -- sampling, forward, backward with its gradient all-reduces (NCCL
        captured in the graph), Adam -- is one graph; with FB_NCCL_IN_GRAPH=0
        several ranks use two graphs around one all-reduce."""
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._eager_step()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        self.g_main = torch.cuda.CUDAGraph()
        one_graph = self.world == 1 or self._overlap()
        with torch.cuda.graph(self.g_main):
            self._sample()
            self._compute(overlap=self._overlap())
            if one_graph:
                if self.world > 1:
                    self._reduce()
                self._apply()
        if not one_graph:
            self.g_opt = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.g_opt, pool=self.g_main.pool()):
                self._apply()
        torch.cuda.synchronize(self.device)

    def _replay(self):
        self.g_main.replay()
        if self.g_opt is not None:
            average_flat(self._flat, self.world)
            self.g_opt.replay()
        if self.world > 1:
            self._memory_ranks()

    def phase_times(self, steps, load):
        """Device time of each phase of the step, for the data-parallel
        breakdown: sampling (this rank's blocks plus, with several ranks, the
        global batch's pointer updates), forward + backward, the gradient
        all-reduce, Adam -- each captured in a graph of its own (the
        all-reduce launched eagerly) and replayed `steps` times between CUDA
        events, load(j) filling the input buffers before step j.  Also the
        sampler with this rank's roots only (sample_device, the one-process
        call).  Returns milliseconds per step; these steps train."""
        dev = self.device
        graphs = {}
        for name, fn in (("sample", self._sample), ("forward_backward", lambda: self._compute(overlap=False)),
                         ("adam", self.opt.step)):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            graphs[name] = g
        if self.world > 1:
            graphs["sample_local_only"] = torch.cuda.CUDAGraph()
            sr, st = self._sample_roots(self.roots_buf, self.ts_buf)
            with torch.cuda.graph(graphs["sample_local_only"]):
                self.sampler.sample_device(sr, st)
        torch.cuda.synchronize(dev)
        acc = {k: 0.0 for k in list(graphs) + (["allreduce"] if self.world > 1 else [])}
        for j in range(steps):
            load(j)
            order = ["sample", "forward_backward"] + (["allreduce"] if self.world > 1 else []) + ["adam"]
            if self.world > 1:
                order.append("sample_local_only")
            for name in order:
                if self.world > 1:
                    dist.barrier()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                if name == "allreduce":
                    average_flat(self._flat, self.world)
                else:
                    graphs[name].replay()
                e1.record()
                torch.cuda.synchronize(dev)
                acc[name] += e0.elapsed_time(e1)
        graphs.clear()
        return {k: v / steps for k, v in acc.items()}

    def load_device_roots(self, b0, b1):
        """Fills the input buffers with this rank's slice of the global batch
        [b0, b1) (and, with several ranks, the global roots)."""
        assert (b1 - b0) // self.world == self.B, "graph was captured for a local batch of %d" % self.B
        groots, gts = self.batch_roots(b0, b1)
        roots, ts = self.local_of(groots, gts)
        self.roots_buf.copy_(roots)
        self.ts_buf.copy_(ts)
        self.e0_buf.fill_(b0)
        if self.world > 1:
            self.groots_buf.copy_(groots)
            self.gts_buf.copy_(gts)

    def step_device(self, roots=None, root_ts=None, global_roots=None, global_ts=None, e0=None):
        """One replayed step on the device-resident input buffers (or the given
        device tensors); returns the loss tensor (no host round trip)."""
        if e0 is not None:
            self.e0_buf.fill_(int(e0))
        if roots is not None:
            self.roots_buf.copy_(roots)
            self.ts_buf.copy_(root_ts)
        if global_roots is not None and self.world > 1:
            self.groots_buf.copy_(global_roots)
            self.gts_buf.copy_(global_ts)
        if self.g_main is None:
            self.capture()
        self._replay()
        return self.loss_buf

    def release(self):
        """Drops the captured graphs after the device has finished with them.
        A graph that holds NCCL calls must be released before the process
        group is destroyed, or the process waits on exit for good."""
        torch.cuda.synchronize()
        self.g_main = self.g_opt = None
        import gc
        gc.collect()
        torch.cuda.synchronize()

    def step_host_pipelined(self, roots_np, ts_np, global_roots_np=None, global_ts_np=None, e0=None):
        """step_host without waiting for this step: the inputs go through pinned
        slot i % 2, the loss comes back into that slot's pinned word, and the
        call returns the previous step's loss (None on the first call) once that
        step has completed -- so the host prepares and copies batch i + 1 while
        the device runs step i.  finish_pipelined() returns the last loss."""
        sl = self._slots[self._slot]
        if sl["done"] is not None:
            sl["done"].synchronize()           # the step that used this slot two calls ago
        self._set_e0(e0)
        sl["roots"].numpy()[:] = roots_np
        sl["ts"].numpy()[:] = ts_np
        self.roots_buf.copy_(sl["roots"], non_blocking=True)
        self.ts_buf.copy_(sl["ts"], non_blocking=True)
        if self.world > 1:
            assert global_roots_np is not None, "several ranks: pass the global batch's roots too"
            sl["groots"].numpy()[:] = global_roots_np
            sl["gts"].numpy()[:] = global_ts_np
            self.groots_buf.copy_(sl["groots"], non_blocking=True)
            self.gts_buf.copy_(sl["gts"], non_blocking=True)
        if self.g_main is None:
            self.capture()
        self._replay()
        if sl["loss"] is None:
            sl["loss"] = torch.zeros_like(self.loss_buf, device="cpu").pin_memory()
        sl["loss"].copy_(self.loss_buf, non_blocking=True)
        sl["done"] = torch.cuda.Event()
        sl["done"].record()
        prev, self._pending = self._pending, self._slot
        self._slot ^= 1
        return None if prev is None else self._read_slot(prev)

    def finish_pipelined(self):
        """The loss of the last step_host_pipelined call (None if none is pending)."""
        prev, self._pending = self._pending, None
        return None if prev is None else self._read_slot(prev)

    def _read_slot(self, i):
        self._slots[i]["done"].synchronize()
        return float(self._slots[i]["loss"])

    def step_host(self, roots_np, ts_np, global_roots_np=None, global_ts_np=None, e0=None):
        """End-to-end step: host roots -> pinned staging -> device buffers ->
        replay -> loss read back to the host."""
        self._set_e0(e0)
        self.h_roots.numpy()[:] = roots_np
        self.h_ts.numpy()[:] = ts_np
        self.roots_buf.copy_(self.h_roots, non_blocking=True)
        self.ts_buf.copy_(self.h_ts, non_blocking=True)
        if self.world > 1:
            assert global_roots_np is not None, "several ranks: pass the global batch's roots too"
            self.h_groots.numpy()[:] = global_roots_np
            self.h_gts.numpy()[:] = global_ts_np
            self.groots_buf.copy_(self.h_groots, non_blocking=True)
            self.gts_buf.copy_(self.h_gts, non_blocking=True)
        if self.g_main is None:
            self.capture()
        self._replay()
        return float(self.loss_buf)
