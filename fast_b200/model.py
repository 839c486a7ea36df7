"""TGAT-style temporal attention model on the fast_b200 kernels.

Module tree and parameter names follow the reference GeneralModel
(NoneBone/FAST modules.py:8-70, layers.py:8-240), so a state_dict saved by one
loads into the other.  The attention core of every layer runs on the device
kernels (``ops.AttentionCore``); the small per-destination tail (w_out, ReLU,
LayerNorm, edge predictor) stays in PyTorch.
"""
import numpy as np
import torch

from . import ops
from .ops import AttentionCore


class DeviceBlock:
    """One sampled block resident on the GPU (replaces the DGL block built by
    utils.py:67-87), sized from host-read dims.  Destinations are the block's
    roots; sources are [roots | one node per edge]; edges are grouped by
    destination."""

    static = False
    n_dst_static = True
    n_dst_dev = None
    n_edges_dev = None
    n_src_dev = None

    def __init__(self, view, dims):
        R, E, S, dim_in = (int(x) for x in dims[:4])
        self.n_dst, self.n_edges, self.n_seg, self.n_src = R, E, S, dim_in
        self.row = view["row"][:E]
        self.eid = view["eid"][:E]
        self.nodes = view["nodes"][:dim_in]
        self.ts = view["ts"][:dim_in]
        self.dst_nodes = view["nodes"][:R]
        self.src_nodes = view["nbr"][:E]
        self.dt_edges = view["dte"][:E]
        self.rptr = view["rptr"][:R + 1]
        self.cntE = view["cntE"][:S + 1] if E > 0 else view["cntE"][:0]

    def num_dst_nodes(self):
        return self.n_dst

    def num_src_nodes(self):
        return self.n_src

    def num_edges(self):
        return self.n_edges


class StaticBlock:
    """Capacity-sized views of a sampled block with its sizes left on the
    device (dims[0] = roots, dims[1] = edges): every kernel launched on it has
    a fixed shape, so a training step over static blocks can be captured in a
    CUDA graph and replayed.  `n_roots` fixes the root count when the host
    knows it (the batch roots of block 0)."""

    static = True

    def __init__(self, view, n_roots=None):
        cap_r, cap_e = int(view["max_roots"]), max(int(view["max_edges"]), 1)
        self.n_dst_static = n_roots is not None
        self.n_dst = int(n_roots) if n_roots is not None else cap_r
        self.n_edges = cap_e
        self.n_src = self.n_dst + cap_e
        self.n_dst_dev = view["dims"][0:1]
        self.n_edges_dev = view["dims"][1:2]
        self.eid = view["eid"][:cap_e]
        self.dst_nodes = view["nodes"][:self.n_dst]
        self.src_nodes = view["nbr"][:cap_e]
        self.dt_edges = view["dte"][:cap_e]
        self.rptr = view["rptr"][:self.n_dst + 1]
        self.row = view["row"][:cap_e]
        # all source rows [roots | one per edge] and their times (node memory)
        self.nodes = view["nodes"][:self.n_src]
        self.ts = view["ts"][:self.n_src]
        self.n_src_dev = view["dims"][3:4]

    def num_dst_nodes(self):
        return self.n_dst

    def num_edges(self):
        return self.n_edges


class TimeEncode(torch.nn.Module):
    """cos(w * t + b), w initialised to 1 / 10^linspace(0, 9, d) (layers.py:8-29)."""

    def __init__(self, dim):
        super().__init__()
        self.dim = dim
        self.w = torch.nn.Linear(1, dim)
        self.w.weight = torch.nn.Parameter(torch.from_numpy(1 / 10 ** np.linspace(0, 9, dim, dtype=np.float32))
                                           .reshape(dim, -1))
        self.w.bias = torch.nn.Parameter(torch.zeros(dim))

    def forward(self, t):
        return torch.cos(self.w(t.reshape((-1, 1))))


class EdgePredictor(torch.nn.Module):
    """layers.py:31-50."""

    def __init__(self, dim_in):
        super().__init__()
        self.dim_in = dim_in
        self.src_fc = torch.nn.Linear(dim_in, dim_in)
        self.dst_fc = torch.nn.Linear(dim_in, dim_in)
        self.out_fc = torch.nn.Linear(dim_in, 1)

    def forward(self, h, neg_samples=1):
        num_edge = h.shape[0] // (neg_samples + 2)
        h_src = self.src_fc(h[:num_edge])
        h_pos_dst = self.dst_fc(h[num_edge:2 * num_edge])
        h_neg_dst = self.dst_fc(h[2 * num_edge:])
        h_pos_edge = torch.nn.functional.relu(h_src + h_pos_dst)
        h_neg_edge = torch.nn.functional.relu(h_src.tile(neg_samples, 1) + h_neg_dst)
        return self.out_fc(h_pos_edge), self.out_fc(h_neg_edge)


class TransfomerAttentionLayer(torch.nn.Module):
    """Parameters as layers.py:53-96 (non-combined branch)."""

    def __init__(self, dim_node_feat, dim_edge_feat, dim_time, num_head, dropout, att_dropout, dim_out,
                 combined=False):
        super().__init__()
        if combined:
            raise NotImplementedError("combine_neighs layers are not part of the device path")
        if dim_time + dim_node_feat + dim_edge_feat <= 0:
            raise ValueError("layer needs at least one input")
        self.num_head = num_head
        self.dim_node_feat = dim_node_feat
        self.dim_edge_feat = dim_edge_feat
        self.dim_time = dim_time
        self.dim_out = dim_out
        self.dropout = torch.nn.Dropout(dropout)
        self.att_dropout_p = att_dropout
        self.negative_slope = 0.2
        if dim_time > 0:
            self.time_enc = TimeEncode(dim_time)
        if dim_node_feat + dim_time > 0:
            self.w_q = torch.nn.Linear(dim_node_feat + dim_time, dim_out)
        self.w_k = torch.nn.Linear(dim_node_feat + dim_edge_feat + dim_time, dim_out)
        self.w_v = torch.nn.Linear(dim_node_feat + dim_edge_feat + dim_time, dim_out)
        self.w_out = torch.nn.Linear(dim_node_feat + dim_out, dim_out)
        self.layer_norm = torch.nn.LayerNorm(dim_out)
        self.step_seed = 0

    def forward(self, blk, h_all=None, node_table=None, edge_table=None, seed=0, offset_dev=None):
        """blk: DeviceBlock or StaticBlock; h_all: [n_src, dim_node_feat]
        previous-layer output, or node_table + blk node ids for the input layer.
        offset_dev: int64 device counter keying the attention dropout."""
        dev = self.w_k.weight.device
        if not blk.static and blk.n_edges == 0:
            return torch.zeros((blk.n_dst, self.dim_out), device=dev)
        if self.dim_node_feat + self.dim_time == 0:
            raise NotImplementedError("Q = ones branch (layers.py:137-140) is not on the device path")
        W_kv = torch.cat([self.w_k.weight, self.w_v.weight], 0)
        b_kv = torch.cat([self.w_k.bias, self.w_v.bias], 0)
        te_w = self.time_enc.w.weight if self.dim_time > 0 else None
        te_b = self.time_enc.w.bias if self.dim_time > 0 else None
        p = self.att_dropout_p if self.training else 0.0
        agg = AttentionCore.apply(h_all, te_w, te_b, self.w_q.weight, self.w_q.bias, W_kv, b_kv, blk,
                                  node_table if h_all is None else None,
                                  edge_table if self.dim_edge_feat > 0 else None,
                                  self.num_head, self.negative_slope, p, seed, offset_dev)
        if self.dim_node_feat != 0:
            if h_all is not None:
                h_dst = h_all[:blk.n_dst]
            elif blk.static:
                h_dst = ops.gather_time_encode(blk.n_dst, h=node_table, h_idx=blk.dst_nodes,
                                               out=torch.zeros(blk.n_dst, self.dim_node_feat, device=dev),
                                               n_rows_dev=blk.n_dst_dev)
            else:
                h_dst = node_table[blk.dst_nodes.long()]
            rst = torch.cat([agg, h_dst], dim=1)
        else:
            rst = agg
        rst = self.w_out(rst)
        rst = torch.nn.functional.relu(self.dropout(rst))
        out = self.layer_norm(rst)
        if blk.static:
            # layers.py:101-102: a block without edges outputs zeros
            out = torch.where(blk.n_edges_dev > 0, out, 0.0)
        return out


class GeneralModel(torch.nn.Module):
    """Memory-less GeneralModel (modules.py:8-70) over device blocks."""

    def __init__(self, dim_node, dim_edge, sample_param, memory_param, gnn_param, train_param, combined=False):
        super().__init__()
        if memory_param.get("type", "none") != "none":
            raise NotImplementedError("node memory models use fast_b200.memory.MemoryModel")
        if gnn_param["arch"] != "transformer_attention":
            raise NotImplementedError("only transformer_attention layers are on the device path")
        if sample_param.get("history", 1) != 1:
            raise NotImplementedError("snapshot history > 1 is not on the device path")
        self.dim_node = dim_node
        self.dim_edge = dim_edge
        self.sample_param = sample_param
        self.memory_param = memory_param
        if "dim_out" not in gnn_param:
            gnn_param["dim_out"] = memory_param["dim_out"]
        self.gnn_param = gnn_param
        self.train_param = train_param
        self.layers = torch.nn.ModuleDict()
        self.layers["l0h0"] = TransfomerAttentionLayer(dim_node, dim_edge, gnn_param["dim_time"],
                                                       gnn_param["att_head"], train_param["dropout"],
                                                       train_param["att_dropout"], gnn_param["dim_out"])
        for l in range(1, gnn_param["layer"]):
            self.layers["l%dh0" % l] = TransfomerAttentionLayer(gnn_param["dim_out"], dim_edge,
                                                                gnn_param["dim_time"], gnn_param["att_head"],
                                                                train_param["dropout"],
                                                                train_param["att_dropout"], gnn_param["dim_out"])
        self.edge_predictor = EdgePredictor(gnn_param["dim_out"])
        self._drop_step = None      # device counter keying attention dropout (not part of the state_dict)

    def embed(self, blocks, node_table=None, edge_table=None):
        """blocks: Device/StaticBlocks in sampler order (hop 1 first); returns
        the root embeddings [n_roots, dim_out]."""
        mfgs = list(reversed(blocks))      # layer order, as to_dgl_blocks(...).reverse()
        dev = self.edge_predictor.out_fc.weight.device
        if self._drop_step is None or self._drop_step.device != dev:
            self._drop_step = torch.zeros(1, dtype=torch.int64, device=dev)
        if self.training:
            self._drop_step += 1
        h = None
        for l in range(self.gnn_param["layer"]):
            layer = self.layers["l%dh0" % l]
            h = layer(mfgs[l], h_all=h, node_table=node_table if l == 0 else None, edge_table=edge_table,
                      seed=0x5EED + l, offset_dev=self._drop_step)
        return h

    def forward(self, blocks, node_table=None, edge_table=None, neg_samples=1):
        return self.edge_predictor(self.embed(blocks, node_table, edge_table), neg_samples=neg_samples)
