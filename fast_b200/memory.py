"""TGN node memory on the device (reference memorys.py:6-182, 270-304;
modules.py:8-47).

`MailBox` keeps the node memory, its timestamps, the mailbox and the mail
timestamps as device tensors for the whole run; the gather of a block's
source rows and the writes after a step are kernels (fb_mem_gather,
fb_mailbox_update_self, fb_memory_update), so the step needs no host round
trip and can be captured in a CUDA graph.  `GRUMemoryUpdater` and
`MemoryModel` carry the reference's module tree and parameter names
(memory_updater.updater.weight_ih, ...), so a state_dict loads across; their
forward and backward run in `engine.FusedStep`.

Covered: memory 'node' with
  * updater 'gru', deliver_to 'self', mail_combine 'last', memory combined
    into the node input without node features (TGN-1);
  * updater 'transformer', deliver_to 'neighbors', mail_combine 'last', the
    'identity' GNN and no_neg sampling (APAN-1).
Other variants raise NotImplementedError.
"""
import torch

from .capi import call, ptr, stream_ptr
from .model import EdgePredictor, TimeEncode, TransfomerAttentionLayer


class MailBox:
    """MailBox (memorys.py:6-41) with every table on `device`.  Duplicate
    writes keep the last occurrence, as the reference's index assignments do
    on the CPU (memorys.py:98, 139)."""

    def __init__(self, memory_param, num_nodes, dim_edge_feat, device):
        if memory_param["type"] != "node":
            raise NotImplementedError("memory type %r" % memory_param["type"])
        if memory_param["deliver_to"] not in ("self", "neighbors") or memory_param["mail_combine"] != "last":
            raise NotImplementedError("mailbox delivery %r / %r" % (memory_param["deliver_to"],
                                                                    memory_param["mail_combine"]))
        self.deliver_to = memory_param["deliver_to"]
        dev = torch.device(device)
        self.memory_param = memory_param
        self.dim_mem = memory_param["dim_out"]
        self.dim_edge_feat = dim_edge_feat
        self.size = memory_param["mailbox_size"]
        self.dim_mail = 2 * self.dim_mem + dim_edge_feat
        self.num_nodes = num_nodes
        f32 = dict(device=dev, dtype=torch.float32)
        self.node_memory = torch.zeros(num_nodes, self.dim_mem, **f32)
        self.node_memory_ts = torch.zeros(num_nodes, **f32)
        self.mailbox = torch.zeros(num_nodes, self.size, self.dim_mail, **f32)
        self.mailbox_ts = torch.zeros(num_nodes, self.size, **f32)
        self.next_mail_pos = torch.zeros(num_nodes, dtype=torch.int32, device=dev)
        # write-order bookkeeping of the last-occurrence-wins writes
        self._last_mail = torch.zeros(num_nodes, dtype=torch.int64, device=dev)
        self._last_mem = torch.zeros(num_nodes, dtype=torch.int64, device=dev)
        self._gen = torch.ones(2, dtype=torch.int32, device=dev)
        self._done = torch.zeros(2, dtype=torch.int32, device=dev)

    def reset(self):
        """MailBox.reset (memorys.py:23-28)."""
        for t in (self.node_memory, self.node_memory_ts, self.mailbox, self.mailbox_ts, self.next_mail_pos):
            t.zero_()

    def gather(self, nodes, ts, n, n_dev, time_enc, out_x, out_h0, out_dt):
        """prep_input_mails (memorys.py:51-73) + the updater's time encoding
        (memorys.py:286-289) for source rows [0, n) (*n_dev on the device)."""
        dt = time_enc.dim if time_enc is not None else 0
        w = time_enc.w.weight.view(-1) if dt else None
        b = time_enc.w.bias if dt else None
        call("fb_mem_gather", ptr(nodes), ptr(ts), n, ptr(n_dev), ptr(self.node_memory), self.dim_mem,
             ptr(self.node_memory_ts), ptr(self.mailbox), self.size * self.dim_mail, ptr(w), ptr(b), dt, ptr(out_x),
             out_x.stride(0), ptr(out_h0), ptr(out_dt), stream_ptr())

    def gather_slots(self, nodes, ts, n, n_dev, time_enc, out_x, out_h0, out_dt):
        """APAN's updater input (memorys.py:360-372): one row per (root, mailbox
        slot) with the time encoding of ts - mail_ts, and the roots' memory."""
        dt = time_enc.dim if time_enc is not None else 0
        w = time_enc.w.weight.view(-1) if dt else None
        b = time_enc.w.bias if dt else None
        call("fb_mail_slots_gather", ptr(nodes), ptr(ts), n, ptr(n_dev), ptr(self.node_memory), self.dim_mem,
             ptr(self.mailbox), ptr(self.mailbox_ts), self.size, self.dim_mail, ptr(w), ptr(b), dt, ptr(out_x),
             out_x.stride(0), ptr(out_h0), ptr(out_dt), stream_ptr())

    def update(self, roots, root_ts, h, edge_feats, e0_dev, block=None):
        """update_mailbox then update_memory (memorys.py:101-178, 84-99) after a
        step: roots / root_ts the batch's [src | dst | neg] roots, h the updated
        memory of those roots (rows in the same order), edge_feats the edge
        table and e0_dev (device int64) the id of the batch's first edge.
        deliver_to 'neighbors' also takes the block sampled for the positive
        roots (its nodes and each edge's root)."""
        n = roots.shape[0] // 3
        de = self.dim_edge_feat
        if self.deliver_to == "neighbors":
            call("fb_mailbox_update_neighbors", ptr(block.nodes), ptr(block.row), ptr(root_ts), n,
                 ptr(block.n_edges_dev), block.n_edges, ptr(h), h.stride(0), self.dim_mem,
                 ptr(edge_feats) if de else None, edge_feats.stride(0) if de else 0, de, ptr(e0_dev),
                 ptr(self.mailbox), ptr(self.mailbox_ts), ptr(self.next_mail_pos), self.size, ptr(self._last_mail),
                 ptr(self._gen[0:1]), ptr(self._done[0:1]), stream_ptr())
            self._update_memory(roots, root_ts, h, n)
            return
        call("fb_mailbox_update_self", ptr(roots), ptr(root_ts), n, ptr(h), h.stride(0), self.dim_mem,
             ptr(edge_feats) if de else None, edge_feats.stride(0) if de else 0, de, ptr(e0_dev), ptr(self.mailbox),
             ptr(self.mailbox_ts), ptr(self.next_mail_pos), self.size, ptr(self._last_mail), ptr(self._gen[0:1]),
             ptr(self._done[0:1]), stream_ptr())
        self._update_memory(roots, root_ts, h, n)

    def _update_memory(self, roots, root_ts, h, n):
        call("fb_memory_update", ptr(roots), ptr(root_ts), n, ptr(h), h.stride(0), self.dim_mem,
             ptr(self.node_memory), ptr(self.node_memory_ts), ptr(self._last_mem), ptr(self._gen[1:2]),
             ptr(self._done[1:2]), stream_ptr())


class GRUMemoryUpdater(torch.nn.Module):
    """GRUMemeoryUpdater (memorys.py:270-304): h' = GRUCell([mail | cos(w (ts
    - mem_ts) + b)], mem).  Parameters as the reference's."""

    def __init__(self, memory_param, dim_in, dim_hid, dim_time, dim_node_feat):
        super().__init__()
        if memory_param["combine_node_feature"] and dim_node_feat > 0:
            raise NotImplementedError("node features combined with the memory")
        if not memory_param["combine_node_feature"]:
            raise NotImplementedError("memory not combined into the node input")
        self.dim_hid = dim_hid
        self.dim_node_feat = dim_node_feat
        self.memory_param = memory_param
        self.dim_time = dim_time
        self.updater = torch.nn.GRUCell(dim_in + dim_time, dim_hid)
        if dim_time > 0:
            self.time_enc = TimeEncode(dim_time)


class TransformerMemoryUpdater(torch.nn.Module):
    """TransformerMemoryUpdater (memorys.py:342-385): attention of the memory
    over the mailbox slots, residual, LayerNorm, mlp, dropout, ReLU.
    Parameters as the reference's."""

    def __init__(self, memory_param, dim_in, dim_out, dim_time, train_param):
        super().__init__()
        self.memory_param = memory_param
        self.dim_time = dim_time
        self.dim_out = dim_out
        self.att_h = memory_param["attention_head"]
        if dim_time > 0:
            self.time_enc = TimeEncode(dim_time)
        self.w_q = torch.nn.Linear(dim_out, dim_out)
        self.w_k = torch.nn.Linear(dim_in + dim_time, dim_out)
        self.w_v = torch.nn.Linear(dim_in + dim_time, dim_out)
        self.layer_norm = torch.nn.LayerNorm(dim_out)
        self.mlp = torch.nn.Linear(dim_out, dim_out)
        self.dropout = torch.nn.Dropout(train_param["dropout"])
        self.att_dropout_p = train_param["att_dropout"]
        self.negative_slope = 0.2


class IdentityNormLayer(torch.nn.Module):
    """IdentityNormLayer (layers.py:242-249): LayerNorm of the node input."""

    def __init__(self, dim_out):
        super().__init__()
        self.norm = torch.nn.LayerNorm(dim_out)


class MemoryModel(torch.nn.Module):
    """GeneralModel with node memory (modules.py:8-47): memory_updater,
    layers['l0h0'.. ] over the memory as node input, edge_predictor."""

    def __init__(self, dim_node, dim_edge, sample_param, memory_param, gnn_param, train_param):
        super().__init__()
        upd = memory_param.get("memory_update")
        if (upd, gnn_param["arch"]) not in (("gru", "transformer_attention"), ("transformer", "identity")):
            raise NotImplementedError("memory updater %r with %r layers" % (upd, gnn_param["arch"]))
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
        dmem = memory_param["dim_out"]
        self.layers = torch.nn.ModuleDict()
        if upd == "transformer":
            # modules.py:23-24, 37-43: the transformer updater feeds an identity (LayerNorm) layer
            self.memory_updater = TransformerMemoryUpdater(memory_param, 2 * dmem + dim_edge, dmem,
                                                           memory_param["dim_time"], train_param)
            self.gnn_param["layer"] = 1
            self.layers["l0h0"] = IdentityNormLayer(dmem)
            self.edge_predictor = EdgePredictor(self.gnn_param["dim_out"])
            self._drop_step = None
            return
        self.memory_updater = GRUMemoryUpdater(memory_param, 2 * dmem + dim_edge, dmem, memory_param["dim_time"],
                                               dim_node)
        self.layers["l0h0"] = TransfomerAttentionLayer(dmem, dim_edge, gnn_param["dim_time"], gnn_param["att_head"],
                                                       train_param["dropout"], train_param["att_dropout"],
                                                       gnn_param["dim_out"])
        for l in range(1, gnn_param["layer"]):
            self.layers["l%dh0" % l] = TransfomerAttentionLayer(gnn_param["dim_out"], dim_edge,
                                                                gnn_param["dim_time"], gnn_param["att_head"],
                                                                train_param["dropout"],
                                                                train_param["att_dropout"], gnn_param["dim_out"])
        self.edge_predictor = EdgePredictor(gnn_param["dim_out"])
        self._drop_step = None

    def forward(self, *a, **k):
        raise NotImplementedError("memory models train and evaluate through engine.FusedStep")
