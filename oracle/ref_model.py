"""TEST INFRASTRUCTURE ONLY -- parameter tree of the reference's memory-less
GeneralModel, for the CPU restatement in ``ref_math``.

Only tests/ and bench.py's CPU legs (``--impl reference`` and
``cpu_baseline``) use this module, and only as the checker / the timed CPU
reference path.  It imports nothing from ``fast_b200``, so the CPU arm never
loads the product's library.

Module tree, parameter names, shapes and initialisation follow NoneBone/FAST:
  TimeEncode                       layers.py:8-18   (w = 1 / 10^linspace(0, 9, d), b = 0)
  EdgePredictor                    layers.py:31-38
  TransfomerAttentionLayer params  layers.py:53-96  (non-combined branch)
  GeneralModel                     modules.py:8-46  (memory-less, transformer_attention)
so a state_dict of the reference model (or of fast_b200.model.GeneralModel,
which keeps the same names) loads into it unchanged.  The forward pass is
``ref_math.model_forward`` (layers.py:98-240, modules.py:48-70, DGL path).
"""
import numpy as np
import torch


class TimeEncode(torch.nn.Module):
    def __init__(self, dim):
        super().__init__()
        self.dim = dim
        self.w = torch.nn.Linear(1, dim)
        self.w.weight = torch.nn.Parameter(torch.from_numpy(1 / 10 ** np.linspace(0, 9, dim, dtype=np.float32))
                                           .reshape(dim, -1))
        self.w.bias = torch.nn.Parameter(torch.zeros(dim))


class EdgePredictor(torch.nn.Module):
    """Parameters of layers.py:31-38; forward as layers.py:40-50."""

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
    """The parameters of one attention layer (layers.py:53-96); ref_math
    computes its forward."""

    def __init__(self, dim_node_feat, dim_edge_feat, dim_time, num_head, dropout, att_dropout, dim_out):
        super().__init__()
        self.num_head = num_head
        self.dim_node_feat = dim_node_feat
        self.dim_edge_feat = dim_edge_feat
        self.dim_time = dim_time
        self.dim_out = dim_out
        self.dropout = torch.nn.Dropout(dropout)
        self.att_dropout = torch.nn.Dropout(att_dropout)
        if dim_time > 0:
            self.time_enc = TimeEncode(dim_time)
        if dim_node_feat + dim_time > 0:
            self.w_q = torch.nn.Linear(dim_node_feat + dim_time, dim_out)
        self.w_k = torch.nn.Linear(dim_node_feat + dim_edge_feat + dim_time, dim_out)
        self.w_v = torch.nn.Linear(dim_node_feat + dim_edge_feat + dim_time, dim_out)
        self.w_out = torch.nn.Linear(dim_node_feat + dim_out, dim_out)
        self.layer_norm = torch.nn.LayerNorm(dim_out)


class GeneralModel(torch.nn.Module):
    """Memory-less GeneralModel (modules.py:8-46): one attention layer per hop
    (the first over node + edge features, the next over the previous layer's
    output + edge features) and the edge predictor."""

    def __init__(self, dim_node, dim_edge, sample_param, memory_param, gnn_param, train_param):
        super().__init__()
        if memory_param.get("type", "none") != "none":
            raise NotImplementedError("the CPU reference arm covers the memory-less TGAT model")
        self.dim_node = dim_node
        self.dim_edge = dim_edge
        self.sample_param = sample_param
        self.memory_param = memory_param
        self.gnn_param = dict(gnn_param)
        self.gnn_param.setdefault("dim_out", memory_param.get("dim_out", 0))
        self.train_param = train_param
        gp, tp = self.gnn_param, train_param
        self.layers = torch.nn.ModuleDict()
        self.layers["l0h0"] = TransfomerAttentionLayer(dim_node, dim_edge, gp["dim_time"], gp["att_head"],
                                                       tp["dropout"], tp["att_dropout"], gp["dim_out"])
        for l in range(1, gp["layer"]):
            self.layers["l%dh0" % l] = TransfomerAttentionLayer(gp["dim_out"], dim_edge, gp["dim_time"],
                                                                gp["att_head"], tp["dropout"], tp["att_dropout"],
                                                                gp["dim_out"])
        self.edge_predictor = EdgePredictor(gp["dim_out"])
