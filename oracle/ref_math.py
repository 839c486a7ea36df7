"""TEST INFRASTRUCTURE ONLY -- CPU fp32 restatement of the reference model math.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline leg use
this module, and only as the checker / reported CPU baseline.

Follows NoneBone/FAST with the DGL code path selected (``--fast_esm 0
--fast_agg 0``):
  TimeEncode                      layers.py:8-29
  EdgePredictor                   layers.py:31-50
  TransfomerAttentionLayer.forward layers.py:98-240 (non-combined branches :137-164)
  GeneralModel.forward            modules.py:48-70
DGL is not vendored by the reference (README.md:13, ``dgl>=0.9.1``); its two
operators are restated from their documented semantics:
  dgl.ops.edge_softmax(block, x)  softmax of x over the in-edges of each destination
  update_all(copy_u('v'), sum)    h[dst] = sum over in-edges of v[src]; 0 if none
The module objects passed in (parameters) may be the product's own layers:
their parameter names and shapes are those of the reference.
"""
import torch


def edge_softmax(x, row, n_dst):
    """x [E, H]; softmax over edges sharing the same destination row."""
    H = x.shape[1]
    idx = row.long().unsqueeze(1).expand(-1, H)
    mx = torch.full((n_dst, H), -float("inf"), dtype=x.dtype).scatter_reduce(0, idx, x, "amax", include_self=True)
    ex = torch.exp(x - mx[row.long()].detach())
    s = torch.zeros((n_dst, H), dtype=x.dtype).index_add_(0, row.long(), ex)
    return ex / s[row.long()]


def time_encode(te, dt):
    """TimeEncode.forward (layers.py:17-29): cos(Linear(1, d)(dt)).  The
    argument is the fp32 value w*dt + b rounded once, which is what torch's
    fp32 Linear(1, d) produces on the CPU; in a wider dtype the argument keeps
    that fp32 value (gradients flow in the wide dtype), so an fp64 run computes
    the same function as the fp32 one."""
    w, b = te.w.weight, te.w.bias
    if w.dtype == torch.float32:
        return torch.cos(te.w(dt.reshape(-1, 1).float()))
    y = dt.reshape(-1, 1).to(w.dtype) * w.reshape(1, -1) + b
    y32 = torch.nn.functional.linear(dt.reshape(-1, 1).float(), w.detach().float(), b.detach().float())
    return torch.cos(y + (y32.to(w.dtype) - y).detach())


def copy_u_sum(v_src, col, row, n_dst):
    """update_all(copy_u('v','m'), sum('m','h')) on a block with edges (col -> row)."""
    out = torch.zeros((n_dst, v_src.shape[1]), dtype=v_src.dtype)
    return out.index_add_(0, row.long(), v_src[col.long()])


def _dtype(layer):
    return layer.w_k.weight.dtype


def layer_forward(layer, row, col, dt, n_dst, h=None, f=None, att_mask=None):
    """One TransfomerAttentionLayer (layers.py:98-240, DGL path).
    h: srcdata['h'] [n_src, dn] or None; f: edata['f'] [E, de] or None;
    dt: edata['dt'] [E]; att_mask: optional dropout multipliers [E, H]."""
    E = row.shape[0]
    dty = _dtype(layer)
    if E == 0:
        return torch.zeros((n_dst, layer.dim_out), dtype=dty)
    if layer.dim_time > 0:
        time_feat = time_encode(layer.time_enc, dt)
        zero_time_feat = time_encode(layer.time_enc, torch.zeros(n_dst, dtype=torch.float32))
    dn, de, dtm = layer.dim_node_feat, layer.dim_edge_feat, layer.dim_time
    rl = row.long()
    if dtm == 0 and dn == 0:
        Q = torch.ones((E, layer.dim_out), dtype=dty)
        K = layer.w_k(f)
        V = layer.w_v(f)
    elif dtm == 0 and de == 0:
        Q = layer.w_q(h[:n_dst])[rl]
        K = layer.w_k(h[n_dst:])
        V = layer.w_v(h[n_dst:])
    elif dtm == 0:
        Q = layer.w_q(h[:n_dst])[rl]
        K = layer.w_k(torch.cat([h[n_dst:], f], dim=1))
        V = layer.w_v(torch.cat([h[n_dst:], f], dim=1))
    elif dn == 0:
        Q = layer.w_q(zero_time_feat)[rl]
        K = layer.w_k(torch.cat([f, time_feat], dim=1))
        V = layer.w_v(torch.cat([f, time_feat], dim=1))
    elif de == 0:
        Q = layer.w_q(torch.cat([h[:n_dst], zero_time_feat], dim=1))[rl]
        K = layer.w_k(torch.cat([h[n_dst:], time_feat], dim=1))
        V = layer.w_v(torch.cat([h[n_dst:], time_feat], dim=1))
    else:
        Q = layer.w_q(torch.cat([h[:n_dst], zero_time_feat], dim=1))[rl]
        K = layer.w_k(torch.cat([h[n_dst:], f, time_feat], dim=1))
        V = layer.w_v(torch.cat([h[n_dst:], f, time_feat], dim=1))
    H = layer.num_head
    Q = Q.reshape(E, H, -1)
    K = K.reshape(E, H, -1)
    V = V.reshape(E, H, -1)
    logits = torch.nn.functional.leaky_relu(torch.sum(Q * K, dim=2), 0.2)
    att = edge_softmax(logits, row, n_dst)
    if att_mask is not None:
        att = att * att_mask
    V = torch.reshape(V * att[:, :, None], (E, -1))
    v_src = torch.cat([torch.zeros((n_dst, V.shape[1]), dtype=dty), V], dim=0)
    agg = copy_u_sum(v_src, col, row, n_dst)
    if dn != 0:
        rst = torch.cat([agg, h[:n_dst]], dim=1)
    else:
        rst = agg
    rst = layer.w_out(rst)
    rst = torch.nn.functional.relu(layer.dropout(rst))
    return layer.layer_norm(rst)


def model_forward(model, blocks, node_feats=None, edge_feats=None, neg_samples=1, layer_fn=None):
    """GeneralModel.forward (modules.py:48-70) for memory-less TGAT models.
    blocks: sampler blocks in get_ret() order (objects with row()/col()/eid()/
    dts()/nodes()/dim_out() accessors returning numpy arrays).  layer_fn
    replaces layer_forward (the bf16-rounding restatement uses it)."""
    layer_fn = layer_fn or layer_forward
    mfgs = list(reversed(blocks))
    h = None
    for l in range(model.gnn_param["layer"]):
        b = mfgs[l]
        layer = model.layers["l%dh0" % l]
        n_dst = int(b.dim_out())
        row = torch.from_numpy(b.row())
        col = torch.from_numpy(b.col())
        dt = torch.from_numpy(b.dts())[n_dst:]
        f = None
        if edge_feats is not None and layer.dim_edge_feat > 0:
            f = edge_feats[torch.from_numpy(b.eid()).long()].to(_dtype(layer))
        if l == 0:
            hin = node_feats[torch.from_numpy(b.nodes()).long()].to(_dtype(layer)) if node_feats is not None else None
        else:
            hin = h
        h = layer_fn(layer, row, col, dt, n_dst, h=hin, f=f)
    return model.edge_predictor(h, neg_samples=neg_samples)


def bce_loss(pred_pos, pred_neg):
    """train.py:373-374."""
    crit = torch.nn.BCEWithLogitsLoss()
    return crit(pred_pos, torch.ones_like(pred_pos)) + crit(pred_neg, torch.zeros_like(pred_neg))
