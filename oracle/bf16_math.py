"""TEST INFRASTRUCTURE ONLY -- the bf16 projection mode restated in fp64 for
the parity tests of fast_b200's bf16 precision mode.

Only tests/ use this module, as the checker.  The reference has no bf16 mode;
this is the reference layer (layers.py:98-240, restated in ref_math.py) with
bf16 rounding (round to nearest even) inserted exactly where the device's
bf16 mode rounds, and nowhere else:
  forward   the K|V projection rows [h_src | f | cos(w dt + b)], the query
            rows [h_dst | cos(b)] (layers with node input), the projected
            K and V (stored as bf16), the attention output entering w_out,
            and the weights w_k, w_v, w_q, w_out;
  backward  the gradients entering the projection-gradient products: dK|dV,
            dQ (layers with node input) and dZ (the w_out output); and the
            gradient of the K|V rows' time encoding cos(w dt + b), which the
            device's product writes as bf16 (an autocast product's input
            gradient is bf16 as well).
Products of rounded operands are exact; everything else (attention,
softmax, LayerNorm, predictor, loss) is fp64.  The Q-side time-encoding
gradient takes the fp32 master w_q, as the device's fb_q_time_bwd does.
A layer without node input keeps its one-row query product unrounded, as
the device does.
"""
import torch

from .ref_math import copy_u_sum, edge_softmax, time_encode


def rbf16(x):
    """x rounded to bf16 (through fp32, as the device rounds fp32 values)."""
    return x.float().to(torch.bfloat16).to(x.dtype)


class _Round(torch.autograd.Function):
    """Forward: round to bf16; backward: the gradient passes unchanged."""

    @staticmethod
    def forward(ctx, x):
        return rbf16(x)

    @staticmethod
    def backward(ctx, g):
        return g


class _RoundGrad(torch.autograd.Function):
    """Forward: identity; backward: the incoming gradient rounded to bf16."""

    @staticmethod
    def forward(ctx, x):
        return x.clone()

    @staticmethod
    def backward(ctx, g):
        return rbf16(g)


class _TimeQ(torch.autograd.Function):
    """The query rows' time-encoding product cos(b) W_q[:, dn:]^T on rounded
    operands, whose input gradient takes the unrounded weight."""

    @staticmethod
    def forward(ctx, te0, wt):
        ctx.save_for_backward(te0, wt)
        return rbf16(te0) @ rbf16(wt).T

    @staticmethod
    def backward(ctx, g):
        te0, wt = ctx.saved_tensors
        return g @ wt, g.T @ rbf16(te0)


def R(x):
    return _Round.apply(x)


def G(x):
    return _RoundGrad.apply(x)


def layer_forward_bf16(layer, row, col, dt, n_dst, h=None, f=None):
    """ref_math.layer_forward (layers with time encoding) in the bf16 mode."""
    E = row.shape[0]
    dty = layer.w_k.weight.dtype
    if E == 0:
        return torch.zeros((n_dst, layer.dim_out), dtype=dty)
    if layer.dim_time == 0:
        raise NotImplementedError("the bf16 restatement covers layers with time encoding")
    dn, de = layer.dim_node_feat, layer.dim_edge_feat
    rl = row.long()
    time_feat = G(time_encode(layer.time_enc, dt))
    zero_time_feat = time_encode(layer.time_enc, torch.zeros(n_dst, dtype=torch.float32))
    parts = ([h[n_dst:]] if dn else []) + ([f] if de else []) + [time_feat]
    X = R(torch.cat(parts, dim=1))
    # K and V are stored as bf16 by the projection (forward rounding), and
    # their gradients are rounded where they enter the gradient products
    K = R(G(X @ R(layer.w_k.weight).T + layer.w_k.bias))
    V = R(G(X @ R(layer.w_v.weight).T + layer.w_v.bias))
    Wq = layer.w_q.weight
    if dn:
        Qh = R(h[:n_dst])
        Q = G(Qh @ R(Wq[:, :dn]).T + _TimeQ.apply(zero_time_feat, Wq[:, dn:]) + layer.w_q.bias)
    else:
        Q = layer.w_q(zero_time_feat)
    Q = Q[rl]
    H = layer.num_head
    Q = Q.reshape(E, H, -1)
    K = K.reshape(E, H, -1)
    V = V.reshape(E, H, -1)
    logits = torch.nn.functional.leaky_relu(torch.sum(Q * K, dim=2), 0.2)
    att = edge_softmax(logits, row, n_dst)
    V = torch.reshape(V * att[:, :, None], (E, -1))
    v_src = torch.cat([torch.zeros((n_dst, V.shape[1]), dtype=dty), V], dim=0)
    agg = copy_u_sum(v_src, col, row, n_dst)
    rst = torch.cat([R(agg), Qh], dim=1) if dn else R(agg)
    rst = G(rst @ R(layer.w_out.weight).T + layer.w_out.bias)
    rst = torch.nn.functional.relu(layer.dropout(rst))
    return layer.layer_norm(rst)
