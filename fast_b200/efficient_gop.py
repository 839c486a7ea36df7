"""The fused attention core for the reference's forwardManager (`fm`), mode 4.

The reference's fast_util/efficientGOP.py dispatches the attention core of
TransfomerAttentionLayer (layers.py:165-223) on two flags: `fm.fastESMFlag`
picks the edge-softmax operator (1: forward/backward_edge_softmax, 2: the CSR
variants; ESM_Function_TGAT, efficientGOP.py:66-95) and `fm.fastAggFlag` the
aggregation (1: forward/backward_tgat, 2: the _shd variants;
MA_Function_TGAT, efficientGOP.py:97-131).  Those flags keep working over the
drop-in `fastAgg` module, with correct semantics.

Mode 4 (`fm.init_gop(fast_agg=4, fast_esm=4)`) replaces the whole chain --
q.k, LeakyReLU, edge softmax, attention dropout, the V * att product, the
[zeros | V] concatenation and the aggregation -- by one kernel forward and one
backward: `FusedSoftmaxAggTGAT` below, over
`fastAgg.forward_fused_softmax_agg` / `backward_fused_softmax_agg`.  Q is
taken per destination (w_q applied to the destination rows, without the
reference's [b.edges()[1]] gather); its gradient comes back per destination.
Attention dropout is drawn inside the kernel from Philox keyed by (seed,
offset, edge, head), not from torch's generator.
"""
import torch

from .ext import fastAgg


class FusedSoftmaxAggTGAT(torch.autograd.Function):
    """agg = sum over each destination's edges of softmax(LeakyReLU(q . k)) * v,
    per head; q [n_dst, D] (or [1, D], broadcast), k, v [E, D] grouped by
    destination, rptr int32 [n_dst + 1] the CSR over every destination
    (empty rows give zeros).  Returns agg [n_dst, D]."""

    @staticmethod
    def forward(ctx, q, k, v, rptr, num_heads, negative_slope=0.2, att_drop=0.0, seed=0, offset=0):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        agg, att = fastAgg.forward_fused_softmax_agg(q, k, v, rptr, int(num_heads), float(negative_slope),
                                                     float(att_drop), int(seed), int(offset))
        ctx.save_for_backward(q, k, v, rptr, att)
        ctx.args = (int(num_heads), float(negative_slope), float(att_drop), int(seed), int(offset))
        return agg

    @staticmethod
    def backward(ctx, d_agg):
        q, k, v, rptr, att = ctx.saved_tensors
        dq, dk, dv = fastAgg.backward_fused_softmax_agg(q, k, v, rptr, att, d_agg.contiguous(), *ctx.args)
        if q.shape[0] == 1 and rptr.shape[0] - 1 != 1:
            dq = dq.sum(0, keepdim=True)       # the broadcast row's gradient
        return dq, dk, dv, None, None, None, None, None, None


def dst_rptr(row, n_dst):
    """CSR offsets over every destination of a block whose edges are grouped
    by destination (the sampler's order), from its row ids, with the drop-in
    operators: exclusive_sum of the per-destination edge counts."""
    counts = torch.bincount(row.long(), minlength=int(n_dst)).int()
    return fastAgg.exclusive_sum(counts)
