"""GPU: the reference's efficientGOP dispatch over the drop-in `fastAgg`.

The reference's attention core (layers.py:165-223) runs, per forwardManager
flags, either DGL or its CUDA operators through two autograd Functions,
ESM_Function_TGAT (fm.fastESMFlag 1 / 2, efficientGOP.py:66-95) and
MA_Function_TGAT (fm.fastAggFlag 1 / 2, efficientGOP.py:97-131).  The two
classes below restate those Functions call for call -- the same fastAgg
operators, argument order and returned list element -- so that every flag
combination runs here on the drop-in module; the reference file itself imports
dgl and is not available on a GPU box.  Mode 4 is the product's
fast_b200.efficient_gop.FusedSoftmaxAggTGAT (one fused kernel each way).

Each mode computes agg = scatter_sum(V * edge_softmax(LeakyReLU(q.k))) with
dropout off, plus the gradients of q, k and v, on a block with empty
destinations, degree-1 and degree-150 segments; all are compared with the
fp64 restatement of the DGL path (oracle/ref_math.py: edge_softmax,
copy_u_sum) at 1e-5 relative / 1e-6 absolute, or as accurate in norm as its
fp32 run.
"""
import pytest
import torch

from conftest import parity
from oracle import ref_math

pytestmark = pytest.mark.gpu


class FM:
    """The flags of forwardManager.init_gop (efficientGOP.py:20-38)."""

    def __init__(self, fast_agg, fast_esm):
        self.fastAggFlag, self.fastESMFlag = fast_agg, fast_esm
        self.reduceSize, self.node_num_per_block = 16, (max(1, int(1024 / 16 / 2)) if fast_esm == 2 else 512)
        self.aggNodePB, self.aggFeat = 8, (32 if fast_agg == 2 else 128)


def _functions(fastAgg, fm):
    class ESM(torch.autograd.Function):
        """ESM_Function_TGAT (efficientGOP.py:66-95)."""

        @staticmethod
        def forward(ctx, indptr, indices, input_feat, num_dst, num_heads=2):
            if fm.fastESMFlag == 1:
                y = fastAgg.forward_edge_softmax(indptr, indices, input_feat, fm.node_num_per_block, num_heads)[0]
            else:
                y = fastAgg.forward_csr_edge_softmax(indptr, indices, input_feat, fm.node_num_per_block,
                                                     fm.reduceSize)[0]
            ctx.num_heads = num_heads
            ctx.save_for_backward(indptr, indices, y)
            return y

        @staticmethod
        def backward(ctx, d_y):
            indptr, indices, y = ctx.saved_tensors
            if fm.fastESMFlag == 1:
                dx = fastAgg.backward_edge_softmax(indptr, indices, d_y.contiguous(), y, fm.node_num_per_block,
                                                   ctx.num_heads)[0]
            else:
                dx = fastAgg.backward_csr_edge_softmax(indptr, indices, d_y.contiguous(), y, fm.node_num_per_block,
                                                       fm.reduceSize)[0]
            return None, None, dx, None, None

    class MA(torch.autograd.Function):
        """MA_Function_TGAT (efficientGOP.py:97-131)."""

        @staticmethod
        def forward(ctx, src_edge, dst_edge, input_feat, num_dst, dense_ptr=None, dense_ind=None):
            if fm.fastAggFlag == 2:
                y = fastAgg.forward_tgat_shd(dense_ptr, dense_ind, src_edge, dst_edge, input_feat, num_dst,
                                             fm.aggNodePB, fm.aggFeat)[0]
                ctx.save_for_backward(src_edge, dst_edge, dense_ptr, dense_ind)
            else:
                y = fastAgg.forward_tgat(src_edge, dst_edge, input_feat, num_dst, fm.aggNodePB, fm.aggFeat)[0]
                ctx.save_for_backward(src_edge, dst_edge)
            ctx.src_nodes = input_feat.size(0)
            return y

        @staticmethod
        def backward(ctx, d_y):
            if fm.fastAggFlag == 2:
                src_edge, dst_edge, dense_ptr, dense_ind = ctx.saved_tensors
                dx = fastAgg.backward_tgat_shd(dense_ptr, dense_ind, src_edge, dst_edge, d_y.contiguous(),
                                               ctx.src_nodes, fm.aggNodePB, fm.aggFeat)[0]
            else:
                src_edge, dst_edge = ctx.saved_tensors
                dx = fastAgg.backward_tgat(src_edge, dst_edge, d_y.contiguous(), ctx.src_nodes, fm.aggNodePB,
                                           fm.aggFeat)[0]
            return None, None, dx, None, None, None

    return ESM, MA


def _block(dev, seed=0):
    """Destinations with degrees 0..150 (several empty), edges grouped by
    destination as the sampler writes them; col = n_dst + e."""
    g = torch.Generator().manual_seed(seed)
    deg = torch.randint(0, 12, (300,), generator=g)
    deg[::17] = 0
    deg[5], deg[6], deg[7] = 150, 1, 64
    nd = deg.numel()
    row = torch.repeat_interleave(torch.arange(nd), deg)
    E = row.numel()
    col = nd + torch.arange(E)
    return nd, E, row.to(dev), col.to(dev)


def _core_reference(Qe, K, V, row, col, nd, H):
    """layers.py:165-207 on the DGL path (ref_math's edge_softmax and copy_u_sum)."""
    E = K.shape[0]
    logits = torch.nn.functional.leaky_relu(torch.sum(Qe.view(E, H, -1) * K.view(E, H, -1), dim=2), 0.2)
    att = ref_math.edge_softmax(logits, row, nd)
    Vw = torch.reshape(V.view(E, H, -1) * att[:, :, None], (E, -1))
    v_src = torch.cat([torch.zeros((nd, Vw.shape[1]), dtype=Vw.dtype), Vw], dim=0)
    return ref_math.copy_u_sum(v_src, col, row, nd)


@pytest.mark.parametrize("fast_esm,fast_agg", [(1, 1), (2, 2), (1, 2), (2, 1), (4, 4)])
def test_fm_modes_over_dropin_fastagg(cuda, fast_esm, fast_agg):
    from fast_b200.efficient_gop import FusedSoftmaxAggTGAT, dst_rptr
    from fast_b200.ext import fastAgg
    H, D = 2, 100
    nd, E, row, col = _block(cuda)
    g = torch.Generator().manual_seed(1)
    Qd = torch.randn(nd, D, generator=g, dtype=torch.float64) * 0.5
    K = torch.randn(E, D, generator=g, dtype=torch.float64) * 0.5
    V = torch.randn(E, D, generator=g, dtype=torch.float64)
    dY = torch.randn(nd, D, generator=g, dtype=torch.float64)
    rl, cl = row.cpu(), col.cpu()
    refs = {}
    for tag, dt in (("64", torch.float64), ("32", torch.float32)):
        q, k, v = (t.to(dt).clone().requires_grad_(True) for t in (Qd, K, V))
        out = _core_reference(q[rl], k, v, rl, cl, nd, H)
        out.backward(dY.to(dt))
        refs[tag] = (out.detach(), q.grad, k.grad, v.grad)
    q, k, v = (t.float().to(cuda).requires_grad_(True) for t in (Qd, K, V))
    if fast_esm == 4:
        out = FusedSoftmaxAggTGAT.apply(q, k, v, dst_rptr(row, nd), H, 0.2, 0.0, 0, 0)
    else:
        fm = FM(fast_agg, fast_esm)
        ESM, MA = _functions(fastAgg, fm)
        # layers.py:165-207 with fm flags: Q gathered per edge, LeakyReLU, the
        # segment pointer over non-empty destinations (unique2indptr,
        # efficientGOP.py:133-136), ESM, V * att, [zeros | V], MA
        f_tmp = torch.nn.functional.leaky_relu(torch.sum(q[row].view(E, H, -1) * k.view(E, H, -1), dim=2), 0.2)
        _, deg_t = torch.unique(row, return_counts=True)
        dense_ptr = fastAgg.exclusive_sum(deg_t.int())
        att = ESM.apply(dense_ptr, dense_ptr, f_tmp.contiguous(), nd)
        Vw = torch.reshape(v.view(E, H, -1) * att[:, :, None], (E, -1))
        v_src = torch.cat([torch.zeros((nd, Vw.shape[1]), device=cuda), Vw], dim=0)
        if fast_agg == 2:
            out = MA.apply(row, col, v_src, nd, dense_ptr, dense_ptr)
        else:
            out = MA.apply(row, col, v_src, nd)
    out.backward(dY.float().to(cuda))
    for name, got, r64, r32 in (("agg", out, refs["64"][0], refs["32"][0]), ("dq", q.grad, refs["64"][1], refs["32"][1]),
                                ("dk", k.grad, refs["64"][2], refs["32"][2]),
                                ("dv", v.grad, refs["64"][3], refs["32"][3])):
        parity(got, r64, r32, name="mode esm=%d agg=%d %s" % (fast_esm, fast_agg, name))
