"""GPU: fused LeakyReLU(q.k) -> segment softmax -> dropout -> aggregate, forward
and backward, against plain PyTorch references of the same op
(oracle/ref_math.py restates DGL's edge_softmax and copy_u/sum), run in fp64
and in fp32.

Tolerance: the north-star bound rtol 1e-5 / atol 1e-6 against the fp64
result, elementwise -- or, where fp32 rounding itself exceeds that bound, the
device result must be as accurate as the fp32 reference (conftest.parity).
"""
import numpy as np
import pytest
import torch

from conftest import parity
from oracle.ref_math import edge_softmax

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-5, 1e-6


def _segments(rng, n_dst, max_deg, big=()):
    deg = rng.integers(0, max_deg + 1, n_dst)
    for j, d in big:
        deg[j] = d
    rptr = np.concatenate([[0], np.cumsum(deg)]).astype(np.int32)
    row = np.repeat(np.arange(n_dst), deg).astype(np.int64)
    return rptr, row


def _avoid_kinks(q, k, row, heads, margin=1e-3):
    """Re-draws K rows whose q.k logit lies within `margin` of 0 for some head:
    at the LeakyReLU kink two correct fp32 evaluations can land on different
    sides and change the derivative by the slope factor."""
    g = torch.Generator().manual_seed(99)
    for _ in range(20):
        qe = (q.expand(int(row.max()) + 1, -1) if q.shape[0] == 1 else q)[torch.from_numpy(row)]
        z = (qe.double().view(len(row), heads, -1) * k.double().view(len(row), heads, -1)).sum(-1)
        bad = (z.abs() < margin).any(1)
        if not bool(bad.any()):
            return
        k[bad] = torch.randn(int(bad.sum()), k.shape[1], generator=g) * 0.5
    raise RuntimeError("could not move logits off the kink")


def _reference(q, k, v, row, n_dst, heads, slope, scale=None, per_edge_q=False):
    E, D = k.shape
    qe = q if per_edge_q else (q.expand(n_dst, -1) if q.shape[0] == 1 else q)[row]
    z = (qe.view(E, heads, -1) * k.view(E, heads, -1)).sum(-1)
    att = edge_softmax(torch.nn.functional.leaky_relu(z, slope), torch.from_numpy(row), n_dst)
    a = att if scale is None else att * scale
    vv = (v.view(E, heads, -1) * a[:, :, None]).reshape(E, D)
    agg = torch.zeros(n_dst, D, dtype=v.dtype).index_add_(0, torch.from_numpy(row), vv)
    return agg, att


@pytest.mark.parametrize("layout", ["kv_rows", "separate"])
@pytest.mark.parametrize("heads,dim", [(2, 100), (2, 128), (4, 200), (1, 64)])
@pytest.mark.parametrize("drop_p", [0.0, 0.1])
def test_attention_fwd_bwd(cuda, heads, dim, drop_p, layout):
    """layout kv_rows: K and V interleaved in [E, 2D] rows (a destination's
    rows move to shared memory by bulk copy); separate: K and V in their own
    [E, D] tensors (register-fed kernels)."""
    from fast_b200 import ops
    from fast_b200.capi import call, ptr, stream_ptr
    rng = np.random.default_rng(heads * 1000 + dim)
    n_dst = 700
    rptr, row = _segments(rng, n_dst, 12, big=((3, 70), (10, 150), (11, 1)))
    E = int(rptr[-1])
    torch.manual_seed(0)
    q = torch.randn(n_dst, dim) * 0.5
    kv = torch.randn(E, 2 * dim) * 0.5
    dagg = torch.randn(n_dst, dim)
    k, v = kv[:, :dim], kv[:, dim:]
    _avoid_kinks(q, k, row, heads)
    scale = None
    if drop_p > 0:
        sc = torch.empty(E, heads, device=cuda)
        call("fb_dropout_scale", E, heads, drop_p, 123, 7, ptr(sc), stream_ptr())
        scale = sc.cpu()
        kept = (scale > 0).float().mean().item()
        assert abs(kept - (1 - drop_p)) < 0.02
    # references (CPU fp64 and fp32, autograd)
    refs = {}
    for dt in (torch.float64, torch.float32):
        qr, kr, vr = (t.to(dt).clone().requires_grad_(True) for t in (q, k, v))
        agg_r, att_r = _reference(qr, kr, vr, row, n_dst, heads, 0.2, None if scale is None else scale.to(dt))
        agg_r.backward(dagg.to(dt))
        refs[dt] = dict(att=att_r.detach(), agg=agg_r.detach(), dq=qr.grad, dk=kr.grad, dv=vr.grad)
    # device
    qd, kvd, rp = q.to(cuda), kv.to(cuda), torch.from_numpy(rptr).to(cuda)
    if layout == "kv_rows":
        kd, vd = kvd[:, :dim], kvd[:, dim:]
    else:
        kd, vd = kvd[:, :dim].contiguous(), kvd[:, dim:].contiguous()
    agg, att = ops.attn_fwd(qd, kd, vd, rp, heads, 0.2, drop_p, 123, 7)
    dq, dkv = ops.attn_bwd(qd, kd, vd, rp, att, dagg.to(cuda), heads, 0.2, drop_p, 123, 7)
    got = dict(att=att, agg=agg, dq=dq, dk=dkv[:, :dim], dv=dkv[:, dim:])
    for name in got:
        parity(got[name], refs[torch.float64][name], refs[torch.float32][name], name)
    # rows without edges are exact zeros; results are bit-identical on rerun
    empty = np.where(np.diff(rptr) == 0)[0]
    assert torch.count_nonzero(agg[torch.from_numpy(empty).to(cuda)]) == 0
    agg2, _ = ops.attn_fwd(qd, kd, vd, rp, heads, 0.2, drop_p, 123, 7)
    assert torch.equal(agg, agg2)
    from fast_b200.capi import call as c_call
    import ctypes
    flags = ctypes.c_int(0)
    c_call("fb_attn_error", ctypes.byref(flags), 1)
    assert flags.value == 0


def test_attention_broadcast_q(cuda):
    """ldq == 0: one query row for every destination (layers.py:149-152, d_node == 0)."""
    from fast_b200 import ops
    rng = np.random.default_rng(5)
    n_dst, dim, heads = 300, 100, 2
    rptr, row = _segments(rng, n_dst, 10)
    E = int(rptr[-1])
    q = torch.randn(1, dim) * 0.5
    kv = torch.randn(E, 2 * dim) * 0.5
    dagg = torch.randn(n_dst, dim)
    _avoid_kinks(q, kv[:, :dim], row, heads)
    refs = {}
    for dt in (torch.float64, torch.float32):
        qr = q.to(dt).clone().requires_grad_(True)
        kr, vr = (kv[:, :dim].to(dt).clone().requires_grad_(True), kv[:, dim:].to(dt).clone().requires_grad_(True))
        agg_r, _ = _reference(qr, kr, vr, row, n_dst, heads, 0.2)
        agg_r.backward(dagg.to(dt))
        refs[dt] = (agg_r.detach(), qr.grad, kr.grad)
    kvd = kv.to(cuda)
    rp = torch.from_numpy(rptr).to(cuda)
    agg, att = ops.attn_fwd(q.to(cuda), kvd[:, :dim], kvd[:, dim:], rp, heads, 0.2)
    dq, dkv = ops.attn_bwd(q.to(cuda), kvd[:, :dim], kvd[:, dim:], rp, att, dagg.to(cuda), heads, 0.2)
    parity(agg, refs[torch.float64][0], refs[torch.float32][0], "agg")
    parity(dq.sum(0, keepdim=True), refs[torch.float64][1], refs[torch.float32][1], "dq")
    parity(dkv[:, :dim], refs[torch.float64][2], refs[torch.float32][2], "dk")


def test_fastagg_fused_attn_logits(cuda):
    """forward_fused_attn / backward_fused_attn of the drop-in module (precomputed logits)."""
    from fast_b200.ext import fastAgg
    rng = np.random.default_rng(8)
    n_dst, heads, dh = 200, 2, 50
    rptr_all, row = _segments(rng, n_dst, 9)
    nonempty = np.where(np.diff(rptr_all) > 0)[0]
    cnt = np.concatenate([[0], np.cumsum(np.diff(rptr_all)[nonempty])]).astype(np.int32)
    E = int(cnt[-1])
    x = torch.randn(E, heads)
    x[x.abs() < 1e-3] = 0.5          # keep logits off the LeakyReLU kink
    V = torch.randn(E, heads, dh)
    xr = x.clone().requires_grad_(True)
    Vr = V.clone().requires_grad_(True)
    att_r = edge_softmax(torch.nn.functional.leaky_relu(xr, 0.2), torch.from_numpy(row), n_dst)
    agg_r = torch.zeros(n_dst, heads * dh).index_add_(0, torch.from_numpy(row),
                                                      (Vr * att_r[:, :, None]).reshape(E, -1))
    dy = torch.randn(n_dst, heads * dh)
    agg_r.backward(dy)
    dev = [t.to(cuda) for t in (x, V, torch.from_numpy(cnt), torch.from_numpy(row))]
    out_agg, att, mask = fastAgg.forward_fused_attn(dev[0], dev[1], dev[2], dev[2], dev[3], dev[3] + n_dst,
                                                    n_dst, heads, 0.2, 0.0)
    torch.testing.assert_close(out_agg.cpu(), agg_r.detach(), rtol=RTOL, atol=ATOL)
    torch.testing.assert_close(att.cpu(), att_r.detach(), rtol=RTOL, atol=ATOL)
    dx, dV = fastAgg.backward_fused_attn(dy.to(cuda), dev[1], att, mask, dev[2], dev[2], dev[3], dev[3] + n_dst,
                                         n_dst, heads, 0.2, 0.0, input_feat=dev[0])
    torch.testing.assert_close(dx.cpu(), xr.grad, rtol=RTOL, atol=ATOL)
    torch.testing.assert_close(dV.cpu(), Vr.grad, rtol=RTOL, atol=ATOL)


def test_fastagg_legacy_ops(cuda):
    """edge softmax, forward/backward_tgat(_shd), exclusive_sum, cal_deg with the reference names."""
    from fast_b200.ext import fastAgg
    rng = np.random.default_rng(3)
    n_dst, heads, D = 150, 2, 100
    rptr_all, row = _segments(rng, n_dst, 11)
    deg = np.diff(rptr_all)
    nonempty = np.where(deg > 0)[0]
    cnt = np.concatenate([[0], np.cumsum(deg[nonempty])]).astype(np.int32)
    E = int(cnt[-1])
    x = torch.randn(E, heads)
    y_r = edge_softmax(x, torch.from_numpy(row), n_dst)
    c = torch.from_numpy(cnt).to(cuda)
    for fwd in (lambda: fastAgg.forward_edge_softmax(c, c, x.to(cuda), 512, heads)[0],
                lambda: fastAgg.forward_csr_edge_softmax(c, c, x.to(cuda), 32, 16)[0]):
        torch.testing.assert_close(fwd().cpu(), y_r, rtol=RTOL, atol=ATOL)
    dy = torch.randn(E, heads)
    dx_r = y_r * (dy - torch.zeros(n_dst, heads).index_add_(0, torch.from_numpy(row), y_r * dy)[row])
    dx = fastAgg.backward_edge_softmax(c, c, dy.to(cuda), y_r.to(cuda), 512, heads)[0]
    torch.testing.assert_close(dx.cpu(), dx_r, rtol=RTOL, atol=ATOL)
    # aggregation over the block's src table [Nd zeros | V]
    V = torch.randn(n_dst + E, D)
    rowt = torch.from_numpy(row)
    colt = torch.arange(n_dst, n_dst + E, dtype=torch.int64)
    agg_r = torch.zeros(n_dst, D).index_add_(0, rowt, V[colt])
    for out in (fastAgg.forward_tgat(rowt.to(cuda), colt.to(cuda), V.to(cuda), n_dst, 8, 128)[0],
                fastAgg.forward_tgat_shd(c, c, rowt.to(cuda), colt.to(cuda), V.to(cuda), n_dst, 8, 32)[0]):
        torch.testing.assert_close(out.cpu(), agg_r, rtol=RTOL, atol=ATOL)
    dyn = torch.randn(n_dst, D)
    dv_r = torch.zeros(n_dst + E, D)
    dv_r[colt] = dyn[rowt]
    for out in (fastAgg.backward_tgat(rowt.to(cuda), colt.to(cuda), dyn.to(cuda), n_dst + E, 8, 128)[0],
                fastAgg.backward_tgat_shd(c, c, rowt.to(cuda), colt.to(cuda), dyn.to(cuda), n_dst + E, 8, 32)[0]):
        torch.testing.assert_close(out.cpu(), dv_r, rtol=RTOL, atol=ATOL)
    degs = torch.from_numpy(deg.astype(np.int32)).to(cuda)
    np.testing.assert_array_equal(fastAgg.exclusive_sum(degs).cpu().numpy(),
                                  np.concatenate([[0], np.cumsum(deg)]).astype(np.int32))
    ids = torch.from_numpy(rng.integers(0, 50, 999).astype(np.int32)).to(cuda)
    np.testing.assert_array_equal(fastAgg.cal_deg(ids, 50).cpu().numpy(),
                                  np.bincount(ids.cpu().numpy(), minlength=50))
    big = torch.from_numpy(rng.integers(0, 5, 300_000).astype(np.int32)).to(cuda)
    np.testing.assert_array_equal(fastAgg.exclusive_sum(big).cpu().numpy()[1:],
                                  np.cumsum(big.cpu().numpy()))


@pytest.mark.parametrize("bcast", [False, True])
@pytest.mark.parametrize("kv_bf16", [False, True])
def test_attention_device_count_launch_is_the_exact_launch(cuda, bcast, kv_bf16):
    """Graph mode launches the attention over capacity-sized blocks with the
    destination count and the dropout offset on the device.  Over the live
    rows that launch must give the exact-size launch's results bit for bit
    (agg rows past the count are zeros); the capacity rows past the count
    hold NaN K|V rows and segments that must be ignored."""
    from fast_b200 import ops
    rng = np.random.default_rng(17)
    n_dst, cap, dim, heads, drop = 500, 640, 100, 2, 0.2
    rptr, row = _segments(rng, n_dst, 8, big=((7, 40),))
    E = int(rptr[-1])
    extra = np.cumsum(rng.integers(0, 9, cap - n_dst)) + E
    rptr_cap = np.concatenate([rptr, extra]).astype(np.int32)
    E_cap = int(rptr_cap[-1])
    torch.manual_seed(3)
    q = torch.randn(1 if bcast else cap, dim) * 0.5
    kv = torch.full((E_cap, 2 * dim), float("nan"))
    kv[:E] = torch.randn(E, 2 * dim) * 0.5
    dagg = torch.randn(cap, dim)
    qd, dg = q.to(cuda), dagg.to(cuda)
    kvd = kv.to(cuda).to(torch.bfloat16).float() if kv_bf16 else kv.to(cuda)
    nd_dev = torch.tensor([n_dst], dtype=torch.int32, device=cuda)
    off_dev = torch.tensor([7], dtype=torch.int64, device=cuda)
    qe = qd if bcast else qd[:n_dst]
    rp, rpc = torch.from_numpy(rptr).to(cuda), torch.from_numpy(rptr_cap).to(cuda)
    if kv_bf16:
        kvb = kvd.to(torch.bfloat16)
        agg0, att0 = ops.attn_fwd_kvbf16(qe, kvb[:E], rp, heads, 0.2, drop, 123, 7)
        agg1, att1 = ops.attn_fwd_kvbf16(qd, kvb, rpc, heads, 0.2, drop, 123, 0, n_dst_dev=nd_dev, offset_dev=off_dev)
        dq0, dkv0 = ops.attn_bwd_kvbf16(qe, kvb[:E], rp, att0, dg[:n_dst], heads, 0.2, drop, 123, 7)
        dq1, dkv1 = ops.attn_bwd_kvbf16(qd, kvb, rpc, att1, dg, heads, 0.2, drop, 123, 0, n_dst_dev=nd_dev,
                                        offset_dev=off_dev)
    else:
        agg0, att0 = ops.attn_fwd(qe, kvd[:E, :dim], kvd[:E, dim:], rp, heads, 0.2, drop, 123, 7)
        agg1, att1 = ops.attn_fwd(qd, kvd[:, :dim], kvd[:, dim:], rpc, heads, 0.2, drop, 123, 0, n_dst_dev=nd_dev,
                                  offset_dev=off_dev)
        dq0, dkv0 = ops.attn_bwd(qe, kvd[:E, :dim], kvd[:E, dim:], rp, att0, dg[:n_dst], heads, 0.2, drop, 123, 7)
        dq1, dkv1 = ops.attn_bwd(qd, kvd[:, :dim], kvd[:, dim:], rpc, att1, dg, heads, 0.2, drop, 123, 0,
                                 n_dst_dev=nd_dev, offset_dev=off_dev)
    torch.cuda.synchronize()
    assert torch.equal(agg1[:n_dst], agg0)
    assert int(torch.count_nonzero(agg1[n_dst:])) == 0
    assert torch.equal(att1[:E], att0)
    assert torch.equal(dq1[:n_dst], dq0)
    assert torch.equal(dkv1[:E].float(), dkv0.float())
