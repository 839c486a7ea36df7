"""GPU: the reference's own CUDA operators (getFastAgg) beside the fused
attention, as a parity cross-check and a speed point.

oracle/build_ref_fastagg.py builds the reference's pybind module for sm_100a
from a patched copy of its sources into oracle/_ref/fastAgg_ref.so (skipped
when it was not built).  The reference attention forward is efficientGOP's
chain (layers.py:165-212): logits by torch, K1 = forward_edge_softmax
(edge_softmax.cu:255-293), V * att by torch, then the aggregation K9 =
forward_tgat_shd (aggregate_shd_kernel.cu:161-209, fm.fastAggFlag 2).  The
default K7 = forward_tgat (fm.fastAggFlag 1) adds only the first
ceil8(n_dst) edges (aggregate_acc_kernel.cu:72-94), so it is timed but not
compared.  K9 waits at a block barrier after an early return for threads past
the last destination or feature, so it runs only where none returns early:
D a multiple of 32 and n_dst a multiple of 8.
"""
import json
import os
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def _ref():
    import build_ref_fastagg
    if not os.path.exists(build_ref_fastagg.OUT):
        pytest.skip("oracle/_ref/fastAgg_ref.so not built (oracle/build_ref_fastagg.py)")
    return build_ref_fastagg.load_built()


def _block(dev, n_dst, fan, D, seed):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    E = n_dst * fan
    rptr = torch.arange(0, E + 1, fan, device=dev, dtype=torch.int32)
    row = torch.arange(n_dst, device=dev, dtype=torch.int64).repeat_interleave(fan)
    col = n_dst + torch.arange(E, device=dev, dtype=torch.int64)
    q = torch.randn(n_dst, D, device=dev, generator=g) * 0.5
    kv = torch.randn(E, 2 * D, device=dev, generator=g) * 0.5
    return E, rptr, row, col, q, kv


def _ref_forward(ref, q, k, v, rptr, row, col, n_dst, H, shd):
    E, D = k.shape
    z = torch.nn.functional.leaky_relu(torch.sum(q[row].view(E, H, -1) * k.view(E, H, -1), dim=2), 0.2)
    att = ref.forward_edge_softmax(rptr, rptr, z.contiguous(), 512, H)[0]
    vw = torch.reshape(v.view(E, H, -1) * att[:, :, None], (E, -1))
    v_src = torch.cat([torch.zeros(n_dst, D, device=q.device), vw], dim=0)
    if shd:
        return ref.forward_tgat_shd(rptr, rptr, row, col, v_src, n_dst, 8, 32)[0]
    return ref.forward_tgat(row, col, v_src, n_dst, 8, 128)[0]


def test_reference_k1_k9_agrees_with_the_fused_attention(cuda):
    """The reference's correct CUDA chain (K1 + K9) and the fused kernel give
    the same aggregate to fp32 accuracy (both against an fp64 torch result)."""
    from fast_b200 import ops
    ref = _ref()
    n_dst, fan, D, H = 2048, 10, 128, 2
    E, rptr, row, col, q, kv = _block(cuda, n_dst, fan, D, 3)
    k, v = kv[:, :D].contiguous(), kv[:, D:].contiguous()
    out9 = _ref_forward(ref, q, k, v, rptr, row, col, n_dst, H, True)
    agg, _ = ops.attn_fwd(q, kv[:, :D], kv[:, D:], rptr, H, 0.2)
    q64, k64, v64 = q.double(), k.double(), v.double()
    z = torch.nn.functional.leaky_relu((q64[row].view(E, H, -1) * k64.view(E, H, -1)).sum(2), 0.2)
    att = torch.softmax(z.view(n_dst, fan, H), dim=1).view(E, H)
    exact = (v64.view(E, H, -1) * att[:, :, None]).view(n_dst, fan, D).sum(1)
    tol = 1e-5 * exact.abs() + 1e-6
    assert bool(((out9.double() - exact).abs() <= tol).all())
    assert bool(((agg.double() - exact).abs() <= tol).all())


def test_reference_cuda_speed_point(cuda):
    """Times the fused attention forward beside the reference's K1 + K7 and
    K1 + K9 chains at config 2's and config 5's hop-2 block sizes (fan-out 10,
    2 heads); prints one JSON line per shape (and appends it to the file named
    by FB_SPEED_POINT_OUT).  The reference times include its torch launches and
    the device synchronisations inside its wrappers."""
    from fast_b200 import ops
    ref = _ref()
    H, fan = 2, 10

    def timed(fn, reps=10):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1000.0 / reps

    lines = []
    for name, n_dst in (("config 2 hop 2", 19_800), ("config 5 hop 2", 132_000)):
        for D in (100, 128):
            E, rptr, row, col, q, kv = _block(cuda, n_dst, fan, D, 4)
            kc, vc = kv[:, :D].contiguous(), kv[:, D:].contiguous()
            line = {"shape": "%s: n_dst=%d, E=%d, D=%d, H=%d" % (name, n_dst, E, D, H),
                    "fast_b200_attn_fwd_us": round(timed(lambda: ops.attn_fwd(q, kv[:, :D], kv[:, D:], rptr, H,
                                                                                0.2)), 2),
                    "reference_K1_K7_us": round(timed(lambda: _ref_forward(ref, q, kc, vc, rptr, row, col, n_dst,
                                                                           H, False)), 2)}
            if D % 32 == 0 and n_dst % 8 == 0:
                line["reference_K1_K9_us"] = round(timed(lambda: _ref_forward(ref, q, kc, vc, rptr, row, col,
                                                                              n_dst, H, True)), 2)
            lines.append(line)
            print(json.dumps(line))
    out = os.environ.get("FB_SPEED_POINT_OUT")
    if out:
        with open(out, "a") as f:
            for line in lines:
                f.write(json.dumps(line) + "\n")
    assert all(v > 0 for line in lines for k, v in line.items() if k.endswith("_us"))
