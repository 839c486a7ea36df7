"""GPU: the tcgen05 projection GEMM (TMA + TMEM, 3xTF32 split) against an
fp64 product, with the criterion of conftest.parity (elementwise rtol 1e-5 /
atol 1e-6, or as accurate as the fp32 CPU GEMM), across the projection
shapes of the configs, partial tiles, bias, accumulate, strided A and a
device-side row count.
"""
import pytest
import torch

from conftest import parity

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(128, 200, 272), (777, 200, 272), (20000, 200, 372), (300, 100, 200),
                                   (1000, 100, 100), (513, 64, 32), (129, 256, 36), (4096, 128, 512)])
def test_gemm_nt_tc(cuda, M, N, K):
    from fast_b200 import ops
    torch.manual_seed(M + N + K)
    A = torch.randn(M, K)
    W = torch.randn(N, K) / K ** 0.5
    bias = torch.randn(N)
    out = ops.gemm_nt_tc(A.to(cuda), W.to(cuda), bias.to(cuda))
    ref64 = A.double() @ W.double().t() + bias.double()
    ref32 = A @ W.t() + bias
    parity(out, ref64, ref32, "C")
    assert ops.tc_error() == 0


def test_gemm_nt_tc_strided_accumulate_device_rows(cuda):
    from fast_b200 import ops
    torch.manual_seed(0)
    M, N, K = 3000, 200, 272
    wide = torch.randn(M, K + 12)
    A = wide[:, 4:4 + K]
    W = torch.randn(N, K) / K ** 0.5
    acc = torch.randn(M, N)
    out = acc.to(cuda)
    m_dev = torch.tensor([2345], dtype=torch.int32, device=cuda)
    ops.gemm_nt_tc(wide.to(cuda)[:, 4:4 + K], W.to(cuda), None, out=out, accumulate=True, M_dev=m_dev)
    ref64 = acc.double() + A.double() @ W.double().t()
    ref32 = acc + A @ W.t()
    parity(out[:2345], ref64[:2345], ref32[:2345], "C rows < M_dev")
    assert torch.equal(out[2345:].cpu(), acc[2345:])       # rows past the device count untouched
    assert ops.tc_error() == 0
