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


# ---------------------------------------------------------------------------
# Grouped launches (fb_gemm_group): NT / NN / TN problems on the tensor cores.
# TMA moves the NN weight and both TN operands as they lie in memory
# (MN-major tiles); these cases pin that layout against fp64 products.

def _backend(monkeypatch, name):
    if name == "ffma":
        monkeypatch.setenv("FB_GEMM", "ffma")
    else:
        monkeypatch.delenv("FB_GEMM", raising=False)


@pytest.mark.parametrize("backend", ["tc", "ffma"])
@pytest.mark.parametrize("M,N,K", [(777, 72, 200), (20000, 100, 200), (300, 272, 100), (5, 100, 372)])
def test_group_nn(cuda, monkeypatch, backend, M, N, K):
    from fast_b200 import ops
    _backend(monkeypatch, backend)
    torch.manual_seed(M + N)
    A = torch.randn(M, K)
    Wfull = torch.randn(K, N + 28) / K ** 0.5           # strided B: a column slice of a wider weight
    Bm = Wfull[:, 28:]
    out = torch.full((M, N), 0.5, device=cuda)
    ops.gemm_group([dict(kind=ops.NN, A=A.to(cuda), B=Wfull.to(cuda)[:, 28:], out=out, accumulate=True)])
    assert ops.tc_error() == 0
    parity(out - 0.5, A.double() @ Bm.double(), A @ Bm, "C")


@pytest.mark.parametrize("backend", ["tc", "ffma"])
@pytest.mark.parametrize("M,N,K,db", [(2500, 200, 272, True), (3073, 400, 272, True), (200000, 200, 372, True),
                                      (1000, 100, 100, False), (77, 100, 200, True), (4000, 100, 0, True)])
def test_group_tn(cuda, monkeypatch, backend, M, N, K, db):
    """Weight (+ bias) gradients.  Rows past the device count hold NaN and
    must not reach the sums; (3073, 400, 272) leaves the last split of the
    reduction empty on 148 SMs."""
    from fast_b200 import ops
    _backend(monkeypatch, backend)
    torch.manual_seed(M + K)
    m_true = M - 3
    G = torch.randn(M, N)
    X = torch.randn(M, max(K, 1))[:, :K] if K else None
    Gd = G.to(cuda)
    Gd[m_true:] = float("nan")
    Xd = None
    if K:
        Xd = X.to(cuda)
        Xd[m_true:] = float("nan")
    cnt = torch.tensor([m_true], dtype=torch.int32, device=cuda)
    C = torch.ones(N, K, device=cuda) if K else None
    dbv = torch.full((N,), 2.0, device=cuda) if db else None
    ops.gemm_group([dict(kind=ops.TN, A=Gd, B=Xd, out=C, accumulate=True, M_dev=cnt, db=dbv)])
    assert ops.tc_error() == 0
    if K:
        parity(C - 1.0, G[:m_true].double().t() @ X[:m_true].double(), G[:m_true].t() @ X[:m_true], "dW")
    if db:
        parity(dbv - 2.0, G[:m_true].double().sum(0), G[:m_true].sum(0), "db")


@pytest.mark.parametrize("backend", ["tc", "ffma"])
def test_group_nt_concat_and_device_rows(cuda, monkeypatch, backend):
    """NT with A = [agg | h] concatenated along K (k1 not a multiple of the
    32-wide slice), bias, a device row count, and a second NT problem in the
    same launch."""
    from fast_b200 import ops
    _backend(monkeypatch, backend)
    torch.manual_seed(11)
    M, D, dn = 3000, 100, 100
    agg, h = torch.randn(M, D), torch.randn(M, dn)
    Wo, bo = torch.randn(D, D + dn) / 14, torch.randn(D)
    Xq, Wq = torch.randn(M, 200), torch.randn(100, 200) / 14
    m_true = 2345
    cnt = torch.tensor([m_true], dtype=torch.int32, device=cuda)
    hw = torch.cat([h, torch.zeros(M, 28)], 1).to(cuda)
    Z = torch.full((M, D), 7.0, device=cuda)
    Q = torch.empty(M, 100, device=cuda)
    ops.gemm_group([dict(kind=ops.NT, A=agg.to(cuda), A2=hw[:, :dn], B=Wo.to(cuda), bias=bo.to(cuda), out=Z,
                         M_dev=cnt),
                    dict(kind=ops.NT, A=Xq.to(cuda), B=Wq.to(cuda), out=Q)])
    assert ops.tc_error() == 0
    cat = torch.cat([agg, h], 1)
    parity(Z[:m_true], cat[:m_true].double() @ Wo.double().t() + bo.double(), cat[:m_true] @ Wo.t() + bo, "Z")
    assert bool((Z[m_true:] == 7.0).all())
    parity(Q, Xq.double() @ Wq.double().t(), Xq @ Wq.t(), "Q")
