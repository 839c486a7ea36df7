"""GPU: the layer-tail, edge-predictor/loss, NN-GEMM and bias-folded TN-GEMM
kernels against fp64 PyTorch references of the same math
(layers.py:213-223, layers.py:31-50, train.py:205-206).

Tolerance: elementwise |dev - ref64| <= 1e-6 + 1e-5 |ref64|, or, for long
sums, the norm form of the parity criterion (conftest.parity)."""
import pytest
import torch

from conftest import parity

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-5, 1e-6


def _close(dev, ref64, ref32=None, name=""):
    dev = dev.double().cpu()
    ref64 = ref64.double().cpu()
    err = (dev - ref64).abs()
    if bool((err <= ATOL + RTOL * ref64.abs()).all()):
        return
    assert ref32 is not None, "%s: max err %g" % (name, float(err.max()))
    assert parity(dev, ref64, ref32.double().cpu()), "%s: max err %g" % (name, float(err.max()))


def _tail_ref(z, gamma, beta, keep, p, dout, dtype):
    z = z.to(dtype).requires_grad_(True)
    g = gamma.to(dtype).requires_grad_(True)
    b = beta.to(dtype).requires_grad_(True)
    y = torch.relu(z * keep.to(dtype) / (1 - p))
    out = torch.nn.functional.layer_norm(y, (z.shape[1],), g, b, 1e-5)
    out.backward(dout.to(dtype))
    return y.detach(), out.detach(), z.grad, g.grad, b.grad


@pytest.mark.parametrize("n,d,p", [(1000, 100, 0.0), (777, 100, 0.3), (300, 256, 0.1), (50, 12, 0.0)])
def test_layer_tail_fwd_bwd(cuda, n, d, p):
    from fast_b200 import ops
    torch.manual_seed(n + d)
    z = torch.randn(n, d)
    gamma, beta = 1 + 0.1 * torch.randn(d), 0.1 * torch.randn(d)
    u = torch.rand(n, d)
    keep = (u >= p).float()
    dout = torch.randn(n, d)
    n_true = n - 7
    y64, o64, dz64, dg64, db64 = _tail_ref(z[:n_true], gamma, beta, keep[:n_true], p, dout[:n_true], torch.float64)
    _, o32, dz32, dg32, db32 = _tail_ref(z[:n_true], gamma, beta, keep[:n_true], p, dout[:n_true], torch.float32)
    zc, gc, bc = z.to(cuda), gamma.to(cuda), beta.to(cuda)
    cnt = torch.tensor([n_true], dtype=torch.int32, device=cuda)
    y, out = ops.layer_tail_fwd(zc, gc, bc, drop_p=p, mask_u=u.to(cuda) if p > 0 else None, n_dev=cnt)
    _close(y[:n_true], y64, name="y")
    _close(out[:n_true], o64, o32, "out")
    assert bool((out[n_true:] == 0).all())
    dgamma = torch.full((d,), 0.5, device=cuda)      # accumulates
    dbeta = torch.zeros(d, device=cuda)
    dz = ops.layer_tail_bwd(dout.to(cuda), y, gc, dgamma, dbeta, drop_p=p, n_dev=cnt)
    _close(dz[:n_true], dz64, dz32, "dz")
    _close(dgamma - 0.5, dg64, dg32, "dgamma")
    _close(dbeta, db64, db32, "dbeta")


def test_layer_tail_gate_zeroes_an_edgeless_block(cuda):
    from fast_b200 import ops
    n, d = 64, 100
    z = torch.randn(n, d, device=cuda)
    gamma, beta = torch.ones(d, device=cuda), torch.randn(d, device=cuda)
    gate = torch.zeros(1, dtype=torch.int32, device=cuda)
    y, out = ops.layer_tail_fwd(z, gamma, beta, gate_dev=gate)
    assert bool((out == 0).all())
    dg, db = torch.zeros(d, device=cuda), torch.zeros(d, device=cuda)
    dz = ops.layer_tail_bwd(torch.randn(n, d, device=cuda), y, gamma, dg, db, gate_dev=gate)
    assert bool((dz == 0).all()) and bool((dg == 0).all()) and bool((db == 0).all())


def _pred_ref(S, P, w, b, dtype):
    S = S.to(dtype).requires_grad_(True)
    P = P.to(dtype).requires_grad_(True)
    w = w.to(dtype).requires_grad_(True)
    b = b.to(dtype).requires_grad_(True)
    B = S.shape[0]
    xp = torch.relu(S + P[:B]) @ w + b
    xn = torch.relu(S + P[B:]) @ w + b
    crit = torch.nn.BCEWithLogitsLoss()
    loss = crit(xp, torch.ones_like(xp)) + crit(xn, torch.zeros_like(xn))
    loss.backward()
    return loss.detach(), torch.cat([xp, xn]).detach(), S.grad, P.grad, w.grad, b.grad


@pytest.mark.parametrize("B,d", [(600, 100), (37, 8), (2000, 172)])
def test_edge_predictor_loss(cuda, B, d):
    from fast_b200 import ops
    torch.manual_seed(B)
    S, P = torch.randn(B, d), torch.randn(2 * B, d)
    w, b = torch.randn(d) * 0.3, torch.randn(1)
    r64 = _pred_ref(S, P, w, b, torch.float64)
    r32 = _pred_ref(S, P, w, b, torch.float32)
    loss = torch.zeros((), device=cuda)
    dS, dP = torch.empty(B, d, device=cuda), torch.empty(2 * B, d, device=cuda)
    dw, db = torch.zeros(d, device=cuda), torch.zeros(1, device=cuda)
    scores = torch.empty(2 * B, device=cuda)
    ops.edge_predictor_loss(S.to(cuda), P.to(cuda), w.to(cuda), b.to(cuda), loss, dS, dP, dw, db, scores=scores)
    for name, dev, a, c in zip(["loss", "scores", "dS", "dP", "dw", "db"], [loss, scores, dS, dP, dw, db], r64, r32):
        _close(dev, a, c, name)


@pytest.mark.parametrize("M,N,K", [(1000, 100, 100), (333, 172, 200), (5, 100, 372), (4000, 100, 200)])
def test_gemm_nn(cuda, M, N, K):
    from fast_b200 import ops
    torch.manual_seed(M)
    A, Bfull = torch.randn(M, K), torch.randn(K, N + 3)
    B = Bfull[:, :N]                                             # strided B (ldb = N + 3)
    ref64 = A.double() @ B.double()
    ref32 = A @ B
    C = torch.full((M, N), 2.0, device=cuda)
    ops.gemm_nn(A.to(cuda), Bfull.to(cuda)[:, :N], out=C, accumulate=True)
    _close(C - 2.0, ref64, ref32, "C")


@pytest.mark.parametrize("M,N,K", [(1000, 200, 272), (37, 100, 100), (5000, 100, 1), (20000, 200, 372)])
def test_gemm_tn_bias(cuda, M, N, K):
    from fast_b200 import ops
    torch.manual_seed(K)
    G, X = torch.randn(M, N), torch.randn(M, K)
    m_true = M - 3
    ref64 = G[:m_true].double().t() @ X[:m_true].double()
    ref32 = G[:m_true].t() @ X[:m_true]
    db64, db32 = G[:m_true].double().sum(0), G[:m_true].sum(0)
    cnt = torch.tensor([m_true], dtype=torch.int32, device=cuda)
    C = torch.ones(N, K, device=cuda)
    db = torch.ones(N, device=cuda)
    ops.gemm_tn(G.to(cuda), X.to(cuda), out=C, accumulate=True, M_dev=cnt, db=db)
    _close(C - 1.0, ref64, ref32, "dW")
    _close(db - 1.0, db64, db32, "db")
    v = torch.full((N,), 7.0, device=cuda)
    ops.gemm_tn(G.to(cuda), X.to(cuda), M_dev=cnt, db=v, db_accumulate=False)
    _close(v, db64, db32, "db (overwrite)")


@pytest.mark.parametrize("dn,with_row", [(0, True), (100, False)])
def test_q_time_bwd(cuda, dn, with_row):
    from fast_b200 import ops
    D, dtime = 100, 100
    torch.manual_seed(dn)
    v = torch.randn(D)
    Wq = torch.randn(D, dn + dtime)
    bt = torch.randn(dtime)
    qin0 = torch.cos(bt) if with_row else None
    dbq = torch.randn(D)
    dbt = torch.randn(dtime)
    dWq = torch.randn(D, dn + dtime)
    def expect(t):
        return (dbq.to(t) + v.to(t), dbt.to(t) - torch.sin(bt.to(t)) * (v.to(t) @ Wq[:, dn:].to(t)),
                dWq.to(t) + (torch.outer(v.to(t), qin0.to(t)) if with_row else 0))
    e64, e32 = expect(torch.float64), expect(torch.float32)
    g_dbq, g_dbt, g_dWq = dbq.to(cuda), dbt.to(cuda), dWq.to(cuda)
    ops.q_time_bwd(v.to(cuda), Wq.to(cuda), dn, dtime, bt.to(cuda), g_dbq, g_dbt,
                   qin0=qin0.to(cuda) if with_row else None, dW_q=g_dWq if with_row else None)
    for name, dev, a, c in zip(["db_q", "db_t", "dW_q"], [g_dbq, g_dbt, g_dWq], e64, e32):
        _close(dev, a, c, name)


def test_gemm_group_mixed(cuda):
    """One grouped launch: NT with A concatenated along K, NN, TN with the bias
    column, TN column sums only (K == 0), and a device-side row count."""
    from fast_b200 import ops
    torch.manual_seed(5)
    M, D, dn, E = 900, 100, 100, 2500
    agg, hd = torch.randn(M, D), torch.randn(M, dn + 100)[:, :dn]
    Wo, bo = torch.randn(D, D + dn), torch.randn(D)
    dKV, A, Wkv = torch.randn(E, 2 * D), torch.randn(E, 272), torch.randn(2 * D, 272)
    dQ = torch.randn(M, D)
    e_true = E - 11
    cnt = torch.tensor([e_true], dtype=torch.int32, device=cuda)
    c = lambda t: t.to(cuda)                  # noqa: E731
    hd_d = c(torch.cat([hd, torch.zeros(M, 100)], 1))[:, :dn]
    Z = torch.empty(M, D, device=cuda)
    dA = torch.full((E, 72), 3.0, device=cuda)
    gW = torch.ones(2 * D, 272, device=cuda)
    gb = torch.ones(2 * D, device=cuda)
    v = torch.full((D,), 9.0, device=cuda)
    ops.gemm_group([
        dict(kind=ops.NT, A=c(agg), A2=hd_d, B=c(Wo), bias=c(bo), out=Z),
        dict(kind=ops.NN, A=c(dKV), B=c(Wkv)[:, 200:], out=dA, M_dev=cnt),
        dict(kind=ops.TN, A=c(dKV), B=c(A), out=gW, accumulate=True, M_dev=cnt, db=gb),
        dict(kind=ops.TN, A=c(dQ), B=None, out=None, db=v, db_accumulate=False)])
    r = lambda t: t.double()                  # noqa: E731
    exp = {
        "Z": (torch.cat([agg, hd], 1).double() @ r(Wo).t() + r(bo), torch.cat([agg, hd], 1) @ Wo.t() + bo, Z),
        "dA": (r(dKV[:e_true]) @ r(Wkv[:, 200:]), dKV[:e_true] @ Wkv[:, 200:], dA[:e_true]),
        "gW": (r(dKV[:e_true]).t() @ r(A[:e_true]), dKV[:e_true].t() @ A[:e_true], gW - 1.0),
        "gb": (r(dKV[:e_true]).sum(0), dKV[:e_true].sum(0), gb - 1.0),
        "v": (r(dQ).sum(0), dQ.sum(0), v),
    }
    for name, (e64, e32, got) in exp.items():
        _close(got, e64, e32, name)
    assert bool((dA[e_true:] == 3.0).all())           # rows past the count untouched
