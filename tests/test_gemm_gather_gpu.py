"""GPU: projection GEMMs, the fused gather + time encoding and its backward,
against plain PyTorch references.

GEMM outputs are compared with an fp64 product at rtol 1e-5 / atol 1e-6,
plus the classical fp32 dot-product error bound gamma_K * sum_k |a_k b_k|
where a K-long sum can exceed atol on near-zero outputs.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _close_fp32(got, a, b, rtol=1e-5, atol=1e-6):
    """got ~= a @ b within rtol/atol or the fp32 summation bound."""
    exact = a.double() @ b.double()
    bound = (a.double().abs() @ b.double().abs()) * (a.shape[1] * 2.0 ** -24) * 2
    err = (got.double() - exact).abs()
    ok = (err <= atol + rtol * exact.abs()) | (err <= bound)
    assert bool(ok.all()), float((err - atol - rtol * exact.abs()).max())


@pytest.mark.parametrize("M,N,K", [(1, 100, 100), (777, 200, 272), (5000, 200, 372), (300, 100, 101),
                                   (129, 57, 33)])
def test_gemm_nt(cuda, M, N, K):
    from fast_b200 import ops
    torch.manual_seed(M + N + K)
    A = torch.randn(M, K)
    W = torch.randn(N, K) / K ** 0.5
    bias = torch.randn(N)
    out = ops.gemm_nt(A.to(cuda), W.to(cuda), bias.to(cuda)).cpu()
    _close_fp32(out - bias, A, W.t())
    # strided A (a column window of a wider matrix) and accumulate
    wide = torch.randn(M, K + 8)
    acc = torch.randn(M, N)
    outd = acc.to(cuda)
    ops.gemm_nt(wide.to(cuda)[:, 4:4 + K], W.to(cuda), None, out=outd, accumulate=True)
    _close_fp32(outd.cpu() - acc, wide[:, 4:4 + K], W.t())


@pytest.mark.parametrize("M,N,K", [(1000, 200, 272), (70000, 200, 372), (33, 100, 200), (4099, 100, 101)])
def test_gemm_tn_and_colsum(cuda, M, N, K):
    from fast_b200 import ops
    torch.manual_seed(M)
    G = torch.randn(M, N)
    X = torch.randn(M, K)
    out = ops.gemm_tn(G.to(cuda), X.to(cuda)).cpu()
    _close_fp32(out, G.t(), X)
    cs = ops.colsum(G.to(cuda)).cpu()
    _close_fp32(cs.unsqueeze(1), G.t(), torch.ones(M, 1))
    out2 = ops.gemm_tn(G.to(cuda), X.to(cuda)).cpu()
    assert torch.equal(out, out2)    # fixed-order split reduction


def test_gather_time_encode(cuda):
    """[h[idx] | f[eid] | cos(w dt + b)] against torch's Linear(1, d) + cos on the CPU."""
    from fast_b200 import ops
    rng = np.random.default_rng(0)
    n_nodes, n_e_tab, E = 500, 3000, 2000
    h = torch.randn(n_nodes, 100)
    f = torch.randn(n_e_tab, 172)
    hid = torch.from_numpy(rng.integers(0, n_nodes, E).astype(np.int32))
    eid = torch.from_numpy(rng.integers(0, n_e_tab, E).astype(np.int32))
    dt = torch.from_numpy((rng.random(E) * 1.4e8).astype(np.float32).round())
    lin = torch.nn.Linear(1, 100)
    lin.weight.data = torch.from_numpy(1 / 10 ** np.linspace(0, 9, 100, dtype=np.float32)).reshape(100, 1)
    lin.bias.data = torch.randn(100) * 0.1
    with torch.no_grad():
        ref = torch.cat([h[hid.long()], f[eid.long()], torch.cos(lin(dt.reshape(-1, 1)))], 1)
    out = ops.gather_time_encode(E, h=h.to(cuda), h_idx=hid.to(cuda), f=f.to(cuda), f_idx=eid.to(cuda),
                                 dt=dt.to(cuda), w=lin.weight.data.reshape(-1).to(cuda), b=lin.bias.data.to(cuda))
    torch.testing.assert_close(out.cpu()[:, :272], ref[:, :272], rtol=0, atol=0)
    torch.testing.assert_close(out.cpu()[:, 272:], ref[:, 272:], rtol=1e-5, atol=1e-6)
    # offset form (previous-layer rows nd + e), rows 7 .. 7 + 400 of a 500-row table
    out2 = ops.gather_time_encode(400, h=h.to(cuda), h_off=7, device=cuda)
    torch.testing.assert_close(out2.cpu(), h[7:407], rtol=0, atol=0)
    # time-only rows (dt = NULL -> cos(b), the zero-time query features)
    out3 = ops.gather_time_encode(3, w=lin.weight.data.reshape(-1).to(cuda), b=lin.bias.data.to(cuda))
    torch.testing.assert_close(out3.cpu(), torch.cos(lin.bias.data).expand(3, -1), rtol=1e-6, atol=1e-7)


def test_time_encode_bwd_sine_accuracy(cuda):
    """The sine inside the time-encoding backward, one argument per column:
    one row with dt = 1, w = 0 and b = the arguments gives db[c] = -sin(b[c])
    exactly (x = fma(1, 0, b) = b, one term per sum).  Arguments: log-uniform
    magnitudes from 1e-6 to 1e9, the floats nearest to k pi/2 (the hardest
    reductions) for k up to 1e8, the floats nearest to (k + 1/2) pi/2 just
    below 2^22 (the largest reduced arguments of the fp32 reduction) and the
    edges of each reduction range (2^22: fp32 / double, 2^28: double / the
    library's sine).  Every value is within 2 ulp of the double sine of the
    same float."""
    from fast_b200 import ops
    rng = np.random.default_rng(7)
    mags = 10.0 ** rng.uniform(-6, 9, 6000)
    args = [(mags * rng.choice([-1.0, 1.0], mags.size)).astype(np.float32)]
    ks = np.concatenate([np.arange(1, 4000), rng.integers(4000, 340000, 3000), rng.integers(340000, 10 ** 8, 2000)])
    near = (ks.astype(np.float64) * (np.pi / 2)).astype(np.float32)
    args += [near, -near, np.nextafter(near, np.float32(np.inf)), np.nextafter(near, np.float32(0))]
    edges = np.array([2.0 ** 19, 2.0 ** 22, 2.0 ** 28, 0.7853981633974483, 1.5707963267948966], dtype=np.float32)
    args += [edges, np.nextafter(edges, np.float32(0)), np.nextafter(edges, np.float32(np.inf)), -edges,
             np.array([0.0, -0.0, 1e-30, -1e-30, 1e-38], dtype=np.float32),
             ((np.arange(2600000, 2670000, 7) + 0.5) * (np.pi / 2)).astype(np.float32)]
    x = np.concatenate(args)
    d = 512
    x = np.concatenate([x, np.zeros((-x.size) % d, dtype=np.float32)])
    got = np.empty_like(x)
    one = torch.ones(1, device=cuda)
    g = torch.ones(1, d, device=cuda)
    w = torch.zeros(d, device=cuda)
    for i in range(0, x.size, d):
        b = torch.from_numpy(x[i:i + d]).to(cuda)
        dw = torch.zeros(d, device=cuda)
        db = torch.zeros(d, device=cuda)
        ops.time_encode_bwd(g, one, w, b, dw, db)
        got[i:i + d] = -db.cpu().numpy()
        assert torch.equal(dw, db)
    ref = np.sin(x.astype(np.float64))
    err = np.abs(got.astype(np.float64) - ref)
    ulp = np.spacing(np.abs(ref).astype(np.float32)).astype(np.float64)
    assert np.all(err <= 2 * ulp), float(np.max(err / ulp))


@pytest.mark.parametrize("d", [100, 50, 37])
@pytest.mark.parametrize("dt_max", [1e4, 2e8, 3e8])
def test_time_encode_bwd(cuda, dt_max, d):
    """dw, db of cos(w dt + b) against an fp64 sum over the same single-rounded
    arguments; E-term sums are compared within the fp32 summation bound
    sum|terms| * E * 2^-24.  dt up to 2e8 (the timestamps of the synthetic
    graphs) exercises the kernel's own argument reduction, 3e8 the fallback
    beyond it.  Widths 100 and 50 take the kernel with four and two columns
    per thread, 37 the one-column kernel."""
    from fast_b200 import ops
    rng = np.random.default_rng(1)
    E = 5000
    dt = torch.from_numpy((rng.random(E) * dt_max).astype(np.float32))
    w = torch.from_numpy(1 / 10 ** np.linspace(0, 9, d, dtype=np.float32))
    b = torch.randn(d) * 0.1
    g = torch.randn(E, d)
    y = (dt.double().unsqueeze(1) * w.double().unsqueeze(0) + b.double()).float()   # fma rounding
    s = torch.sin(y.double())
    ref_w = (-s * g.double() * dt.double().unsqueeze(1)).sum(0)
    ref_b = (-s * g.double()).sum(0)
    terms_w = (s * g.double() * dt.double().unsqueeze(1)).abs().sum(0)
    terms_b = (s * g.double()).abs().sum(0)
    dw = torch.zeros(d, device=cuda)
    db = torch.zeros(d, device=cuda)
    ops.time_encode_bwd(g.to(cuda), dt.to(cuda), w.to(cuda), b.to(cuda), dw, db)
    for got, ref, terms in ((dw.cpu(), ref_w, terms_w), (db.cpu(), ref_b, terms_b)):
        err = (got.double() - ref).abs()
        assert bool((err <= 1e-6 + 1e-5 * ref.abs() + terms * E * 2.0 ** -24).all())
