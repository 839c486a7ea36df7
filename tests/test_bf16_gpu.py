"""GPU: the bf16 precision mode's kernels.

* fb_gemm_bf16_group (tcgen05 kind::f16) against an fp64 product of the same
  bf16 operands: the products of bf16 values are exact in fp32, so the only
  difference is the fp32 accumulation, bounded by K * 2^-23 * sum |a b|.
  NT (with bias, accumulate, A | A2 concatenation), NN on a column block of a
  bf16 weight copy, TN with the bias gradient; operand rows past the
  device-side count hold NaN and must not reach the result.
* fb_cast_bf16, fb_gather_time_encode_bf16, fb_attn_bwd_bf16kv and the bf16
  output of the GEMM are bit-exact against round-to-nearest-even of the fp32
  kernels' outputs; the attention on bf16 K|V rows (fb_attn_fwd_kvbf16 /
  fb_attn_bwd_kvbf16) equals the fp32 attention on the same, rounded, rows;
  fb_time_encode_bwd_bf16 equals fb_time_encode_bwd on the widened gradient.
* A whole FusedStep in the bf16 mode against oracle/bf16_math.py: the
  reference layer in fp64 with bf16 rounding at exactly the device's
  rounding points, on the oracle sampler's blocks.  Relative L2 error
  <= 2e-3 per gradient tensor, or no more than 5x the error of the oracle's
  own fp32 run (the form of the fp32 step's parity rule; the device's K
  passes through the tensor cores' fp32 accumulation before its bf16
  rounding, so it meets more ties than the CPU run), with the key and value
  biases as one vector (the
  key bias's exact gradient nearly vanishes) and <= 1e-3 for the loss and
  predictions
  (what remains is fp32 arithmetic and the rare operand that fp32 and fp64
  round to neighbouring bf16 values), with node / edge widths (413 / 186)
  that exercise every padded segment, on a model whose ReLU inputs sit away
  from the kink.  The plain bf16 error against the exact fp64 reference is
  reported beside it: at initialisation the positive and negative loss
  gradients nearly cancel, which lifts it to several percent.
"""
import copy

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _bf(x):
    return x.to(torch.bfloat16)


def _check(got, a64, b64, K, name, base=None):
    """|got - (base + a64 @ b64)| <= K 2^-23 (|a| @ |b|) + 2^-23 (|base| + |ref|),
    elementwise: the accumulation bound plus the fp32 roundings of adding
    bias / the accumulated output."""
    ref = a64 @ b64
    bound = K * 2.0 ** -23 * (a64.abs() @ b64.abs()) + 1e-30
    if base is not None:
        base = base.double()
        ref = ref + base
        bound = bound + 2.0 ** -23 * (base.abs() + ref.abs())
    err = (got.double() - ref).abs()
    bad = (err > bound) | ~torch.isfinite(got)
    assert not bool(bad.any()), "%s: %d of %d outside the fp32-accumulation bound (max err %.3e)" % (
        name, int(bad.sum()), bad.numel(), float(err.max()))


def test_gemm_bf16_nt_bias_accumulate(cuda):
    from fast_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(3)
    M, N, K = 1000, 200, 708
    A = _bf(torch.randn(M, 712, generator=g)).to(cuda)[:, :K]
    W = _bf(torch.randn(N, 712, generator=g) * 0.05).to(cuda)[:, :K]
    bias = torch.randn(N, generator=g).to(cuda)
    C0 = torch.randn(M, N, generator=g).to(cuda)
    C = C0.clone()
    ops.gemm_bf16_group([dict(kind=ops.NT, A=A, B=W, bias=bias, out=C, accumulate=True)])
    torch.cuda.synchronize()
    _check(C, A.double(), W.double().T, K, "NT", base=C0.double() + bias.double())


def test_gemm_bf16_nt_concat_and_device_rows(cuda):
    from fast_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(4)
    M, D, dn = 777, 100, 413
    agg = _bf(torch.randn(M, 104, generator=g)).to(cuda)
    agg[:, D:] = float("nan")                  # past A's width (ka): must read as zeros
    qin = _bf(torch.randn(M, 520, generator=g)).to(cuda)
    W = torch.zeros(D, 104 + 416, dtype=torch.bfloat16, device=cuda)
    W[:, :D] = _bf(torch.randn(D, D, generator=g) * 0.05).to(cuda)
    W[:, 104:104 + dn] = _bf(torch.randn(D, dn, generator=g) * 0.05).to(cuda)
    n_dev = torch.tensor([700], dtype=torch.int32, device=cuda)
    C = torch.full((M, D), 7.0, device=cuda)
    ops.gemm_bf16_group([dict(kind=ops.NT, A=agg[:, :D], A2=qin[:, :dn], k1=104, B=W[:, :104 + dn], out=C,
                              M_dev=n_dev)])
    torch.cuda.synchronize()
    a64 = torch.cat([agg[:700, :D].double(), torch.zeros(700, 4, dtype=torch.float64, device=cuda),
                     qin[:700, :dn].double()], 1)
    _check(C[:700], a64, W[:, :104 + dn].double().T, 104 + dn, "NT concat")
    assert bool((C[700:] == 7.0).all())


def test_gemm_bf16_nn_on_weight_columns(cuda):
    from fast_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(5)
    M, K = 2500, 200
    G = _bf(torch.randn(M, K, generator=g)).to(cuda)
    Wf = _bf(torch.randn(K, 712, generator=g) * 0.05).to(cuda)
    for c0, n in ((608, 100), (0, 413), (416, 186)):
        B = Wf[:, c0:c0 + n]
        C = torch.empty(M, n, device=cuda)
        ops.gemm_bf16_group([dict(kind=ops.NN, A=G, B=B, out=C)])
        torch.cuda.synchronize()
        _check(C, G.double(), B.double(), K, "NN cols %d" % c0)


@pytest.mark.parametrize("c16", [True, False])
def test_gemm_bf16_nt_epilogue_adds_table_rows(cuda, c16):
    """NT with an fp32 table added per output row (C[m] += add[add_idx[m]]):
    the node-feature block of layer 0's K|V product, computed once per table
    row.  Equal to the product plus the gathered rows within the fp32
    accumulation bound (then one bf16 rounding for a bf16 C); rows past the
    device-side count carry out-of-range indices and stay untouched."""
    from fast_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(12)
    M, m_dev, N, K, rows = 5000, 4700, 200, 292, 777
    X = _bf(torch.randn(M, 296, generator=g)).to(cuda)[:, :K]
    W = _bf(torch.randn(N, 296, generator=g) * 0.05).to(cuda)[:, :K]
    P = torch.randn(rows, N, generator=g).to(cuda)
    idx = torch.randint(0, rows, (M,), generator=g, dtype=torch.int32)
    idx[m_dev:] = 10 ** 7
    idx = idx.to(cuda)
    bias = torch.randn(N, generator=g).to(cuda)
    n_dev = torch.tensor([m_dev], dtype=torch.int32, device=cuda)
    C = torch.full((M, N), 7.0, device=cuda, dtype=torch.bfloat16 if c16 else torch.float32)
    ops.gemm_bf16_group([dict(kind=ops.NT, A=X, B=W, bias=bias, out=C, M_dev=n_dev, add=P, add_idx=idx)])
    torch.cuda.synchronize()
    base = bias.double() + P[idx[:m_dev].long()].double()
    if c16:
        a64, w64 = X[:m_dev].double(), W.double().T
        exact = a64 @ w64 + base
        # the fp32 accumulation bound, then one bf16 rounding of a value that fp32
        # may have moved across a rounding boundary
        acc = K * 2.0 ** -23 * (a64.abs() @ w64.abs()) + 2.0 ** -22 * (bias.double().abs() +
                                                                      P[idx[:m_dev].long()].double().abs() +
                                                                      exact.abs())
        err = (C[:m_dev].double() - exact).abs()
        assert bool((err <= acc + 2.0 ** -7 * (exact.abs() + acc)).all())
    else:
        _check(C[:m_dev], X[:m_dev].double(), W.double().T, K, "NT + rows", base=base)
    assert bool((C[m_dev:].float() == 7.0).all())


@pytest.mark.parametrize("M,m_dev,dn,layout", [(3000, 2777, 413, "tables"), (70001, 70001, 413, "tables"),
                                                (20000, 1, 413, "tables"), (5000, 4321, 0, "tables"),
                                                (3000, 2777, 413, "node_rows"), (70001, 70001, 413, "node_rows")])
def test_gemm_bf16_gathered_rows(cuda, M, m_dev, dn, layout):
    """The projection rows [h | f | t] gathered inside the GEMM (ops.RowGather:
    node rows by node id, edge rows by edge id, the time block row by row,
    64-column segments; "node_rows": node rows by node id, then one matrix
    [f | t] read row by row, the layer-0 weight gradient's operand) give, for
    NT and for the segmented TN with the bias gradient, the products of the
    materialised rows within the fp32 accumulation bound.  Rows past the
    device-side count carry indices far outside the tables and NaN rows: they
    must reach no output."""
    from fast_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(11)
    de, dt, D2 = 186, 100, 200
    n_nodes, n_edge_rows = 1667, 9000
    ntab = torch.zeros(n_nodes, 416, dtype=torch.bfloat16)
    ntab[:, :dn] = _bf(torch.randn(n_nodes, dn, generator=g))
    etab = torch.zeros(n_edge_rows, 192, dtype=torch.bfloat16)
    etab[:, :de] = _bf(torch.randn(n_edge_rows, de, generator=g))
    ntab, etab = ntab.to(cuda), etab.to(cuda)
    nid = torch.randint(0, n_nodes, (M,), generator=g, dtype=torch.int32)
    nid[::7] = 3                                             # repeated rows
    eid = torch.randint(0, n_edge_rows, (M,), generator=g, dtype=torch.int32)
    nid[m_dev:], eid[m_dev:] = 2 ** 30, -5                     # stale indices past the count
    nid, eid = nid.to(cuda), eid.to(cuda)
    T = torch.zeros(M, 104, dtype=torch.bfloat16)
    T[:, :dt] = _bf(torch.rand(M, dt, generator=g) * 2 - 1)
    T[m_dev:] = float("nan")
    T = T.to(cuda)
    segs, cols, wid = [], [], []
    if dn:
        segs.append((ntab, dn, nid, 448)); cols.append(dn); wid.append(448)
    if layout == "tables":
        segs += [(etab, de, eid, 192), (T, dt, None, 128)]
        cols += [de, dt]; wid += [192, 128]
    else:
        # [f | t] rows written by the gather: f at 0, t at 192, 296 columns
        XF = torch.zeros(M, 296, dtype=torch.bfloat16, device=cuda)
        XF[:m_dev, :de] = etab[eid[:m_dev].long(), :de]
        XF[:, 192:192 + dt] = T[:, :dt]
        segs.append((XF, 192 + dt, None, 320)); cols.append(192 + dt); wid.append(320)
    gat = ops.RowGather(segs)
    K = gat.K
    # the materialised rows (past the count: zeros) and the weights in the same column layout
    X = torch.zeros(m_dev, K, dtype=torch.float64, device=cuda)
    at = 0
    for (tab, c, idx, w) in segs:
        X[:, at:at + c] = (tab[idx[:m_dev].long(), :c] if idx is not None else tab[:m_dev, :c]).double()
        at += w
    W = torch.zeros(D2, K, dtype=torch.bfloat16, device=cuda)
    at = 0
    for c, w in zip(cols, wid):
        W[:, at:at + c] = _bf(torch.randn(D2, c, generator=g) * 0.05).to(cuda)
        at += w
    bias = torch.randn(D2, generator=g).to(cuda)
    n_dev = torch.tensor([m_dev], dtype=torch.int32, device=cuda)
    C = torch.full((M, D2), 7.0, device=cuda)
    ops.gemm_bf16_group([dict(kind=ops.NT, gather=gat, M=M, B=W, bias=bias, out=C, M_dev=n_dev)])
    torch.cuda.synchronize()
    _check(C[:m_dev], X, W.double().T, K, "gathered NT", base=bias.double().expand(m_dev, D2))
    assert bool((C[m_dev:] == 7.0).all())
    # segmented TN with the bias gradient: dW[:, to + j] += sum_m G[m] X[m, at + j]
    G = _bf(torch.randn(M, D2, generator=g)).to(cuda)
    G[m_dev:] = float("nan")
    dW0 = torch.randn(D2, sum(cols), generator=g).to(cuda)
    dW = dW0.clone()
    db = torch.zeros(D2, device=cuda)
    tn_segs, at, to = [], 0, 0
    for c, w in zip(cols, wid):
        tn_segs.append((at, c, to))
        at, to = at + w, to + c
    ops.gemm_bf16_group([dict(kind=ops.TN, A=G, gather=gat, out=dW, accumulate=True, db=db, db_accumulate=False,
                              M_dev=n_dev, segs=tn_segs)])
    torch.cuda.synchronize()
    Xc = torch.cat([X[:, a:a + c] for a, c, _ in tn_segs], 1)
    g64 = G[:m_dev].double()
    _check(dW, g64.T, Xc, m_dev, "gathered TN dW", base=dW0)
    _check(db.reshape(-1, 1), g64.T, torch.ones(m_dev, 1, dtype=torch.float64, device=cuda), m_dev, "gathered TN db")


@pytest.mark.parametrize("M,m_dev", [(3000, 2777), (70000, 70000), (20000, 1)])
def test_gemm_bf16_tn_bias_gradient_masks_stale_rows(cuda, M, m_dev):
    from fast_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(6)
    N, K = 200, 413
    G = _bf(torch.randn(M, N, generator=g)).to(cuda)
    X = _bf(torch.randn(M, 712, generator=g)).to(cuda)
    G[m_dev:] = float("nan")
    X[m_dev:] = float("nan")
    dW0 = torch.randn(N, K, generator=g).to(cuda)
    dW = dW0.clone()
    db = torch.zeros(N, device=cuda)
    n_dev = torch.tensor([m_dev], dtype=torch.int32, device=cuda)
    ops.gemm_bf16_group([dict(kind=ops.TN, A=G, B=X[:, :K], out=dW, accumulate=True, db=db, db_accumulate=False,
                              M_dev=n_dev)])
    torch.cuda.synchronize()
    g64, x64 = G[:m_dev].double(), X[:m_dev, :K].double()
    _check(dW, g64.T, x64, m_dev, "TN dW", base=dW0)
    ones = torch.ones(m_dev, 1, dtype=torch.float64, device=cuda)
    _check(db.reshape(-1, 1), g64.T, ones, m_dev, "TN db")


@pytest.mark.parametrize("M,m_dev", [(5000, 4321), (200000, 200000)])
def test_gemm_bf16_tn_column_segments(cuda, M, m_dev):
    """The K|V weight gradient over a bf16 projection row in one TN problem:
    X's columns in three segments at 8-column boundaries (the gaps hold NaN
    and are skipped), the bias gradient, accumulate; rows past the device
    count hold NaN."""
    from fast_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(12)
    N, segs = 200, [(0, 413, 0), (416, 186, 413), (608, 100, 599)]
    G = _bf(torch.randn(M, N, generator=g)).to(cuda)
    X = _bf(torch.randn(M, 712, generator=g)).to(cuda)
    X[:, 413:416] = float("nan")
    X[:, 602:608] = float("nan")
    G[m_dev:] = float("nan")
    X[m_dev:] = float("nan")
    dW0 = torch.randn(N, 699, generator=g).to(cuda)
    dW = dW0.clone()
    db0 = torch.randn(N, generator=g).to(cuda)
    db = db0.clone()
    n_dev = torch.tensor([m_dev], dtype=torch.int32, device=cuda)
    ops.gemm_bf16_group([dict(kind=ops.TN, A=G, B=X[:, :708], out=dW, accumulate=True, db=db, M_dev=n_dev,
                              segs=segs)])
    torch.cuda.synchronize()
    g64 = G[:m_dev].double()
    for at, ln, to in segs:
        _check(dW[:, to:to + ln], g64.T, X[:m_dev, at:at + ln].double(), m_dev, "TN seg %d" % at,
               base=dW0[:, to:to + ln])
    _check(db.reshape(-1, 1), g64.T, torch.ones(m_dev, 1, dtype=torch.float64, device=cuda), m_dev, "TN db",
           base=db0.reshape(-1, 1))


def test_gemm_bf16_group_mixed(cuda):
    """One launch: NT, NN and two TN problems, as a layer's backward level issues them."""
    from fast_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(7)
    M, D = 5000, 100
    dKV = _bf(torch.randn(M, 2 * D, generator=g)).to(cuda)
    X = _bf(torch.randn(M, 400, generator=g)).to(cuda)
    W = _bf(torch.randn(2 * D, 400, generator=g) * 0.05).to(cuda)
    gW = torch.zeros(2 * D, 396, device=cuda)
    gb = torch.zeros(2 * D, device=cuda)
    dt_ = torch.empty(M, 100, device=cuda)
    dh = torch.empty(M, 100, device=cuda)
    KV = torch.empty(M, 2 * D, device=cuda)
    ops.gemm_bf16_group([dict(kind=ops.TN, A=dKV, B=X[:, :290], out=gW[:, :290]),
                         dict(kind=ops.TN, A=dKV, B=X[:, 296:396], out=gW[:, 290:390], db=gb),
                         dict(kind=ops.NN, A=dKV, B=W[:, 296:396], out=dt_),
                         dict(kind=ops.NN, A=dKV, B=W[:, 0:100], out=dh),
                         dict(kind=ops.NT, A=X[:, :396], B=W[:, :396], out=KV)])
    torch.cuda.synchronize()
    d64, x64, w64 = dKV.double(), X.double(), W.double()
    _check(gW[:, :290], d64.T, x64[:, :290], M, "TN seg 0")
    _check(gW[:, 290:390], d64.T, x64[:, 296:396], M, "TN seg 1")
    _check(gb.reshape(-1, 1), d64.T, torch.ones(M, 1, dtype=torch.float64, device=cuda), M, "TN db")
    _check(dt_, d64, w64[:, 296:396], 2 * D, "NN te")
    _check(dh, d64, w64[:, :100], 2 * D, "NN h")
    _check(KV, x64[:, :396], w64[:, :396].T, 396, "NT")


def test_gemm_bf16_output_is_the_rounded_fp32_output(cuda):
    from fast_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(13)
    M, N, K = 3333, 200, 708
    A = _bf(torch.randn(M, 712, generator=g)).to(cuda)[:, :K]
    W = _bf(torch.randn(N, 712, generator=g) * 0.05).to(cuda)[:, :K]
    bias = torch.randn(N, generator=g).to(cuda)
    n_dev = torch.tensor([3000], dtype=torch.int32, device=cuda)
    C32 = torch.empty(M, N, device=cuda)
    C16 = torch.full((M, N), 5.0, device=cuda, dtype=torch.bfloat16)
    ops.gemm_bf16_group([dict(kind=ops.NT, A=A, B=W, bias=bias, out=C32, M_dev=n_dev)])
    ops.gemm_bf16_group([dict(kind=ops.NT, A=A, B=W, bias=bias, out=C16, M_dev=n_dev)])
    torch.cuda.synchronize()
    assert torch.equal(C16[:3000], C32[:3000].to(torch.bfloat16))
    assert bool((C16[3000:] == 5.0).all())


@pytest.mark.parametrize("drop", [0.0, 0.1])
def test_attention_on_bf16_kv_rows(cuda, drop):
    from fast_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(14)
    nd, D, H = 3000, 100, 2
    deg = torch.randint(0, 30, (nd,), generator=g)             # segments longer than one bulk group too
    rptr = torch.zeros(nd + 1, dtype=torch.int32)
    rptr[1:] = torch.cumsum(deg, 0)
    E = int(rptr[-1])
    rptr = rptr.to(cuda)
    q = torch.randn(nd, D, generator=g).to(cuda)
    kv16 = _bf(torch.randn(E, 2 * D, generator=g)).to(cuda)
    kv32 = kv16.float()
    dagg = torch.randn(nd, D, generator=g).to(cuda)
    agg, att = ops.attn_fwd_kvbf16(q, kv16, rptr, H, 0.2, drop, 7, 3)
    agg_r, att_r = ops.attn_fwd(q, kv32[:, :D], kv32[:, D:], rptr, H, 0.2, drop, 7, 3)
    dq, dkv = ops.attn_bwd_kvbf16(q, kv16, rptr, att, dagg, H, 0.2, drop, 7, 3)
    dq_r, dkv_r = ops.attn_bwd(q, kv32[:, :D], kv32[:, D:], rptr, att_r, dagg, H, 0.2, drop, 7, 3)
    torch.cuda.synchronize()
    assert torch.equal(agg, agg_r) and torch.equal(att, att_r)
    assert torch.equal(dq, dq_r)
    assert torch.equal(dkv, dkv_r.to(torch.bfloat16))


def test_cast_bf16_is_round_to_nearest_even(cuda):
    from fast_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(8)
    W = torch.randn(200, 699, generator=g).to(cuda)
    H = torch.randn(500, 100, generator=g).to(cuda)
    Wb = torch.zeros(200, 712, dtype=torch.bfloat16, device=cuda)
    Hb = torch.full((500, 104), 3.0, dtype=torch.bfloat16, device=cuda)
    rows = torch.tensor([321], dtype=torch.int32, device=cuda)
    ops.cast_bf16([(W[:, :413], Wb[:, :413]), (W[:, 413:599], Wb[:, 416:602]), (W[:, 599:], Wb[:, 608:708]),
                   (H, Hb[:, :100], rows)])
    torch.cuda.synchronize()
    assert torch.equal(Wb[:, :413], W[:, :413].to(torch.bfloat16))
    assert torch.equal(Wb[:, 416:602], W[:, 413:599].to(torch.bfloat16))
    assert torch.equal(Wb[:, 608:708], W[:, 599:].to(torch.bfloat16))
    assert bool((Wb[:, 413:416] == 0).all()) and bool((Wb[:, 602:608] == 0).all())
    assert torch.equal(Hb[:321, :100], H[:321].to(torch.bfloat16))
    assert bool((Hb[321:] == 3.0).all()) and bool((Hb[:, 100:] == 3.0).all())


def test_gather_bf16_matches_rounded_fp32_gather(cuda):
    from fast_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(9)
    n_nodes, n_edges, dn, de, dtime, E = 300, 5000, 413, 186, 100, 4099
    nf = torch.randn(n_nodes, dn, generator=g)
    ef = torch.randn(n_edges, de, generator=g)
    nf_b = torch.zeros(n_nodes, ops.pad8(dn), dtype=torch.bfloat16)
    nf_b[:, :dn] = nf.to(torch.bfloat16)
    ef_b = torch.zeros(n_edges, ops.pad8(de), dtype=torch.bfloat16)
    ef_b[:, :de] = ef.to(torch.bfloat16)
    nf_b, ef_b = nf_b.to(cuda), ef_b.to(cuda)
    nid = torch.randint(0, n_nodes, (E,), generator=g, dtype=torch.int32).to(cuda)
    eid = torch.randint(0, n_edges, (E,), generator=g, dtype=torch.int32).to(cuda)
    dt = (torch.rand(E, generator=g) * 1e5).to(cuda)
    w = torch.randn(dtime, generator=g).to(cuda)
    b = torch.randn(dtime, generator=g).to(cuda)
    X, width = ops.gather_time_encode_bf16(E, h=nf_b, h_idx=nid, f=ef_b, f_idx=eid, dt=dt, w=w, b=b, dn=dn, de=de)
    ref = ops.gather_time_encode(E, dt=dt, w=w, b=b)             # fp32 cos(w dt + b) from the fp32 kernel
    torch.cuda.synchronize()
    assert width == 416 + 192 + 100 and X.shape[1] == 712
    assert torch.equal(X[:, :416], nf_b[nid.long()])
    assert torch.equal(X[:, 416:608], ef_b[eid.long()])
    assert torch.equal(X[:, 608:708], ref.to(torch.bfloat16))
    # fp32 source (a layer's output) with a device row count
    h = torch.randn(E, 100, generator=g).to(cuda)
    n_dev = torch.tensor([4000], dtype=torch.int32, device=cuda)
    out = torch.full((E, 400), 5.0, dtype=torch.bfloat16, device=cuda)
    ops.gather_time_encode_bf16(E, h=h, f=ef_b, f_idx=eid, dt=dt, w=w, b=b, de=de, out=out, n_rows_dev=n_dev)
    torch.cuda.synchronize()
    assert torch.equal(out[:4000, :100], h[:4000].to(torch.bfloat16))
    assert bool((out[:4000, 100:104] == 0).all())
    assert torch.equal(out[:4000, 104:296], ef_b[eid[:4000].long()])
    assert torch.equal(out[:4000, 296:396], ref[:4000].to(torch.bfloat16))
    assert bool((out[4000:] == 5.0).all())


def test_attn_bwd_bf16kv_is_the_rounded_fp32_gradient(cuda):
    from fast_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(10)
    nd, fan, D, H = 2000, 10, 100, 2
    E = nd * fan
    rptr = torch.arange(0, E + 1, fan, dtype=torch.int32).to(cuda)
    q = torch.randn(nd, D, generator=g).to(cuda)
    kv = torch.randn(E, 2 * D, generator=g).to(cuda)
    dagg = torch.randn(nd, D, generator=g).to(cuda)
    agg, att = ops.attn_fwd(q, kv[:, :D], kv[:, D:], rptr, H, 0.2, 0.1, 11, 0)
    dq, dkv = ops.attn_bwd(q, kv[:, :D], kv[:, D:], rptr, att, dagg, H, 0.2, 0.1, 11, 0)
    dq_b, dkv_b = ops.attn_bwd_bf16kv(q, kv[:, :D], kv[:, D:], rptr, att, dagg, H, 0.2, 0.1, 11, 0)
    torch.cuda.synchronize()
    assert torch.equal(dq_b, dq)
    assert torch.equal(dkv_b, dkv.to(torch.bfloat16))


@pytest.mark.parametrize("E,e_dev,d", [(5000, 4444, 100), (330000, 330000, 100), (5000, 4999, 600)])
def test_time_encode_bwd_bf16_is_the_fp32_sum_of_the_widened_gradient(cuda, E, e_dev, d):
    """fb_time_encode_bwd_bf16 on bf16 g gives fb_time_encode_bwd's result
    on g widened to fp32, bit for bit (same partition, same summation order),
    with the row count read on the device; 600 columns take the 32-column
    tile kernel instead of the one for rows of up to 512."""
    from fast_b200 import ops
    rng = np.random.default_rng(7)
    dt = torch.from_numpy((rng.random(E) * 2e8).astype(np.float32)).to(cuda)
    w = torch.from_numpy(1 / 10 ** np.linspace(0, 9, d, dtype=np.float32)).to(cuda)
    b = (torch.randn(d) * 0.1).to(cuda)
    g16 = torch.randn(E, d).to(torch.bfloat16).to(cuda)
    n_dev = torch.tensor([e_dev], dtype=torch.int32, device=cuda)
    out = []
    for g in (g16, g16.float()):
        dw = torch.full((d,), 0.5, device=cuda)
        db = torch.full((d,), -0.25, device=cuda)
        ops.time_encode_bwd(g, dt, w, b, dw, db, n_dev=n_dev)
        out.append((dw, db))
    torch.cuda.synchronize()
    assert torch.equal(out[0][0], out[1][0]) and torch.equal(out[0][1], out[1][1])
    assert not torch.equal(out[0][0], torch.full_like(out[0][0], 0.5))


def _bound(name):
    """Relative L2 bound against the bf16-rounding oracle (a tensor also
    passes when it is within 5x the error of the oracle's own fp32 run: each
    operand that fp32 and fp64 round to neighbouring bf16 values moves by one
    bf16 step, and the softmax backward's cancellation amplifies those moves
    in the query / key gradients)."""
    return 1e-3 if name in ("pos", "neg", "loss") else 2e-3


def _kv_bias_joined(grads):
    """w_k.bias and w_v.bias of each layer as one vector (the device computes
    them as one bias gradient).  Alone, the key bias's gradient is no test:
    adding a constant to every logit of a destination leaves its softmax
    unchanged, so that gradient is zero but for the LeakyReLU's negative
    side, and what is left is rounding noise of large sums."""
    out = {}
    for n, g in grads.items():
        if n.endswith("w_k.bias"):
            out[n[:-len("w_k.bias")] + "kv.bias"] = torch.cat([g, grads[n[:-len("k.bias")] + "v.bias"]])
        elif not n.endswith("w_v.bias"):
            out[n] = g
    return out


@pytest.mark.parametrize("dn,de", [(413, 186), (0, 172)])
def test_bf16_step_matches_fp64_oracle_to_bf16_accuracy(cuda, dn, de):
    from conftest import small_graph
    from fast_b200.engine import FusedStep
    from fast_b200.ext import sampler_core
    from fast_b200.model import DeviceBlock, GeneralModel
    from fast_b200.train import _bf16_table
    from oracle import bf16_math, ref_math
    from oracle.sampler import OracleSampler
    layers, fanout, n_nodes, n_edges = 2, [10, 10], 300, 30000
    g = small_graph(n_nodes=n_nodes, n_edges=n_edges, seed=21, int_ts=False, t_max=2e4, zipf=1.0)
    torch.manual_seed(1)
    # features exactly representable in bf16, so the tables carry no rounding of their own
    nf = torch.randn(n_nodes, dn).to(torch.bfloat16).float() if dn else None
    ef = torch.randn(n_edges, de).to(torch.bfloat16).float()
    sp = dict(layer=layers, neighbor=fanout, strategy="recent", prop_time=False, history=1, duration=0)
    gnn = dict(arch="transformer_attention", layer=layers, att_head=2, dim_time=100, dim_out=100)
    tr = dict(lr=1e-4, dropout=0.0, att_dropout=0.0)
    m64 = GeneralModel(dn, de, sp, dict(type="none", dim_out=0), gnn, tr).double()
    # ReLU pre-activations away from the kink (biases of w_out and of the
    # predictor's two projections + 4): at the kink the gradient jumps, and a
    # 1e-4 forward difference (an operand that fp32 and fp64 round to
    # neighbouring bf16 values) would switch a whole gradient term
    with torch.no_grad():
        for l in range(layers):
            m64.layers["l%dh0" % l].w_out.bias += 4.0
        m64.edge_predictor.src_fc.bias += 4.0
        m64.edge_predictor.dst_fc.bias += 4.0
    m_gpu = copy.deepcopy(m64).float().to(cuda)
    m32 = copy.deepcopy(m64).float()
    eng = FusedStep(m_gpu, precision="bf16")
    dev = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    smp = sampler_core.ParallelSampler(dev(g["indptr"]), dev(g["indices"]), dev(g["eid"]), dev(g["ts"]), 1, 1,
                                       layers, fanout, True, False, 1, 0.0)
    ora = OracleSampler(g["indptr"], g["indices"], g["eid"], g["ts"], 1, 1, layers, fanout, True, False, 1, 0.0)
    nf_d = _bf16_table(nf.to(cuda), dn) if dn else None
    ef_d = _bf16_table(ef.to(cuda), de)
    rng = np.random.default_rng(0)
    B = 200
    for b0 in range(5000, 5000 + 3 * B, B):
        src, dst, t = g["src"][b0:b0 + B], g["dst"][b0:b0 + B], g["t"][b0:b0 + B]
        roots = np.concatenate([src, dst, rng.integers(0, n_nodes, B).astype(np.int32)])
        rts = np.concatenate([t, t, t]).astype(np.float32)
        smp.sample_device(dev(roots), dev(rts))
        blocks = [DeviceBlock(v, d) for v, d in zip(smp.block_views(), smp.dims())]
        ora.sample(roots, rts)
        loss_g = torch.zeros((), device=cuda)
        scores = torch.empty(2 * B, device=cuda)
        eng.step(blocks, nf_d, ef_d, loss_g, scores=scores)
        torch.cuda.synchronize()
        rel = lambda a, b: float((a.double().cpu() - b.double()).norm() / (b.double().norm() + 1e-12))  # noqa
        gdev = _kv_bias_joined({n: pg.grad.double().cpu() for (n, p64), pg in zip(m64.named_parameters(),
                                                                                 m_gpu.parameters())
                                if pg.grad is not None})
        runs = {}
        for tag, model, fn in (("bf16", m64, bf16_math.layer_forward_bf16),
                               ("bf16_fp32", m32, bf16_math.layer_forward_bf16),
                               ("exact", m64, None)):
            model.zero_grad()
            dty = next(model.parameters()).dtype
            nfx = nf.to(dty) if dn else None
            rp, rn = ref_math.model_forward(model, ora.get_ret(), nfx, ef.to(dty), layer_fn=fn)
            loss = ref_math.bce_loss(rp, rn)
            loss.backward()
            runs[tag] = (rp.detach().view(-1), rn.detach().view(-1), float(loss),
                         _kv_bias_joined({n: p.grad.detach() for n, p in model.named_parameters()
                                          if p.grad is not None}))
        ref = runs["bf16"]
        out = {}
        for tag in ("bf16", "exact"):
            rp, rn, lv, gr = runs[tag]
            out[tag] = dict(pos=rel(scores[:B], rp), neg=rel(scores[B:], rn),
                            loss=abs(float(loss_g) - lv) / abs(lv), **{n: rel(gdev[n], gr[n]) for n in gr})
        # the fp32 run of the same bf16 algorithm, against its fp64 run
        own = {n: rel(runs["bf16_fp32"][3][n], ref[3][n]) for n in ref[3]}
        print("relative L2 error vs the bf16-rounding oracle:", {k: "%.1e" % v for k, v in out["bf16"].items()})
        print("fp32 run of that oracle vs its fp64 run:", {k: "%.1e" % v for k, v in own.items()})
        print("relative L2 error vs the exact fp64 reference:", {k: "%.1e" % v for k, v in out["exact"].items()})
        bad = {k: (v, own.get(k)) for k, v in out["bf16"].items()
               if not (v < _bound(k) or (k in own and v <= 5 * own[k]))}
        assert not bad, bad
        assert max(out["exact"].values()) < 0.25      # sanity: bf16 accuracy, not another function
