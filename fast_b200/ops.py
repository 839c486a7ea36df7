"""Tensor-level wrappers of the fast_b200 kernels and the autograd function
of one temporal-attention layer core.

Every wrapper launches on torch's current CUDA stream through the C ABI
(`capi`) and allocates its outputs / workspaces with torch's caching
allocator.  Inputs must be fp32 (int32 for ids) with unit column stride.
"""
import contextlib
import ctypes
import os

import torch

from .capi import call, ptr, stream_ptr, lib


class KernelTimer:
    """Times every kernel wrapper with CUDA events on the current stream.
    Each wrapped launch is issued `reps` times back to back between one event
    pair, so the host runs ahead of the device and the events bracket device
    time, not launch gaps.  Records carry the algorithmic bytes and flops of
    one launch (for the roofline).  Repeated launches of accumulating kernels
    change their outputs: time only steps whose results are thrown away."""

    def __init__(self, reps=10):
        self.reps = reps
        self.records = []

    def run(self, name, nbytes, flops, fn):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(self.reps):
            fn()
        e.record()
        self.records.append((name, s, e, nbytes, flops, self.reps))

    def summary(self):
        torch.cuda.synchronize()
        out = {}
        for name, s, e, nb, fl, reps in self.records:
            r = out.setdefault(name, dict(launches=0, ms=0.0, bytes=0, flops=0))
            r["launches"] += 1
            r["ms"] += s.elapsed_time(e) / reps
            r["bytes"] += nb
            r["flops"] += fl
        return out


TIMER = None            # set to a KernelTimer to time every kernel wrapper
USE_TC = False          # route eligible gemm_nt calls to the tcgen05 kernel
LAUNCHES = [0]          # kernels launched through these wrappers
# FB_NVTX=1: each wrapper's launches inside an NVTX range named like its timer
# entry (eager steps), so a profiler can select one group by name
NVTX = os.environ.get("FB_NVTX", "0") == "1"


def _launch(name, nbytes, flops, kernels, fn):
    LAUNCHES[0] += kernels
    if NVTX:
        torch.cuda.nvtx.range_push(name)
    if TIMER is None:
        fn()
    else:
        TIMER.run(name, nbytes, flops, fn)
    if NVTX:
        torch.cuda.nvtx.range_pop()


def timed(name, fn):
    """Runs fn (device work launched elsewhere, e.g. the sampler) under TIMER
    when one is set; adds nothing to LAUNCHES."""
    if TIMER is None:
        fn()
    else:
        TIMER.run(name, 0, 0, fn)


def _f32_rows(t, name):
    if t.dtype != torch.float32 or t.dim() != 2 or t.stride(1) != 1 or not t.is_cuda:
        raise ValueError("%s must be a CUDA fp32 matrix with unit column stride" % name)


def _p(t):
    """Device pointer of an optional device-count tensor."""
    return None if t is None else t.data_ptr()


def gemm_nt(A, B, bias=None, out=None, accumulate=False, M_dev=None):
    """out[m, n] (+)= sum_k A[m, k] B[n, k] + bias[n]; rows m < *M_dev when given."""
    _f32_rows(A, "A")
    _f32_rows(B, "B")
    M, K = A.shape
    N = B.shape[0]
    if B.shape[1] != K:
        raise ValueError("gemm_nt: inner dimensions differ")
    if out is None:
        out = torch.empty(M, N, device=A.device, dtype=torch.float32)
    if USE_TC and M >= 256 and lib.fb_gemm_nt_tc_supported(ptr(A), A.stride(0), ptr(B), B.stride(0), N, K):
        return gemm_nt_tc(A, B, bias, out, accumulate, M_dev)
    _launch("gemm_nt", 4 * (M * K + N * K + M * N), 2 * M * N * K, 1,
            lambda: call("fb_gemm_nt", ptr(A), A.stride(0), ptr(B), B.stride(0), ptr(bias), ptr(out),
                         out.stride(0), M, _p(M_dev), N, K, int(accumulate), stream_ptr()))
    return out


def gemm_nt_tc(A, B, bias=None, out=None, accumulate=False, M_dev=None):
    """gemm_nt on the tcgen05 tensor cores (3xTF32 split, fp32 accuracy)."""
    _f32_rows(A, "A")
    _f32_rows(B, "B")
    M, K = A.shape
    N = B.shape[0]
    if out is None:
        out = torch.empty(M, N, device=A.device, dtype=torch.float32)
    _launch("gemm_nt_tc", 4 * (M * K + N * K + M * N), 2 * M * N * K, 1,
            lambda: call("fb_gemm_nt_tc", ptr(A), A.stride(0), ptr(B), B.stride(0), ptr(bias), ptr(out),
                         out.stride(0), M, _p(M_dev), N, K, int(accumulate), stream_ptr()))
    return out


def tc_error(clear=True):
    import ctypes
    f = ctypes.c_int(0)
    call("fb_gemm_tc_error", ctypes.byref(f), int(clear))
    return f.value


def gemm_nn(A, B, bias=None, out=None, accumulate=False, M_dev=None):
    """out[m, n] (+)= sum_k A[m, k] B[k, n] + bias[n]  (B stored [K, N]); rows m < *M_dev when given."""
    _f32_rows(A, "A")
    _f32_rows(B, "B")
    M, K = A.shape
    N = B.shape[1]
    if B.shape[0] != K:
        raise ValueError("gemm_nn: inner dimensions differ")
    if out is None:
        out = torch.empty(M, N, device=A.device, dtype=torch.float32)
    _launch("gemm_nn", 4 * (M * K + N * K + M * N), 2 * M * N * K, 1,
            lambda: call("fb_gemm_nn", ptr(A), A.stride(0), ptr(B), B.stride(0), ptr(bias), ptr(out),
                         out.stride(0), M, _p(M_dev), N, K, int(accumulate), stream_ptr()))
    return out


def gemm_tn(G, X, out=None, accumulate=False, M_dev=None, db=None, db_accumulate=None):
    """out[n, k] (+)= sum_m G[m, n] X[m, k]  (weight gradient); rows m < *M_dev when given.
    With db, also db[n] (+)= sum_m G[m, n] in the same pass (db_accumulate
    defaults to accumulate)."""
    _f32_rows(G, "G")
    _f32_rows(X, "X")
    M, N = G.shape
    K = X.shape[1]
    if out is None:
        out = torch.empty(N, K, device=G.device, dtype=torch.float32)
    dba = accumulate if db_accumulate is None else db_accumulate
    ws = torch.empty(int(lib.fb_gemm_tn_ws_bytes(M, N, K)), device=G.device, dtype=torch.uint8)
    _launch("gemm_tn", 4 * (M * N + M * K + N * K), 2 * M * N * K, 2,
            lambda: call("fb_gemm_tn_bias", ptr(G), G.stride(0), ptr(X), X.stride(0), ptr(out), out.stride(0), M,
                         _p(M_dev), N, K, int(accumulate), ptr(db), int(dba), ptr(ws), stream_ptr()))
    return out


NT, NN, TN = 0, 1, 2


def gemm_group(problems, name="gemm_group"):
    """Runs independent GEMMs in one launch (+ one split-reduce for the TN
    ones): on the tcgen05 tensor cores (3xTF32), or on the CUDA cores when
    FB_GEMM=ffma is set in the environment.  Each problem is a dict: kind (NT / NN / TN), A, B (TN: X; may be
    None for a TN with K == 0), out, and optionally A2 / k1 (NT / NN: A's
    columns >= k1 come from A2), bias, M_dev, accumulate, db, db_accumulate.
    Shapes: NT A [M, K], B [N, K]; NN A [M, K], B [K, N]; TN A = G [M, N],
    B = X [M, K], out [N, K]."""
    from .capi import GemmProblem
    arr = (GemmProblem * len(problems))()
    nbytes, flops = 0, 0
    keep = []
    for i, p in enumerate(problems):
        A, B, out = p["A"], p.get("B"), p.get("out")
        A2 = p.get("A2")
        kind = p["kind"]
        for t in (A, B, A2, out):
            if t is not None:
                _f32_rows(t, "gemm_group operand")
        M = A.shape[0]
        if kind == TN:
            N, K = A.shape[1], (0 if B is None else B.shape[1])
        elif kind == NT:
            N, K = B.shape[0], A.shape[1] + (0 if A2 is None else A2.shape[1])
        else:
            N, K = B.shape[1], A.shape[1] + (0 if A2 is None else A2.shape[1])
        k1 = A.shape[1] if A2 is not None else K
        db = p.get("db")
        acc = int(bool(p.get("accumulate", False)))
        dba = p.get("db_accumulate")
        if out is None:                      # TN column sums only (K == 0): nothing lands in C
            assert kind == TN and K == 0 and db is not None
            c_ptr, ldc = ptr(db), 0
        else:
            c_ptr, ldc = ptr(out), out.stride(0)
        arr[i] = GemmProblem(kind, ptr(A), A.stride(0), ptr(A2), 0 if A2 is None else A2.stride(0), k1,
                             ptr(B), 0 if B is None else B.stride(0), ptr(p.get("bias")), c_ptr, ldc,
                             M, _p(p.get("M_dev")), N, K, acc, ptr(db), int(acc if dba is None else bool(dba)))
        keep.append((A, B, A2, out, db))
        nbytes += 4 * (M * K + N * K + M * N)
        flops += 2 * M * N * K
    n = len(problems)
    dev = problems[0]["A"].device
    ws = torch.empty(int(lib.fb_gemm_group_ws_bytes(arr, n)), device=dev, dtype=torch.uint8)
    # the grouped GEMM, plus the split reduction when the group holds a TN problem
    _launch(name, nbytes, flops, 1 + int(any(p["kind"] == TN for p in problems)),
            lambda: call("fb_gemm_group", arr, n, ptr(ws), ws.numel(), stream_ptr()))


def pad8(n):
    """n rounded up to a multiple of 8 (16 bytes of bf16)."""
    return (n + 7) // 8 * 8


def _bf16_rows(t, name):
    if t.dtype != torch.bfloat16 or t.dim() != 2 or t.stride(1) != 1 or not t.is_cuda:
        raise ValueError("%s must be a CUDA bf16 matrix with unit column stride" % name)


class RowGather:
    """Rows of a bf16 GEMM operand gathered from up to three sources
    (fb_bf16_row_gather): segments [(table, cols, idx, width)] in column
    order -- a bf16 table [rows, ld] (ld a multiple of 8) whose first `cols`
    columns are data, the int32 row index of every operand row (None: row r
    of the table), and the segment's width in the operand, a multiple of 64.
    Columns past `cols` read as zeros."""

    def __init__(self, segments):
        if not 1 <= len(segments) <= 3:
            raise ValueError("RowGather: 1 to 3 segments")
        self.segments = list(segments)
        self.starts, end = [], 0
        for tab, cols, idx, width in self.segments:
            _bf16_rows(tab, "RowGather table")
            if width % 64 or width < 1 or cols > tab.shape[1]:
                raise ValueError("RowGather: segment widths are multiples of 64 columns")
            if idx is not None and (idx.dtype != torch.int32 or not idx.is_contiguous()):
                raise ValueError("RowGather: row indices must be contiguous int32")
            self.starts.append(end)
            end += width
        self.K = end

    def struct(self):
        from .capi import Bf16RowGather
        g = Bf16RowGather()
        g.nseg = len(self.segments)
        for s, (tab, cols, idx, width) in enumerate(self.segments):
            g.end[s] = self.starts[s] + width
            g.tab[s] = ptr(tab)
            g.tab_rows[s] = tab.shape[0]
            g.tab_ld[s] = tab.stride(0)
            g.tab_cols[s] = cols
            g.idx[s] = ptr(idx)
        return g

    def read_bytes(self, M):
        """Algorithmic bytes of M gathered rows: each source row's data and its index."""
        return sum(M * (2 * cols + (4 if idx is not None else 0)) for _, cols, idx, _ in self.segments)


def gemm_bf16_group(problems, name="gemm_bf16_group"):
    """gemm_group with bf16 operands (torch.bfloat16 matrices; C, bias, db
    fp32) on the tcgen05 kind::f16 kernel: products of bf16 values
    accumulated in fp32.  Same problem dicts as gemm_group (B required); with
    A2, k1 (a multiple of 8, >= A's width) is the column of B where A2's
    block starts.  A TN problem may give segs = [(at, len, to), ...]: B's
    columns [at, at + len) land in out's columns from `to`, the rest of B's
    columns are skipped (a weight gradient over a bf16 projection row)."""
    from .capi import Bf16RowGather, GemmBf16Problem
    arr = (GemmBf16Problem * len(problems))()
    gathers = (Bf16RowGather * len(problems))()
    nbytes, flops = 0, 0
    keep = []
    for i, p in enumerate(problems):
        A, B, out, A2 = p.get("A"), p.get("B"), p.get("out"), p.get("A2")
        gat = p.get("gather")
        kind = p["kind"]
        for t in (A, B, A2):
            if t is not None:
                _bf16_rows(t, "gemm_bf16_group operand")
        c16 = out.dtype == torch.bfloat16
        if c16:
            _bf16_rows(out, "gemm_bf16_group output")
        else:
            _f32_rows(out, "gemm_bf16_group output")
        if gat is not None:
            # NT: A's rows gathered (A absent, M from p["M"]); TN: X's rows gathered (B absent)
            gathers[i] = gat.struct()
            if kind == NT:
                M, N, K = int(p["M"]), B.shape[0], gat.K
            elif kind == TN:
                M, N, K = A.shape[0], A.shape[1], gat.K
            else:
                raise ValueError("gemm_bf16_group: a gathered operand is NT's A or a segmented TN's X")
        else:
            M = A.shape[0]
        if gat is not None:
            pass
        elif kind == TN:
            N, K = A.shape[1], B.shape[1]
        elif kind == NT:
            N, K = B.shape[0], A.shape[1] + (0 if A2 is None else A2.shape[1])
        else:
            N, K = B.shape[1], A.shape[1] + (0 if A2 is None else A2.shape[1])
        k1 = p.get("k1", A.shape[1]) if A2 is not None else K
        if A2 is not None:
            K = k1 + A2.shape[1]
        db = p.get("db")
        acc = int(bool(p.get("accumulate", False)))
        dba = p.get("db_accumulate")
        segs = p.get("segs") or ()
        if len(segs) > 3:
            raise ValueError("gemm_bf16_group: at most 3 column segments")
        pad3 = lambda v: (ctypes.c_int * 3)(*(list(v) + [0] * (3 - len(v))))  # noqa: E731
        arr[i] = GemmBf16Problem(kind, ptr(A), 0 if A is None else A.stride(0), ptr(A2),
                                 0 if A2 is None else A2.stride(0), k1,
                                 ptr(B), 0 if B is None else B.stride(0), ptr(p.get("bias")), ptr(out), out.stride(0),
                                 M, _p(p.get("M_dev")), N, K, acc, ptr(db), int(acc if dba is None else bool(dba)),
                                 A.shape[1] if A2 is not None else 0, len(segs), pad3([g[0] for g in segs]),
                                 pad3([g[1] for g in segs]), pad3([g[2] for g in segs]), int(c16),
                                 ctypes.pointer(gathers[i]) if gat is not None else None)
        add, add_idx = p.get("add"), p.get("add_idx")
        if add is not None:
            # C[m] += add[add_idx[m]] in the epilogue: an fp32 table [rows, >= N] and int32 indices
            _f32_rows(add, "gemm_bf16_group add table")
            if add_idx is None or add_idx.dtype != torch.int32 or add.shape[1] < N:
                raise ValueError("gemm_bf16_group: add needs an fp32 [rows, >= N] table and int32 add_idx")
            arr[i].add, arr[i].add_idx = ptr(add), ptr(add_idx)
            arr[i].ld_add, arr[i].add_rows = add.stride(0), add.shape[0]
            nbytes += 4 * M * (N + 1)
        keep.append((A, B, A2, out, db, gat, add, add_idx))
        if gat is not None and kind == NT:  # gathered rows in once, weights, C out
            nbytes += gat.read_bytes(M) + 2 * N * K + (2 if c16 else 4) * M * N
        elif gat is not None:               # G [M, N] and the gathered rows in, the gradient out
            nbytes += 2 * M * N + gat.read_bytes(M) + 4 * N * K
        elif kind == TN:                   # reads A [M, N] and B [M, K]; writes the [N, K] gradient
            nbytes += 2 * M * (N + K) + 4 * N * K
        else:                              # reads A [M, K] and B; writes C [M, N] (bf16 or fp32)
            nbytes += 2 * (M * K + N * K) + (2 if c16 else 4) * M * N
        flops += 2 * M * N * K
    n = len(problems)
    dev = out.device
    ws = torch.empty(int(lib.fb_gemm_bf16_group_ws_bytes(arr, n)), device=dev, dtype=torch.uint8)
    # the grouped GEMM, plus the split reduction when the group holds a TN problem
    _launch(name, nbytes, flops, 1 + int(any(p["kind"] == TN for p in problems)),
            lambda: call("fb_gemm_bf16_group", arr, n, ptr(ws), ws.numel(), stream_ptr()))


def cast_bf16(jobs, name="cast_bf16"):
    """One launch of fp32 -> bf16 (round to nearest even) block copies: jobs
    are (src fp32 [rows, cols] view, dst bf16 [rows, cols] view[, rows_dev])."""
    from .capi import CastJob, CAST_MAX_JOBS
    if not jobs:
        return
    if len(jobs) > CAST_MAX_JOBS:
        for i in range(0, len(jobs), CAST_MAX_JOBS):
            cast_bf16(jobs[i:i + CAST_MAX_JOBS], name)
        return
    arr = (CastJob * len(jobs))()
    nbytes = 0
    for i, j in enumerate(jobs):
        src, dst = j[0], j[1]
        rows_dev = j[2] if len(j) > 2 else None
        _f32_rows(src, "cast_bf16 source")
        _bf16_rows(dst, "cast_bf16 destination")
        if tuple(src.shape) != tuple(dst.shape):
            raise ValueError("cast_bf16: source %s and destination %s differ" % (tuple(src.shape), tuple(dst.shape)))
        arr[i] = CastJob(ptr(src), src.stride(0), ptr(dst), dst.stride(0), src.shape[0], _p(rows_dev), src.shape[1],
                         0)
        nbytes += 6 * src.numel()
    _launch(name, nbytes, 0, 1, lambda: call("fb_cast_bf16", arr, len(jobs), stream_ptr()))


def bf16_layout(*dims):
    """Column offsets of the segments of a bf16 projection row (each at a
    multiple of 8) and the row's width (data columns; the last segment unpadded)."""
    offs, at = [], 0
    for d in dims:
        offs.append(at)
        at += pad8(d)
    width = offs[-1] + dims[-1] if dims else 0
    return offs, width


def gather_time_encode_bf16(n_rows, h=None, h_idx=None, h_off=0, f=None, f_idx=None, dt=None, w=None, b=None,
                            out=None, device=None, n_rows_dev=None, h_off_dev=None, dn=None, de=None):
    """bf16 rows [h | f | cos(w*dt + b)] with segments at multiples of 8 columns
    (zeros between).  h / f: fp32 matrices, or bf16 tables with rows padded
    with zeros to a multiple of 8 (then dn / de give the true widths)."""
    dn = 0 if h is None else (dn if dn is not None else h.shape[1])
    de = 0 if f is None else (de if de is not None else f.shape[1])
    dtime = 0 if w is None else w.numel()
    dev = device or (h.device if h is not None else (f.device if f is not None else w.device))
    width = pad8(dn) + pad8(de) + dtime
    if out is None:
        out = torch.empty(n_rows, pad8(width), device=dev, dtype=torch.bfloat16)
    hb = int(h is not None and h.dtype == torch.bfloat16)
    fb_ = int(f is not None and f.dtype == torch.bfloat16)
    nbytes = n_rows * (2 * width + (2 if hb else 4) * dn + (2 if fb_ else 4) * de + 4 * (dt is not None)
                       + 4 * (h_idx is not None) + 4 * (f_idx is not None))
    _launch("gather_time_encode", nbytes, 0, 1,
            lambda: call("fb_gather_time_encode_bf16", ptr(h), hb, 0 if h is None else h.stride(0), ptr(h_idx),
                         int(h_off), _p(h_off_dev), dn, ptr(f), fb_, 0 if f is None else f.stride(0), ptr(f_idx), de,
                         ptr(dt), ptr(w), ptr(b), dtime, ptr(out), out.stride(0), n_rows, _p(n_rows_dev),
                         stream_ptr()))
    return out, width


def attn_fwd_kvbf16(q, kv, rptr, heads, slope, drop_p=0.0, seed=0, offset=0, n_dst_dev=None, offset_dev=None):
    """attn_fwd on bf16 K|V rows kv [E, 2D] (K then V): agg, att fp32."""
    nd = rptr.numel() - 1
    E, D2 = kv.shape
    D = D2 // 2
    _bf16_rows(kv, "attn_fwd_kvbf16 kv")
    ldq = 0 if (q.shape[0] == 1 and nd != 1) else q.stride(0)
    att = torch.empty(E, heads, device=kv.device, dtype=torch.float32)
    agg = torch.empty(nd, D, device=kv.device, dtype=torch.float32)
    qrows = nd if ldq else 1
    nbytes = 4 * (qrows * D + (nd + 1) + nd * D + E * heads) + 2 * 2 * E * D
    _launch("attn_fwd", nbytes, 0, 1,
            lambda: call("fb_attn_fwd_kvbf16", ptr(q), ldq, ptr(kv), kv.stride(0), ptr(rptr), nd, _p(n_dst_dev),
                         heads, D, slope, drop_p, seed, offset, _p(offset_dev), ptr(att), ptr(agg), agg.stride(0),
                         stream_ptr()))
    return agg, att


def attn_bwd_kvbf16(q, kv, rptr, att, dagg, heads, slope, drop_p=0.0, seed=0, offset=0, n_dst_dev=None,
                    offset_dev=None):
    """attn_bwd on bf16 K|V rows: dq fp32 [Nd, D], dK|dV bf16 [E, 2D]."""
    nd = rptr.numel() - 1
    E, D2 = kv.shape
    D = D2 // 2
    _bf16_rows(kv, "attn_bwd_kvbf16 kv")
    ldq = 0 if (q.shape[0] == 1 and nd != 1) else q.stride(0)
    dq = torch.empty(nd, D, device=kv.device, dtype=torch.float32)
    dkv = torch.empty(E, 2 * D, device=kv.device, dtype=torch.bfloat16)
    qrows = nd if ldq else 1
    nbytes = 4 * (qrows * D + nd * D + E * heads + (nd + 1) + nd * D) + 2 * 4 * E * D
    _launch("attn_bwd", nbytes, 0, 1,
            lambda: call("fb_attn_bwd_kvbf16", ptr(q), ldq, ptr(kv), kv.stride(0), ptr(rptr), nd, _p(n_dst_dev),
                         heads, D, slope, drop_p, seed, offset, _p(offset_dev), ptr(att), ptr(dagg),
                         dagg.stride(0), ptr(dq), ptr(dkv), dkv.stride(0), stream_ptr()))
    return dq, dkv


def attn_fwd_kvbf16_bf16out(q, kv, rptr, heads, slope, agg_bf, drop_p=0.0, seed=0, offset=0, n_dst_dev=None,
                            offset_dev=None):
    """attn_fwd_kvbf16 writing the aggregate as bf16 into agg_bf ([Nd, D] view,
    rows 8-byte aligned); returns att fp32."""
    nd = rptr.numel() - 1
    E, D2 = kv.shape
    D = D2 // 2
    _bf16_rows(kv, "attn_fwd_kvbf16_bf16out kv")
    if agg_bf.dtype != torch.bfloat16 or tuple(agg_bf.shape) != (nd, D):
        raise ValueError("attn_fwd_kvbf16_bf16out: agg_bf must be a bf16 [n_dst, D] view")
    ldq = 0 if (q.shape[0] == 1 and nd != 1) else q.stride(0)
    att = torch.empty(E, heads, device=kv.device, dtype=torch.float32)
    qrows = nd if ldq else 1
    nbytes = 4 * (qrows * D + (nd + 1) + E * heads) + 2 * nd * D + 2 * 2 * E * D
    _launch("attn_fwd", nbytes, 0, 1,
            lambda: call("fb_attn_fwd_kvbf16_bf16out", ptr(q), ldq, ptr(kv), kv.stride(0), ptr(rptr), nd,
                         _p(n_dst_dev), heads, D, slope, drop_p, seed, offset, _p(offset_dev), ptr(att), ptr(agg_bf),
                         agg_bf.stride(0), stream_ptr()))
    return att


def attn_bwd_kvbf16_bf16dq(q, kv, rptr, att, dagg, heads, slope, dq_bf, drop_p=0.0, seed=0, offset=0,
                           n_dst_dev=None, offset_dev=None):
    """attn_bwd_kvbf16 writing dq as bf16 into dq_bf ([Nd, D] view); returns dK|dV bf16 [E, 2D]."""
    nd = rptr.numel() - 1
    E, D2 = kv.shape
    D = D2 // 2
    _bf16_rows(kv, "attn_bwd_kvbf16_bf16dq kv")
    if dq_bf.dtype != torch.bfloat16 or tuple(dq_bf.shape) != (nd, D):
        raise ValueError("attn_bwd_kvbf16_bf16dq: dq_bf must be a bf16 [n_dst, D] view")
    ldq = 0 if (q.shape[0] == 1 and nd != 1) else q.stride(0)
    dkv = torch.empty(E, 2 * D, device=kv.device, dtype=torch.bfloat16)
    qrows = nd if ldq else 1
    nbytes = 4 * (qrows * D + nd * D + E * heads + (nd + 1)) + 2 * nd * D + 2 * 4 * E * D
    _launch("attn_bwd", nbytes, 0, 1,
            lambda: call("fb_attn_bwd_kvbf16_bf16dq", ptr(q), ldq, ptr(kv), kv.stride(0), ptr(rptr), nd,
                         _p(n_dst_dev), heads, D, slope, drop_p, seed, offset, _p(offset_dev), ptr(att), ptr(dagg),
                         dagg.stride(0), ptr(dq_bf), dq_bf.stride(0), ptr(dkv), dkv.stride(0), stream_ptr()))
    return dkv


def attn_bwd_bf16kv(q, k, v, rptr, att, dagg, heads, slope, drop_p=0.0, seed=0, offset=0, n_dst_dev=None,
                    offset_dev=None, dq=None):
    """attn_bwd with dk | dv written as one bf16 [E, 2D] matrix (the operand of
    the bf16 projection-gradient GEMMs); dq fp32."""
    nd = rptr.numel() - 1
    E, D = k.shape
    ldq = 0 if (q.shape[0] == 1 and nd != 1) else q.stride(0)
    if dq is None:
        dq = torch.empty(nd, D, device=k.device, dtype=torch.float32)
    dkv = torch.empty(E, 2 * D, device=k.device, dtype=torch.bfloat16)
    qrows = nd if ldq else 1
    nbytes = 4 * (qrows * D + nd * D + 2 * E * D + E * heads + (nd + 1) + nd * D) + 2 * 2 * E * D
    _launch("attn_bwd", nbytes, 0, 1,
            lambda: call("fb_attn_bwd_bf16kv", ptr(q), ldq, ptr(k), ptr(v), k.stride(0), ptr(rptr), nd,
                         _p(n_dst_dev), heads, D, slope, drop_p, seed, offset, _p(offset_dev), ptr(att), ptr(dagg),
                         dagg.stride(0), ptr(dq), ptr(dkv), dkv.data_ptr() + 2 * D, dkv.stride(0), stream_ptr()))
    return dq, dkv


def gru_fwd(gi, gh, h0, h1, n_dev=None):
    """GRUCell gates from the products gi = x W_ih^T + b_ih, gh = h0 W_hh^T + b_hh
    ([n, 3H]); writes h1 and keeps (r, z, n) in gi (memorys.py:272-304)."""
    n, H = h0.shape
    for t, w in ((gi, 3 * H), (gh, 3 * H), (h1, H)):
        if t.shape != (n, w) or not t.is_contiguous():
            raise ValueError("gru_fwd: expected contiguous [n, 3H] gates and [n, H] states")
    _launch("gru_fwd", 4 * n * (9 * H), 0, 1,
            lambda: call("fb_gru_fwd", ptr(gi), ptr(gh), ptr(h0), ptr(h1), n, _p(n_dev), H, stream_ptr()))
    return h1


def gru_bwd(gi, gh, h0, dh1, n_dev=None):
    """Backward of gru_fwd: gi <- d(gi), gh <- d(gh) for the gradient dh1."""
    n, H = h0.shape
    _launch("gru_bwd", 4 * n * (14 * H), 0, 1,
            lambda: call("fb_gru_bwd", ptr(gi), ptr(gh), ptr(h0), ptr(dh1), dh1.stride(0), n, _p(n_dev), H,
                         stream_ptr()))


def add_layernorm_fwd(x, res, gamma, beta, eps=1e-5, n_dev=None):
    """out = LayerNorm(x + res) per row; returns (out, xhat, rstd) for the backward
    (the residual step of memorys.py:378-379)."""
    n, D = x.shape
    out = torch.empty_like(x)
    xhat = torch.empty_like(x)
    rstd = torch.empty(n, device=x.device, dtype=torch.float32)
    _launch("add_layernorm_fwd", 4 * n * D * 4, 0, 1,
            lambda: call("fb_add_layernorm_fwd", ptr(x), ptr(res), ptr(gamma), ptr(beta), float(eps), ptr(out),
                         ptr(xhat), ptr(rstd), n, _p(n_dev), D, stream_ptr()))
    return out, xhat, rstd


def add_layernorm_bwd(dout, xhat, rstd, gamma, dgamma, dbeta, n_dev=None):
    """Gradient of add_layernorm_fwd's input (x and res alike); accumulates
    dgamma, dbeta."""
    n, D = dout.shape
    dx = torch.empty_like(dout)
    ws = torch.empty(int(lib.fb_add_layernorm_bwd_ws_bytes(n, D)), device=dout.device, dtype=torch.uint8)
    _launch("add_layernorm_bwd", 4 * n * D * 3, 0, 2,
            lambda: call("fb_add_layernorm_bwd", ptr(dout), ptr(xhat), ptr(rstd), ptr(gamma), ptr(dx), ptr(dgamma),
                         ptr(dbeta), n, _p(n_dev), D, ptr(ws), stream_ptr()))
    return dx


def layer_tail_fwd(z, gamma, beta, eps=1e-5, drop_p=0.0, seed=0, offset=0, offset_dev=None, mask_u=None,
                   y=None, out=None, n_dev=None, gate_dev=None):
    """y = relu(dropout(z)), out = LayerNorm(y) per row (rows >= *n_dev: out = 0;
    all rows when *gate_dev == 0)."""
    n, d = z.shape
    y = torch.empty_like(z) if y is None else y
    out = torch.empty_like(z) if out is None else out
    _launch("layer_tail_fwd", 4 * (3 * n * d + 2 * d), 0, 1,
            lambda: call("fb_layer_tail_fwd", ptr(z), z.stride(0), ptr(gamma), ptr(beta), float(eps),
                         float(drop_p), int(seed), int(offset), _p(offset_dev), ptr(mask_u), ptr(y), y.stride(0),
                         ptr(out), out.stride(0), n, _p(n_dev), _p(gate_dev), d, stream_ptr()))
    return y, out


def layer_tail_bwd(dout, y, gamma, dgamma, dbeta, eps=1e-5, drop_p=0.0, dz=None, n_dev=None, gate_dev=None):
    """dz from dout and the saved y; dgamma / dbeta accumulate."""
    n, d = y.shape
    dz = torch.empty_like(y) if dz is None else dz
    ws = torch.empty(int(lib.fb_layer_tail_bwd_ws_bytes(n, d)), device=y.device, dtype=torch.uint8)
    _launch("layer_tail_bwd", 4 * (3 * n * d + 3 * d), 0, 2,
            lambda: call("fb_layer_tail_bwd", ptr(dout), dout.stride(0), ptr(y), y.stride(0), ptr(gamma),
                         float(eps), float(drop_p), ptr(dz), dz.stride(0), ptr(dgamma), ptr(dbeta), n, _p(n_dev),
                         _p(gate_dev), d, ptr(ws), stream_ptr()))
    return dz


def edge_predictor_loss(S, P, w_o, b_o, loss, dS, dP, dw_o, db_o, scores=None):
    """Scores relu(S_i + P_.) . w_o + b_o of the B positive and B negative
    pairs, the BCE-with-logits loss (written to `loss`), dS / dP, and the
    out_fc gradients (accumulated)."""
    B, d = S.shape
    ws = torch.empty(int(lib.fb_edge_predictor_loss_ws_bytes(B, d)), device=S.device, dtype=torch.uint8)
    _launch("edge_predictor_loss", 4 * (2 * 3 * B * d + 2 * d), 0, 2,
            lambda: call("fb_edge_predictor_loss", ptr(S), S.stride(0), ptr(P), P.stride(0), ptr(w_o), ptr(b_o), B,
                         d, ptr(loss), ptr(dS), dS.stride(0), ptr(dP), dP.stride(0), ptr(dw_o), ptr(db_o),
                         ptr(scores), ptr(ws), stream_ptr()))


def q_time_bwd(v, W_q, dn, dtime, b_t, db_q, db_t, qin0=None, dW_q=None):
    """db_q += v; db_t -= sin(b_t) * (v @ W_q[:, dn:]); with qin0, dW_q += outer(v, qin0)."""
    D = v.numel()
    _launch("q_time_bwd", 4 * (D * (dn + dtime) + 2 * D + 2 * dtime), 0, 1,
            lambda: call("fb_q_time_bwd", ptr(v), D, ptr(W_q), W_q.stride(0), dn, dtime, ptr(b_t), ptr(qin0),
                         ptr(dW_q), 0 if dW_q is None else dW_q.stride(0), ptr(db_q), ptr(db_t), stream_ptr()))


def colsum(G, out=None, accumulate=False, M_dev=None):
    _f32_rows(G, "G")
    M, N = G.shape
    if out is None:
        out = torch.empty(N, device=G.device, dtype=torch.float32)
    ws = torch.empty(int(lib.fb_colsum_ws_bytes(M, N)), device=G.device, dtype=torch.uint8)
    _launch("colsum", 4 * (M * N + N), M * N, 2,
            lambda: call("fb_colsum", ptr(G), G.stride(0), ptr(out), M, _p(M_dev), N, int(accumulate), ptr(ws),
                         stream_ptr()))
    return out


def gather_time_encode(n_rows, h=None, h_idx=None, h_off=0, f=None, f_idx=None, dt=None, w=None, b=None,
                       out=None, device=None, n_rows_dev=None, h_off_dev=None):
    """Rows [h[h_idx or r + h_off (+ *h_off_dev)] | f[f_idx or r] | cos(w*dt + b)] for r < n_rows
    (r < *n_rows_dev when given; the rest of `out` is left untouched)."""
    dn = 0 if h is None else h.shape[1]
    de = 0 if f is None else f.shape[1]
    dtime = 0 if w is None else w.numel()
    dev = device or (h.device if h is not None else (f.device if f is not None else w.device))
    if out is None:
        out = torch.empty(n_rows, dn + de + dtime, device=dev, dtype=torch.float32)
    nbytes = 4 * n_rows * (2 * (dn + de) + dtime + (1 if dt is not None else 0)
                           + (1 if h_idx is not None else 0) + (1 if f_idx is not None else 0))
    _launch("gather_time_encode", nbytes, 0, 1,
            lambda: call("fb_gather_time_encode", ptr(h), 0 if h is None else h.stride(0), ptr(h_idx),
                         int(h_off), _p(h_off_dev), dn, ptr(f), 0 if f is None else f.stride(0), ptr(f_idx), de,
                         ptr(dt), ptr(w), ptr(b), dtime, ptr(out), out.stride(0), n_rows, _p(n_rows_dev),
                         stream_ptr()))
    return out


def time_encode_bwd(g, dt, w, b, dw, db, n_dev=None):
    """dw/db += gradient of cos(w*dt + b) given g = dL/dcos (rows at g.stride(0));
    g fp32 or bf16 (summed in fp32)."""
    n, dtime = g.shape
    if g.dtype not in (torch.float32, torch.bfloat16) or g.stride(1) != 1:
        raise ValueError("time_encode_bwd: g must be fp32 or bf16 with unit column stride")
    fn, es = ("fb_time_encode_bwd_bf16", 2) if g.dtype == torch.bfloat16 else ("fb_time_encode_bwd", 4)
    ws = torch.empty(int(lib.fb_time_encode_bwd_ws_bytes(n, dtime)), device=g.device, dtype=torch.uint8)
    _launch("time_encode_bwd", es * n * dtime + 4 * n, 0, 2,
            lambda: call(fn, ptr(g), g.stride(0), ptr(dt), ptr(w), ptr(b), dtime, n, _p(n_dev),
                         ptr(dw), ptr(db), ptr(ws), stream_ptr()))


def attn_fwd(q, k, v, rptr, heads, slope, drop_p=0.0, seed=0, offset=0, n_dst_dev=None, offset_dev=None):
    """agg, att = fused LeakyReLU(q.k) -> segment softmax -> dropout -> sum(att * v).
    q: [Nd, D] or [1, D] (broadcast); k, v: [E, D] views sharing a row stride."""
    nd = rptr.numel() - 1
    E, D = k.shape
    ldq = 0 if (q.shape[0] == 1 and nd != 1) else q.stride(0)
    att = torch.empty(E, heads, device=k.device, dtype=torch.float32)
    agg = torch.empty(nd, D, device=k.device, dtype=torch.float32)
    qrows = nd if ldq else 1
    nbytes = 4 * (qrows * D + 2 * E * D + (nd + 1) + nd * D + E * heads)
    _launch("attn_fwd", nbytes, 0, 1,
            lambda: call("fb_attn_fwd", ptr(q), ldq, ptr(k), ptr(v), k.stride(0), ptr(rptr), nd, _p(n_dst_dev),
                         heads, D, slope, drop_p, seed, offset, _p(offset_dev), ptr(att), ptr(agg),
                         agg.stride(0), stream_ptr()))
    return agg, att


def attn_bwd(q, k, v, rptr, att, dagg, heads, slope, drop_p=0.0, seed=0, offset=0, dkv=None, n_dst_dev=None,
             offset_dev=None):
    """dq [Nd, D] per destination, dk/dv [E, D] written interleaved into dkv [E, 2D]."""
    nd = rptr.numel() - 1
    E, D = k.shape
    ldq = 0 if (q.shape[0] == 1 and nd != 1) else q.stride(0)
    dq = torch.empty(nd, D, device=k.device, dtype=torch.float32)
    if dkv is None:
        dkv = torch.empty(E, 2 * D, device=k.device, dtype=torch.float32)
    qrows = nd if ldq else 1
    nbytes = 4 * (qrows * D + nd * D + 2 * E * D + E * heads + (nd + 1) + 2 * E * D + nd * D)
    _launch("attn_bwd", nbytes, 0, 1,
            lambda: call("fb_attn_bwd", ptr(q), ldq, ptr(k), ptr(v), k.stride(0), ptr(rptr), nd, _p(n_dst_dev),
                         heads, D, slope, drop_p, seed, offset, _p(offset_dev), ptr(att), ptr(dagg),
                         dagg.stride(0), ptr(dq), ptr(dkv), dkv.data_ptr() + 4 * D, dkv.stride(0), stream_ptr()))
    return dq, dkv


class AttentionCore(torch.autograd.Function):
    """One TransfomerAttentionLayer core on device (layers.py:98-223, TGAT/TGN branch):

        Qin = [h_dst | cos(b_t)]              Q = Qin W_q^T + b_q      ([Nd, D], or one row if dn == 0)
        A   = [h_src | f[eid] | cos(w_t dt + b_t)]
        KV  = A [W_k; W_v]^T + [b_k; b_v]     ([E, 2D])
        agg = sum_e dropout(softmax_seg(LeakyReLU(Q[row] . K))) V

    Node inputs come either from the previous layer's output h_all
    ([Nd + E, dn], differentiable; dst rows first, then one row per edge) or
    from a node-feature table gathered by node id.  Returns agg [Nd, D].

    With a static block (capacity-sized views and device-resident counts,
    blk.static) every launch has a fixed shape and reads the true sizes on
    the device, so the whole step can be captured in a CUDA graph."""

    @staticmethod
    def forward(ctx, h_all, w_t, b_t, W_q, b_q, W_kv, b_kv, blk, node_table, edge_table, heads, slope, drop_p,
                seed, offset_dev):
        nd, E = blk.n_dst, blk.n_edges
        nd_dev, E_dev = blk.n_dst_dev, blk.n_edges_dev
        if blk.static and h_all is not None and not blk.n_dst_static:
            raise NotImplementedError("graph mode feeds h_all only to blocks with a host-known root count")
        dn = h_all.shape[1] if h_all is not None else (node_table.shape[1] if node_table is not None else 0)
        de = edge_table.shape[1] if edge_table is not None else 0
        dtime = 0 if w_t is None else w_t.numel()
        D = W_kv.shape[0] // 2
        wv = w_t.reshape(-1) if w_t is not None else None
        dv = W_kv.device
        if h_all is not None:
            hsrc = dict(h=h_all, h_off=nd)
            hdst = dict(h=h_all, h_off=0)
        elif node_table is not None:
            hsrc = dict(h=node_table, h_idx=blk.src_nodes)
            hdst = dict(h=node_table, h_idx=blk.dst_nodes)
        else:
            hsrc = hdst = {}
        A = gather_time_encode(E, f=edge_table, f_idx=blk.eid, dt=blk.dt_edges, w=wv, b=b_t, device=dv,
                               n_rows_dev=E_dev, **hsrc)
        KV = gemm_nt(A, W_kv, b_kv, M_dev=E_dev)
        if dn > 0:
            Qin = torch.zeros(nd, dn + dtime, device=dv) if blk.static else None
            Qin = gather_time_encode(nd, w=wv, b=b_t, device=dv, out=Qin, n_rows_dev=nd_dev, **hdst)
            Q = gemm_nt(Qin, W_q, b_q, M_dev=nd_dev)
        else:
            Qin = gather_time_encode(1, w=wv, b=b_t, device=dv)
            Q = gemm_nt(Qin, W_q, b_q)
        agg, att = attn_fwd(Q, KV[:, :D], KV[:, D:], blk.rptr, heads, slope, drop_p, seed, 0, n_dst_dev=nd_dev,
                            offset_dev=offset_dev)
        ctx.save_for_backward(A, KV, Qin, Q, att, W_q, W_kv, wv, b_t, offset_dev)
        ctx.blk = blk
        ctx.cfg = (dn, de, dtime, D, heads, slope, drop_p, seed, h_all is not None)
        return agg

    @staticmethod
    def backward(ctx, dagg):
        A, KV, Qin, Q, att, W_q, W_kv, wv, b_t, offset_dev = ctx.saved_tensors
        dn, de, dtime, D, heads, slope, drop_p, seed, has_h = ctx.cfg
        blk = ctx.blk
        nd, E = blk.n_dst, blk.n_edges
        nd_dev, E_dev = blk.n_dst_dev, blk.n_edges_dev
        dagg = dagg.contiguous()
        dQ, dKV = attn_bwd(Q, KV[:, :D], KV[:, D:], blk.rptr, att, dagg, heads, slope, drop_p, seed, 0,
                           n_dst_dev=nd_dev, offset_dev=offset_dev)
        dW_kv = gemm_tn(dKV, A, M_dev=E_dev)
        db_kv = colsum(dKV, M_dev=E_dev)
        g_h = g_w = g_b = None
        if has_h and ctx.needs_input_grad[0]:
            g_h = torch.zeros(nd + E, dn, device=dagg.device, dtype=torch.float32)
            gemm_nt(dKV, W_kv[:, :dn].t().contiguous(), out=g_h[nd:], M_dev=E_dev)
        if dtime > 0:
            g_w = torch.zeros(dtime, device=dagg.device, dtype=torch.float32)
            g_b = torch.zeros(dtime, device=dagg.device, dtype=torch.float32)
            dA_t = gemm_nt(dKV, W_kv[:, dn + de:].t().contiguous(), M_dev=E_dev)
            time_encode_bwd(dA_t, blk.dt_edges, wv, b_t, g_w, g_b, n_dev=E_dev)
        # Q side
        if Qin.shape[0] == 1 and nd != 1:
            dq_vec = colsum(dQ, M_dev=nd_dev)
            dW_q = torch.outer(dq_vec, Qin[0])
            db_q = dq_vec
            dQin = (dq_vec @ W_q).unsqueeze(0)
        else:
            dW_q = gemm_tn(dQ, Qin, M_dev=nd_dev)
            db_q = colsum(dQ, M_dev=nd_dev)
            dQin = gemm_nt(dQ, W_q.t().contiguous(), M_dev=nd_dev)
        if g_h is not None and dn > 0:
            g_h[:nd].copy_(dQin[:, :dn])
        if dtime > 0:
            # every Q row's time block is cos(b_t) (TimeEncode of dt = 0); rows
            # past the device-side count carry no gradient
            rows = dQin[:, dn:] if nd_dev is None or Qin.shape[0] == 1 else \
                torch.where((torch.arange(nd, device=dagg.device) < nd_dev).unsqueeze(1), dQin[:, dn:], 0.0)
            g_b -= torch.sin(b_t) * rows.sum(0)
        return (g_h, None if g_w is None else g_w.view(-1, 1), g_b, dW_q, db_q, dW_kv, db_kv,
                None, None, None, None, None, None, None, None)
