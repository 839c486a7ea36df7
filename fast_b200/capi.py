"""ctypes binding of the libfast_b200 C ABI (include/fast_b200.h).

The training path calls the kernels through these wrappers with raw device
pointers taken from torch tensors, on torch's current stream.  A non-zero
status raises ``FastB200Error`` with the library's message.  There is no
fallback: if the library is missing the import fails.
"""
import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libfast_b200.so")


class FastB200Error(RuntimeError):
    pass


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            "fast_b200: %s is missing; build it with `python -m fast_b200.build` "
            "(or __graft_entry__.build())" % LIB_PATH)
    return ctypes.CDLL(LIB_PATH)


lib = _load()

c_i32p = ctypes.c_void_p
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float
_U64 = ctypes.c_uint64
_SZ = ctypes.c_size_t

_SIGS = {
    "fb_last_error": (ctypes.c_char_p, []),
    "fb_version": (ctypes.c_char_p, []),
    "fb_sampler_create": (_I, [_P, _P, _P, _P, _I64, _I64, _I, _I, _P, _I, _I, _I, _F, _U64, _P]),
    "fb_sampler_destroy": (_I, [_P]),
    "fb_sampler_reset": (_I, [_P, _P]),
    "fb_sampler_sample": (_I, [_P, _P, _P, _I64, _I, _P]),
    "fb_sampler_update_pointers": (_I, [_P, _P, _P, _I64, _P]),
    "fb_sampler_sample_shard": (_I, [_P, _P, _P, _I64, _P, _P, _I64, _P]),
    "fb_sampler_num_blocks": (_I, [_P]),
    "fb_sampler_block": (_I, [_P, _I, _P]),
    "fb_sampler_dims": (_I, [_P, _P, _P]),
    "fb_sampler_dedup": (_I, [_P, _I, _P]),
    "fb_sampler_set_call_index": (_I, [_P, _U64]),
    "fb_attn_fwd": (_I, [_P, _I64, _P, _P, _I64, _P, _I64, _P, _I, _I, _F, _F, _U64, _U64, _P, _P, _P, _I64, _P]),
    "fb_attn_bwd": (_I, [_P, _I64, _P, _P, _I64, _P, _I64, _P, _I, _I, _F, _F, _U64, _U64, _P, _P, _P, _I64,
                         _P, _P, _P, _I64, _P]),
    "fb_attn_logits_fwd": (_I, [_P, _P, _I64, _P, _I64, _P, _I64, _I, _I, _F, _F, _P, _P, _P, _P]),
    "fb_attn_logits_bwd": (_I, [_P, _P, _I64, _P, _I64, _P, _I64, _I, _I, _F, _F, _P, _P, _P, _P, _P, _P]),
    "fb_dropout_scale": (_I, [_I64, _I, _F, _U64, _U64, _P, _P]),
    "fb_count_ids": (_I, [_P, _I64, _P, _I64, _P]),
    "fb_balanced_mask": (_I, [_P, _I64, _I, _P, _P]),
    "fb_edge_softmax_fwd": (_I, [_P, _I64, _P, _I, _P, _P]),
    "fb_edge_softmax_bwd": (_I, [_P, _I64, _P, _P, _I, _P, _P]),
    "fb_scatter_rows": (_I, [_P, _P, _I64, _P, _I64, _I, _P, _I64, _P]),
    "fb_segment_rows": (_I, [_P, _I64, _P, _P, _P, _I64, _I, _P, _I64, _P]),
    "fb_exclusive_sum_ws_bytes": (_SZ, [_I64]),
    "fb_exclusive_sum": (_I, [_P, _I64, _P, _P, _P]),
    "fb_exclusive_sum_noalloc": (_I, [_P, _I64, _P, _P]),
    "fb_gather_time_encode": (_I, [_P, _I64, _P, _I64, _P, _I, _P, _I64, _P, _I, _P, _P, _P, _I, _P, _I64, _I64, _P,
                                   _P]),
    "fb_time_encode_bwd_ws_bytes": (_SZ, [_I64, _I]),
    "fb_time_encode_bwd": (_I, [_P, _I64, _P, _P, _P, _I, _I64, _P, _P, _P, _P, _P]),
    "fb_time_encode_bwd_bf16": (_I, [_P, _I64, _P, _P, _P, _I, _I64, _P, _P, _P, _P, _P]),
    "fb_gather_rows_tiered": (_I, [_P, _I64, _P, _P, _I64, _P, _I64, _I64, _P, _I64, _I, _I, _P, _I64, _P, _P, _P]),
    "fb_host_rows_device_pointer": (_I, [_P, _P]),
    "fb_gemm_nt": (_I, [_P, _I64, _P, _I64, _P, _P, _I64, _I64, _P, _I, _I, _I, _P]),
    "fb_gemm_nt_tc_supported": (_I, [_P, _I64, _P, _I64, _I, _I]),
    "fb_gemm_nt_tc": (_I, [_P, _I64, _P, _I64, _P, _P, _I64, _I64, _P, _I, _I, _I, _P]),
    "fb_gemm_tc_error": (_I, [_P, _I]),
    "fb_gemm_tn_ws_bytes": (_SZ, [_I64, _I, _I]),
    "fb_gemm_tn": (_I, [_P, _I64, _P, _I64, _P, _I64, _I64, _P, _I, _I, _I, _P, _P]),
    "fb_colsum_ws_bytes": (_SZ, [_I64, _I]),
    "fb_colsum": (_I, [_P, _I64, _P, _I64, _P, _I, _I, _P, _P]),
    "fb_gemm_nn": (_I, [_P, _I64, _P, _I64, _P, _P, _I64, _I64, _P, _I, _I, _I, _P]),
    "fb_gemm_tn_bias": (_I, [_P, _I64, _P, _I64, _P, _I64, _I64, _P, _I, _I, _I, _P, _I, _P, _P]),
    "fb_layer_tail_fwd": (_I, [_P, _I64, _P, _P, _F, _F, _U64, _U64, _P, _P, _P, _I64, _P, _I64, _I64, _P, _P,
                               _I, _P]),
    "fb_layer_tail_bwd_ws_bytes": (_SZ, [_I64, _I]),
    "fb_layer_tail_bwd": (_I, [_P, _I64, _P, _I64, _P, _F, _F, _P, _I64, _P, _P, _I64, _P, _P, _I, _P, _P]),
    "fb_edge_predictor_loss_ws_bytes": (_SZ, [_I64, _I]),
    "fb_edge_predictor_loss": (_I, [_P, _I64, _P, _I64, _P, _P, _I64, _I, _P, _P, _I64, _P, _I64, _P, _P, _P,
                                    _P, _P]),
    "fb_q_time_bwd": (_I, [_P, _I, _P, _I64, _I, _I, _P, _P, _P, _I64, _P, _P, _P]),
    "fb_adam_step": (_I, [_P, _P, _P, _P, _I64, _F, _F, _F, _F, _P, _P, _P]),
    "fb_attn_error": (_I, [_P, _I]),
    "fb_mem_gather": (_I, [_P, _P, _I64, _P, _P, _I, _P, _P, _I, _P, _P, _I, _P, _I64, _P, _P, _P]),
    "fb_gru_fwd": (_I, [_P, _P, _P, _P, _I64, _P, _I, _P]),
    "fb_gru_bwd": (_I, [_P, _P, _P, _P, _I64, _I64, _P, _I, _P]),
    "fb_mailbox_update_self": (_I, [_P, _P, _I64, _P, _I64, _I, _P, _I64, _I, _P, _P, _P, _P, _I, _P, _P, _P, _P]),
    "fb_memory_update": (_I, [_P, _P, _I64, _P, _I64, _I, _P, _P, _P, _P, _P, _P]),
    "fb_mail_slots_gather": (_I, [_P, _P, _I64, _P, _P, _I, _P, _P, _I, _I, _P, _P, _I, _P, _I64, _P, _P, _P]),
    "fb_add_layernorm_fwd": (_I, [_P, _P, _P, _P, _F, _P, _P, _P, _I64, _P, _I, _P]),
    "fb_add_layernorm_bwd_ws_bytes": (ctypes.c_size_t, [_I64, _I]),
    "fb_add_layernorm_bwd": (_I, [_P, _P, _P, _P, _P, _P, _P, _I64, _P, _I, _P, _P]),
    "fb_mailbox_update_neighbors": (_I, [_P, _P, _P, _I64, _P, _I64, _P, _I64, _I, _P, _I64, _I, _P, _P, _P, _P, _I,
                                         _P, _P, _P, _P]),
    "fb_gather_time_encode_bf16": (_I, [_P, _I, _I64, _P, _I64, _P, _I, _P, _I, _I64, _P, _I, _P, _P, _P, _I, _P,
                                        _I64, _I64, _P, _P]),
    "fb_attn_bwd_bf16kv": (_I, [_P, _I64, _P, _P, _I64, _P, _I64, _P, _I, _I, _F, _F, _U64, _U64, _P, _P, _P, _I64,
                                _P, _P, _P, _I64, _P]),
    "fb_attn_fwd_kvbf16": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I, _I, _F, _F, _U64, _U64, _P, _P, _P, _I64, _P]),
    "fb_attn_bwd_kvbf16": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I, _I, _F, _F, _U64, _U64, _P, _P, _P, _I64, _P,
                                _P, _I64, _P]),
    "fb_attn_fwd_kvbf16_bf16out": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I, _I, _F, _F, _U64, _U64, _P, _P, _P, _I64,
                                        _P]),
    "fb_attn_bwd_kvbf16_bf16dq": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I, _I, _F, _F, _U64, _U64, _P, _P, _P, _I64,
                                       _P, _I64, _P, _I64, _P]),
}

class GemmProblem(ctypes.Structure):
    """fb_gemm_problem (include/fast_b200.h)."""
    _fields_ = [("kind", ctypes.c_int),
                ("A", ctypes.c_void_p), ("lda", ctypes.c_int64),
                ("A2", ctypes.c_void_p), ("lda2", ctypes.c_int64), ("k1", ctypes.c_int),
                ("B", ctypes.c_void_p), ("ldb", ctypes.c_int64),
                ("bias", ctypes.c_void_p),
                ("C", ctypes.c_void_p), ("ldc", ctypes.c_int64),
                ("M", ctypes.c_int64), ("M_dev", ctypes.c_void_p),
                ("N", ctypes.c_int), ("K", ctypes.c_int),
                ("accumulate", ctypes.c_int),
                ("db", ctypes.c_void_p), ("db_accumulate", ctypes.c_int)]


_SIGS["fb_gemm_group_ws_bytes"] = (_SZ, [ctypes.POINTER(GemmProblem), _I])
_SIGS["fb_gemm_group"] = (_I, [ctypes.POINTER(GemmProblem), _I, _P, _SZ, _P])


class Bf16RowGather(ctypes.Structure):
    """fb_bf16_row_gather (include/fast_b200.h): an operand's rows gathered
    from up to three bf16 sources, in 64-column-aligned segments."""
    _fields_ = [("nseg", ctypes.c_int), ("end", ctypes.c_int * 3), ("tab", ctypes.c_void_p * 3),
                ("tab_rows", ctypes.c_int64 * 3), ("tab_ld", ctypes.c_int64 * 3), ("tab_cols", ctypes.c_int * 3),
                ("idx", ctypes.c_void_p * 3)]


class GemmBf16Problem(ctypes.Structure):
    """fb_gemm_bf16_problem (include/fast_b200.h): fb_gemm_problem's fields
    (operand pointers to bf16) plus ka, the TN column segments, the bf16
    output flag and the optional gathered operand."""
    _fields_ = GemmProblem._fields_ + [("ka", ctypes.c_int), ("nseg", ctypes.c_int),
                                       ("seg_at", ctypes.c_int * 3), ("seg_len", ctypes.c_int * 3),
                                       ("seg_to", ctypes.c_int * 3), ("c_bf16", ctypes.c_int),
                                       ("gather", ctypes.POINTER(Bf16RowGather)), ("add", ctypes.c_void_p),
                                       ("add_idx", ctypes.c_void_p), ("ld_add", ctypes.c_int64),
                                       ("add_rows", ctypes.c_int64)]


_SIGS["fb_gemm_bf16_group_ws_bytes"] = (_SZ, [ctypes.POINTER(GemmBf16Problem), _I])
_SIGS["fb_gemm_bf16_group"] = (_I, [ctypes.POINTER(GemmBf16Problem), _I, _P, _SZ, _P])


class CastJob(ctypes.Structure):
    """fb_cast_job (include/fast_b200.h)."""
    _fields_ = [("src", ctypes.c_void_p), ("lds", ctypes.c_int64), ("dst", ctypes.c_void_p), ("ldd", ctypes.c_int64),
                ("rows", ctypes.c_int64), ("rows_dev", ctypes.c_void_p), ("cols", ctypes.c_int),
                ("pad_", ctypes.c_int)]


CAST_MAX_JOBS = 32
_SIGS["fb_cast_bf16"] = (_I, [ctypes.POINTER(CastJob), _I, _P])
_SIGS["fb_fill_normal_bf16"] = (_I, [_P, _I64, _I, _I64, _U64, _P])

for _name, (_res, _args) in _SIGS.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


class BlockView(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in
                ("row", "col", "eid", "ts", "dts", "nodes", "rptr", "cntE", "uniE", "invE", "dims")] + \
               [("max_roots", ctypes.c_int64), ("max_edges", ctypes.c_int64), ("dte", ctypes.c_void_p),
                ("nbr", ctypes.c_void_p)]


def exported_symbols():
    """Names this binding expects the library to export."""
    return list(_SIGS)


def check(rc):
    if rc != 0:
        raise FastB200Error("fast_b200: " + lib.fb_last_error().decode())


def call(name, *args):
    """Calls an fb_* entry point and raises on a non-zero status."""
    check(getattr(lib, name)(*args))


def ptr(t):
    """Device pointer of a tensor (None -> NULL)."""
    return None if t is None else t.data_ptr()


def stream_ptr(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class CSampler:
    """Direct C-ABI handle of the device sampler (fb_sampler_*), for callers
    that do not go through the pybind `sampler_core` module."""

    def __init__(self, indptr, indices, eid, ts, num_layers, num_neighbors, recent, prop_time=False,
                 num_history=1, window_duration=0.0, seed=0):
        import numpy as np
        self._keep = [np.ascontiguousarray(a) for a in (indptr, indices, eid, ts)]
        nn = (ctypes.c_int32 * len(num_neighbors))(*num_neighbors)
        h = ctypes.c_void_p()
        ip, ix, ei, t = self._keep
        check(lib.fb_sampler_create(ip.ctypes.data, ix.ctypes.data, ei.ctypes.data, t.ctypes.data, ip.size - 1,
                                    ix.size, 0, num_layers, nn, int(recent), int(prop_time), num_history,
                                    float(window_duration), seed, ctypes.byref(h)))
        self.h = h
        self.nblocks = lib.fb_sampler_num_blocks(h)

    def __del__(self):
        if getattr(self, "h", None):
            lib.fb_sampler_destroy(self.h)
            self.h = None

    def reset(self):
        check(lib.fb_sampler_reset(self.h, stream_ptr()))

    def sample(self, roots, root_ts):
        import numpy as np
        r = np.ascontiguousarray(roots, dtype=np.int32)
        t = np.ascontiguousarray(root_ts, dtype=np.float32)
        check(lib.fb_sampler_sample(self.h, r.ctypes.data, t.ctypes.data, r.size, 0, stream_ptr()))

    def sample_shard(self, roots, root_ts, global_roots, global_ts):
        """One data-parallel rank's sample(): device (torch) tensors of this
        rank's roots and of the global batch's (fb_sampler_sample_shard)."""
        check(lib.fb_sampler_sample_shard(self.h, roots.data_ptr(), root_ts.data_ptr(), roots.numel(),
                                          global_roots.data_ptr(), global_ts.data_ptr(), global_roots.numel(),
                                          stream_ptr()))

    def dims(self):
        import numpy as np
        d = np.zeros(8 * self.nblocks, np.int32)
        check(lib.fb_sampler_dims(self.h, d.ctypes.data, stream_ptr()))
        return d.reshape(self.nblocks, 8)

    def dedup(self, i):
        check(lib.fb_sampler_dedup(self.h, i, stream_ptr()))

    def block_arrays(self, i, dedup=True):
        """Host copies of block i (reference TemporalGraphBlock fields)."""
        import numpy as np
        import torch
        if dedup:
            self.dedup(i)
        d = self.dims()[i]
        R, E, S, dim_in, nu = (int(x) for x in d[:5])
        v = BlockView()
        check(lib.fb_sampler_block(self.h, i, ctypes.byref(v)))

        def grab(p, n, dt):
            if n == 0:
                return np.empty(0, dt)
            return device_array(p, n, dt).cpu().numpy().copy()
        return dict(row=grab(v.row, E, np.int32), col=grab(v.col, E, np.int32), eid=grab(v.eid, E, np.int32),
                    ts=grab(v.ts, dim_in, np.float32), dts=grab(v.dts, dim_in, np.float32),
                    nodes=grab(v.nodes, dim_in, np.int32), rptr=grab(v.rptr, R + 1, np.int32),
                    cntE=grab(v.cntE, S + 1 if E else 0, np.int32), uniE=grab(v.uniE, nu if dedup else 0, np.int32),
                    invE=grab(v.invE, E if dedup else 0, np.int32), dim_in=dim_in, dim_out=R)


class _CudaArray:
    def __init__(self, p, n, typestr):
        self.__cuda_array_interface__ = {"shape": (int(n),), "typestr": typestr, "data": (int(p), False),
                                         "version": 3, "strides": None}


def device_array(p, n, dtype):
    """Zero-copy torch view of n elements of numpy dtype at device pointer p."""
    import numpy as np
    import torch
    return torch.as_tensor(_CudaArray(p, n, np.dtype(dtype).str), device="cuda")
