"""TEST INFRASTRUCTURE ONLY -- CPU oracle for the temporal sampler.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline leg import
this module, and only as the checker.  It drives the C restatement in
``sampler_oracle.c`` with the same orchestration as the reference
``ParallelSampler::sample`` (NoneBone/FAST getSamplerCore/sampler_core.cpp:597-712)
and ``sample_layer`` (sampler_core.cpp:458-595), and exposes the same Python
surface as the reference pybind module (sampler_core.cpp:1115-1149).

``load_reference()`` loads the reference sampler compiled from its own source
into ``oracle/_ref`` (see oracle/Makefile), when that build exists.
"""
import ctypes
import glob
import importlib.util
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")


def _lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "_build", "libsampler_oracle.so")
        if not os.path.exists(path):
            subprocess.check_call(["make", "-s", "-C", _HERE, "all"])
        lib = ctypes.CDLL(path)
        lib.orc_reset.argtypes = [_i32p, _i32p, ctypes.c_int64]
        lib.orc_update_ptr.argtypes = [_i32p, _f32p, _i32p, _i32p, _f32p, ctypes.c_int64, ctypes.c_float]
        lib.orc_sample_layer.restype = ctypes.c_int64
        lib.orc_sample_layer.argtypes = [
            _i32p, _i32p, _i32p, _f32p, _i32p, _i32p, ctypes.c_int, ctypes.c_int, ctypes.c_float,
            ctypes.c_float, _i32p, _f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.POINTER(ctypes.c_uint), _i32p, _i32p, _i32p, _f32p, _f32p, _i32p]
        lib.orc_cnt.restype = ctypes.c_int64
        lib.orc_cnt.argtypes = [_i32p, ctypes.c_int64, _i32p]
        lib.orc_dedup.restype = ctypes.c_int64
        lib.orc_dedup.argtypes = [_i32p, ctypes.c_int64, _i32p, _i32p]
        _LIB = lib
    return _LIB


class OracleBlock:
    """Same accessors as the reference TemporalGraphBlock (sampler_core.cpp:31-65)."""

    def __init__(self, row, col, eid, ts, dts, nodes, uniE, invE, cntE, dim_in, dim_out):
        self._d = dict(row=row, col=col, eid=eid, ts=ts, dts=dts, nodes=nodes,
                       uniE=uniE, invE=invE, cntE=cntE)
        self._dim_in, self._dim_out = dim_in, dim_out

    def __getattr__(self, k):
        d = self.__dict__.get("_d")
        if d is not None and k in d:
            return lambda: d[k].copy()
        raise AttributeError(k)

    def dim_in(self):
        return self._dim_in

    def dim_out(self):
        return self._dim_out


class OracleSampler:
    """CPU restatement of ParallelSampler with one worker thread."""

    def __init__(self, indptr, indices, eid, ts, num_thread_per_worker, num_workers, num_layers,
                 num_neighbors, recent, prop_time, num_history, window_duration):
        self.indptr = np.ascontiguousarray(indptr, dtype=np.int32)
        self.indices = np.ascontiguousarray(indices, dtype=np.int32)
        self.eid = np.ascontiguousarray(eid, dtype=np.int32)
        self.ts = np.ascontiguousarray(ts, dtype=np.float32)
        self.num_layers = int(num_layers)
        self.num_neighbors = list(num_neighbors)
        self.recent = bool(recent)
        self.prop_time = bool(prop_time)
        self.num_history = int(num_history)
        self.window_duration = np.float32(window_duration)
        self.n_nodes = self.indptr.shape[0] - 1
        self.ts_ptr = [np.empty(self.n_nodes, np.int32) for _ in range(self.num_history + 1)]
        self.ret = []
        self.reset()

    def reset(self):
        for p in self.ts_ptr:
            _lib().orc_reset(self.indptr, p, self.n_nodes)

    def _update(self, slot, roots, rts, offset):
        _lib().orc_update_ptr(self.indptr, self.ts, self.ts_ptr[slot], roots, rts,
                              roots.shape[0], ctypes.c_float(offset))

    def _sample_layer(self, roots0, rts0, neighs, use_ptr, from_root):
        nh = self.num_history
        lib = _lib()
        if from_root:
            roots, rts = roots0, rts0
        else:
            prev = self.ret[len(self.ret) - 1 - nh]
            roots, rts = prev._d["nodes"], prev._d["ts"]
        if use_ptr:
            self._update(nh, roots, rts, 0.0)
        for i in range(nh):
            if not from_root:
                prev = self.ret[len(self.ret) - 1 - i - nh]
                roots, rts = prev._d["nodes"], prev._d["ts"]
            offset = np.float32(-i) * self.window_duration
            if use_ptr and abs(float(self.window_duration)) > 1e-7:
                self._update(nh - 1 - i, roots, rts, np.float32(offset - self.window_duration))
            R = roots.shape[0]
            cap = R * neighs
            row = np.empty(cap, np.int32)
            col = np.empty(cap, np.int32)
            eo = np.empty(cap, np.int32)
            tso = np.empty(R + cap, np.float32)
            dtso = np.zeros(R + cap, np.float32)
            nodes = np.empty(R + cap, np.int32)
            state = ctypes.c_uint(0)
            E = lib.orc_sample_layer(self.indptr, self.indices, self.eid, self.ts,
                                     self.ts_ptr[nh - 1 - i], self.ts_ptr[nh - i], int(use_ptr), nh,
                                     ctypes.c_float(self.window_duration), ctypes.c_float(offset),
                                     roots, rts, R, int(neighs), int(self.recent), int(self.prop_time),
                                     ctypes.byref(state), row, col, eo, tso, dtso, nodes)
            tso[:R] = rts
            nodes[:R] = roots
            dtso[:R] = 0
            cnt = np.empty(E + 1, np.int32)
            m = lib.orc_cnt(row[:E].copy(), E, cnt)
            uni = np.empty(E, np.int32)
            inv = np.empty(E, np.int32)
            nu = lib.orc_dedup(eo[:E].copy(), E, uni, inv)
            blk = OracleBlock(row[:E].copy(), col[:E].copy(), eo[:E].copy(), tso[:R + E].copy(),
                              dtso[:R + E].copy(), nodes[:R + E].copy(), uni[:nu].copy(),
                              inv[:E].copy(), cnt[:m].copy(), R + E, R)
            self.ret[len(self.ret) - 1 - i] = blk

    def sample(self, root_nodes, root_ts, csrFlag=()):
        roots = np.ascontiguousarray(root_nodes, dtype=np.int32)
        rts = np.ascontiguousarray(root_ts, dtype=np.float32)
        self.ret = []
        first = True
        for layer in range(self.num_layers):
            self.ret.extend([None] * self.num_history)
            if first or (self.prop_time and self.num_history == 1) or self.recent:
                first = False
                use_ptr = True
            else:
                use_ptr = False
            self._sample_layer(roots, rts, self.num_neighbors[layer], use_ptr, layer == 0)

    def get_ret(self):
        return list(self.ret)

    # host-CPU tuning hooks of the reference; no-ops here
    def configOMP(self, *a, **k):
        return None


def reference_path():
    """Path of the reference sampler built from its own source, or None."""
    hits = glob.glob(os.path.join(_HERE, "_ref", "sampler_core_ref*.so"))
    return hits[0] if hits else None


def load_reference():
    """Import the compiled reference sampler (module ``sampler_core_ref``: the
    reference source built with its module renamed, so it can sit beside the
    product module ``sampler_core`` in one process)."""
    path = reference_path()
    if path is None:
        return None
    spec = importlib.util.spec_from_file_location("sampler_core_ref", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod
