"""CPU: the C-ABI library loads without a GPU and exports every entry point
include/fast_b200.h declares; the ctypes table covers them all; the drop-in
modules expose the reference's names (operators.cpp:606-624,
sampler_core.cpp:1115-1149).  No kernel is called here."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    with open(os.path.join(ROOT, "include", "fast_b200.h")) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fb_[a-z0-9_]+)\s*\(", text)))


def test_header_symbols_are_exported():
    from fast_b200.capi import LIB_PATH
    lib = ctypes.CDLL(LIB_PATH)
    names = _declared()
    assert len(names) > 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_ctypes_table_covers_the_header():
    from fast_b200 import capi
    declared = set(_declared())
    table = set(capi.exported_symbols())
    assert declared - table == set(), sorted(declared - table)
    assert table - declared == set(), sorted(table - declared)


def test_version_and_error_string_without_a_gpu():
    from fast_b200.capi import lib
    assert lib.fb_version().decode()
    assert isinstance(lib.fb_last_error(), bytes)


def test_dropin_modules_expose_reference_names():
    from fast_b200.ext import fastAgg, sampler_core
    for name in ["forward_edge_softmax", "backward_edge_softmax", "forward_csr_edge_softmax",
                 "backward_csr_edge_softmax", "forward_tgat", "backward_tgat", "forward_tgat_shd",
                 "backward_tgat_shd"]:
        assert hasattr(fastAgg, name), name
    assert hasattr(sampler_core, "ParallelSampler")
    assert hasattr(sampler_core, "TemporalGraphBlock")
    for meth in ["sample", "get_ret", "reset"]:
        assert hasattr(sampler_core.ParallelSampler, meth), meth
    for acc in ["row", "col", "eid", "ts", "dts", "nodes", "dim_in", "dim_out", "uniE", "invE", "cntE"]:
        assert hasattr(sampler_core.TemporalGraphBlock, acc), acc


def test_wrappers_reject_bad_operands_before_any_launch():
    """Host-side checks of the ops wrappers: operands of the wrong type or
    layout raise ValueError before the library is called (no GPU needed)."""
    import pytest
    import torch
    from fast_b200 import ops
    d = torch.zeros(4, dtype=torch.float32)
    with pytest.raises(ValueError):                          # fp16 gradient
        ops.time_encode_bwd(torch.zeros(4, 3, dtype=torch.float16), d, d[:3], d[:3], d[:3], d[:3])
    with pytest.raises(ValueError):                          # column stride != 1
        ops.time_encode_bwd(torch.zeros(3, 4).t(), d, d[:3], d[:3], d[:3], d[:3])
    a = torch.zeros(16, 8, dtype=torch.float32)
    with pytest.raises(ValueError):                          # fp32 operand to the bf16 GEMM
        ops.gemm_bf16_group([dict(kind=ops.NT, A=a, B=a, out=torch.zeros(16, 16))])


def test_tiered_gather_rejects_bad_arguments_before_any_launch():
    """fb_gather_rows_tiered checks its arguments on the host: element width,
    row width, leading dimensions and missing tables return FB_ERR_ARG (1)
    without touching a GPU."""
    from fast_b200.capi import lib
    buf = ctypes.create_string_buffer(64)
    p = ctypes.addressof(buf)
    args = dict(ids=p, n=4, n_dev=None, slot_of=p, n_rows_total=8, dev_rows=p, ld_dev=4, n_dev_rows=2,
                host_rows=p, ld_host=4, d=4, elem_bytes=4, out=p, ld_out=4, misses=None, err=None, stream=None)
    for bad in (dict(elem_bytes=3), dict(d=0), dict(ld_out=3), dict(ld_host=2), dict(host_rows=None),
                dict(dev_rows=None), dict(ids=None), dict(n=-1)):
        a = dict(args, **bad)
        assert lib.fb_gather_rows_tiered(*a.values()) == 1, bad
    assert lib.fb_host_rows_device_pointer(None, None) == 1


def test_import_fails_loudly_without_the_library():
    """No fallback: with libfast_b200.so absent, importing the binding (and
    so every op) raises ImportError naming the build command."""
    import subprocess
    import sys
    code = ("import os, sys\n"
            "real = os.path.exists\n"
            "os.path.exists = lambda p: False if str(p).endswith('libfast_b200.so') else real(p)\n"
            "try:\n"
            "    import fast_b200.ops\n"
            "except ImportError as e:\n"
            "    print('IMPORT-ERROR', e)\n"
            "    sys.exit(0)\n"
            "sys.exit(3)\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr[-2000:]
    assert "IMPORT-ERROR" in r.stdout and "fast_b200.build" in r.stdout
