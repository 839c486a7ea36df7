"""GPU: the allocation-free exclusive sum (fb_exclusive_sum_noalloc), for
callers that cannot allocate device memory -- inside a CUDA graph capture,
under a fixed memory budget, or where an allocator call would stall the
device.  Called through the C ABI, twice in a row, it must return exactly
what fb_exclusive_sum (caller-provided workspace) returns; sizes past its
stated maximum must be refused before any launch.

This file is named to run last, so a run that stops at its first failure has
already run every other test.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu
MAX_N = 4096 * 256


def _scan_with_workspace(x, lib, stream):
    n = x.numel()
    out = torch.empty(n + 1, dtype=torch.int32, device=x.device)
    ws = torch.empty(int(lib.fb_exclusive_sum_ws_bytes(n)), dtype=torch.uint8, device=x.device)
    assert lib.fb_exclusive_sum(x.data_ptr(), n, out.data_ptr(), ws.data_ptr(), stream) == 0
    return out


def test_exclusive_sum_noalloc_matches(cuda):
    from fast_b200.capi import lib, stream_ptr
    st = stream_ptr()
    g = torch.Generator(device=cuda).manual_seed(3)
    for n in (MAX_N, 100_003):      # two calls in a row, the second shorter than the first
        x = torch.randint(0, 9, (n,), dtype=torch.int32, device=cuda, generator=g)
        ref = _scan_with_workspace(x, lib, st)
        out = torch.full((n + 1,), -1, dtype=torch.int32, device=cuda)
        rc = lib.fb_exclusive_sum_noalloc(x.data_ptr(), n, out.data_ptr(), st)
        assert rc == 0, lib.fb_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    small = torch.ones(4, dtype=torch.int32, device=cuda)
    out = torch.empty(5, dtype=torch.int32, device=cuda)
    assert lib.fb_exclusive_sum_noalloc(small.data_ptr(), MAX_N + 1, out.data_ptr(), st) == 3   # unsupported
    assert b"1048576" in lib.fb_last_error()
