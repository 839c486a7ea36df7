"""GPU: the allocation-free exclusive sum (fb_exclusive_sum_noalloc).

Some callers cannot allocate device memory: a host that gives this library a
fixed memory budget and owns every allocation itself, or a loop where an
allocator call would synchronise the device.  This entry point serves them by
keeping its scratch in a static device array of the library.  Called through
the C ABI, twice in a row, it must return exactly what fb_exclusive_sum
(caller-provided workspace) returns, and what torch.cumsum gives with a
leading zero; n = 0 must give out[0] = 0; sizes past its stated maximum must
be refused before any launch.

The file is named so that pytest collects it last: a run that stops at its
first failure has then already run every other test.  It also passes alone in
a fresh process, where its first call does the per-device set-up.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu
MAX_N = 4096 * 256


def _scan_with_workspace(x, lib, stream):
    n = x.numel()
    out = torch.empty(n + 1, dtype=torch.int32, device=x.device)
    ws = torch.empty(max(1, int(lib.fb_exclusive_sum_ws_bytes(n))), dtype=torch.uint8, device=x.device)
    assert lib.fb_exclusive_sum(x.data_ptr(), n, out.data_ptr(), ws.data_ptr(), stream) == 0
    return out


def _cumsum_ref(x):
    return torch.cat([torch.zeros(1, dtype=torch.int64, device=x.device), torch.cumsum(x.long(), 0)]).int()


def test_exclusive_sum_noalloc_matches(cuda):
    from fast_b200.capi import lib, stream_ptr
    st = stream_ptr()
    g = torch.Generator(device=cuda).manual_seed(3)
    # two calls in a row at the maximum and below it, then edge sizes: an exact
    # multiple of the 256-element chunk, one element, none
    for n in (MAX_N, 100_003, 256, 1, 0):
        x = torch.randint(0, 9, (max(n, 1),), dtype=torch.int32, device=cuda, generator=g)[:n]
        ref = _scan_with_workspace(x, lib, st) if n else torch.zeros(1, dtype=torch.int32, device=cuda)
        out = torch.full((n + 1,), -1, dtype=torch.int32, device=cuda)
        rc = lib.fb_exclusive_sum_noalloc(x.data_ptr() if n else 0, n, out.data_ptr(), st)
        assert rc == 0, lib.fb_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(out, ref), n
        assert torch.equal(out, _cumsum_ref(x)), n
    small = torch.ones(4, dtype=torch.int32, device=cuda)
    out = torch.empty(5, dtype=torch.int32, device=cuda)
    assert lib.fb_exclusive_sum_noalloc(small.data_ptr(), MAX_N + 1, out.data_ptr(), st) == 3   # unsupported
    assert b"1048576" in lib.fb_last_error()
