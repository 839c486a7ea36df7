"""GPU: the device-built synthetic workload of config 5.

* make_graph_device keeps the reference preprocessing contract that
  make_graph keeps (fast_util/preprocess/gen_graph.py), with every array a
  device tensor: chronological edge
  ids, non-decreasing float32 timestamps, a CSR keyed by the source whose
  every adjacency list is in chronological order (a stable sort on the
  source), indices / ts / eid consistent with the edge list.
* fb_fill_normal_bf16 gives N(0, 1) samples (moments within sampling error)
  and zero padding columns; the same seed gives the same table.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_device_graph_keeps_the_csr_contract(cuda):
    import dataclasses
    from fast_b200.data import CONFIGS, make_graph_device
    cfg = dataclasses.replace(CONFIGS[5], edges=200_000)
    g = make_graph_device(cfg, cuda, seed=3)
    E, N = cfg.edges, cfg.nodes
    assert g.src.is_cuda and g.dst.is_cuda and g.ts.is_cuda       # the edge list stays on the device
    src, dst, ts = g.src.cpu().numpy(), g.dst.cpu().numpy(), g.ts.cpu().numpy()
    assert src.shape == (E,) and dst.shape == (E,) and ts.dtype == np.float32
    assert bool(np.all(np.diff(ts) >= 0))
    indptr = g.indptr.cpu().numpy().astype(np.int64)
    eid = g.eid.cpu().numpy().astype(np.int64)
    assert indptr[0] == 0 and indptr[-1] == E and bool(np.all(np.diff(indptr) >= 0))
    assert np.array_equal(np.sort(eid), np.arange(E))
    assert np.array_equal(np.bincount(src, minlength=N), np.diff(indptr))
    order = np.argsort(src, kind="stable")
    assert np.array_equal(eid, order)                       # chronological within each source
    assert np.array_equal(g.indices.cpu().numpy(), dst[order])
    assert np.array_equal(g.ts_csr.cpu().numpy(), ts[order])
    # Zipf(1.05) endpoints: the most frequent node takes a large share
    share = np.bincount(src, minlength=N).max() / E
    assert 0.05 < share < 0.3


def test_fill_normal_bf16(cuda):
    from fast_b200.capi import call, ptr, stream_ptr
    rows, cols, ld = 20000, 186, 192
    t = torch.full((rows, ld), 9.0, device=cuda, dtype=torch.bfloat16)
    call("fb_fill_normal_bf16", ptr(t), rows, cols, ld, 11, stream_ptr())
    u = torch.full_like(t, 9.0)
    call("fb_fill_normal_bf16", ptr(u), rows, cols, ld, 11, stream_ptr())
    torch.cuda.synchronize()
    assert torch.equal(t, u)
    assert bool((t[:, cols:] == 0).all())
    x = t[:, :cols].float().double()
    n = x.numel()
    assert abs(float(x.mean())) < 5 / n ** 0.5
    assert abs(float(x.var()) - 1.0) < 0.01
    assert abs(float((x ** 3).mean())) < 0.02                 # symmetric
    assert abs(float((x ** 4).mean()) - 3.0) < 0.05           # normal kurtosis
