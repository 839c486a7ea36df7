"""GPU: the on-disk dataset format read into device memory.

* build_ext_full_device (the CSR of gen_graph.py built with device sorts)
  equals the reference's own ext_full.npz, recorded by
  tests/golden/make_loader_golden.py, bit for bit, with and without
  --add_reverse, on a raw edge list with sparse ids, hubs and many equal
  timestamps; and equals build_ext_full on a synthetic graph.
* load_graph(dir, device) puts the files' arrays on the device unchanged, and
  the device sampler on them returns the oracle's recent-k blocks.
"""
import os

import numpy as np
import pytest
import torch

from fast_b200 import dataio

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "loader_golden.npz")


def test_device_csr_matches_reference(cuda, tmp_path):
    import pandas as pd
    z = np.load(GOLDEN)
    csv = str(tmp_path / "edges.csv")
    pd.DataFrame(dict(src=z["csv_src"], dst=z["csv_dst"], time=z["csv_time"],
                      ext_roll=z["csv_ext_roll"])).to_csv(csv)
    for prefix, rev in (("ext_", False), ("rev_", True)):
        g = dataio.build_ext_full_device(csv, cuda, add_reverse=rev)
        for k in ("indptr", "indices", "ts", "eid"):
            assert g[k].is_cuda
            got = g[k].cpu().numpy()
            assert got.dtype == z[prefix + k].dtype, (prefix, k)
            assert np.array_equal(got, z[prefix + k]), (prefix, k)


def test_device_csr_and_loader_on_a_synthetic_graph(cuda, tmp_path):
    from fast_b200.data import WorkloadConfig, make_graph
    from fast_b200.capi import CSampler
    from oracle.sampler import OracleSampler
    cfg = WorkloadConfig("ld", 500, 60000, ("zipf", 1.1), ("uniform",), 3e4, True, 0, 8, "normal", "TGAT",
                         "recent", (5,), 64)
    g = make_graph(cfg, seed=8)                 # integer timestamps: many ties inside lists
    d = str(tmp_path / "LD")
    dataio.write_dataset(g, d)
    host = dataio.build_ext_full(os.path.join(d, "edges.csv"))
    dev = dataio.build_ext_full_device(os.path.join(d, "edges.csv"), cuda)
    for k in ("indptr", "indices", "ts", "eid"):
        assert np.array_equal(dev[k].cpu().numpy(), host[k]), k
    hg, dg = dataio.load_graph(d), dataio.load_graph(d, device=cuda)
    for k in ("src", "dst", "ts", "indptr", "indices", "eid", "ts_csr"):
        a = getattr(dg, k)
        assert a.is_cuda and np.array_equal(a.cpu().numpy(), getattr(hg, k)), k
    assert (dg.n_nodes, dg.train_end, dg.val_end) == (hg.n_nodes, hg.train_end, hg.val_end)
    s = CSampler(dg.indptr.cpu().numpy(), dg.indices.cpu().numpy(), dg.eid.cpu().numpy(), dg.ts_csr.cpu().numpy(),
                 2, [5, 5], True)
    o = OracleSampler(hg.indptr, hg.indices, hg.eid, hg.ts_csr, 1, 1, 2, [5, 5], True, False, 1, 0.0)
    b0 = 40000
    roots = np.concatenate([hg.src[b0:b0 + 100], hg.dst[b0:b0 + 100]]).astype(np.int32)
    rts = np.concatenate([hg.ts[b0:b0 + 100]] * 2).astype(np.float32)
    s.sample(roots, rts)
    o.sample(roots, rts)
    for i, ob in enumerate(o.get_ret()):
        d_ = s.block_arrays(i)
        for k in ("row", "col", "eid", "ts", "dts", "nodes"):
            np.testing.assert_array_equal(d_[k], getattr(ob, k)(), err_msg="block %d %s" % (i, k))
