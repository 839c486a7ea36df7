"""GPU: the device sampler (through the C ABI and the sampler_core drop-in)
against the CPU oracle, which tests/test_oracle_sampler.py pins to the
reference.  Recent sampling must match bit for bit, including the stateful
time pointers across batches; uniform sampling must match in distribution.
"""
import os

import numpy as np
import pytest

from conftest import small_graph
from oracle.sampler import OracleSampler

pytestmark = pytest.mark.gpu
FIELDS = ["row", "col", "eid", "ts", "dts", "nodes", "cntE", "uniE", "invE"]
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "sampler_golden.npz")


def _check_block(dev, ob, where):
    for k in FIELDS:
        np.testing.assert_array_equal(dev[k], getattr(ob, k)(), err_msg="%s %s" % (where, k))
    assert dev["dim_in"] == ob.dim_in() and dev["dim_out"] == ob.dim_out(), where
    # rptr over every root agrees with the row ids
    row, rptr = dev["row"], dev["rptr"]
    assert rptr[0] == 0 and rptr[-1] == row.size
    counts = np.bincount(row, minlength=dev["dim_out"]) if row.size else np.zeros(dev["dim_out"], np.int64)
    np.testing.assert_array_equal(np.diff(rptr), counts, err_msg=where + " rptr")


@pytest.mark.parametrize("layers,neigh", [(1, [10]), (2, [10, 10]), (2, [3, 40])])
def test_recent_bit_exact(cuda, layers, neigh):
    from fast_b200.capi import CSampler
    g = small_graph(n_nodes=150, n_edges=12000, seed=7, empty_nodes=(3, 4), zipf=1.1, int_ts=False, t_max=1e7)
    dev = CSampler(g["indptr"], g["indices"], g["eid"], g["ts"], layers, neigh, True)
    ora = OracleSampler(g["indptr"], g["indices"], g["eid"], g["ts"], 1, 1, layers, neigh, True, False, 1, 0.0)
    rng = np.random.default_rng(1)
    for bt in range(8):
        R = int(rng.integers(1, 400))
        roots = rng.integers(0, 150, R).astype(np.int32)
        rts = (rng.random(R) * 1e6 + 1.2e6 * bt).astype(np.float32)
        dev.sample(roots, rts)
        ora.sample(roots, rts)
        for i, ob in enumerate(ora.get_ret()):
            _check_block(dev.block_arrays(i), ob, "batch %d block %d" % (bt, i))
        if bt == 4:
            dev.reset()
            ora.reset()


def test_golden_vectors_device(cuda):
    """The device sampler reproduces the reference's own outputs (recent cases)."""
    from fast_b200.capi import CSampler
    gold = np.load(GOLDEN)
    cases = sorted({k.split("/")[0] for k in gold.files})
    for case in cases:
        g = {k.split("/", 1)[1]: gold[k] for k in gold.files if k.startswith(case + "/")}
        layers, recent, nh, wd = (int(g["params"][0]), bool(g["params"][1]), int(g["params"][2]),
                                  float(g["params"][3]))
        if not recent:
            continue
        s = CSampler(g["indptr"], g["indices"], g["eid"], g["ts"], layers, list(g["neighbors"]), True, False, nh, wd)
        for bt in range(int(g["n_batches"][0])):
            s.sample(g["roots_%d" % bt], g["rts_%d" % bt])
            for i in range(s.nblocks):
                d = s.block_arrays(i)
                for k in FIELDS:
                    np.testing.assert_array_equal(d[k], g["b%d_%d_%s" % (bt, i, k)],
                                                  err_msg="%s batch %d block %d %s" % (case, bt, i, k))


def test_dropin_module_matches_oracle(cuda):
    """The pybind drop-in (`sampler_core`) with numpy in / numpy out."""
    from fast_b200.ext import sampler_core
    g = small_graph(n_nodes=90, n_edges=7000, seed=9)
    a = sampler_core.ParallelSampler(g["indptr"], g["indices"], g["eid"], g["ts"], 8, 1, 2, [10, 10], True, False,
                                     1, 0.0)
    b = OracleSampler(g["indptr"], g["indices"], g["eid"], g["ts"], 8, 1, 2, [10, 10], True, False, 1, 0.0)
    rng = np.random.default_rng(4)
    for bt in range(5):
        roots = rng.integers(0, 90, 300).astype(np.int32)
        rts = np.full(300, 120.0 * (bt + 1), np.float32)
        a.configOMP(8, 3, [])
        a.sample(roots, rts, [1, 1, 1])
        b.sample(roots, rts)
        for ra, rb in zip(a.get_ret(), b.get_ret()):
            for k in FIELDS:
                np.testing.assert_array_equal(getattr(ra, k)(), getattr(rb, k)(), err_msg=k)
            assert ra.dim_in() == rb.dim_in() and ra.dim_out() == rb.dim_out()


def test_empty_and_invalid_roots(cuda):
    from fast_b200.capi import CSampler, FastB200Error
    g = small_graph(n_nodes=20, n_edges=500, seed=2)
    s = CSampler(g["indptr"], g["indices"], g["eid"], g["ts"], 2, [5, 5], True)
    s.sample(np.zeros(0, np.int32), np.zeros(0, np.float32))
    d = s.dims()
    assert (d[:, :4] == 0).all()
    s.sample(np.array([0, 25, 1], np.int32), np.array([10, 10, 10], np.float32))
    with pytest.raises(FastB200Error):
        s.dims()
    s.sample(np.array([0, 1], np.int32), np.array([900, 900], np.float32))
    assert s.dims()[0, 0] == 2


def _chi2(counts):
    counts = np.asarray(counts, np.float64)
    exp = counts.sum() / counts.size
    return ((counts - exp) ** 2 / exp).sum(), counts.size - 1


def test_uniform_distribution(cuda):
    """Per-root chi-square: picks are uniform over the time-valid window, and
    the device histogram matches the reference's (oracle, 1 thread)."""
    from fast_b200.capi import CSampler
    from scipy.stats import chi2 as chi2d
    n_e = 50
    indptr = np.array([0, n_e, n_e], np.int32)
    indices = np.ones(n_e, np.int32)
    eid = np.arange(n_e, dtype=np.int32)
    ts = np.arange(1, n_e + 1, dtype=np.float32)
    R, K = 4000, 10
    dev = CSampler(indptr, indices, eid, ts, 1, [K], False, seed=99)
    ora = OracleSampler(indptr, indices, eid, ts, 1, 1, 1, [K], False, False, 1, 0.0)
    for t_root, n_bins in ((60.0, 50), (30.5, 30)):
        roots = np.zeros(R, np.int32)
        rts = np.full(R, t_root, np.float32)
        if t_root < 60:
            # advance the pointer first so the window still spans all 50 edges
            dev.sample(np.zeros(1, np.int32), np.full(1, 60.0, np.float32))
            ora.sample(np.zeros(1, np.int32), np.full(1, 60.0, np.float32))
        dev.sample(roots, rts)
        ora.sample(roots, rts)
        d = dev.block_arrays(0, dedup=False)
        o = ora.get_ret()[0]
        hd = np.bincount(d["eid"], minlength=n_e)[:n_bins]
        ho = np.bincount(o.eid(), minlength=n_e)[:n_bins]
        assert d["eid"].max() < n_bins and o.eid().max() < n_bins       # rejection of ts >= root ts
        # keep rate: every draw survives with probability n_bins / 50
        exp_kept = R * K * n_bins / n_e
        assert abs(d["eid"].size - exp_kept) < 6 * np.sqrt(exp_kept)
        for h in (hd, ho):
            stat, dof = _chi2(h)
            assert chi2d.sf(stat, dof) > 1e-4, (t_root, stat, dof)
        # two-sample test between the device and reference histograms
        tab = np.vstack([hd, ho]).astype(np.float64)
        exp = tab.sum(1, keepdims=True) * tab.sum(0, keepdims=True) / tab.sum()
        stat = ((tab - exp) ** 2 / exp).sum()
        assert chi2d.sf(stat, n_bins - 1) > 1e-4


def test_full_size_recent_config2_graph(cuda):
    """Config-2-sized graph (1.14 M nodes, 7.83 M edges): two chronological
    batches of 1,800 roots, 2-hop recent 10x10, bit-exact against the oracle."""
    from fast_b200.data import CONFIGS, make_graph
    from fast_b200.capi import CSampler
    g = make_graph(CONFIGS[2])
    dev = CSampler(g.indptr, g.indices, g.eid, g.ts_csr, 2, [10, 10], True)
    ora = OracleSampler(g.indptr, g.indices, g.eid, g.ts_csr, 1, 1, 2, [10, 10], True, False, 1, 0.0)
    rng = np.random.default_rng(0)
    for b0 in (1_000_000, 4_000_000):
        src, dst, t = g.src[b0:b0 + 600], g.dst[b0:b0 + 600], g.ts[b0:b0 + 600]
        roots = np.concatenate([src, dst, rng.integers(0, g.n_nodes, 600).astype(np.int32)])
        rts = np.concatenate([t, t, t]).astype(np.float32)
        dev.sample(roots, rts)
        ora.sample(roots, rts)
        for i, ob in enumerate(ora.get_ret()):
            _check_block(dev.block_arrays(i), ob, "b0 %d block %d" % (b0, i))
