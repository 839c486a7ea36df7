"""CPU: the C restatement of the sampler (oracle/) pinned against the reference.

Two pins: (1) the golden vectors in tests/golden/sampler_golden.npz, written by
tests/golden/make_golden.py from the reference sampler compiled from its own
source; (2) when oracle/_ref holds that build, a live comparison on seeded
random graphs.  Recent sampling is thread-count independent in the
reference; uniform sampling matches it bit for bit with one reference thread.
"""
import os

import numpy as np
import pytest

from conftest import small_graph
from oracle.sampler import OracleSampler, load_reference

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "sampler_golden.npz")
FIELDS = ["row", "col", "eid", "ts", "dts", "nodes", "cntE", "uniE", "invE"]


def _compare(ra, rb, fields):
    for k in fields:
        a, b = getattr(ra, k)(), getattr(rb, k)()
        assert a.dtype == b.dtype or k in ("uniE", "invE"), k
        np.testing.assert_array_equal(a, b, err_msg=k)
    assert ra.dim_in() == rb.dim_in() and ra.dim_out() == rb.dim_out()


def test_golden_vectors():
    gold = np.load(GOLDEN, allow_pickle=False)
    cases = sorted({k.split("/")[0] for k in gold.files})
    assert len(cases) >= 6
    for case in cases:
        g = {k.split("/", 1)[1]: gold[k] for k in gold.files if k.startswith(case + "/")}
        p = g["params"]
        layers, recent, nh, wd = int(p[0]), bool(p[1]), int(p[2]), float(p[3])
        neigh = list(g["neighbors"])
        s = OracleSampler(g["indptr"], g["indices"], g["eid"], g["ts"], 1, 1, layers, neigh, recent, False, nh, wd)
        nb = int(g["n_batches"][0])
        for bt in range(nb):
            s.sample(g["roots_%d" % bt], g["rts_%d" % bt], [])
            for i, blk in enumerate(s.get_ret()):
                for k in FIELDS:
                    np.testing.assert_array_equal(getattr(blk, k)(), g["b%d_%d_%s" % (bt, i, k)],
                                                  err_msg="%s batch %d block %d %s" % (case, bt, i, k))


def test_hand_graph_truncated_window():
    """Node 0: 12 edges at ts 1..12; node 1: 3 edges at 5,6,7.  A root at ts 4
    sampled after a root at 13 in the same batch sees only edges below its own
    time inside the already-advanced window (sampler_core.cpp:133-157,555-566)."""
    indptr = np.array([0, 12, 15, 15], np.int32)
    indices = np.array([1] * 12 + [0, 0, 0], np.int32)
    eid = np.arange(15, dtype=np.int32)
    ts = np.array(list(range(1, 13)) + [5, 6, 7], np.float32)
    s = OracleSampler(indptr, indices, eid, ts, 1, 1, 1, [3], True, False, 1, 0.0)
    s.sample(np.array([0, 0, 1, 2], np.int32), np.array([13, 4, 13, 5], np.float32))
    b = s.get_ret()[0]
    np.testing.assert_array_equal(b.row(), [0, 0, 0, 2, 2])
    np.testing.assert_array_equal(b.eid(), [11, 10, 9, 14, 13])
    np.testing.assert_array_equal(b.cntE(), [0, 3, 5])


@pytest.mark.parametrize("recent", [True, False])
@pytest.mark.parametrize("threads", [1, 3])
def test_oracle_matches_reference_build(recent, threads):
    ref = load_reference()
    if ref is None:
        pytest.skip("reference sampler not built (make -C oracle ref)")
    if not recent and threads > 1:
        pytest.skip("uniform draws depend on the reference thread count; distribution-tested on GPU")
    g = small_graph(n_nodes=80, n_edges=6000, seed=3, empty_nodes=(5, 6), zipf=1.1)
    a = ref.ParallelSampler(g["indptr"], g["indices"], g["eid"], g["ts"], threads, 1, 2, [7, 4], recent, False, 1, 0.0)
    b = OracleSampler(g["indptr"], g["indices"], g["eid"], g["ts"], 1, 1, 2, [7, 4], recent, False, 1, 0.0)
    rng = np.random.default_rng(11)
    for bt in range(12):
        roots = rng.integers(0, 80, 90).astype(np.int32)
        rts = np.full(90, 80.0 * (bt + 1), np.float32)
        rts[::7] -= 50.0       # earlier duplicates of the same nodes inside a batch
        a.sample(roots, rts, [])
        b.sample(roots, rts, [])
        for ra, rb in zip(a.get_ret(), b.get_ret()):
            _compare(ra, rb, FIELDS if threads == 1 else FIELDS[:7])
        if bt == 5:
            a.reset()
            b.reset()


def test_oracle_history_window_matches_reference():
    ref = load_reference()
    if ref is None:
        pytest.skip("reference sampler not built")
    g = small_graph(n_nodes=40, n_edges=3000, seed=5, t_max=2000)
    a = ref.ParallelSampler(g["indptr"], g["indices"], g["eid"], g["ts"], 1, 1, 2, [5, 3], True, False, 3, 150.0)
    b = OracleSampler(g["indptr"], g["indices"], g["eid"], g["ts"], 1, 1, 2, [5, 3], True, False, 3, 150.0)
    rng = np.random.default_rng(2)
    for bt in range(6):
        roots = rng.integers(0, 40, 50).astype(np.int32)
        rts = np.full(50, 300.0 * (bt + 1), np.float32)
        a.sample(roots, rts, [])
        b.sample(roots, rts, [])
        for ra, rb in zip(a.get_ret(), b.get_ret()):
            _compare(ra, rb, FIELDS)
