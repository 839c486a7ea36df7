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


def _per_root_picks(d):
    """eid, ts and dts of every root's picks, from a block's arrays."""
    rp = d["rptr"]
    R = d["dim_out"]
    return [(d["eid"][rp[j]:rp[j + 1]], d["ts"][R + rp[j]:R + rp[j + 1]], d["dts"][R + rp[j]:R + rp[j + 1]])
            for j in range(R)]


def _shard_index(world, r, B):
    """Positions of rank r's roots [src_r | dst_r | neg_r] in the global list [src | dst | neg]."""
    per = B // world
    return np.concatenate([s * B + r * per + np.arange(per) for s in range(3)])


@pytest.mark.parametrize("world,neigh", [(2, [10, 10]), (3, [4, 6]), (2, [5, 5, 5])])
def test_shard_sampling_equals_global(cuda, world, neigh):
    """Data-parallel sampling (fb_sampler_sample_shard), `world` ranks emulated
    by one sampler each on this GPU: over chronological batches, every rank's
    blocks of every layer hold, root by root, exactly the picks (eid, ts, dts)
    one sampler of the global batch makes (sampler_core.cpp:133-157, :700-710:
    every recent layer advances the shared pointers with the global batch's
    roots of that layer).  Also checks that advancing the pointers with the
    global roots of layer 0 alone (the earlier scheme) misses that: some
    deeper picks then differ."""
    import torch
    from fast_b200.capi import CSampler, check, lib, stream_ptr
    g = small_graph(n_nodes=120, n_edges=30000, seed=11, zipf=1.1, int_ts=False, t_max=1e6)
    L = len(neigh)
    args = (g["indptr"], g["indices"], g["eid"], g["ts"], L, neigh, True)
    glob = CSampler(*args)
    ranks = [CSampler(*args) for _ in range(world)]
    old = [CSampler(*args) for _ in range(world)]          # layer-0 global update only
    B = 30 * world
    rng = np.random.default_rng(5)
    differs = 0
    for bt in range(6):
        b0 = 8000 + 2500 * bt
        t = g["t"][b0:b0 + B]
        groots = np.concatenate([g["src"][b0:b0 + B], g["dst"][b0:b0 + B],
                                 rng.integers(0, 120, B).astype(np.int32)])
        gts = np.concatenate([t, t, t]).astype(np.float32)
        glob.sample(groots, gts)
        gl = [_per_root_picks(glob.block_arrays(i, dedup=False)) for i in range(L)]
        gdim = [glob.dims()[i][0] for i in range(L)]
        d_groots, d_gts = torch.from_numpy(groots).cuda(), torch.from_numpy(gts).cuda()
        for r in range(world):
            sel = _shard_index(world, r, B)
            dr = torch.from_numpy(groots[sel]).cuda()
            dt = torch.from_numpy(gts[sel]).cuda()
            ranks[r].sample_shard(dr, dt, d_groots, d_gts)
            check(lib.fb_sampler_update_pointers(old[r].h, d_groots.data_ptr(), d_gts.data_ptr(), 3 * B,
                                                 stream_ptr()))
            old[r].sample(groots[sel], gts[sel])
            gmap = sel                                   # local root -> global root of layer 0
            for l in range(L):
                loc = ranks[r].block_arrays(l, dedup=False)
                lp = _per_root_picks(loc)
                assert len(lp) == len(gmap)
                for j, gj in enumerate(gmap):
                    for a, b in zip(lp[j], gl[l][gj]):
                        np.testing.assert_array_equal(a, b, err_msg="batch %d rank %d layer %d root %d"
                                                      % (bt, r, l, j))
                ol = _per_root_picks(old[r].block_arrays(l, dedup=False))
                differs += sum(not np.array_equal(ol[j][0], gl[l][gj][0]) for j, gj in enumerate(gmap))
                # next layer's roots: this layer's nodes (roots, then each root's picks in order)
                grp = glob.block_arrays(l, dedup=False)["rptr"]
                nxt = list(gmap)
                for j, gj in enumerate(gmap):
                    nxt += [gdim[l] + grp[gj] + i for i in range(len(lp[j][0]))]
                gmap = np.array(nxt, np.int64)
    assert differs > 0


def _advance_pointers(ptr, indptr, ts, roots, rts):
    """update_ts_ptr (sampler_core.cpp:133-157) in numpy: ptr[n] becomes the
    last edge of n with ts <= root_ts - 1e-7f (fp32), never moving back."""
    thr = (rts.astype(np.float32) - np.float32(1e-7)).astype(np.float32)
    for n, t in zip(roots, thr):
        b, e = indptr[n], indptr[n + 1]
        ub = b + int(np.searchsorted(ts[b:e], t, side="right"))
        if ub > b:
            ptr[n] = max(ptr[n], ub - 1)


def _window_upper_bound(indptr, ts, n, t):
    """The window of a layer that samples without the pointers, num_history 1
    (sampler_core.cpp:531-538): [indptr[n], max(upper_bound(t) - 1, indptr[n])]."""
    b, e = indptr[n], indptr[n + 1]
    ub = b + int(np.searchsorted(ts[b:e], np.float32(t), side="right"))
    return b, max(ub - 1, b)


def _recent_picks(ts, s, e, K, t):
    """The recent-k picks of window [s, e] (sampler_core.cpp:555-565): k from e
    down to max(s, e - K) + 1 (exclusive), kept when ts[k] < t - 1e-7f."""
    thr = np.float32(np.float32(t) - np.float32(1e-7))
    return [k for k in range(e, max(s, e - K), -1) if ts[k] < thr]


def test_uniform_two_layer_windows_config2(cuda):
    """Uniform 10x10 on the config-2 graph, structural pin of both layers over
    chronological batches: every device pick lies in its root's window (layer
    0: [indptr, time pointer]; layer 1: the upper_bound window,
    sampler_core.cpp:700-706, :522-552); roots with a window narrower than the
    fan-out give the recent picks bit for bit (:555); every pick has
    ts < root_ts; the kept counts and the picks' positions among each root's
    time-valid edges are uniform (pooled chi-square over wide-window roots).
    The numpy windows are checked against the C oracle in recent mode first."""
    from scipy.stats import chi2 as chi2d
    from fast_b200.capi import CSampler
    from fast_b200.data import CONFIGS, make_graph
    g = make_graph(CONFIGS[2])
    K = 10
    indptr, ts, indices = g.indptr, g.ts_csr, g.indices
    pos_of_eid = np.empty_like(g.eid)
    pos_of_eid[g.eid] = np.arange(g.eid.size, dtype=np.int32)
    dev = CSampler(indptr, indices, g.eid, ts, 2, [K, K], False, seed=2024)
    ora = OracleSampler(indptr, indices, g.eid, ts, 1, 1, 1, [K], True, False, 1, 0.0)
    ptr = indptr[:-1].astype(np.int64).copy()
    rng = np.random.default_rng(3)
    u_hist, u_exp = np.zeros(20), np.zeros(20)
    kept = exp_kept = var_kept = 0.0
    n_fallback = 0
    for b0 in (2_000_000, 3_500_000, 5_000_000):
        src, dst, t = g.src[b0:b0 + 600], g.dst[b0:b0 + 600], g.ts[b0:b0 + 600]
        roots = np.concatenate([src, dst, rng.integers(0, g.n_nodes, 600).astype(np.int32)])
        rts = np.concatenate([t, t, t]).astype(np.float32)
        _advance_pointers(ptr, indptr, ts, roots, rts)
        # the numpy windows of layer 0 against the oracle's recent picks
        ora.sample(roots, rts)
        ob = ora.get_ret()[0]
        orp = np.concatenate([[0], np.cumsum(np.bincount(ob.row(), minlength=roots.size))])
        for j in range(roots.size):
            want = _recent_picks(ts, indptr[roots[j]], ptr[roots[j]], K, rts[j])
            np.testing.assert_array_equal(pos_of_eid[ob.eid()[orp[j]:orp[j + 1]]], want, err_msg="oracle root %d" % j)
        dev.sample(roots, rts)
        layer_roots = (roots, rts)
        for layer in range(2):
            d = dev.block_arrays(layer, dedup=False)
            R = d["dim_out"]
            lr, lt = layer_roots
            assert R == lr.size
            np.testing.assert_array_equal(d["nodes"][:R], lr)
            rp = d["rptr"]
            for j in range(R):
                n, tj = int(lr[j]), np.float32(lt[j])
                s, e = (indptr[n], int(ptr[n])) if layer == 0 else _window_upper_bound(indptr, ts, n, tj)
                ks = pos_of_eid[d["eid"][rp[j]:rp[j + 1]]]
                where = "batch %d layer %d root %d" % (b0, layer, j)
                assert ks.size <= K, where
                np.testing.assert_array_equal(indices[ks], d["nodes"][R + rp[j]:R + rp[j + 1]], err_msg=where)
                np.testing.assert_array_equal(ts[ks], d["ts"][R + rp[j]:R + rp[j + 1]], err_msg=where)
                thr = np.float32(tj - np.float32(1e-7))
                assert (ts[ks] < thr).all(), where
                if e - s < K:
                    n_fallback += 1
                    np.testing.assert_array_equal(ks, _recent_picks(ts, s, e, K, tj), err_msg=where)
                    continue
                assert ((ks >= s) & (ks <= e)).all(), where
                valid = np.nonzero(ts[s:e + 1] < thr)[0] + s
                p = valid.size / (e - s + 1)
                kept += ks.size
                exp_kept += K * p
                var_kept += K * p * (1 - p)
                if valid.size >= 20:
                    # each kept pick's rank among the valid edges, in 20 bins; the
                    # expected count of a bin is its share of the valid edges
                    bins = (np.arange(valid.size) * 20) // valid.size
                    u_hist += np.bincount(bins[np.searchsorted(valid, ks)], minlength=20)
                    u_exp += ks.size * np.bincount(bins, minlength=20) / valid.size
            layer_roots = (d["nodes"], d["ts"])
    assert n_fallback > 0
    assert abs(kept - exp_kept) < 6 * np.sqrt(var_kept) + 1, (kept, exp_kept)
    stat = ((u_hist - u_exp) ** 2 / u_exp).sum()
    assert u_hist.sum() > 2000 and chi2d.sf(stat, 19) > 1e-4, (stat, u_hist, u_exp)


def test_uniform_per_root_chi2_hub(cuda):
    """Per-root chi-square on the config-2 graph: the highest-degree node as
    2,000 roots at one time, 10 draws each.  Its kept picks are uniform over
    the time-valid edges of its window [indptr, time pointer], and the kept
    count is the draws times the valid share of the window."""
    from scipy.stats import chi2 as chi2d
    from fast_b200.capi import CSampler
    from fast_b200.data import CONFIGS, make_graph
    g = make_graph(CONFIGS[2])
    deg = np.diff(g.indptr)
    hub = int(np.argmax(deg))
    b, e_all = g.indptr[hub], g.indptr[hub + 1]
    t_root = np.float32(g.ts_csr[b + (e_all - b) * 3 // 4])
    pos_of_eid = np.empty_like(g.eid)
    pos_of_eid[g.eid] = np.arange(g.eid.size, dtype=np.int32)
    dev = CSampler(g.indptr, g.indices, g.eid, g.ts_csr, 1, [10], False, seed=7)
    R, K = 2000, 10
    dev.sample(np.full(R, hub, np.int32), np.full(R, t_root, np.float32))
    ks = pos_of_eid[dev.block_arrays(0, dedup=False)["eid"]]
    ptr = g.indptr[:-1].astype(np.int64).copy()
    _advance_pointers(ptr, g.indptr, g.ts_csr, np.array([hub]), np.array([t_root], np.float32))
    s, e = b, int(ptr[hub])
    assert e - s >= K
    valid = np.nonzero(g.ts_csr[s:e + 1] < np.float32(t_root - np.float32(1e-7)))[0] + s
    assert ((ks >= s) & (ks <= e)).all() and np.isin(ks, valid).all()
    p = valid.size / (e - s + 1)
    assert abs(ks.size - R * K * p) < 6 * np.sqrt(R * K * p * (1 - p)) + 1
    nb = min(40, valid.size)
    bins = (np.arange(valid.size) * nb) // valid.size
    h = np.bincount(bins[np.searchsorted(valid, ks)], minlength=nb)
    exp = ks.size * np.bincount(bins, minlength=nb) / valid.size
    stat = ((h - exp) ** 2 / exp).sum()
    assert chi2d.sf(stat, nb - 1) > 1e-4, (stat, h)
