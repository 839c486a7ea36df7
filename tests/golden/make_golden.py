"""Writes tests/golden/sampler_golden.npz from the REFERENCE sampler.

Run in the build container, where the reference sampler has been compiled
from its own source into oracle/_ref (``make -C oracle ref``):

    python tests/golden/make_golden.py

Each case stores the graph, the sampler parameters, the batches of roots and
every output array of every block the reference returned.  Every case uses
one reference thread: with more, the reference appends uniE in the order its
threads finish (sampler_core.cpp:300-304) and uniform draws follow per-thread
rand_r streams; the one-thread order is the deterministic one the oracle and
the device sampler reproduce.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

from conftest import small_graph  # noqa: E402
from oracle.sampler import load_reference  # noqa: E402

FIELDS = ["row", "col", "eid", "ts", "dts", "nodes", "cntE", "uniE", "invE"]


def hand_graph():
    indptr = np.array([0, 12, 15, 15], np.int32)
    indices = np.array([1] * 12 + [0, 0, 0], np.int32)
    eid = np.arange(15, dtype=np.int32)
    ts = np.array(list(range(1, 13)) + [5, 6, 7], np.float32)
    return dict(indptr=indptr, indices=indices, eid=eid, ts=ts)


def run_case(ref, out, name, g, layers, neigh, recent, nh, wd, batches, threads):
    s = ref.ParallelSampler(g["indptr"], g["indices"], g["eid"], g["ts"], threads, 1, layers, neigh, recent, False,
                            nh, wd)
    out[name + "/indptr"] = g["indptr"]
    out[name + "/indices"] = g["indices"]
    out[name + "/eid"] = g["eid"]
    out[name + "/ts"] = g["ts"]
    out[name + "/params"] = np.array([layers, int(recent), nh, wd], np.float64)
    out[name + "/neighbors"] = np.array(neigh, np.int32)
    out[name + "/n_batches"] = np.array([len(batches)], np.int32)
    for bt, (roots, rts) in enumerate(batches):
        out[name + "/roots_%d" % bt] = roots
        out[name + "/rts_%d" % bt] = rts
        s.sample(roots, rts, [])
        for i, blk in enumerate(s.get_ret()):
            for k in FIELDS:
                out[name + "/b%d_%d_%s" % (bt, i, k)] = getattr(blk, k)()


def main():
    ref = load_reference()
    if ref is None:
        raise SystemExit("build the reference sampler first: make -C oracle ref")
    out = {}
    rng = np.random.default_rng(2024)
    h = hand_graph()
    run_case(ref, out, "hand_recent", h, 1, [3], True, 1, 0.0,
             [(np.array([0, 1], np.int32), np.array([13, 13], np.float32)),
              (np.array([0, 0, 1, 2], np.int32), np.array([13, 4, 13, 5], np.float32))], 1)
    g1 = small_graph(n_nodes=50, n_edges=3000, seed=1, zipf=1.1)
    b1 = [(rng.integers(0, 50, 60).astype(np.int32), np.full(60, 150.0 * (i + 1), np.float32)) for i in range(5)]
    run_case(ref, out, "recent_1layer", g1, 1, [10], True, 1, 0.0, b1, 1)
    g2 = small_graph(n_nodes=120, n_edges=5000, seed=2, int_ts=False, t_max=2e8)
    b2 = [(rng.integers(0, 120, 45).astype(np.int32), np.full(45, 4e7 * (i + 1), np.float32)) for i in range(4)]
    run_case(ref, out, "recent_2layer", g2, 2, [10, 10], True, 1, 0.0, b2, 1)
    b3 = [(rng.integers(0, 120, 45).astype(np.int32), np.full(45, 4e7 * (i + 1), np.float32)) for i in range(3)]
    run_case(ref, out, "uniform_2layer_1thread", g2, 2, [5, 5], False, 1, 0.0, b3, 1)
    g4 = small_graph(n_nodes=30, n_edges=800, seed=4, empty_nodes=(0, 7, 8), t_max=500)
    roots = np.array([0, 7, 8, 1, 1, 1, 2, 3, 29, 3], np.int32)
    rts = np.array([100, 400, 100, 0, 250, 499, 1, 600, 300, 2], np.float32)   # before/after all edges, dups
    run_case(ref, out, "edge_cases", g4, 2, [4, 40], True, 1, 0.0, [(roots, rts), (roots[::-1].copy(), rts + 1)], 1)
    g5 = small_graph(n_nodes=40, n_edges=3000, seed=5, t_max=2000)
    b5 = [(rng.integers(0, 40, 50).astype(np.int32), np.full(50, 300.0 * (i + 1), np.float32)) for i in range(4)]
    run_case(ref, out, "history3_window", g5, 2, [5, 3], True, 3, 150.0, b5, 1)
    path = os.path.join(HERE, "sampler_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, len(out), "arrays")


if __name__ == "__main__":
    main()
