"""Writes tests/golden/loader_golden.npz by running the REFERENCE preprocessing
scripts on a small synthetic raw edge list.

Run in the build container, where the reference tree is readable:

    python tests/golden/make_loader_golden.py

The raw list has sparse node ids (so txt2csv's reindexing matters), hub nodes
with dozens of edges and integer times from a narrow range (so both
sort_values and gen_graph's per-node np.argsort meet many equal keys).  The
reference's fast_util/preprocess/txt2csv.py and gen_graph.py (with and
without --add_reverse) run unmodified in a temporary DATA directory; the
fixture keeps the raw list and their outputs.
"""
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle.paths import REF_ROOT as REF  # noqa: E402


def raw_edges(seed=5, n=3000):
    rng = np.random.default_rng(seed)
    ids = rng.choice(100000, 180, replace=False) * 7 + 3          # sparse ids
    w = np.arange(1, 181, dtype=np.float64) ** -1.1
    src = ids[rng.choice(180, n, p=w / w.sum())]
    dst = ids[rng.integers(0, 180, n)]
    t = rng.integers(1_000_000, 1_000_300, n)                      # many equal times
    return src.astype(np.int64), dst.astype(np.int64), t.astype(np.int64)


def main():
    if not os.path.isdir(REF):
        raise SystemExit("reference tree not found")
    src, dst, t = raw_edges()
    out = dict(raw_src=src, raw_dst=dst, raw_t=t)
    with tempfile.TemporaryDirectory() as tmp:
        d = os.path.join(tmp, "DATA", "SYN")
        os.makedirs(d)
        txt = os.path.join(d, "syn.edges")
        with open(txt, "w") as f:
            f.write("% header line\n")
            for a, b, c in zip(src, dst, t):
                f.write("%d %d %d\n" % (a, b, c))
        pre = os.path.join(REF, "fast_util", "preprocess")
        run = lambda *a: subprocess.run([sys.executable] + list(a), cwd=tmp, check=True,  # noqa: E731
                                        stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        run(os.path.join(pre, "txt2csv.py"), "--data", "SYN", "--txt", txt)
        import pandas as pd
        df = pd.read_csv(os.path.join(d, "edges.csv"))
        for c in ("src", "dst", "time", "ext_roll"):
            out["csv_" + c] = df[c].values
        run(os.path.join(pre, "gen_graph.py"), "--data", "SYN")
        g = np.load(os.path.join(d, "ext_full.npz"))
        for k in ("indptr", "indices", "ts", "eid"):
            out["ext_" + k] = g[k]
        run(os.path.join(pre, "gen_graph.py"), "--data", "SYN", "--add_reverse")
        g = np.load(os.path.join(d, "ext_full.npz"))
        for k in ("indptr", "indices", "ts", "eid"):
            out["rev_" + k] = g[k]
    path = os.path.join(HERE, "loader_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, len(out), "arrays")


if __name__ == "__main__":
    main()
