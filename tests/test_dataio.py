"""CPU: the on-disk dataset format (fast_b200/dataio.py) against the
reference's own preprocessing scripts, recorded by
tests/golden/make_loader_golden.py: txt2csv.py's edges.csv and gen_graph.py's
ext_full.npz (with and without --add_reverse) on a raw edge list with sparse
ids, hub nodes and many equal timestamps.  Bit-exact.  Then a round trip: a
synthetic graph written in that format loads back unchanged and samples the
same blocks."""
import os

import numpy as np

from fast_b200 import dataio

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "loader_golden.npz")


def test_txt_to_edges_csv_matches_reference(tmp_path):
    z = np.load(GOLDEN)
    txt = tmp_path / "syn.edges"
    with open(txt, "w") as f:
        f.write("% header line\n")
        for a, b, c in zip(z["raw_src"], z["raw_dst"], z["raw_t"]):
            f.write("%d %d %d\n" % (a, b, c))
    dataio.txt_to_edges_csv(str(txt), str(tmp_path / "edges.csv"))
    import pandas as pd
    df = pd.read_csv(tmp_path / "edges.csv")
    for c in ("src", "dst", "time", "ext_roll"):
        assert np.array_equal(df[c].values, z["csv_" + c]), c


def _golden_csv(z, path):
    import pandas as pd
    pd.DataFrame(dict(src=z["csv_src"], dst=z["csv_dst"], time=z["csv_time"], ext_roll=z["csv_ext_roll"])).to_csv(path)


def test_build_ext_full_matches_reference(tmp_path):
    z = np.load(GOLDEN)
    csv = str(tmp_path / "edges.csv")
    _golden_csv(z, csv)
    for prefix, rev in (("ext_", False), ("rev_", True)):
        g = dataio.build_ext_full(csv, add_reverse=rev)
        for k in ("indptr", "indices", "ts", "eid"):
            assert g[k].dtype == z[prefix + k].dtype, (prefix, k)
            assert np.array_equal(g[k], z[prefix + k]), (prefix, k)


def test_write_and_load_round_trip(tmp_path):
    from fast_b200.data import WorkloadConfig, make_graph
    # float timestamps: no ties, so the generator's stable order is the only order
    cfg = WorkloadConfig("rt", 300, 20000, ("zipf", 1.1), ("uniform",), 5e3, False, 0, 8, "normal", "TGAT",
                         "recent", (5,), 64)
    g = make_graph(cfg, seed=4)
    dataio.write_dataset(g, str(tmp_path / "RT"))
    h = dataio.load_graph(str(tmp_path / "RT"))
    for k in ("src", "dst", "ts", "indptr", "indices", "eid", "ts_csr"):
        assert np.array_equal(getattr(g, k), getattr(h, k)), k
    assert (h.n_nodes, h.train_end, h.val_end) == (g.n_nodes, g.train_end, g.val_end)
    # the oracle sampler draws the same blocks from both
    from oracle.sampler import OracleSampler
    roots = np.concatenate([g.src[15000:15050], g.dst[15000:15050]]).astype(np.int32)
    rts = np.concatenate([g.ts[15000:15050]] * 2).astype(np.float32)
    blocks = []
    for gr in (g, h):
        s = OracleSampler(gr.indptr, gr.indices, gr.eid, gr.ts_csr, 1, 1, 1, [5], True, False, 1, 0.0)
        s.sample(roots, rts)
        blocks.append(s.get_ret()[0])
    for k in ("row", "col", "eid", "ts", "dts", "nodes"):
        assert np.array_equal(getattr(blocks[0], k)(), getattr(blocks[1], k)()), k
