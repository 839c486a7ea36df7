"""On-disk dataset format of the reference, read straight into the training
graph (and written, for data prepared here).

The reference prepares a dataset in two steps and loads it with
utils.py:54-57 (load_graph):
  fast_util/preprocess/txt2csv.py   raw "src dst time" edge list -> DATA/<d>/edges.csv
  fast_util/preprocess/gen_graph.py edges.csv -> DATA/<d>/ext_full.npz (CSR)
and train.py:99-100 takes the train / validation ends from the ext_roll
column.  This module restates both steps and the load:

  txt_to_edges_csv    ids reindexed densely in sorted order, times shifted to
                      start at 0, rows ordered by time with the same pandas
                      call, ext_roll 0/1/2 for the 70/15/15 chronological split
  build_ext_full      CSR keyed by src (optionally with reverse edges), each
                      node's list ordered by np.argsort of its timestamps
  load_graph          edges.csv + ext_full.npz -> data.TemporalGraph

Ordering of equal timestamps: gen_graph sorts every node's list with
np.argsort's default kind, which is not stable (and for float32 may run a
SIMD sort).  build_ext_full sorts all lists at once with a stable sort --
the same order wherever a node's timestamps are distinct -- and calls
np.argsort on exactly the lists that hold ties, so the result is the
reference's on the same NumPy build.
"""
import os

import numpy as np

from .data import TemporalGraph


def txt_to_edges_csv(txt_path, csv_path):
    """txt2csv.py: the first line is a header and is skipped; columns src,
    dst, time; ids reindexed by np.unique over [src | dst]; time made integer
    and shifted to start at 0; rows sorted by time (pandas sort_values, its
    default quicksort); ext_roll = 0 / 1 / 2 at 70% / 85%."""
    import pandas as pd
    with open(txt_path) as f:
        rows = [line.split() for line in f.readlines()]
    df = pd.DataFrame(rows[1:])
    df.columns = ["src", "dst", "time"]
    src = df.src.astype(int)
    dst = df.dst.astype(int)
    cut = len(src)
    total, inv = np.unique(np.concatenate((src, dst)), return_inverse=True)
    new = np.arange(len(total))
    df["src"] = new[inv][:cut]
    df["dst"] = new[inv][cut:]
    df.time = df.time.astype(int)
    df.time -= df.time.min()
    df = df.sort_values(by=["time"])
    df = df.reset_index(drop=True)
    roll = np.zeros(len(df), dtype=int)
    roll[int(0.7 * len(df)):int(0.85 * len(df))] = 1
    roll[int(0.85 * len(df)):] = 2
    df["ext_roll"] = roll
    df.to_csv(csv_path)
    return df


def build_ext_full(csv_path, npz_path=None, add_reverse=False):
    """gen_graph.py: returns (and with npz_path saves) indptr, indices, ts,
    eid of the CSR keyed by src (and dst with add_reverse), every node's
    list ordered by np.argsort of its timestamps."""
    import pandas as pd
    df = pd.read_csv(csv_path)
    src = df["src"].values.astype(np.int32)
    dst = df["dst"].values.astype(np.int32)
    t = df["time"].values.astype(np.float32)
    idx = np.arange(len(df), dtype=np.int32)
    num_nodes = max(int(df["src"].max()), int(df["dst"].max())) + 1
    if add_reverse:
        # per edge in order: the src list gets (dst, t, idx), then the dst list (src, t, idx)
        key = np.stack([src, dst], 1).reshape(-1)
        nbr = np.stack([dst, src], 1).reshape(-1)
        tt = np.repeat(t, 2)
        ii = np.repeat(idx, 2)
    else:
        key, nbr, tt, ii = src, dst, t, idx
    # lists in insertion order (a stable sort on the node id), then by time
    order = np.argsort(key, kind="stable")
    key, nbr, tt, ii = key[order], nbr[order], tt[order], ii[order]
    indptr = np.zeros(num_nodes + 1, dtype=np.int64)
    np.add.at(indptr, key.astype(np.int64) + 1, 1)
    indptr = np.cumsum(indptr).astype(np.int32)
    by_time = np.lexsort((tt, key))            # stable within each node; key stays grouped
    out_nbr, out_t, out_i = nbr[by_time], tt[by_time], ii[by_time]
    # lists with equal timestamps: the reference's own np.argsort decides their order
    same = (key[1:] == key[:-1]) & (out_t[1:] == out_t[:-1])
    for n in np.unique(key[:-1][same]):
        b, e = int(indptr[n]), int(indptr[n + 1])
        s = np.argsort(tt[b:e])
        out_nbr[b:e], out_t[b:e], out_i[b:e] = nbr[b:e][s], tt[b:e][s], ii[b:e][s]
    res = dict(indptr=indptr, indices=out_nbr.astype(np.int32), ts=out_t.astype(np.float32),
               eid=out_i.astype(np.int32))
    if npz_path is not None:
        np.savez(npz_path, **res)
    return res


def build_ext_full_device(csv_path, device, add_reverse=False):
    """build_ext_full on the GPU: the same CSR (indptr, indices, ts, eid;
    gen_graph.py's contract), as device tensors, byte for byte.  The lists are
    grouped by node with a stable sort and ordered by time with a second
    stable sort, both on the device; a list holding equal timestamps takes
    the order of the reference's own np.argsort of its times (run on the host
    for those lists only, as build_ext_full does), since an unstable sort's
    order among ties is the one thing a device sort cannot reproduce."""
    import pandas as pd
    import torch
    df = pd.read_csv(csv_path)
    dev = torch.device(device)
    src = torch.from_numpy(df["src"].values.astype(np.int32)).to(dev)
    dst = torch.from_numpy(df["dst"].values.astype(np.int32)).to(dev)
    t = torch.from_numpy(df["time"].values.astype(np.float32)).to(dev)
    idx = torch.arange(len(df), dtype=torch.int32, device=dev)
    num_nodes = max(int(df["src"].max()), int(df["dst"].max())) + 1
    if add_reverse:
        key, nbr = torch.stack([src, dst], 1).reshape(-1), torch.stack([dst, src], 1).reshape(-1)
        tt, ii = t.repeat_interleave(2), idx.repeat_interleave(2)
    else:
        key, nbr, tt, ii = src, dst, t, idx
    _, order = torch.sort(key, stable=True)                  # insertion order within each node
    key, nbr, tt, ii = key[order], nbr[order], tt[order], ii[order]
    indptr = torch.zeros(num_nodes + 1, dtype=torch.int64, device=dev)
    indptr[1:] = torch.cumsum(torch.bincount(key.long(), minlength=num_nodes), 0)
    _, by_t = torch.sort(tt, stable=True)                      # lexsort((tt, key)): time, then node
    _, by_k = torch.sort(key[by_t], stable=True)
    by_time = by_t[by_k]
    out_nbr, out_t, out_i = nbr[by_time].clone(), tt[by_time].clone(), ii[by_time].clone()
    same = (key[1:] == key[:-1]) & (out_t[1:] == out_t[:-1])
    tie_nodes = torch.unique(key[:-1][same]).cpu().numpy()
    if tie_nodes.size:
        ip = indptr.cpu().numpy()
        for n in tie_nodes:
            b, e = int(ip[n]), int(ip[n + 1])
            s = torch.from_numpy(np.argsort(tt[b:e].cpu().numpy())).to(dev)
            out_nbr[b:e], out_t[b:e], out_i[b:e] = nbr[b:e][s], tt[b:e][s], ii[b:e][s]
    return dict(indptr=indptr.to(torch.int32), indices=out_nbr, ts=out_t, eid=out_i)


def load_graph(data_dir, device=None):
    """utils.py:54-57 + train.py:99-100: edges.csv and ext_full.npz of a
    dataset directory as a TemporalGraph (edge list in chronological order,
    CSR, train / validation ends from ext_roll).  With `device`, every array
    goes straight from the files into device memory (one copy each, nothing
    rebuilt on the host), as make_graph_device's graphs are."""
    import pandas as pd
    df = pd.read_csv(os.path.join(data_dir, "edges.csv"))
    g = np.load(os.path.join(data_dir, "ext_full.npz"))
    roll = df["ext_roll"].values
    n = len(df)
    train_end = int(np.argmax(roll > 0)) if (roll > 0).any() else n
    val_end = int(np.argmax(roll > 1)) if (roll > 1).any() else n
    arrays = dict(src=df["src"].values.astype(np.int32), dst=df["dst"].values.astype(np.int32),
                  ts=df["time"].values.astype(np.float32), indptr=g["indptr"].astype(np.int32),
                  indices=g["indices"].astype(np.int32), eid=g["eid"].astype(np.int32),
                  ts_csr=g["ts"].astype(np.float32))
    if device is not None:
        import torch
        arrays = {k: torch.from_numpy(v).to(torch.device(device)) for k, v in arrays.items()}
    return TemporalGraph(n_nodes=int(g["indptr"].shape[0] - 1), train_end=train_end, val_end=val_end, **arrays)


def write_dataset(graph, data_dir):
    """A TemporalGraph (e.g. the synthetic generators') in the reference's
    on-disk format: edges.csv with the ext_roll split, and ext_full.npz."""
    import pandas as pd
    os.makedirs(data_dir, exist_ok=True)
    E = len(graph.src)
    roll = np.zeros(E, dtype=int)
    roll[graph.train_end:graph.val_end] = 1
    roll[graph.val_end:] = 2
    pd.DataFrame(dict(src=graph.src, dst=graph.dst, time=graph.ts, ext_roll=roll)).to_csv(
        os.path.join(data_dir, "edges.csv"))
    build_ext_full(os.path.join(data_dir, "edges.csv"), os.path.join(data_dir, "ext_full.npz"))
