"""Feature tables split between HBM and page-locked host memory: the B200 form
of the reference's slim feature cache (fast_util/slimCache.py:184-403).

The reference picks hot rows by pre-sampling (get_hot_cts: how often each node
and edge id appears in sampled batches), keeps them in a GPU table with an
id -> cache-slot map (init_cache, fresh_cache :184-259) and, per batch, copies
the other rows from the CPU table (trans2Device :261-403).  Here the full table
stays in page-locked host memory and the hot rows are copied once into a
device table; `gather` is one kernel (fb_gather_rows_tiered) that reads each
row from the device table when its id has a slot and from host memory
otherwise, with no host step in between.  For a workload whose tables fit in
HBM (every config here, config 5's bf16 edge table included) the trainers keep
them device-resident instead; this is for tables that do not.
"""
import ctypes

import numpy as np
import torch

from .capi import call, ptr, stream_ptr


def _p(t):
    return None if t is None else t.data_ptr()


def hot_ids_by_count(counts, capacity):
    """Ids of the `capacity` most frequent rows (ties: smaller id first), from
    per-id counts such as the reference's pre-sampling scores."""
    counts = np.asarray(counts)
    capacity = int(max(0, min(capacity, counts.shape[0])))
    order = np.lexsort((np.arange(counts.shape[0]), -counts.astype(np.int64)))
    return order[:capacity].astype(np.int64)


def count_ids(id_batches, n_rows):
    """How often each id appears in an iterable of id arrays (the reference's
    pre-sampling count, get_hot_cts)."""
    c = np.zeros(int(n_rows), dtype=np.int64)
    for ids in id_batches:
        ids = np.asarray(ids, dtype=np.int64).ravel()
        ids = ids[(ids >= 0) & (ids < n_rows)]
        c += np.bincount(ids, minlength=int(n_rows))
    return c


def slot_map(hot_ids, n_rows):
    """int32 [n_rows]: the device slot of each hot id, -1 for the others."""
    m = np.full(int(n_rows), -1, dtype=np.int32)
    hot = np.asarray(hot_ids, dtype=np.int64)
    if hot.size and (hot.min() < 0 or hot.max() >= n_rows or np.unique(hot).size != hot.size):
        raise ValueError("slot_map: hot ids must be distinct and inside the table")
    m[hot] = np.arange(hot.size, dtype=np.int32)
    return m


class TieredFeatureTable:
    """A [rows, d] fp32 or bf16 feature table: all rows in page-locked host
    memory, the hot ones also in HBM.

    table: CPU tensor (fp32 or bf16; copied into page-locked memory unless it
    is pinned already, so a table near the size of host memory should be
    allocated pinned from the start: torch.empty(rows, d, pin_memory=True)).
    hot_ids: row ids to place in HBM (e.g. hot_ids_by_count(count_ids(
    sampled_ids, rows), capacity)).
    """

    def __init__(self, table, hot_ids, device="cuda"):
        if table.device.type != "cpu" or table.dim() != 2 or table.dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("TieredFeatureTable: table must be a 2-D fp32 or bf16 CPU tensor")
        dev = torch.device(device)
        self.device = torch.device(dev.type, torch.cuda.current_device() if dev.index is None else dev.index)
        self.rows, self.d = table.shape
        self.dtype = table.dtype
        pinned = table.is_pinned() and table.is_contiguous()
        self.host = table if pinned else table.contiguous().pin_memory()
        dp = ctypes.c_void_p(0)
        call("fb_host_rows_device_pointer", ctypes.c_void_p(self.host.data_ptr()), ctypes.byref(dp))
        self._host_dev = dp.value
        hot = np.asarray(hot_ids, dtype=np.int64)
        self.slot_of = torch.from_numpy(slot_map(hot, self.rows)).to(self.device)
        self.dev = self.host[torch.from_numpy(hot)].to(self.device) if hot.size else \
            torch.empty(0, self.d, dtype=self.dtype, device=self.device)
        self.misses = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)

    @property
    def hot_rows(self):
        return self.dev.shape[0]

    def gather(self, ids, out=None, n_dev=None):
        """out[r] = table[ids[r]] for the rows of int32 device ids (n_dev: a
        device row count, rows past it are left as they are)."""
        if ids.dtype != torch.int32 or ids.device != self.device or ids.dim() != 1:
            raise ValueError("TieredFeatureTable.gather: ids must be a 1-D int32 tensor on the table's device")
        n = ids.shape[0]
        if out is None:
            out = torch.empty(n, self.d, dtype=self.dtype, device=self.device)
        if out.dtype != self.dtype or out.dim() != 2 or out.shape[1] < self.d or out.stride(1) != 1:
            raise ValueError("TieredFeatureTable.gather: out must be [n, >= d] of the table's dtype")
        es = 4 if self.dtype == torch.float32 else 2
        call("fb_gather_rows_tiered", ptr(ids), n, _p(n_dev), ptr(self.slot_of), self.rows,
             ptr(self.dev) if self.dev.numel() else None, self.dev.stride(0) if self.dev.numel() else self.d,
             self.dev.shape[0], ctypes.c_void_p(self._host_dev), self.host.stride(0), self.d, es, ptr(out),
             out.stride(0), ptr(self.misses), ptr(self.err), stream_ptr())
        return out

    def read_misses(self):
        """Rows read from host memory since construction (synchronises)."""
        return int(self.misses.item())

    def read_bad_ids(self):
        """True when a gather met an id outside the table (its row came out as
        zeros); synchronises."""
        return bool(self.err.item() & 1)
