import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); parity tests through the C ABI")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def small_graph(n_nodes=60, n_edges=4000, seed=0, t_max=1000, int_ts=True, empty_nodes=(), zipf=None):
    """Chronological random temporal graph in the reference CSR layout."""
    rng = np.random.default_rng(seed)
    if zipf is None:
        src = rng.integers(0, n_nodes, n_edges).astype(np.int32)
    else:
        w = np.arange(1, n_nodes + 1, dtype=np.float64) ** (-zipf)
        src = rng.choice(n_nodes, n_edges, p=w / w.sum()).astype(np.int32)
    for n in empty_nodes:
        src[src == n] = (n + 1) % n_nodes
    dst = rng.integers(0, n_nodes, n_edges).astype(np.int32)
    if int_ts:
        t = np.sort(rng.integers(0, t_max, n_edges)).astype(np.float32)
    else:
        t = np.sort(rng.random(n_edges) * t_max).astype(np.float32)
    order = np.argsort(src, kind="stable")
    indptr = np.zeros(n_nodes + 1, np.int64)
    np.add.at(indptr, src.astype(np.int64) + 1, 1)
    indptr = np.cumsum(indptr).astype(np.int32)
    return dict(indptr=indptr, indices=dst[order].astype(np.int32), eid=order.astype(np.int32), ts=t[order],
                src=src, dst=dst, t=t)
