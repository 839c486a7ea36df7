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


RTOL, ATOL = 1e-5, 1e-6


def parity(dev, ref64, ref32, name="", rtol=RTOL, atol=ATOL):
    """Device result vs the fp64 restatement T64 and the fp32 one T32 (the
    reference's own arithmetic).  Passes when, elementwise,
    |dev - T64| <= atol + rtol |T64|, or when the device result is as
    accurate as the fp32 reference: ||dev - T64|| <= 2 ||T32 - T64|| + atol sqrt(n).
    Returns the form that passed ("elem" / "norm"); raises otherwise."""
    import torch
    dev, ref64, ref32 = (t.detach().cpu().double() for t in (dev, ref64, ref32))
    err = (dev - ref64).abs()
    if bool((err <= atol + rtol * ref64.abs()).all()):
        return "elem"
    e_dev, e_ref = float(err.norm()), float((ref32 - ref64).norm())
    if e_dev <= 2 * e_ref + atol * err.numel() ** 0.5:
        return "norm"
    worst = int(torch.argmax(err / (atol + rtol * ref64.abs())))
    raise AssertionError("%s: device error %.3e (norm) vs fp32 reference %.3e; worst element %d: dev %.9g ref %.9g"
                         % (name, e_dev, e_ref, worst, float(dev.reshape(-1)[worst]),
                            float(ref64.reshape(-1)[worst])))
