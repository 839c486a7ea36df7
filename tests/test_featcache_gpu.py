"""fb_gather_rows_tiered through TieredFeatureTable: rows of an fp32 / bf16
table, the hot ones from HBM and the others read by the kernel from
page-locked host memory, must equal table[ids] bit for bit; the host-read
count, a device row count and an out-of-table id are checked too."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,d", [(torch.float32, 37), (torch.float32, 64), (torch.bfloat16, 192),
                                     (torch.bfloat16, 37)])
def test_tiered_gather_equals_indexing(cuda, dtype, d):
    from fast_b200.featcache import TieredFeatureTable, count_ids, hot_ids_by_count
    rows = 5000
    g = torch.Generator().manual_seed(3)
    table = torch.randn(rows, d, generator=g).to(dtype)
    rng = np.random.default_rng(4)
    ids = rng.zipf(1.3, 6000) % rows                      # skewed, with repeats
    hot = hot_ids_by_count(count_ids([ids[:3000]], rows), 700)
    t = TieredFeatureTable(table, hot, device=cuda)
    ids_d = torch.from_numpy(ids.astype(np.int32)).to(cuda)
    out = t.gather(ids_d)
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), table[torch.from_numpy(ids)])
    assert t.read_misses() == int((~np.isin(ids, hot)).sum())
    assert not t.read_bad_ids()
    # a device row count: rows past it stay as they were
    n_dev = torch.tensor([100], dtype=torch.int32, device=cuda)
    out2 = torch.full((ids.size, d), 7, dtype=dtype, device=cuda)
    t.gather(ids_d, out=out2, n_dev=n_dev)
    assert torch.equal(out2[:100].cpu(), table[torch.from_numpy(ids[:100])])
    assert bool((out2[100:] == 7).all())
    # an id outside the table: a zero row and the error bit
    bad = torch.tensor([0, rows, 1], dtype=torch.int32, device=cuda)
    o3 = t.gather(bad)
    assert torch.equal(o3[1].cpu(), torch.zeros(d, dtype=dtype))
    assert torch.equal(o3[0].cpu(), table[0]) and torch.equal(o3[2].cpu(), table[1])
    assert t.read_bad_ids()


def test_tiered_gather_without_hot_rows(cuda):
    from fast_b200.featcache import TieredFeatureTable
    table = torch.arange(300 * 8, dtype=torch.float32).reshape(300, 8)
    t = TieredFeatureTable(table, [], device=cuda)
    ids = torch.tensor([5, 299, 0, 5], dtype=torch.int32, device=cuda)
    assert torch.equal(t.gather(ids).cpu(), table[ids.cpu().long()])
    assert t.read_misses() == 4
