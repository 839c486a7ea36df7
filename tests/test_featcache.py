"""Host logic of the tiered feature table (fast_b200/featcache.py): the
pre-sampling count and hot-row choice of the reference's slim feature cache
(slimCache.py:184-259, get_hot_cts / init_cache) and the id -> slot map."""
import numpy as np
import pytest

from fast_b200.featcache import count_ids, hot_ids_by_count, slot_map


def test_count_ids_counts_every_batch_and_skips_outside_ids():
    c = count_ids([np.array([0, 3, 3, 9]), [3, 1, -1, 10]], 10)
    assert c.tolist() == [1, 1, 0, 3, 0, 0, 0, 0, 0, 1]


def test_hot_ids_by_count_takes_the_most_frequent_smaller_ids_first():
    counts = np.array([2, 7, 2, 0, 7, 1])
    assert hot_ids_by_count(counts, 3).tolist() == [1, 4, 0]
    assert hot_ids_by_count(counts, 0).tolist() == []
    assert sorted(hot_ids_by_count(counts, 99).tolist()) == list(range(6))


def test_slot_map_places_hot_ids_and_rejects_bad_ones():
    m = slot_map([5, 2, 7], 8)
    assert m.dtype == np.int32
    assert m.tolist() == [-1, -1, 1, -1, -1, 0, -1, 2]
    assert slot_map([], 3).tolist() == [-1, -1, -1]
    for bad in ([1, 1], [8], [-1]):
        with pytest.raises(ValueError):
            slot_map(bad, 8)
