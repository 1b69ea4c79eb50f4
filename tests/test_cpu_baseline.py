"""The sharded CPU baseline (one CpuIndex per row shard, cpu.ts:66-88, merged
with mergePartials, gpuTopk.ts:160-189) returns what one CpuIndex over all rows
returns: uneven shards, an empty shard, and filtered shards given as row maps."""
import numpy as np

from oracle import oracle as O


def test_sharded_baseline_equals_single_index():
    rng = np.random.default_rng(0)
    n, d, k = 5000, 96, 10
    x = O.normalize_rows(rng.standard_normal((n, d)).astype(np.float32))
    q = O.normalize_rows(rng.standard_normal((7, d)).astype(np.float32))
    r1, s1 = O.cpu_index_query_batch(x, d, q, k, threads=4)
    bounds = [0, 1000, 2500, 2500, 4999, 5000]
    shards = [x[a:b] for a, b in zip(bounds[:-1], bounds[1:])]
    r2, s2, c = O.cpu_sharded_query_batch(shards, bounds[:-1], n, d, q, k, threads=3)
    assert np.array_equal(r1, r2) and np.array_equal(s1.view(np.uint32), s2.view(np.uint32))
    assert np.all(c == k)


def test_filtered_shards_with_row_maps():
    rng = np.random.default_rng(1)
    n, d, k = 3000, 32, 5
    x = O.normalize_rows(rng.standard_normal((n, d)).astype(np.float32))
    q = O.normalize_rows(rng.standard_normal((3, d)).astype(np.float32))
    keep = np.flatnonzero(rng.random(n) < 0.3).astype(np.uint32)
    r1, s1 = O.cpu_index_query_batch(x[keep], d, q, k, threads=2)
    parts = np.array_split(keep, 4)
    r2, s2, _ = O.cpu_sharded_query_batch([x[p] for p in parts], [0] * 4, n, d, q, k, threads=2, maps=parts)
    assert np.array_equal(keep[r1], r2) and np.array_equal(s1.view(np.uint32), s2.view(np.uint32))
