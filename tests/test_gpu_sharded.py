"""Row-sharded search on one GPU: W shard indexes (row_base = their first
global row) write shard records through bv_search_async, the records are
concatenated in rank order (what the all-gather produces) and bv_merge_shards
must return exactly what one index over all rows returns -- rows bit-exact,
scores bit-identical -- and what the oracle's merge returns.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _rows(n, d, seed):
    rng = np.random.default_rng(seed)
    return O.normalize_rows(rng.standard_normal((n, d)).astype(np.float32))


@pytest.mark.parametrize("bits,scoring,world,n,d,k,fetch", [
    (8, "asym", 2, 20000, 384, 10, 40),
    (8, "int", 3, 9001, 768, 10, 40),
    (4, "asym", 8, 30000, 384, 10, 80),
    (4, "int", 4, 12345, 128, 10, 80),
    (1, "hamming", 8, 40000, 768, 100, 1000),
    (1, "asym", 3, 5000, 256, 10, 320),
    (8, "asym", 4, 3, 64, 2, 8),  # fewer rows than shards: one shard is empty
])
def test_merge_equals_single_index(bits, scoring, world, n, d, k, fetch):
    import torch

    from browservec_b200.index import AddonQuantIndex
    from browservec_b200.sharded import CudaShardEngine, record_words, shard_bounds

    x = _rows(n, d, bits * 13 + world)
    nq = 5
    qs = _rows(nq, d, 77)
    engines, single = [], None
    try:
        for r in range(world):
            lo, hi = shard_bounds(n, world, r)
            e = CudaShardEngine(d, bits, scoring, O.DEFAULT_SEED, 2, "cosine", 0, lo)
            if hi > lo:
                e.append(x[lo:hi])
            engines.append(e)
        single = AddonQuantIndex(d, bits=bits, scoring=scoring)
        single.append(x, n)
        want_rows, want_scores, want_counts, *_ = single.search_arrays(qs, k, fetch)

        stream = torch.cuda.Stream()
        q = torch.from_numpy(qs).cuda()
        torch.cuda.synchronize()
        recs = []
        with torch.cuda.stream(stream):
            for e in engines:
                rec = e.new_record(nq, fetch)
                e.search_record(q, k, fetch, rec, stream.cuda_stream)
                recs.append(rec)
            gathered = torch.cat(recs)
            rows, scores, counts = engines[0].merge(gathered, world, nq, k, fetch, stream.cuda_stream)
        stream.synchronize()
        rows, scores, counts = rows.cpu().numpy(), scores.cpu().numpy(), counts.cpu().numpy()
        assert gathered.numel() == world * record_words(nq, fetch)

        g = gathered.cpu().numpy().reshape(world, -1)
        for i in range(nq):
            c = int(counts[i])
            assert c == int(want_counts[i]) == min(k, n)
            assert np.array_equal(rows[i, :c].view(np.uint32), want_rows[i, :c].astype(np.uint32)), i
            assert np.array_equal(scores[i, :c].view(np.uint32), want_scores[i, :c].view(np.uint32)), i
            recs_np = []
            for w in range(world):
                plane = nq * fetch
                cnt = int(g[w, 3 * plane + i])
                sl = slice(i * fetch, i * fetch + cnt)
                recs_np.append((g[w, :plane][sl].view(np.uint32), g[w, plane:2 * plane][sl].view(np.float32),
                                g[w, 2 * plane:3 * plane][sl].view(np.float32)))
            orow, oscore = O.merge_shard_records(recs_np, fetch, k)
            assert np.array_equal(orow, rows[i, :c].view(np.uint32))
            assert np.array_equal(oscore.view(np.uint32), scores[i, :c].view(np.uint32))
    finally:
        for e in engines:
            e.destroy()
        if single is not None:
            single.destroy()


def test_merge_rejects_bad_arguments():
    import torch

    from browservec_b200 import _lib
    from browservec_b200.sharded import CudaShardEngine

    e = CudaShardEngine(64, 8, "asym", O.DEFAULT_SEED, 2, "cosine", 0, 0)
    try:
        g = torch.zeros(1024, dtype=torch.int32, device="cuda")
        with pytest.raises(_lib.BvError, match="k <= fetch"):
            e.merge(g, 2, 1, 10, 5, 0)
        with pytest.raises(_lib.BvError, match="world 65"):
            e.merge(g, 65, 1, 1, 5, 0)
    finally:
        e.destroy()


@pytest.mark.parametrize("bits,scoring,world,n,d,k,fetch,nq", [
    (1, "hamming", 8, 40000, 768, 100, 1000, 70),
    (1, "int", 4, 30011, 768, 100, 1000, 130),
    (4, "int", 3, 20000, 384, 10, 80, 200),
    (8, "int", 2, 9001, 128, 10, 40, 64),
    (8, "int", 5, 12, 64, 2, 8, 3),  # fewer rows per shard than fetch: every key is a member
])
def test_two_phase_batched_shards_equal_single_index(bits, scoring, world, n, d, k, fetch, nq):
    """bv_batch_select on every shard, the keys concatenated in rank order (the
    all-gather), bv_keys_threshold, bv_batch_finish with that threshold, then
    bv_merge_shards: bit-identical to one index's bv_search_batch, with the
    shards' members partitioning the global best F."""
    import torch

    from browservec_b200.index import AddonQuantIndex
    from browservec_b200.sharded import CudaShardEngine, record_views, shard_bounds

    x = _rows(n, d, bits * 17 + world)
    qs = _rows(nq, d, 78)
    engines, single = [], None
    try:
        for r in range(world):
            lo, hi = shard_bounds(n, world, r)
            e = CudaShardEngine(d, bits, scoring, O.DEFAULT_SEED, 2, "cosine", 0, lo, batched=True)
            if hi > lo:
                e.append(x[lo:hi])
            engines.append(e)
        single = AddonQuantIndex(d, bits=bits, scoring=scoring)
        single.append(x, n)
        stream = torch.cuda.Stream()
        q = torch.from_numpy(qs).cuda()
        F = max(fetch, k)
        wr = torch.zeros((nq, k), dtype=torch.int32, device="cuda")
        ws = torch.zeros((nq, k), dtype=torch.float32, device="cuda")
        wc = torch.zeros(nq, dtype=torch.int32, device="cuda")
        single.search_batch_device(q.data_ptr(), nq, k, F, True, wr.data_ptr(), ws.data_ptr(), wc.data_ptr(),
                                   stream=stream.cuda_stream)
        torch.cuda.synchronize()
        keys = [e.select_keys(q, k, F, stream.cuda_stream) for e in engines]
        gk = torch.cat(keys)
        thr = engines[0].keys_threshold(gk, world, nq, F, stream.cuda_stream)
        stream.synchronize()
        # the threshold against a host selection over the gathered keys
        g = gk.cpu().numpy().view(np.uint64).reshape(world, nq, F)
        t = thr.cpu().numpy().view(np.uint64)
        for i in range(nq):
            ks = g[:, i, :].reshape(-1)
            ks = ks[ks != 0]
            assert int((ks >= t[i]).sum()) == min(F, ks.size), i
        # full member records (rows, approximate and exact scores) merged by bv_merge_shards
        recs = []
        for e in engines:
            rec = e.new_record(nq, F)
            e.finish_record(q, k, F, rec, stream.cuda_stream, None, thr)
            recs.append(rec)
        gathered = torch.cat(recs)
        rows, scores, counts = engines[0].merge(gathered, world, nq, k, F, stream.cuda_stream)
        stream.synchronize()
        members = sum(int(record_views(r, nq, F).counts.sum().item()) for r in recs)
        assert members == nq * min(F, n)
        assert torch.equal(counts, wc)
        assert torch.equal(rows, wr)
        assert torch.equal(scores.view(torch.int32), ws.view(torch.int32))
        # and the top-k records of the bench path, merged by bv_merge_topk
        for e in engines:  # the members are re-selected: select again (the finish consumed them)
            e.select_keys(q, k, F, stream.cuda_stream)
        tops = [e.finish_topk(q, k, F, stream.cuda_stream, None, thr) for e in engines]
        rows2, scores2, counts2 = engines[0].merge_topk(torch.cat(tops), world, nq, k, stream.cuda_stream)
        stream.synchronize()
        assert torch.equal(counts2, wc)
        assert torch.equal(rows2, wr)
        assert torch.equal(scores2.view(torch.int32), ws.view(torch.int32))
    finally:
        for e in engines:
            e.destroy()
        if single is not None:
            single.destroy()


@pytest.mark.parametrize("bits,scoring,n,d,k,fetch,nq", [
    (1, "int", 40000, 768, 100, 1000, 300),
    (8, "asym", 20000, 384, 10, 40, 7),
    (4, "int", 30000, 384, 10, 80, 300),
])
def test_one_rank_shortcut_equals_record_merge(bits, scoring, n, d, k, fetch, nq):
    """A one-rank ShardedIndex answers with its shard's own best k (no record,
    no merge): the same rows and score bits as the record + merge path."""
    import socket

    import torch
    import torch.distributed as dist

    from browservec_b200.sharded import ShardedIndex

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", world_size=1, rank=0)
    try:
        x = _rows(n, d, bits * 29 + 1)
        qs = torch.from_numpy(_rows(nq, d, 5)).cuda()
        idx = ShardedIndex(d, n, bits=bits, scoring=scoring, metric="cosine", device=0)
        idx.load(torch.from_numpy(x).cuda())
        got = [t.cpu().numpy() for t in idx.search(qs, k, fetch)]
        eng, st = idx.engine, torch.cuda.Stream()
        with torch.cuda.stream(st):
            rec = eng.new_record(nq, fetch)
            eng.search_record(qs, k, fetch, rec, st.cuda_stream)
            want = [t.cpu().numpy() for t in eng.merge(rec, 1, nq, k, fetch, st.cuda_stream)]
        torch.cuda.synchronize()
        np.testing.assert_array_equal(got[2], want[2])
        for q in range(nq):
            m = int(want[2][q])
            np.testing.assert_array_equal(got[0][q, :m], want[0][q, :m])
            assert got[1][q, :m].view(np.uint32).tolist() == want[1][q, :m].view(np.uint32).tolist()
        idx.destroy()
    finally:
        dist.destroy_process_group()
