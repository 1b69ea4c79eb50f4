"""Row-sharded search on CPU: the merge rule and the distributed plumbing.

1. Oracle level: splitting the rows into W contiguous shards, taking each
   shard's best F with exact scores and merging gives exactly the single-store
   answer (rows and scores), for every scoring mode and uneven splits.
2. Plumbing: two gloo ranks run ``ShardedIndex`` with an oracle-backed test
   engine (shard records, all-gather in rank order, merge) and must return
   the single-store answer on every rank.
"""
import os
import socket

import numpy as np
import pytest
import torch

from browservec_b200.sharded import ShardedIndex, record_views, record_words, shard_bounds, topk_words
from oracle import oracle as O


def _rows(n, d, seed):
    rng = np.random.default_rng(seed)
    return O.normalize_rows(rng.standard_normal((n, d)).astype(np.float32))


def test_shard_bounds():
    for n in (0, 1, 7, 100, 1001):
        for w in (1, 2, 3, 8):
            b = [shard_bounds(n, w, r) for r in range(w)]
            assert b[0][0] == 0 and b[-1][1] == n
            assert all(b[i][1] == b[i + 1][0] for i in range(w - 1))
            sizes = [hi - lo for lo, hi in b]
            assert max(sizes) - min(sizes) <= 1 and sizes == sorted(sizes, reverse=True)
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


def test_vector_keys_match_scalar_key():
    s = np.array([1.5, -1.5, 0.0, -0.0, 3.4e38, -3.4e38, 1e-30, -1e-30], np.float32)
    r = np.array([0, 1, 2, 3, 4, 5, 6, 0xFFFFFFFE], np.uint32)
    k = O.keys(s, r)
    assert [int(x) for x in k] == [O.key(float(a), int(b)) for a, b in zip(s, r)]


@pytest.mark.parametrize("bits,mode,world,k,fetch", [
    (8, O.MODE_ASYM, 2, 10, 40), (8, O.MODE_INT, 3, 10, 40), (4, O.MODE_ASYM, 4, 10, 80),
    (1, O.MODE_HAMMING, 8, 20, 200), (1, O.MODE_ASYM, 5, 5, 160)])
def test_oracle_merge_equals_single_store(bits, mode, world, k, fetch):
    n, d = 1203, 64
    x = _rows(n, d, bits * 7 + world)
    full = O.Corpus(x, d, bits)
    for qi in range(3):
        q = _rows(1, d, 1000 + qi)[0]
        want_rows, want_scores, _, _ = full.query(q, k, fetch, mode)
        recs = []
        for r in range(world):
            lo, hi = shard_bounds(n, world, r)
            recs.append(O.shard_record(O.Corpus(x[lo:hi], d, bits), lo, q, k, fetch, mode))
        got_rows, got_scores = O.merge_shard_records(recs, fetch, k)
        assert np.array_equal(got_rows, want_rows)
        assert np.array_equal(got_scores.view(np.uint32), want_scores.view(np.uint32))


class OracleShardEngine:
    """Test engine: the shard-local search and the merge restated by the oracle."""

    def __init__(self, d, bits, mode, row_base):
        self.d, self.bits, self.mode, self.row_base = d, bits, mode, row_base
        self.corpus = None

    @property
    def size(self):
        return 0 if self.corpus is None else self.corpus.n

    def append(self, rows):
        self.corpus = O.Corpus(np.asarray(rows, np.float32), self.d, self.bits)

    def new_record(self, nq, fetch):
        return torch.zeros(record_words(nq, fetch), dtype=torch.int32)

    def search_record(self, q, k, fetch, rec, stream, mask=None):
        nq = q.shape[0]
        v = record_views(rec.numpy(), nq, fetch)
        for i in range(nq):
            rows, approx, exact = O.shard_record(self.corpus, self.row_base, q[i].numpy(), k, fetch, self.mode)
            n = rows.size
            v.rows[i * fetch:i * fetch + n] = rows.view(np.int32)
            v.approx[i * fetch:i * fetch + n] = approx.view(np.int32)
            v.exact[i * fetch:i * fetch + n] = exact.view(np.int32)
            v.counts[i] = n

    def search_topk(self, q, k, fetch, stream, mask=None):
        """A one-rank group's whole answer: the shard's own best k (global rows)."""
        nq = q.shape[0]
        rows = np.zeros((nq, k), np.int32)
        scores = np.zeros((nq, k), np.float32)
        counts = np.zeros(nq, np.int32)
        self.topk_calls = getattr(self, "topk_calls", 0) + 1
        for i in range(nq):
            r, s, _, _ = self.corpus.query(q[i].numpy(), k, fetch, self.mode)
            rows[i, :r.size] = (r + np.uint32(self.row_base)).view(np.int32)
            scores[i, :r.size] = s
            counts[i] = r.size
        return torch.from_numpy(rows), torch.from_numpy(scores), torch.from_numpy(counts)

    # two-phase batched flow (select keys -> all-gather -> global threshold ->
    # re-rank only this shard's members of the global best F)
    two_phase = False

    def select_keys(self, q, k, fetch, stream, mask=None):
        nq = q.shape[0]
        out = np.zeros((nq, fetch), np.uint64)
        self._cands = []
        for i in range(nq):
            _, _, cr, cs = self.corpus.query(q[i].numpy(), k, fetch, self.mode)
            self._cands.append((cr, cs))
            out[i, :cr.size] = O.keys(cs, cr.astype(np.uint32) + np.uint32(self.row_base))
        return torch.from_numpy(out.reshape(-1).view(np.int64))

    def keys_threshold(self, gathered, world, nq, fetch, stream):
        g = gathered.numpy().view(np.uint64).reshape(world, nq, fetch)
        thr = np.ones(nq, np.uint64)
        for i in range(nq):
            ks = np.sort(g[:, i, :].reshape(-1))[::-1]
            ks = ks[ks != 0]
            if ks.size > fetch:
                thr[i] = ks[fetch - 1]
        return torch.from_numpy(thr.view(np.int64))

    def finish_topk(self, q, k, fetch, stream, mask, thr):
        """This shard's members of the global best F (keys >= thr), re-ranked
        exactly; its best k of them as [rows nq*k | scores nq*k | counts nq]."""
        nq = q.shape[0]
        out = np.zeros(topk_words(nq, k), np.int32)
        t = thr.numpy().view(np.uint64)
        self.members = 0
        for i in range(nq):
            cr, cs = self._cands[i]
            rows = cr.astype(np.uint32) + np.uint32(self.row_base)
            keep = O.keys(cs, rows) >= t[i]
            rows = rows[keep]
            self.members += int(rows.size)
            exact = np.array([np.float32(O.dot_row(self.corpus.originals[r - self.row_base], q[i].numpy()))
                              for r in rows], np.float32)
            order = np.argsort(O.keys(exact, rows))[::-1][:k]
            n = order.size
            out[i * k:i * k + n] = rows[order].view(np.int32)
            out[nq * k + i * k:nq * k + i * k + n] = exact[order].view(np.int32)
            out[2 * nq * k + i] = n
        return torch.from_numpy(out)

    def merge_topk(self, gathered, world, nq, k, stream):
        g = gathered.numpy().reshape(world, topk_words(nq, k))
        rows = np.zeros((nq, k), np.int32)
        scores = np.zeros((nq, k), np.float32)
        counts = np.zeros(nq, np.int32)
        for i in range(nq):
            rr, ss = [], []
            for w in range(world):
                c = int(g[w, 2 * nq * k + i])
                rr.append(g[w, i * k:i * k + c].view(np.uint32))
                ss.append(g[w, nq * k + i * k:nq * k + i * k + c].view(np.float32))
            rr, ss = np.concatenate(rr), np.concatenate(ss)
            order = np.argsort(O.keys(ss, rr))[::-1][:k]
            rows[i, :order.size], scores[i, :order.size], counts[i] = rr[order].view(np.int32), ss[order], order.size
        return torch.from_numpy(rows), torch.from_numpy(scores), torch.from_numpy(counts)

    def merge(self, gathered, world, nq, k, fetch, stream):
        g = gathered.numpy().reshape(world, record_words(nq, fetch))
        rows = np.zeros((nq, k), np.int32)
        scores = np.zeros((nq, k), np.float32)
        counts = np.zeros(nq, np.int32)
        for i in range(nq):
            recs = []
            for w in range(world):
                v = record_views(g[w], nq, fetch)
                c = int(v.counts[i])
                sl = slice(i * fetch, i * fetch + c)
                recs.append((v.rows[sl].view(np.uint32), v.approx[sl].view(np.float32),
                             v.exact[sl].view(np.float32)))
            r, s = O.merge_shard_records(recs, fetch, k)
            rows[i, :r.size], scores[i, :r.size], counts[i] = r.view(np.int32), s, r.size
        return torch.from_numpy(rows), torch.from_numpy(scores), torch.from_numpy(counts)

    def destroy(self):
        pass


N, D, BITS, MODE, K, FETCH, NQ = 777, 32, 8, O.MODE_ASYM, 5, 20, 3


def _rank_main(rank, world, port, out_dir, two_phase=False):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = _rows(N, D, 5)
        lo, _ = shard_bounds(N, world, rank)
        eng = OracleShardEngine(D, BITS, MODE, lo)
        eng.two_phase = two_phase
        idx = ShardedIndex(D, N, bits=BITS, engine=eng)
        idx.load(x, global_rows=True)
        q = torch.from_numpy(_rows(NQ, D, 6))
        rows, scores, counts = idx.search(q, K, FETCH)
        members = torch.tensor([getattr(eng, "members", -1)])
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), rows=rows.numpy(), scores=scores.numpy(),
                 counts=counts.numpy(), members=members.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_gloo_two_ranks_match_single_store(tmp_path):
    import torch.multiprocessing as mp

    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn")
    x = _rows(N, D, 5)
    full = O.Corpus(x, D, BITS)
    qs = _rows(NQ, D, 6)
    for r in range(world):
        got = np.load(tmp_path / f"r{r}.npz")
        for i in range(NQ):
            wr, ws, _, _ = full.query(qs[i], K, FETCH, MODE)
            n = int(got["counts"][i])
            assert n == wr.size
            assert np.array_equal(got["rows"][i, :n].view(np.uint32), wr)
            assert np.array_equal(got["scores"][i, :n].view(np.uint32), ws.view(np.uint32))


def test_gloo_three_ranks_two_phase_members_only(tmp_path):
    """The two-phase flow: every rank re-ranks only its members of the global
    best F (together exactly F per query), and the merged answer is still the
    single-store answer."""
    import torch.multiprocessing as mp

    world = 3
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path), True), nprocs=world,
                       start_method="spawn")
    x = _rows(N, D, 5)
    full = O.Corpus(x, D, BITS)
    qs = _rows(NQ, D, 6)
    members = 0
    for r in range(world):
        got = np.load(tmp_path / f"r{r}.npz")
        members += int(got["members"][0])
        for i in range(NQ):
            wr, ws, _, _ = full.query(qs[i], K, FETCH, MODE)
            n = int(got["counts"][i])
            assert n == wr.size
            assert np.array_equal(got["rows"][i, :n].view(np.uint32), wr)
            assert np.array_equal(got["scores"][i, :n].view(np.uint32), ws.view(np.uint32))
    assert members == NQ * FETCH  # the shards' members partition the global best F


def test_gloo_one_rank_answers_alone(tmp_path):
    """A one-rank group takes the shortcut (its own best k, no record, no
    merge) and returns the single-store answer."""
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()))
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        x = _rows(N, D, 5)
        eng = OracleShardEngine(D, BITS, MODE, 0)
        idx = ShardedIndex(D, N, bits=BITS, engine=eng)
        idx.load(x, global_rows=True)
        qs = _rows(NQ, D, 6)
        rows, scores, counts = idx.search(torch.from_numpy(qs), K, FETCH)
        assert eng.topk_calls == 1
        full = O.Corpus(x, D, BITS)
        for i in range(NQ):
            wr, ws, _, _ = full.query(qs[i], K, FETCH, MODE)
            n = int(counts[i])
            assert n == wr.size
            assert np.array_equal(rows[i, :n].numpy().view(np.uint32), wr)
            assert np.array_equal(scores[i, :n].numpy().view(np.uint32), ws.view(np.uint32))
    finally:
        dist.destroy_process_group()
