"""Row-sharded quantized search: one process per GPU, one all-gather per batch.

The reference splits a large corpus into row chunks that one GPU scans in
turn (``ChunkedCorpus``, src/engine/buffers.ts:92-214, driven by
QuantIndex.search, src/index/quant.ts:194-245).  Here the chunks become
per-GPU shards: rank r of W holds the contiguous global rows
``shard_bounds(n, W, r)`` (codes, scales and fp32 originals), scans them for
every query, re-ranks its local best F exactly, and writes one shard record
per batch.  A single ``all_gather_into_tensor`` (NCCL over NVLink) gives every
rank all W records, and ``bv_merge_shards`` rebuilds the answer a single
store would give: the global best F by approximate score, then the best k of
those by exact score.

Record layout (u32 words, one per rank, ``record_words(nq, F)`` long):
``[rows nq*F | approx nq*F | exact nq*F | counts nq]`` -- rows are global.

Batched engines search in two halves when W > 1: each rank selects its best
F approximate keys (``select_keys``), one all-gather of those keys gives every
rank the global F-th best key per query (``keys_threshold``), and each rank
then re-ranks only its own keys at or above it -- its members of the global
best F, about F / W rows per query instead of F -- and contributes its best k
of them by exact score (``finish_topk``: a record of ``topk_words(nq, k)``
words ``[rows nq*k | scores nq*k | counts nq]``).  A second all-gather and
``merge_topk`` give the single-store answer, since the members of all ranks
are exactly the global best F.

The CUDA engine is the only engine shipped; tests substitute their own
``engine`` object to exercise the distributed plumbing on CPU ranks.
"""
from __future__ import annotations

import ctypes as C
from contextlib import nullcontext
from dataclasses import dataclass

import numpy as np

from . import _lib
from .index import DEFAULT_SEED, AddonQuantIndex


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous split of n rows over world ranks; the first n % world ranks
    take one extra row."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def record_words(nq: int, fetch: int) -> int:
    return 3 * nq * fetch + nq


def topk_words(nq: int, k: int) -> int:
    return 2 * nq * k + nq


@dataclass
class RecordViews:
    """Views of one shard record (a 1-D int32 tensor or ndarray)."""
    rows: object
    approx: object
    exact: object
    counts: object


def record_views(rec, nq: int, fetch: int) -> RecordViews:
    plane = nq * fetch
    return RecordViews(rows=rec[:plane], approx=rec[plane:2 * plane], exact=rec[2 * plane:3 * plane],
                       counts=rec[3 * plane:3 * plane + nq])


class CudaShardEngine:
    """The shard-local work on this rank's GPU: bv_search_async into the
    record, bv_merge_shards over the gathered records."""

    def __init__(self, dim: int, bits: int, scoring: str, seed: int, rounds: int, metric: str,
                 device: int, row_base: int, batched: bool | None = None):
        import torch

        self.torch = torch
        # integer scorings serve a batch on the tensor cores (bv_search_batch);
        # asym scores per query (bv_search_async)
        self.batched = scoring != "asym" if batched is None else batched
        self.device = torch.device("cuda", device)
        self.index = AddonQuantIndex(dim, seed=seed, rounds=rounds, bits=bits, scoring=scoring,
                                     device=device, metric=metric, row_base=row_base)
        self.L = _lib.load()

    @property
    def size(self) -> int:
        return self.index.size

    def append(self, rows) -> None:
        """rows: a float32 CUDA tensor (n, dim) on this rank's device, or a host array."""
        torch = self.torch
        if isinstance(rows, torch.Tensor) and rows.is_cuda:
            rows = rows.contiguous()
            self.index.append_device(rows.data_ptr(), rows.shape[0],
                                     torch.cuda.current_stream(self.device).cuda_stream)
            torch.cuda.current_stream(self.device).synchronize()
        else:
            a = np.ascontiguousarray(rows, dtype=np.float32)
            self.index.append(a, a.shape[0])

    def new_record(self, nq: int, fetch: int):
        return self.torch.empty(record_words(nq, fetch), dtype=self.torch.int32, device=self.device)

    def search_record(self, q, k: int, fetch: int, rec, stream: int, mask=None) -> None:
        nq = q.shape[0]
        v = record_views(rec, nq, fetch)
        if not hasattr(self, "_scratch") or self._scratch.numel() < nq * (2 * k + 1):
            self._scratch = self.torch.empty(nq * (2 * k + 1), dtype=self.torch.int32, device=self.device)
        s = self._scratch
        args = _lib.BvSearchArgs(queries=q.data_ptr(), nq=nq, k=k, fetch=fetch, rerank=1,
                                 mask=None if mask is None else mask.data_ptr(),
                                 mask_words=0 if mask is None else mask.numel(),
                                 out_rows=s.data_ptr(), out_scores=s[nq * k:].data_ptr(),
                                 out_counts=s[2 * nq * k:].data_ptr(), cand_rows=v.rows.data_ptr(),
                                 cand_scores=v.approx.data_ptr(), cand_counts=v.counts.data_ptr(),
                                 cand_exact=v.exact.data_ptr())
        fn = self.L.bv_search_batch if self.batched else self.L.bv_search_async
        _lib.check(fn(self.index._h, C.byref(args), C.c_void_p(stream)))

    @property
    def two_phase(self) -> bool:
        return self.batched

    def _args(self, q, k, fetch, rec, mask):
        nq = q.shape[0]
        v = record_views(rec, nq, fetch) if rec is not None else None
        if not hasattr(self, "_scratch") or self._scratch.numel() < nq * (2 * k + 1):
            self._scratch = self.torch.empty(nq * (2 * k + 1), dtype=self.torch.int32, device=self.device)
        s = self._scratch
        return _lib.BvSearchArgs(queries=q.data_ptr(), nq=nq, k=k, fetch=fetch, rerank=1,
                                 mask=None if mask is None else mask.data_ptr(),
                                 mask_words=0 if mask is None else mask.numel(),
                                 out_rows=s.data_ptr(), out_scores=s[nq * k:].data_ptr(),
                                 out_counts=s[2 * nq * k:].data_ptr(),
                                 cand_rows=v.rows.data_ptr() if v else None,
                                 cand_scores=v.approx.data_ptr() if v else None,
                                 cand_counts=v.counts.data_ptr() if v else None,
                                 cand_exact=v.exact.data_ptr() if v else None)

    def select_keys(self, q, k: int, fetch: int, stream: int, mask=None):
        """First half of a batched shard search: this shard's best `fetch`
        approximate keys per query (int64 view of u64 keys, global rows)."""
        nq = q.shape[0]
        keys = self.torch.empty(nq * fetch, dtype=self.torch.int64, device=self.device)
        args = self._args(q, k, fetch, None, mask)
        _lib.check(self.L.bv_batch_select(self.index._h, C.byref(args), C.c_void_p(keys.data_ptr()),
                                          C.c_void_p(stream)))
        return keys

    def search_topk(self, q, k: int, fetch: int, stream: int, mask=None):
        """The whole answer of a single shard: the best k by exact score
        (global rows), no candidate record (what one rank needs alone)."""
        torch = self.torch
        nq = q.shape[0]
        rows = torch.empty((nq, k), dtype=torch.int32, device=self.device)
        scores = torch.empty((nq, k), dtype=torch.float32, device=self.device)
        counts = torch.empty(nq, dtype=torch.int32, device=self.device)
        args = _lib.BvSearchArgs(queries=q.data_ptr(), nq=nq, k=k, fetch=fetch, rerank=1,
                                 mask=None if mask is None else mask.data_ptr(),
                                 mask_words=0 if mask is None else mask.numel(),
                                 out_rows=rows.data_ptr(), out_scores=scores.data_ptr(),
                                 out_counts=counts.data_ptr())
        fn = self.L.bv_search_batch if self.batched else self.L.bv_search_async
        _lib.check(fn(self.index._h, C.byref(args), C.c_void_p(stream)))
        return rows, scores, counts

    def keys_threshold(self, gathered, world: int, nq: int, fetch: int, stream: int):
        thr = self.torch.empty(nq, dtype=self.torch.int64, device=self.device)
        _lib.check(self.L.bv_keys_threshold(C.c_void_p(gathered.data_ptr()), world, nq, fetch,
                                            C.c_void_p(thr.data_ptr()), C.c_void_p(stream)))
        return thr

    def finish_record(self, q, k: int, fetch: int, rec, stream: int, mask, thr) -> None:
        """Second half, full record: re-rank this shard's candidates at or
        above thr[q] and write them (rows, approximate and exact scores)."""
        args = self._args(q, k, fetch, rec, mask)
        _lib.check(self.L.bv_batch_finish(self.index._h, C.byref(args), C.c_void_p(thr.data_ptr()),
                                          C.c_void_p(stream)))

    def finish_topk(self, q, k: int, fetch: int, stream: int, mask, thr):
        """Second half: re-rank this shard's candidates at or above thr[q];
        returns its best k of them as a top-k record (global rows)."""
        nq = q.shape[0]
        out = self.torch.empty(topk_words(nq, k), dtype=self.torch.int32, device=self.device)
        args = _lib.BvSearchArgs(queries=q.data_ptr(), nq=nq, k=k, fetch=fetch, rerank=1,
                                 mask=None if mask is None else mask.data_ptr(),
                                 mask_words=0 if mask is None else mask.numel(),
                                 out_rows=out.data_ptr(), out_scores=out[nq * k:].data_ptr(),
                                 out_counts=out[2 * nq * k:].data_ptr())
        _lib.check(self.L.bv_batch_finish(self.index._h, C.byref(args), C.c_void_p(thr.data_ptr()),
                                          C.c_void_p(stream)))
        return out

    def merge_topk(self, gathered, world: int, nq: int, k: int, stream: int):
        torch = self.torch
        rows = torch.empty((nq, k), dtype=torch.int32, device=self.device)
        scores = torch.empty((nq, k), dtype=torch.float32, device=self.device)
        counts = torch.empty(nq, dtype=torch.int32, device=self.device)
        _lib.check(self.L.bv_merge_topk(C.c_void_p(gathered.data_ptr()), world, nq, k,
                                        C.c_void_p(rows.data_ptr()), C.c_void_p(scores.data_ptr()),
                                        C.c_void_p(counts.data_ptr()), C.c_void_p(stream)))
        return rows, scores, counts

    def merge(self, gathered, world: int, nq: int, k: int, fetch: int, stream: int):
        torch = self.torch
        rows = torch.empty((nq, k), dtype=torch.int32, device=self.device)
        scores = torch.empty((nq, k), dtype=torch.float32, device=self.device)
        counts = torch.empty(nq, dtype=torch.int32, device=self.device)
        _lib.check(self.L.bv_merge_shards(C.c_void_p(gathered.data_ptr()), world, nq, fetch, k,
                                          C.c_void_p(rows.data_ptr()), C.c_void_p(scores.data_ptr()),
                                          C.c_void_p(counts.data_ptr()), C.c_void_p(stream)))
        return rows, scores, counts

    def destroy(self) -> None:
        self.index.destroy()


class ShardedIndex:
    """Quantized flat index whose rows are split across the ranks of a
    torch.distributed process group (NCCL, one process per GPU).

    Every rank constructs it with the same arguments and the planned corpus
    size ``n_total``; rank r then holds global rows ``shard_bounds(n_total,
    W, r)``.  ``load`` takes each rank's slice (host array or a CUDA tensor of
    just this rank's rows); ``search`` is collective: every rank calls it with
    the same queries and receives the merged global answer.
    """

    def __init__(self, dim: int, n_total: int, bits: int = 8, scoring: str = "asym",
                 seed: int = DEFAULT_SEED, rounds: int = 2, metric: str = "cosine", group=None,
                 device: int | None = None, engine=None, batched: bool | None = None):
        import torch
        import torch.distributed as dist

        if not dist.is_initialized():
            raise RuntimeError("ShardedIndex needs an initialised torch.distributed process group")
        self.torch, self.dist, self.group = torch, dist, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.dim, self.n_total = dim, n_total
        self.lo, self.hi = shard_bounds(n_total, self.world, self.rank)
        if engine is None:
            if device is None:
                device = torch.cuda.current_device()
            engine = CudaShardEngine(dim, bits, scoring, seed, rounds, metric, device, self.lo, batched)
            self._stream = torch.cuda.Stream(device=engine.device)
        else:
            self._stream = None
        self.engine = engine

    def set_scoring(self, scoring: str, batched: bool | None = None) -> None:
        """Score later searches with another mode (every rank must call it)."""
        self.engine.index.set_scoring(scoring)
        self.engine.batched = scoring != "asym" if batched is None else batched

    @property
    def local_rows(self) -> int:
        return self.hi - self.lo

    def load(self, rows, global_rows: bool = False) -> None:
        """Append this rank's rows: ``rows`` is either the full corpus
        (``global_rows=True``, sliced here) or exactly this rank's slice."""
        part = rows[self.lo:self.hi] if global_rows else rows
        if part.shape[0] != self.local_rows:
            raise ValueError(f"rank {self.rank} expects {self.local_rows} rows, got {part.shape[0]}")
        if self.engine.size != 0:
            raise RuntimeError("shard already loaded")
        self.engine.append(part)

    def search(self, q, k: int, fetch: int, mask=None):
        """Collective search of nq queries (a (nq, dim) float32 tensor on this
        rank's device, normalised for cosine).  `mask` (optional): this rank's
        score mask, uint32 words over its local rows (e.g. DeviceColumns.mask
        of its shard's metadata).  Returns (rows, scores, counts) tensors of
        shape (nq, k), (nq, k), (nq,) with global rows."""
        torch = self.torch
        fetch = max(fetch, k)
        nq = q.shape[0]
        if self._stream is not None:
            self._stream.wait_stream(torch.cuda.current_stream(self.engine.device))
        ctx = torch.cuda.stream(self._stream) if self._stream is not None else nullcontext()
        with ctx:
            sid = self._stream.cuda_stream if self._stream is not None else 0
            if self.world == 1 and hasattr(self.engine, "search_topk"):
                # one rank holds every row: its own best k is the answer (no
                # candidate record, no merge)
                out = self.engine.search_topk(q, k, fetch, sid, mask)
            elif self.world > 1 and getattr(self.engine, "two_phase", False):
                keys = self.engine.select_keys(q, k, fetch, sid, mask)
                gk = torch.empty(self.world * keys.numel(), dtype=keys.dtype, device=keys.device)
                self.dist.all_gather_into_tensor(gk, keys, group=self.group)
                thr = self.engine.keys_threshold(gk, self.world, nq, fetch, sid)
                rec = self.engine.finish_topk(q, k, fetch, sid, mask, thr)
                gathered = torch.empty(self.world * rec.numel(), dtype=rec.dtype, device=rec.device)
                self.dist.all_gather_into_tensor(gathered, rec, group=self.group)
                out = self.engine.merge_topk(gathered, self.world, nq, k, sid)
            else:
                rec = self.engine.new_record(nq, fetch)
                self.engine.search_record(q, k, fetch, rec, sid, mask)
                gathered = torch.empty(self.world * rec.numel(), dtype=rec.dtype, device=rec.device)
                self.dist.all_gather_into_tensor(gathered, rec, group=self.group)
                out = self.engine.merge(gathered, self.world, nq, k, fetch, sid)
        if self._stream is not None:
            torch.cuda.current_stream(self.engine.device).wait_stream(self._stream)
        return out

    def destroy(self) -> None:
        self.engine.destroy()
