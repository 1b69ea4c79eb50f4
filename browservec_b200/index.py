"""Python host of the B200 quantized flat-scan path.

``AddonQuantIndex`` is the index the reference's ``buildIndex`` would construct
instead of ``QuantIndex`` (src/index.ts:134-140): it implements the
``VectorIndex`` seam (src/index/flat.ts:30-40) plus the duck-typed extras
``queryMasked``/``queryBatch``/``chunkCount``/``ingestMode`` that ``BrowserVec``
probes, over the C ABI of libbvcuda.so.

``BrowserVec`` mirrors the quantized branch of the reference's orchestration
(src/index.ts): store bookkeeping, normalisation, the filter strategy
(exact scan for <= 4096 matches, else an in-index mask), the fetch/re-rank
rule and the id mapping.  The re-rank runs on the GPU inside the search call,
so ``query_batch`` re-ranks as well (the reference's batched branch skips it,
src/index.ts:495-516).  A filter's mask is built by the GPU predicate over
device copies of the metadata columns, once per (filter, store version) --
the reference rebuilds it in JS for every query (src/index.ts:372-395) -- and
a filtered ``query_batch`` searches all its queries in one call instead of
looping over ``query`` (src/index.ts:477-481).
"""
from __future__ import annotations

import ctypes as C
import json
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Mapping, Sequence

import numpy as np

from . import _lib
from .filter import DeviceColumns, FilterColumns, compile_filter, pack_mask

DEFAULT_SEED = 0x9E3779B9          # src/index.ts:71
FILTER_CPU_SCAN_MAX = 4096         # src/index.ts:76
MASK_CACHE_ENTRIES = 16            # filter masks kept per store (least recently used dropped)


def default_rerank_factor(bits: int) -> int:
    """src/index.ts:99-103 (bits 0: the exact fp32 index needs no re-rank)."""
    if bits == 0:
        return 1
    if bits == 1:
        return 32
    return 16 if bits == 4 else 4


@dataclass
class FlatHit:
    row: int
    score: float


@dataclass
class QueryResult:
    id: str
    score: float
    metadata: Mapping[str, Any] | None = None


def _ptr(a: np.ndarray | None):
    """Address of a contiguous array as an int (c_void_p fields take ints)."""
    return None if a is None else a.__array_interface__["data"][0]


def _outputs(nq: int, k: int, F: int, cand: bool):
    """The result arrays of one search carved from a single zeroed buffer:
    (rows[nq,k], scores[nq,k], counts[nq]) and, with cand, (cand_rows[nq,F],
    cand_scores[nq,F], cand_counts[nq]) -- with their addresses."""
    sizes = [nq * k, nq * k, nq] + ([nq * F, nq * F, nq] if cand else [])
    buf = np.zeros(sum(sizes), np.uint32)
    base = _ptr(buf)
    arrs, addrs, off = [], [], 0
    shapes = [(nq, k), (nq, k), (nq,), (nq, F), (nq, F), (nq,)]
    for i, n in enumerate(sizes):
        a = buf[off:off + n]
        if i % 3 == 1:
            a = a.view(np.float32)
        arrs.append(a.reshape(shapes[i]))
        addrs.append(base + 4 * off)
        off += n
    return arrs, addrs


def normalize_rows(m: np.ndarray) -> np.ndarray:
    """store.ts:209-217 for each row: f64 running sum of squares (sequential),
    sqrt, f64 inverse, f32 store.  np.cumsum accumulates strictly in order."""
    m = np.ascontiguousarray(m, dtype=np.float32)
    x = m.astype(np.float64)
    sums = np.cumsum(x * x, axis=1)[:, -1] if m.shape[1] else np.zeros(m.shape[0])
    norm = np.sqrt(sums)
    inv = np.where(norm > 0, 1.0 / np.where(norm > 0, norm, 1.0), 1.0)
    out = (x * inv[:, None]).astype(np.float32)
    return np.where((norm > 0)[:, None], out, m)


class AddonQuantIndex:
    """VectorIndex over libbvcuda (quantized flat scan on one GPU shard)."""

    def __init__(self, dim: int, seed: int = DEFAULT_SEED, rounds: int = 2, bits: int = 8,
                 scoring: str = "asym", device: int = 0, metric: str = "cosine", row_base: int = 0):
        L = _lib.load()
        if metric == "l2":
            raise ValueError("quantized mode supports metric cosine/dot only (l2 quantization is later work)")
        cfg = _lib.BvConfig(dim=dim, bits=bits, metric=_lib.METRIC_DOT if metric == "dot" else _lib.METRIC_COSINE,
                            seed=seed & 0xFFFFFFFF, rounds=rounds, scoring=_lib.SCORING[scoring],
                            device=device, row_base=row_base)
        h = C.c_void_p()
        _lib.check(L.bv_create(C.byref(cfg), C.byref(h)))
        self._h = h
        self._L = L
        self.dim, self.bits, self.seed, self.rounds, self.scoring = dim, bits, seed, rounds, scoring
        self.device = device
        self.row_base = row_base

    # ---- VectorIndex seam -------------------------------------------------
    @property
    def size(self) -> int:
        n = C.c_uint64()
        _lib.check(self._L.bv_size(self._h, C.byref(n)))
        return int(n.value)

    @property
    def chunk_count(self) -> int:
        return 1

    @property
    def ingest_mode(self) -> str:
        return "gpu"

    def append(self, data: np.ndarray, count: int) -> None:
        """quant.ts:129-141 (the error message of quant.ts:130-132)."""
        data = np.ascontiguousarray(data, dtype=np.float32).reshape(-1)
        if data.size != count * self.dim:
            raise ValueError(f"expected {count * self.dim} floats, got {data.size}")
        _lib.check(self._L.bv_append(self._h, _ptr(data), count))

    def append_device(self, ptr: int, count: int, stream: int = 0) -> None:
        _lib.check(self._L.bv_append_device(self._h, C.c_void_p(ptr), count, C.c_void_p(stream)))

    def query(self, q: np.ndarray, k: int) -> list[FlatHit]:
        """quant.ts:165-167: approximate top-k by quantized score."""
        return self.search(q[None, :], k, k, rerank=False)[0]

    def query_masked(self, q: np.ndarray, k: int, mask_words: np.ndarray) -> list[FlatHit]:
        """quant.ts:174-176"""
        return self.search(q[None, :], k, k, rerank=False, mask=mask_words)[0]

    def query_batch(self, packed: np.ndarray, n: int, k: int, fetch: int | None = None,
                    rerank: bool = True, mask: np.ndarray | None = None) -> list[list[FlatHit]]:
        return self.search(np.asarray(packed, np.float32).reshape(n, self.dim), k,
                           fetch if fetch else k, rerank=rerank, mask=mask)

    def search(self, qs: np.ndarray, k: int, fetch: int, rerank: bool = True,
               mask: np.ndarray | None = None, with_candidates: bool = False):
        """k results per query after (optional) exact re-rank of `fetch` candidates."""
        qs = np.ascontiguousarray(qs, dtype=np.float32).reshape(-1, self.dim)
        nq = qs.shape[0]
        F = max(fetch, k)
        o, a = _outputs(nq, k, F, with_candidates)
        out_rows, out_scores, out_counts = o[:3]
        cand = tuple(o[3:]) if with_candidates else (None, None, None)
        ca = a[3:] if with_candidates else (None, None, None)
        m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint32)
        if m is not None:
            need = (self.size + 31) // 32
            if m.size < need:  # scoreMask.ts:68-70
                raise ValueError(f"mask has {m.size} words, need {need} for {self.size} rows")
        args = _lib.BvSearchArgs(queries=_ptr(qs), nq=nq, k=k, fetch=F, rerank=int(rerank),
                                 mask=_ptr(m), mask_words=0 if m is None else m.size,
                                 out_rows=a[0], out_scores=a[1], out_counts=a[2], cand_rows=ca[0],
                                 cand_scores=ca[1], cand_counts=ca[2])
        _lib.check(self._L.bv_search(self._h, C.byref(args)))
        hits = [[FlatHit(int(out_rows[i, j]), float(out_scores[i, j])) for j in range(int(out_counts[i]))]
                for i in range(nq)]
        if with_candidates:
            return hits, cand
        return hits

    def search_arrays(self, qs: np.ndarray, k: int, fetch: int, rerank: bool = True,
                      mask: np.ndarray | None = None):
        """Like search() but returns (rows[nq,k], scores[nq,k], counts[nq], cand_rows, cand_scores,
        cand_counts) numpy arrays."""
        qs = np.ascontiguousarray(qs, dtype=np.float32).reshape(-1, self.dim)
        nq = qs.shape[0]
        F = max(fetch, k)
        o, a = _outputs(nq, k, F, True)
        m = None if mask is None else np.ascontiguousarray(mask, dtype=np.uint32)
        args = _lib.BvSearchArgs(queries=_ptr(qs), nq=nq, k=k, fetch=F, rerank=int(rerank),
                                 mask=_ptr(m), mask_words=0 if m is None else m.size,
                                 out_rows=a[0], out_scores=a[1], out_counts=a[2],
                                 cand_rows=a[3], cand_scores=a[4], cand_counts=a[5])
        _lib.check(self._L.bv_search(self._h, C.byref(args)))
        return tuple(o)

    def search_device(self, q_ptr: int, nq: int, k: int, fetch: int, rerank: bool,
                      out_rows_ptr: int, out_scores_ptr: int, out_counts_ptr: int,
                      mask_ptr: int = 0, mask_words: int = 0, stream: int = 0) -> None:
        """Device-pointer search enqueued on `stream` (no host synchronisation)."""
        args = _lib.BvSearchArgs(queries=q_ptr, nq=nq, k=k, fetch=max(fetch, k), rerank=int(rerank),
                                 mask=mask_ptr or None, mask_words=mask_words, out_rows=out_rows_ptr,
                                 out_scores=out_scores_ptr, out_counts=out_counts_ptr)
        _lib.check(self._L.bv_search_async(self._h, C.byref(args), C.c_void_p(stream)))

    def search_device_cand(self, q_ptr: int, nq: int, k: int, fetch: int, rerank: bool,
                           out_rows_ptr: int, out_scores_ptr: int, out_counts_ptr: int,
                           mask_ptr: int = 0, mask_words: int = 0, stream: int = 0,
                           cand_rows_ptr: int = 0, cand_scores_ptr: int = 0, cand_counts_ptr: int = 0,
                           cand_exact_ptr: int = 0) -> None:
        """search_device with the candidate outputs (per-query scans)."""
        args = _lib.BvSearchArgs(queries=q_ptr, nq=nq, k=k, fetch=max(fetch, k), rerank=int(rerank),
                                 mask=mask_ptr or None, mask_words=mask_words, out_rows=out_rows_ptr,
                                 out_scores=out_scores_ptr, out_counts=out_counts_ptr,
                                 cand_rows=cand_rows_ptr or None, cand_scores=cand_scores_ptr or None,
                                 cand_counts=cand_counts_ptr or None, cand_exact=cand_exact_ptr or None)
        _lib.check(self._L.bv_search_async(self._h, C.byref(args), C.c_void_p(stream)))

    def search_batch_device(self, q_ptr: int, nq: int, k: int, fetch: int, rerank: bool,
                            out_rows_ptr: int, out_scores_ptr: int, out_counts_ptr: int,
                            mask_ptr: int = 0, mask_words: int = 0, stream: int = 0,
                            cand_rows_ptr: int = 0, cand_scores_ptr: int = 0, cand_counts_ptr: int = 0,
                            cand_exact_ptr: int = 0) -> None:
        """Batched search on the tensor cores (integer scorings), device
        pointers; returns once `stream` has finished the batch."""
        args = _lib.BvSearchArgs(queries=q_ptr, nq=nq, k=k, fetch=max(fetch, k), rerank=int(rerank),
                                 mask=mask_ptr or None, mask_words=mask_words, out_rows=out_rows_ptr,
                                 out_scores=out_scores_ptr, out_counts=out_counts_ptr,
                                 cand_rows=cand_rows_ptr or None, cand_scores=cand_scores_ptr or None,
                                 cand_counts=cand_counts_ptr or None, cand_exact=cand_exact_ptr or None)
        _lib.check(self._L.bv_search_batch(self._h, C.byref(args), C.c_void_p(stream)))

    def search_masked(self, qs: np.ndarray, k: int, fetch: int, rerank: bool, mask_dev) -> list[list[FlatHit]]:
        """Search with a score mask already on the device (uint32 words as a
        CUDA tensor, e.g. DeviceColumns.mask): the queries go to the device,
        integer scorings of 64+ queries run as one tensor-core batch, the
        results come back to the host."""
        import torch

        qs = np.ascontiguousarray(qs, dtype=np.float32).reshape(-1, self.dim)
        nq = qs.shape[0]
        F = max(fetch, k)
        dev = mask_dev.device
        if getattr(self, "_stream", None) is None:
            self._stream = torch.cuda.Stream(device=dev)
        st = self._stream
        st.wait_stream(torch.cuda.current_stream(dev))  # the mask was built on the current stream
        with torch.cuda.stream(st):
            q = torch.from_numpy(qs).to(dev, non_blocking=False)
            out = torch.empty(nq * (2 * k + 1), dtype=torch.int32, device=dev)
            args = _lib.BvSearchArgs(queries=q.data_ptr(), nq=nq, k=k, fetch=F, rerank=int(rerank),
                                     mask=mask_dev.data_ptr(), mask_words=mask_dev.numel(),
                                     out_rows=out.data_ptr(), out_scores=out[nq * k:].data_ptr(),
                                     out_counts=out[2 * nq * k:].data_ptr())
            batched = self.scoring != "asym" and self.bits != 0 and nq >= 64
            fn = self._L.bv_search_batch if batched else self._L.bv_search_async
            _lib.check(fn(self._h, C.byref(args), C.c_void_p(st.cuda_stream)))
            host = out.cpu().numpy()
        st.synchronize()
        rows = host[:nq * k].reshape(nq, k)
        scores = host[nq * k:2 * nq * k].view(np.float32).reshape(nq, k)
        counts = host[2 * nq * k:]
        return [[FlatHit(int(rows[i, j]), float(scores[i, j])) for j in range(int(counts[i]))]
                for i in range(nq)]

    def search_candidates(self, qs: np.ndarray, lists, k: int, fetch: int, rerank: bool = True,
                          with_candidates: bool = False):
        """The IVF x quant candidate-list scan (src/index/ivfquant.ts:468-490):
        query i is scored against the rows lists[i] only (its probed lists'
        rows).  Returns (rows, scores, counts[, cand_rows, cand_scores,
        cand_counts]) numpy arrays, rows global."""
        import torch

        qs = np.ascontiguousarray(qs, dtype=np.float32).reshape(-1, self.dim)
        nq = qs.shape[0]
        F = max(fetch, k)
        lists = [np.ascontiguousarray(x, dtype=np.uint32).reshape(-1) for x in lists]
        if len(lists) != nq:
            raise ValueError(f"{nq} queries but {len(lists)} candidate lists")
        offs = np.zeros(nq + 1, np.uint32)
        offs[1:] = np.cumsum([x.size for x in lists])
        dev = torch.device("cuda", self.device)
        if getattr(self, "_stream", None) is None:
            self._stream = torch.cuda.Stream(device=dev)
        st = self._stream
        with torch.cuda.stream(st):
            q = torch.from_numpy(qs).to(dev)
            flat = np.concatenate(lists) if int(offs[-1]) else np.zeros(1, np.uint32)
            cand = torch.from_numpy(flat.view(np.int32)).to(dev)
            out = torch.empty(nq * (2 * k + 1) + (nq * (2 * F + 1) if with_candidates else 0), dtype=torch.int32,
                              device=dev)
            b = 2 * nq * k + nq
            args = _lib.BvSearchArgs(queries=q.data_ptr(), nq=nq, k=k, fetch=F, rerank=int(rerank),
                                     out_rows=out.data_ptr(), out_scores=out[nq * k:].data_ptr(),
                                     out_counts=out[2 * nq * k:].data_ptr(),
                                     cand_rows=out[b:].data_ptr() if with_candidates else None,
                                     cand_scores=out[b + nq * F:].data_ptr() if with_candidates else None,
                                     cand_counts=out[b + 2 * nq * F:].data_ptr() if with_candidates else None)
            _lib.check(self._L.bv_search_rows(self._h, C.byref(args), _ptr(offs), C.c_void_p(cand.data_ptr()),
                                              C.c_void_p(st.cuda_stream)))
            host = out.cpu().numpy()
        st.synchronize()
        res = (host[:nq * k].view(np.uint32).reshape(nq, k), host[nq * k:2 * nq * k].view(np.float32).reshape(nq, k),
               host[2 * nq * k:b].view(np.uint32))
        if with_candidates:
            res += (host[b:b + nq * F].view(np.uint32).reshape(nq, F),
                    host[b + nq * F:b + 2 * nq * F].view(np.float32).reshape(nq, F),
                    host[b + 2 * nq * F:].view(np.uint32))
        return res

    def set_scoring(self, scoring: str) -> None:
        """Score later searches with another mode (codes are shared by all modes)."""
        _lib.check(self._L.bv_set_scoring(self._h, _lib.SCORING[scoring]))
        self.scoring = scoring

    def set_batch_timing(self, enable: bool) -> None:
        """Record the device time of each phase of batched searches (CUDA events)."""
        _lib.check(self._L.bv_set_batch_timing(self._h, int(enable)))

    def batch_profile(self) -> dict:
        """Phase device times (ms) and counts of the last batched search."""
        pr = _lib.BvBatchProfile()
        _lib.check(self._L.bv_last_batch_profile(self._h, C.byref(pr)))
        return {f: getattr(pr, f) for f, _ in pr._fields_}

    def query_rows_exact(self, q: np.ndarray, rows: np.ndarray, k: int) -> list[FlatHit]:
        """index.ts:445-464 on the GPU (rows <= 4096)."""
        q = np.ascontiguousarray(q, dtype=np.float32)
        rows = np.ascontiguousarray(rows, dtype=np.uint32)
        ro = np.zeros(max(k, 1), np.uint32)
        so = np.zeros(max(k, 1), np.float32)
        n = C.c_uint32()
        _lib.check(self._L.bv_query_rows_exact(self._h, _ptr(q), _ptr(rows), rows.size, k, _ptr(ro),
                                               _ptr(so), C.byref(n)))
        return [FlatHit(int(ro[i]), float(so[i])) for i in range(n.value)]

    def export_codes(self, row0: int = 0, count: int | None = None):
        count = self.size - row0 if count is None else count
        wpr = {8: 4, 4: 8, 1: 32}[self.bits]
        P = 4
        while P < self.dim:
            P <<= 1
        words = np.zeros((count, P // wpr), np.uint32)
        scales = np.zeros(count, np.float32)
        _lib.check(self._L.bv_export_codes(self._h, row0, count, _ptr(words), _ptr(scales)))
        return words, scales

    def export_originals(self, row0: int = 0, count: int | None = None) -> np.ndarray:
        """The stored (normalized) fp32 rows, (count, dim)."""
        count = self.size - row0 if count is None else count
        out = np.empty((count, self.dim), np.float32)
        _lib.check(self._L.bv_export_originals(self._h, row0, count, _ptr(out)))
        return out

    def stats(self) -> dict:
        s = _lib.BvStats()
        _lib.check(self._L.bv_get_stats(self._h, C.byref(s)))
        return {f: getattr(s, f) for f, _ in s._fields_}

    def set_phase_trace(self, ptr: int, capacity: int) -> None:
        """Device buffer (u64) receiving per-phase timestamps of each scan launch."""
        _lib.check(self._L.bv_set_phase_trace(self._h, C.c_void_p(ptr) if ptr else None, capacity))

    def last_launches(self) -> int:
        n = C.c_uint32()
        _lib.check(self._L.bv_launches_last_search(self._h, C.byref(n)))
        return int(n.value)

    def destroy(self) -> None:
        if getattr(self, "_h", None):
            self._L.bv_destroy(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.destroy()
        except Exception:
            pass


class PreparedSearch:
    """A host-memory search request whose buffers and argument block are made
    once: each call copies a batch of queries in and runs bv_search (the
    call search() makes), so a caller issuing one query at a time pays no
    per-call allocation.  The returned arrays are reused by the next call."""

    def __init__(self, index: "AddonQuantIndex", nq: int, k: int, fetch: int, rerank: bool = True):
        self.q = np.zeros((nq, index.dim), np.float32)
        self.rows = np.zeros((nq, k), np.uint32)
        self.scores = np.zeros((nq, k), np.float32)
        self.counts = np.zeros(nq, np.uint32)
        self.args = _lib.BvSearchArgs(queries=self.q.ctypes.data, nq=nq, k=k, fetch=max(fetch, k),
                                      rerank=int(rerank), mask=None, mask_words=0,
                                      out_rows=self.rows.ctypes.data, out_scores=self.scores.ctypes.data,
                                      out_counts=self.counts.ctypes.data)
        self._ref = C.byref(self.args)
        self._fn = index._L.bv_search
        self._index = index

    def __call__(self, qs: np.ndarray):
        np.copyto(self.q, qs.reshape(self.q.shape), casting="same_kind")
        rc = self._fn(self._index._h, self._ref)
        if rc:
            _lib.check(rc)
        return self.rows, self.scores, self.counts


class AsyncSearchList:
    """Device searches submitted together by one bv_search_async_n call.

    entries: (index, q_ptr, k, fetch, rerank, out_rows_ptr, out_scores_ptr, out_counts_ptr) per
    search, nq = 1 each; the argument array is built once and can be submitted any number of times
    (the pointers are fixed)."""

    def __init__(self, entries):
        n = len(entries)
        if n == 0:
            raise ValueError("no searches")
        self.n = n
        self._keep = [e[0] for e in entries]
        self._idx = (C.c_void_p * n)(*[e[0]._h.value for e in entries])
        self._args = (_lib.BvSearchArgs * n)()
        for i, (ix, q, k, fetch, rerank, r, s, c) in enumerate(entries):
            self._args[i] = _lib.BvSearchArgs(queries=q, nq=1, k=k, fetch=max(fetch, k), rerank=int(rerank),
                                              mask=None, mask_words=0, out_rows=r, out_scores=s, out_counts=c)
        self._L = entries[0][0]._L

    def submit(self, stream: int = 0) -> None:
        _lib.check(self._L.bv_search_async_n(self._idx, self._args, self.n, C.c_void_p(stream)))


@dataclass
class _Entry:
    id: str
    row: int
    metadata: Mapping[str, Any] | None = None


@dataclass
class _Store:
    """src/store/store.ts: id<->row map, tombstones, metadata columns."""

    dimension: int
    metric: str
    normalize: bool
    by_id: dict = field(default_factory=dict)
    by_row: list = field(default_factory=list)
    deleted: set = field(default_factory=set)
    columns: FilterColumns = field(default_factory=FilterColumns)


class BrowserVec:
    """The flat branches of src/index.ts over AddonQuantIndex: quantBits 1/4/8
    (the quantized scan, QuantIndex) and 0 (the exact fp32 scan, FlatIndex,
    src/index/flat.ts:132-211, scored with the WASM-SIMD f32 arithmetic of the
    reference's CPU path)."""

    def __init__(self, dimension: int, metric: str = "cosine", normalize: bool | None = None,
                 quant_bits: int = 8, quant: Mapping[str, Any] | None = None, scoring: str = "asym",
                 device: int = 0):
        if not isinstance(dimension, int) or dimension <= 0:
            raise ValueError(f"dimension must be a positive integer, got {dimension}")
        quant = dict(quant or {})
        if quant_bits not in (0, 1, 4, 8):
            raise ValueError(f"quantBits {quant_bits} not supported (ships 0, 1, 4, 8)")
        if quant_bits == 0:
            scoring = "asym"  # exact scores: no quantized scoring mode applies
        self.store = _Store(dimension, metric, metric == "cosine" if normalize is None else normalize)
        self.quant_bits = quant_bits
        self.rerank_factor = int(quant.get("rerankFactor", default_rerank_factor(quant_bits)))
        self.index = AddonQuantIndex(dimension, quant.get("seed", DEFAULT_SEED), quant.get("rounds", 2),
                                     quant_bits, scoring, device, metric)
        self.last_query_ms: float | None = None
        self.last_query_gpu_ms: float | None = None
        self._version = 0       # bumped by every add and delete
        self._dev = None        # (version, DeviceColumns, live-row mask words) on the index's GPU
        self._masks: OrderedDict = OrderedDict()  # (filter, version) -> (mask words, matches, rows)

    @classmethod
    def create(cls, config: Mapping[str, Any]) -> "BrowserVec":
        """BrowserVec.create (src/index.ts:232-263), quantized flat stores only."""
        return cls(config["dimension"], config.get("metric", "cosine"), config.get("normalize"),
                   config.get("quantBits", 8), config.get("quant"), config.get("scoring", "asym"),
                   config.get("device", 0))

    # ---- ingest -----------------------------------------------------------
    def add_batch(self, records: Sequence[Mapping[str, Any]]) -> None:
        """src/index.ts:293-305"""
        if not records:
            return
        d = self.store.dimension
        vecs = np.zeros((len(records), d), np.float32)
        metas = []
        for i, r in enumerate(records):
            v = np.asarray(r["vector"], np.float32)
            if v.size != d:
                raise ValueError(f"vector dim {v.size} != store dim {d}")
            if r["id"] in self.store.by_id:
                raise ValueError(f"duplicate id: {r['id']}")
            vecs[i] = v
            row = len(self.store.by_row)
            e = _Entry(r["id"], row, r.get("metadata"))
            self.store.by_id[r["id"]] = e
            self.store.by_row.append(e)
            metas.append(r.get("metadata"))
        if self.store.normalize:
            vecs = normalize_rows(vecs)
        self.store.columns.append(metas)
        self.index.append(vecs, len(records))
        self._version += 1

    def add(self, record: Mapping[str, Any]) -> None:
        self.add_batch([record])

    def add_arrays(self, vectors: np.ndarray, ids: Sequence[str] | None = None,
                   columns: Mapping[str, np.ndarray] | None = None,
                   dictionaries: Mapping[str, list] | None = None) -> None:
        """Bulk ingest of prepared arrays (rows normalized like store.prepare)."""
        vectors = np.ascontiguousarray(vectors, np.float32)
        n = vectors.shape[0]
        base = len(self.store.by_row)
        for i in range(n):
            rid = ids[i] if ids is not None else f"v{base + i}"
            e = _Entry(rid, base + i, None)
            self.store.by_id[rid] = e
            self.store.by_row.append(e)
        if self.store.normalize:
            vectors = normalize_rows(vectors)
        if columns:
            self.store.columns.append_columns(n, columns, dictionaries)
        else:
            self.store.columns.append([None] * n)
        self.index.append(vectors, n)
        self._version += 1

    # ---- snapshots (src/index.ts:608-700, src/persist/format.ts) ----------
    def export(self) -> bytes:
        """BrowserVec.export: a snapshot of the live rows (tombstones compacted
        out, src/index.ts:646-671), in the reference's format."""
        from .persist import serialize

        live = [e for e in self.store.by_row if e.row not in self.store.deleted]
        vecs = self.index.export_originals() if self.index.size else np.zeros((0, self.store.dimension), np.float32)
        if self.store.deleted:
            vecs = vecs[np.array([e.row for e in live], np.int64)]
        entries = [{"id": e.id, "metadata": e.metadata} for e in live]
        return serialize(self.store.dimension, self.store.metric, self.store.normalize, entries, vecs)

    @classmethod
    def import_(cls, buf, config: Mapping[str, Any] | None = None) -> "BrowserVec":
        """BrowserVec.import (src/index.ts:616-644): a store built from a
        snapshot (quantBits from `config`, default 0 as in the reference)."""
        from .persist import deserialize

        snap = deserialize(buf)
        config = dict(config or {})
        db = cls(snap.dimension, snap.metric, snap.normalize, config.get("quantBits", 0), config.get("quant"),
                 config.get("scoring", "asym"), config.get("device", 0))
        db.load_snapshot(snap)
        return db

    def load_snapshot(self, snap) -> None:
        """src/index.ts:673-700: ids and metadata into the store, and the
        stored vectors (already normalized when the store normalizes) into
        the index in one bulk append -- the GPU encodes them -- instead of a
        per-row insert."""
        if self.count > 0 or self.store.by_row:
            raise ValueError("cannot load into a non-empty store")
        if snap.dimension != self.store.dimension:
            raise ValueError(f"snapshot dim {snap.dimension} != store dim {self.store.dimension}")
        if snap.metric != self.store.metric:
            raise ValueError(f"snapshot metric {snap.metric} != store metric {self.store.metric}")
        metas = []
        for row, e in enumerate(snap.entries):
            if e["id"] in self.store.by_id:
                raise ValueError(f"duplicate id: {e['id']}")
            ent = _Entry(e["id"], row, e.get("metadata"))
            self.store.by_id[e["id"]] = ent
            self.store.by_row.append(ent)
            metas.append(e.get("metadata"))
        self.store.columns.append(metas)
        if snap.count:
            self.index.append(snap.vectors, snap.count)
        self._version += 1

    def delete(self, id: str) -> bool:
        e = self.store.by_id.pop(id, None)
        if e is None:
            return False
        self.store.deleted.add(e.row)
        self._version += 1
        return True

    @property
    def count(self) -> int:
        return len(self.store.by_id)

    # ---- query ------------------------------------------------------------
    def _prep_query(self, query) -> np.ndarray:
        q = np.asarray(query, np.float32).reshape(-1).copy()
        if q.size != self.store.dimension:
            raise ValueError(f"query dim {q.size} != store dim {self.store.dimension}")
        if self.store.normalize:
            q = normalize_rows(q[None, :])[0]
        return q

    def _meta_of(self, row: int):
        return self.store.by_row[row].metadata

    def _device_mask(self, flt: Mapping[str, Any]):
        """The score mask of a filter -- its rows that are not deleted
        (src/index.ts:372-386) -- built by the GPU predicate over device
        copies of the metadata columns and kept per (filter, store version):
        (mask words as a CUDA tensor, match count, the matching rows when at
        most FILTER_CPU_SCAN_MAX, else None)."""
        import torch

        key = (json.dumps(flt, sort_keys=True, default=repr), self._version)
        hit = self._masks.get(key)
        if hit is not None:
            self._masks.move_to_end(key)
            return hit
        dev = torch.device("cuda", self.index.device)
        if self._dev is None or self._dev[0] != self._version:
            dc = DeviceColumns.from_host(self.store.columns, dev)
            live = np.ones(len(self.store.by_row), bool)
            if self.store.deleted:
                live[np.fromiter(self.store.deleted, np.int64)] = False
            live_w = torch.from_numpy(pack_mask(live).view(np.int32)).to(dev)
            self._dev = (self._version, dc, live_w)
            self._masks.clear()  # masks of older versions are stale
        _, dc, live_w = self._dev
        m = dc.mask(flt, live=live_w)
        if not hasattr(self, "_popc"):
            self._popc = torch.tensor([bin(i).count("1") for i in range(256)], dtype=torch.int64, device=dev)
        b = m.view(torch.uint8)
        count = int(self._popc[b.long()].sum().item())
        rows = None
        if 0 < count <= FILTER_CPU_SCAN_MAX:
            bits = ((b.unsqueeze(1) >> torch.arange(8, device=dev, dtype=torch.uint8)) & 1).flatten()
            rows = torch.nonzero(bits).squeeze(1).cpu().numpy().astype(np.uint32)
        entry = (m, count, rows)
        self._masks[key] = entry
        while len(self._masks) > MASK_CACHE_ENTRIES:
            self._masks.popitem(last=False)
        return entry

    def _fetch(self, k: int, masked: bool, rerank: bool | None):
        """src/index.ts:405-417: k_eff (oversampled by the tombstones unless a
        mask already drops them) and the candidate fetch."""
        total = self.index.size
        k_eff = min(total, k) if masked else min(total, k + len(self.store.deleted))
        do_rerank = rerank if rerank is not None else self.rerank_factor > 1
        fetch = min(total, max(k_eff, k_eff * self.rerank_factor)) if do_rerank else k_eff
        return k_eff, fetch, do_rerank

    def query(self, query, k: int = 10, filter: Mapping[str, Any] | None = None,
              rerank: bool | None = None) -> list[QueryResult]:
        """src/index.ts:343-436 (quantized branch)."""
        import time

        q = self._prep_query(query)
        predicate = compile_filter(filter) if filter else None
        t0 = time.perf_counter()
        if predicate is not None:
            m, count, rows = self._device_mask(filter)
            if count == 0:
                return []
            if rows is not None:
                return self._query_rows_exact(q, rows, k)
            k_eff, fetch, do_rerank = self._fetch(k, True, rerank)
            if k_eff <= 0:
                return []
            hits = self.index.search_masked(q[None, :], k_eff, fetch, do_rerank, m)[0]
            self.last_query_ms = (time.perf_counter() - t0) * 1e3
            self.last_query_gpu_ms = None
            return self._map_hits(hits, k, predicate)
        k_eff, fetch, do_rerank = self._fetch(k, False, rerank)
        if k_eff <= 0:
            return []
        hits = self.index.search(q[None, :], k_eff, fetch, rerank=do_rerank)[0]
        self.last_query_ms = (time.perf_counter() - t0) * 1e3
        self.last_query_gpu_ms = min(self.index.stats()["last_query_gpu_ms"], self.last_query_ms)
        return self._map_hits(hits, k, predicate)

    def _map_hits(self, hits, k, predicate=None) -> list[QueryResult]:
        out = []
        for h in hits:
            if self.store.deleted and h.row in self.store.deleted:
                continue
            e = self.store.by_row[h.row]
            if predicate is not None and not predicate(e.metadata):
                continue
            out.append(QueryResult(e.id, h.score, e.metadata))
            if len(out) == k:
                break
        return out

    def _query_rows_exact(self, q, rows, k) -> list[QueryResult]:
        """src/index.ts:445-464"""
        hits = self.index.query_rows_exact(q, rows, k)
        return [QueryResult(self.store.by_row[h.row].id, h.score, self.store.by_row[h.row].metadata)
                for h in hits]

    def query_batch(self, queries, k: int = 10, filter: Mapping[str, Any] | None = None,
                    rerank: bool | None = None) -> list[list[QueryResult]]:
        """src/index.ts:473-517, with the re-rank the batched reference branch
        lacks; a filtered batch shares one device mask and one search call
        (the reference loops over query(), rebuilding the mask each time)."""
        queries = list(queries) if not isinstance(queries, np.ndarray) else queries
        if len(queries) == 0:
            return []
        qs = np.stack([self._prep_query(q) for q in queries])
        if filter:
            predicate = compile_filter(filter)
            m, count, rows = self._device_mask(filter)
            if count == 0:
                return [[] for _ in range(qs.shape[0])]
            if rows is not None:
                return [self._query_rows_exact(q, rows, k) for q in qs]
            k_eff, fetch, do_rerank = self._fetch(k, True, rerank)
            batch = self.index.search_masked(qs, k_eff, fetch, do_rerank, m)
            return [self._map_hits(h, k, predicate) for h in batch]
        k_eff, fetch, do_rerank = self._fetch(k, False, rerank)
        if k_eff <= 0:
            return [[] for _ in range(qs.shape[0])]
        batch = self.index.search(qs, k_eff, fetch, rerank=do_rerank)
        return [self._map_hits(h, k) for h in batch]

    def stats(self) -> dict:
        """src/index.ts:702-750 (fields this path produces)."""
        s = {"count": self.count, "dimension": self.store.dimension, "metric": self.store.metric,
             "device": "cuda", "quantBits": self.quant_bits}
        if self.store.deleted:
            s["deleted"] = len(self.store.deleted)
        if self.last_query_ms is not None:
            s["lastQueryMs"] = self.last_query_ms
            s["lastQueryGpuMs"] = self.last_query_gpu_ms
            s["lastQueryCpuMs"] = self.last_query_ms - (self.last_query_gpu_ms or 0.0)
        s["ingest"] = self.index.ingest_mode
        return s

    def destroy(self) -> None:
        self.index.destroy()
