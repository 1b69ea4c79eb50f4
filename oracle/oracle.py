"""ctypes wrapper over the C oracle (``oracle/libbv_oracle.so``).

TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA path and the CPU
baseline of ``bench.py``.  The product package ``browservec_b200`` never
imports this module.  Each wrapper names the reference file:line (TypeScript,
sharma-open-source/browservec) that the C function restates.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libbv_oracle.so")

MODE_ASYM, MODE_INT, MODE_HAMMING = 0, 1, 2
DEFAULT_SEED = 0x9E3779B9  # index.ts:71


def build() -> str:
    """Compile the oracle with its Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P = C.c_void_p
        i32, i64, u32 = C.c_int, C.c_int64, C.c_uint32
        sig = {
            "bvo_mulberry32_next": (u32, [P]),
            "bvo_mulberry32_doubles": (None, [u32, P, i64]),
            "bvo_random_signs": (None, [P, i32, u32]),
            "bvo_pad_to_pow2": (i32, [i32]),
            "bvo_fwht": (None, [P, i32]),
            "bvo_rotator_signs": (i32, [i32, u32, i32, P]),
            "bvo_rotate": (None, [P, i32, i32, i32, P, P]),
            "bvo_quantize_row8": (i32, [P, i32, P, P]),
            "bvo_quantize_row4": (i32, [P, i32, P, P]),
            "bvo_quantize_row1": (i32, [P, i32, P, P]),
            "bvo_dequant_row8": (None, [P, i32, C.c_float, P]),
            "bvo_dequant_row4": (None, [P, i32, C.c_float, P]),
            "bvo_dequant_row1": (None, [P, i32, C.c_float, P]),
            "bvo_words_per_row": (i32, [i32, i32]),
            "bvo_encode": (i32, [P, i64, i32, u32, i32, i32, P, P, P]),
            "bvo_prepare_query": (None, [P, i32, i32, i32, i32, i32, P, P, P, P]),
            "bvo_score_rows": (None, [i32, i32, i32, P, P, i64, P, P, C.c_float, P]),
            "bvo_key": (C.c_uint64, [C.c_float, u32]),
            "bvo_topk": (i32, [P, i64, P, i32, P, P]),
            "bvo_topk_ref": (i32, [P, i64, i32, P, P]),
            "bvo_merge_partials_ref": (i32, [P, P, i64, i64, i32, P, P]),
            "bvo_dot_row": (C.c_double, [P, P, i32]),
            "bvo_normalize": (None, [P, i32]),
            "bvo_query": (i32, [i32, i32, i32, i32, P, i32, P, P, P, i64, P, P, i32, i32, i32,
                                P, P, P, P]),
            "bvo_query_rows_exact": (i32, [P, i32, P, i64, P, i32, P, P]),
            "bvo_wasm_dot": (None, [P, P, P, i64, i32]),
            "bvo_cpu_index_query": (i32, [P, i64, i32, P, i32, P, P]),
            "bvo_cpu_index_query_batch": (i32, [P, i64, i32, P, i32, i32, i32, P, P]),
            "bvo_query_batch": (i32, [i32, i32, i32, i32, P, i32, P, P, P, i64, P, P, i32, i32,
                                      i32, i32, i32, P, P, P]),
            "bvo_cpu_sharded_query_batch": (i32, [P, P, P, P, i32, i64, i32, P, i32, i32, i32, P, P, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _u32(a):
    return np.ascontiguousarray(a, dtype=np.uint32)


# ---------------------------------------------------------------- prng.ts
def mulberry32(seed: int, n: int) -> np.ndarray:
    """prng.ts:5-14 -- n successive rng() values (f64)."""
    out = np.empty(n, np.float64)
    lib().bvo_mulberry32_doubles(seed & 0xFFFFFFFF, _p(out), n)
    return out


def random_signs(n: int, seed: int) -> np.ndarray:
    """prng.ts:17-22"""
    out = np.empty(n, np.float32)
    lib().bvo_random_signs(_p(out), n, seed & 0xFFFFFFFF)
    return out


# ------------------------------------------------------------- rotator.ts
def pad_to_pow2(n: int) -> int:
    """rotator.ts:16-21"""
    return lib().bvo_pad_to_pow2(n)


def fwht(a) -> np.ndarray:
    """rotator.ts:46-58 (returns a transformed copy)."""
    a = _f32(a).copy()
    lib().bvo_fwht(_p(a), a.size)
    return a


def rotator_signs(dim: int, seed: int = DEFAULT_SEED, rounds: int = 2) -> np.ndarray:
    """rotator.ts:44-58 -- (rounds, P) pre-scaled sign vectors."""
    P = pad_to_pow2(dim)
    out = np.empty((max(rounds, 1), P), np.float32)
    lib().bvo_rotator_signs(dim, seed & 0xFFFFFFFF, rounds, _p(out))
    return out[:rounds]


def rotate(x, dim: int, seed: int = DEFAULT_SEED, rounds: int = 2, signs=None) -> np.ndarray:
    """rotator.ts:60-70"""
    P = pad_to_pow2(dim)
    s = rotator_signs(dim, seed, rounds) if signs is None else _f32(signs)
    x = _f32(x)
    dst = np.empty(P, np.float32)
    lib().bvo_rotate(_p(s), rounds, dim, P, _p(x), _p(dst))
    return dst


# --------------------------------------------------------------- codec.ts
def quantize_row(rot, bits: int):
    """codec.ts:32-54 (8), :85-108 (4), :135-154 (1) -> (words, scale)."""
    rot = _f32(rot)
    n = rot.size
    per = {8: 4, 4: 8, 1: 32}[bits]
    words = np.zeros(max(n // per, 1), np.uint32)
    scale = np.zeros(1, np.float32)
    fn = {8: lib().bvo_quantize_row8, 4: lib().bvo_quantize_row4, 1: lib().bvo_quantize_row1}[bits]
    rc = fn(_p(rot), n, _p(words), _p(scale))
    if rc != 0:
        raise ValueError(f"paddedDim must be a multiple of {per}" if bits != 8 else
                         "paddedDim must be a multiple of 4")
    return words[: n // per], float(scale[0])


def dequant_row(words, scale: float, bits: int) -> np.ndarray:
    """codec.ts:56-66 / :110-120 / :156-167"""
    words = _u32(words)
    per = {8: 4, 4: 8, 1: 32}[bits]
    out = np.empty(words.size * per, np.float32)
    fn = {8: lib().bvo_dequant_row8, 4: lib().bvo_dequant_row4, 1: lib().bvo_dequant_row1}[bits]
    fn(_p(words), words.size, C.c_float(scale), _p(out))
    return out


def words_per_row(P: int, bits: int) -> int:
    return lib().bvo_words_per_row(P, bits)


def encode(data, dim: int, bits: int, seed: int = DEFAULT_SEED, rounds: int = 2,
           want_rotated: bool = False):
    """encode.ts:64-78 -> (words[count, wpr], scales[count], rotated|None)."""
    data = _f32(data).reshape(-1)
    if data.size % dim:
        raise ValueError(f"expected {((data.size // dim) + 1) * dim} floats, got {data.size}")
    count = data.size // dim
    P = pad_to_pow2(dim)
    wpr = words_per_row(P, bits)
    words = np.empty((count, wpr), np.uint32)
    scales = np.empty(count, np.float32)
    rot = np.empty((count, P), np.float32) if want_rotated else None
    rc = lib().bvo_encode(_p(data), count, dim, seed & 0xFFFFFFFF, rounds, bits, _p(words),
                          _p(scales), _p(rot))
    if rc != 0:
        raise ValueError("encode failed")
    return words, scales, rot


# ---------------------------------------------------------------- scoring
def prepare_query(q, dim: int, bits: int, mode: int, seed: int = DEFAULT_SEED, rounds: int = 2):
    P = pad_to_pow2(dim)
    s = rotator_signs(dim, seed, rounds)
    q = _f32(q)
    rq = np.empty(P, np.float32)
    qw = np.zeros(P // 4 + 1, np.uint32)
    qs = np.zeros(1, np.float32)
    lib().bvo_prepare_query(_p(s), rounds, dim, P, bits, mode, _p(q), _p(rq), _p(qw), _p(qs))
    return rq, qw, float(qs[0])


def score_rows(codes, scales, q, dim: int, bits: int, mode: int = MODE_ASYM,
               seed: int = DEFAULT_SEED, rounds: int = 2) -> np.ndarray:
    """Canonical quantized scores of every row (distanceQ8/Q4/Q1 restated)."""
    codes = _u32(codes)
    scales = _f32(scales)
    P = pad_to_pow2(dim)
    rq, qw, qs = prepare_query(q, dim, bits, mode, seed, rounds)
    out = np.empty(scales.size, np.float32)
    lib().bvo_score_rows(bits, mode, P, _p(codes), _p(scales), scales.size, _p(rq), _p(qw),
                         C.c_float(qs), _p(out))
    return out


def key(score: float, row: int) -> int:
    return int(lib().bvo_key(C.c_float(score), row))


def topk(scores, k: int, mask=None):
    """Canonical top-k (score desc, row asc) -> (rows, scores)."""
    scores = _f32(scores)
    m = None if mask is None else _u32(mask)
    rows = np.empty(max(k, 1), np.uint32)
    out = np.empty(max(k, 1), np.float32)
    n = lib().bvo_topk(_p(scores), scores.size, _p(m), k, _p(rows), _p(out))
    return rows[:n], out[:n]


def topk_ref(scores, k: int):
    """flat.ts:217-239 -- the reference heap selection, exactly."""
    scores = _f32(scores)
    rows = np.empty(max(k, 1), np.uint32)
    out = np.empty(max(k, 1), np.float32)
    n = lib().bvo_topk_ref(_p(scores), scores.size, k, _p(rows), _p(out))
    return rows[:n], out[:n]


def merge_partials_ref(scores, rows, n: int, k: int):
    """gpuTopk.ts:160-189"""
    scores, rows = _f32(scores), _u32(rows)
    ro = np.empty(max(k, 1), np.uint32)
    so = np.empty(max(k, 1), np.float32)
    c = lib().bvo_merge_partials_ref(_p(scores), _p(rows), scores.size, n, k, _p(ro), _p(so))
    return ro[:c], so[:c]


def dot_row(row, q) -> float:
    """store.ts:114-130"""
    row, q = _f32(row), _f32(q)
    return float(lib().bvo_dot_row(_p(row), _p(q), row.size))


def normalize(v) -> np.ndarray:
    """store.ts:209-217 (returns a normalized copy)."""
    v = _f32(v).copy()
    lib().bvo_normalize(_p(v), v.size)
    return v


def normalize_rows(m) -> np.ndarray:
    m = _f32(m).copy()
    for i in range(m.shape[0]):
        lib().bvo_normalize(_p(m[i]), m.shape[1])
    return m


def fetch_count(total: int, k: int, rerank_factor: int, rerank: bool = True) -> int:
    """index.ts:414-417: fetch = min(total, max(kEff, kEff*rf)) when re-ranking."""
    k_eff = min(total, k)
    if not rerank:
        return k_eff
    return min(total, max(k_eff, k_eff * rerank_factor))


class Corpus:
    """An encoded corpus held by the oracle (codes, scales, fp32 originals)."""

    def __init__(self, originals, dim: int, bits: int, seed: int = DEFAULT_SEED, rounds: int = 2,
                 codes=None, scales=None):
        self.dim, self.bits, self.seed, self.rounds = dim, bits, seed, rounds
        self.P = pad_to_pow2(dim)
        self.originals = _f32(originals).reshape(-1, dim)
        if codes is None:
            codes, scales, _ = encode(self.originals, dim, bits, seed, rounds)
        self.codes, self.scales = _u32(codes), _f32(scales)
        self.signs = rotator_signs(dim, seed, rounds)

    @property
    def n(self) -> int:
        return self.scales.size

    def query(self, q, k: int, fetch: int, mode: int = MODE_ASYM, mask=None, rerank: bool = True):
        """index.ts:343-436 quant branch -> (rows, scores, cand_rows, cand_scores)."""
        q = _f32(q)
        m = None if mask is None else _u32(mask)
        F = max(fetch, 1)
        ro = np.empty(max(k, 1), np.uint32)
        so = np.empty(max(k, 1), np.float32)
        cr = np.zeros(F, np.uint32)
        cs = np.zeros(F, np.float32)
        n = lib().bvo_query(self.bits, mode, self.dim, self.P, _p(self.signs), self.rounds,
                            _p(self.codes), _p(self.scales), _p(self.originals), self.n, _p(m),
                            _p(q), k, fetch, int(rerank), _p(ro), _p(so), _p(cr), _p(cs))
        nc = min(F, self.n if m is None else int(np.unpackbits(m.view(np.uint8),
                                                               bitorder="little")[: self.n].sum()))
        return ro[:n], so[:n], cr[:nc], cs[:nc]

    def query_candidates(self, q, cand, k: int, fetch: int, mode: int = MODE_ASYM, rerank: bool = True):
        """The indexed (candidate-list) scan of ivfquant.ts:468-490: the same
        query over only the rows `cand`, scored and ranked by candidate slot
        (distanceQ8.ts:25-41 with indexed: true, ties to the earlier slot),
        then mapped back to rows.  -> (rows, scores, cand_rows, cand_scores)."""
        cand = _u32(cand)
        if cand.size == 0:
            e = np.zeros(0, np.uint32)
            return e, np.zeros(0, np.float32), e, np.zeros(0, np.float32)
        wpr = self.codes.size // self.n
        sub = Corpus(self.originals[cand], self.dim, self.bits, self.seed, self.rounds,
                     codes=self.codes.reshape(self.n, wpr)[cand], scales=self.scales[cand])
        r, s, cr, cs = sub.query(q, k, fetch, mode, rerank=rerank)
        return cand[r], s, cand[cr], cs

    def query_batch(self, qs, k: int, fetch: int, mode: int = MODE_ASYM, mask=None,
                    rerank: bool = True, threads: int = 0):
        qs = _f32(qs).reshape(-1, self.dim)
        nq = qs.shape[0]
        m = None if mask is None else _u32(mask)
        threads = threads or os.cpu_count() or 1
        ro = np.zeros((nq, k), np.uint32)
        so = np.zeros((nq, k), np.float32)
        cnt = np.zeros(nq, np.int32)
        lib().bvo_query_batch(self.bits, mode, self.dim, self.P, _p(self.signs), self.rounds,
                              _p(self.codes), _p(self.scales), _p(self.originals), self.n, _p(m),
                              _p(qs), nq, k, fetch, int(rerank), threads, _p(ro), _p(so), _p(cnt))
        return ro, so, cnt


def query_rows_exact(originals, dim: int, rows, q, k: int):
    """index.ts:445-464"""
    originals, rows, q = _f32(originals), _u32(rows), _f32(q)
    ro = np.empty(max(k, 1), np.uint32)
    so = np.empty(max(k, 1), np.float32)
    n = lib().bvo_query_rows_exact(_p(originals), dim, _p(rows), rows.size, _p(q), k, _p(ro), _p(so))
    return ro[:n], so[:n]


def wasm_dot(data, q, dim: int) -> np.ndarray:
    """kernel.wat:6-43"""
    data, q = _f32(data), _f32(q)
    rows = data.size // dim
    out = np.empty(rows, np.float32)
    lib().bvo_wasm_dot(_p(data), _p(q), _p(out), rows, dim)
    return out


def cpu_index_query_batch(data, dim: int, qs, k: int, threads: int = 0):
    """cpu.ts:66-88 over nq queries, split across threads."""
    data, qs = _f32(data), _f32(qs).reshape(-1, dim)
    rows = data.size // dim
    nq = qs.shape[0]
    threads = threads or os.cpu_count() or 1
    ro = np.zeros((nq, k), np.uint32)
    so = np.zeros((nq, k), np.float32)
    lib().bvo_cpu_index_query_batch(_p(data), rows, dim, _p(qs), nq, k, threads, _p(ro), _p(so))
    return ro, so


def cpu_sharded_query_batch(shards, bases, total_rows: int, dim: int, qs, k: int, threads: int = 0,
                            maps=None):
    """One CpuIndex per row shard (cpu.ts:66-88: WASM-SIMD dot + topK of
    flat.ts:217-239), the shards' hits merged with mergePartials
    (gpuTopk.ts:160-189).  shards: float32 arrays (rows_s, dim); bases: the
    global row of each shard's first row; maps (optional): per shard, the
    global row of each of its rows.  Returns (rows, scores, counts)."""
    shards = [_f32(a).reshape(-1, dim) for a in shards]
    qs = _f32(qs).reshape(-1, dim)
    ns, nq = len(shards), qs.shape[0]
    threads = threads or os.cpu_count() or 1
    ptrs = (C.c_void_p * ns)(*[a.ctypes.data for a in shards])
    rows = np.array([a.shape[0] for a in shards], np.int64)
    base = np.array(bases, np.int64)
    mp = None
    if maps is not None:
        maps = [_u32(m) for m in maps]
        mp = (C.c_void_p * ns)(*[m.ctypes.data for m in maps])
    ro = np.zeros((nq, k), np.uint32)
    so = np.zeros((nq, k), np.float32)
    cnt = np.zeros(nq, np.int32)
    lib().bvo_cpu_sharded_query_batch(C.cast(ptrs, C.c_void_p), _p(rows), _p(base),
                                      None if mp is None else C.cast(mp, C.c_void_p), ns, total_rows, dim,
                                      _p(qs), nq, k, threads, _p(ro), _p(so), _p(cnt))
    return ro, so, cnt


def keys(scores, rows) -> np.ndarray:
    """Vectorised bvo_key: orderable(score) << 32 | ~row (score desc, row asc
    when sorted descending); -0.0 counts as +0.0."""
    s = _f32(scores).copy()
    s[s == 0] = 0.0
    u = s.view(np.uint32).astype(np.uint64)
    neg = (u & 0x80000000) != 0
    u = np.where(neg, (~u) & 0xFFFFFFFF, u | 0x80000000)
    return (u << np.uint64(32)) | ((~_u32(rows)).astype(np.uint64) & np.uint64(0xFFFFFFFF))


def shard_record(shard: "Corpus", row_base: int, q, k: int, fetch: int, mode: int = MODE_ASYM):
    """One shard's contribution to a row-sharded search: its best `fetch`
    candidates by approximate score (quant.ts:194-245 per chunk) with global
    rows and their exact re-rank scores (store.ts:114-130)."""
    q = _f32(q)
    _, _, cr, cs = shard.query(q, k, fetch, mode)
    exact = np.array([np.float32(dot_row(shard.originals[r], q)) for r in cr], np.float32)
    return cr.astype(np.uint32) + np.uint32(row_base), cs.astype(np.float32), exact


def merge_shard_records(records, fetch: int, k: int):
    """Global best `fetch` by approximate key over all shard records, then the
    best k by exact key (gpuTopk.ts:160-189 mergePartials, index.ts:583-594),
    canonical order.  records: [(rows, approx, exact), ...]."""
    rows = np.concatenate([r[0] for r in records]).astype(np.uint32)
    approx = np.concatenate([r[1] for r in records]).astype(np.float32)
    exact = np.concatenate([r[2] for r in records]).astype(np.float32)
    ka = keys(approx, rows)
    sel = np.argsort(ka)[::-1][:fetch]
    ke = keys(exact[sel], rows[sel])
    best = sel[np.argsort(ke)[::-1][:k]]
    return rows[best], exact[best].copy()
