"""ctypes binding of libbvcuda.so (include/browservec.h).

The library is required: there is no CPU fallback on this path, so a missing
or unloadable library raises at first use with the build command to run.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libbvcuda.so")

BV_OK, BV_ERR_INVALID, BV_ERR_UNSUPPORTED, BV_ERR_CUDA, BV_ERR_DEVICE_LOST, BV_ERR_TIMEOUT, BV_ERR_NOMEM = range(7)
SCORE_ASYM, SCORE_INT, SCORE_HAMMING = 0, 1, 2
METRIC_COSINE, METRIC_DOT = 0, 1
SCORING = {"asym": SCORE_ASYM, "int": SCORE_INT, "hamming": SCORE_HAMMING}

# Every symbol include/browservec.h declares (checked by the CPU test suite).
EXPORTS = ("bv_create", "bv_destroy", "bv_last_error", "bv_append", "bv_append_device", "bv_size",
           "bv_search", "bv_search_async", "bv_search_async_n", "bv_query_rows_exact", "bv_export_codes", "bv_get_stats",
           "bv_launches_last_search", "bv_set_phase_trace", "bv_search_noalloc",
           "bv_merge_shards", "bv_search_batch", "bv_filter_mask", "bv_batch_select", "bv_batch_finish",
           "bv_keys_threshold", "bv_set_batch_timing", "bv_last_batch_profile", "bv_set_scoring",
           "bv_merge_topk", "bv_check_wait_timeout", "bv_export_originals",
           "bv_search_rows")


class BvConfig(C.Structure):
    _fields_ = [("dim", C.c_uint32), ("bits", C.c_uint32), ("metric", C.c_uint32),
                ("seed", C.c_uint32), ("rounds", C.c_uint32), ("scoring", C.c_uint32),
                ("device", C.c_int32), ("row_base", C.c_uint32)]


class BvSearchArgs(C.Structure):
    _fields_ = [("queries", C.c_void_p), ("nq", C.c_uint32), ("k", C.c_uint32),
                ("fetch", C.c_uint32), ("rerank", C.c_int32), ("mask", C.c_void_p),
                ("mask_words", C.c_uint64), ("out_rows", C.c_void_p), ("out_scores", C.c_void_p),
                ("out_counts", C.c_void_p), ("cand_rows", C.c_void_p), ("cand_scores", C.c_void_p),
                ("cand_counts", C.c_void_p), ("cand_exact", C.c_void_p)]


class BvStats(C.Structure):
    _fields_ = [("rows", C.c_uint64), ("dim", C.c_uint32), ("padded_dim", C.c_uint32),
                ("bits", C.c_uint32), ("words_per_row", C.c_uint32), ("chunks", C.c_uint32),
                ("last_query_gpu_ms", C.c_float), ("device_bytes", C.c_uint64)]


class BvBatchProfile(C.Structure):
    _fields_ = [("prep_ms", C.c_float), ("gemm_ms", C.c_float), ("select_ms", C.c_float),
                ("tail_ms", C.c_float), ("compact_ms", C.c_float), ("gemm_launches", C.c_uint32),
                ("rounds", C.c_uint32), ("kept_rows", C.c_uint32), ("nq", C.c_uint32),
                ("gemm_macs", C.c_double)]


class BvColumn(C.Structure):
    _fields_ = [("tag", C.c_void_p), ("num", C.c_void_p), ("code", C.c_void_p)]


FILTER_MAX_TERMS = 16
FILTER_MAX_IN = 16
TAG_MISSING, TAG_NULL, TAG_BOOL, TAG_NUMBER, TAG_STRING = range(5)
OP_CODES = {"$eq": 0, "$ne": 1, "$in": 2, "$gt": 3, "$gte": 4, "$lt": 5, "$lte": 6}


class BvValue(C.Structure):
    _fields_ = [("tag", C.c_uint32), ("code", C.c_int32), ("num", C.c_double)]


class BvFilterTerm(C.Structure):
    _fields_ = [("column", C.c_uint32), ("op", C.c_uint32), ("nvals", C.c_uint32),
                ("vals", BvValue * FILTER_MAX_IN)]


class BvError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


_lib = None


def load(path: str = LIB_PATH):
    """Load libbvcuda.so, raising if it is absent (no fallback path exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with `python -m browservec_b200.build` "
                           "(the quantized scan has no CPU fallback)")
    L = C.CDLL(path)
    P = C.c_void_p
    sig = {
        "bv_create": (C.c_int, [C.POINTER(BvConfig), C.POINTER(C.c_void_p)]),
        "bv_destroy": (C.c_int, [P]),
        "bv_last_error": (C.c_char_p, []),
        "bv_append": (C.c_int, [P, P, C.c_uint64]),
        "bv_append_device": (C.c_int, [P, P, C.c_uint64, P]),
        "bv_size": (C.c_int, [P, C.POINTER(C.c_uint64)]),
        "bv_search": (C.c_int, [P, C.POINTER(BvSearchArgs)]),
        "bv_search_async": (C.c_int, [P, C.POINTER(BvSearchArgs), P]),
        "bv_search_async_n": (C.c_int, [C.POINTER(P), C.POINTER(BvSearchArgs), C.c_uint32, P]),
        "bv_query_rows_exact": (C.c_int, [P, P, P, C.c_uint32, C.c_uint32, P, P, P]),
        "bv_export_codes": (C.c_int, [P, C.c_uint64, C.c_uint64, P, P]),
        "bv_get_stats": (C.c_int, [P, C.POINTER(BvStats)]),
        "bv_launches_last_search": (C.c_int, [P, C.POINTER(C.c_uint32)]),
        "bv_set_phase_trace": (C.c_int, [P, P, C.c_uint64]),
        "bv_search_noalloc": (C.c_int, [P, C.POINTER(BvSearchArgs), P]),
        "bv_merge_shards": (C.c_int, [P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, P, P, P, P]),
        "bv_search_batch": (C.c_int, [P, C.POINTER(BvSearchArgs), P]),
        "bv_filter_mask": (C.c_int, [C.POINTER(BvColumn), C.c_uint32, C.POINTER(BvFilterTerm), C.c_uint32,
                                     C.c_uint64, P, P, P]),
        "bv_batch_select": (C.c_int, [P, C.POINTER(BvSearchArgs), P, P]),
        "bv_batch_finish": (C.c_int, [P, C.POINTER(BvSearchArgs), P, P]),
        "bv_keys_threshold": (C.c_int, [P, C.c_uint32, C.c_uint32, C.c_uint32, P, P]),
        "bv_set_batch_timing": (C.c_int, [P, C.c_int]),
        "bv_last_batch_profile": (C.c_int, [P, C.POINTER(BvBatchProfile)]),
        "bv_set_scoring": (C.c_int, [P, C.c_uint32]),
        "bv_merge_topk": (C.c_int, [P, C.c_uint32, C.c_uint32, C.c_uint32, P, P, P, P]),
        "bv_check_wait_timeout": (C.c_int, [P, C.c_uint32]),
        "bv_export_originals": (C.c_int, [P, C.c_uint64, C.c_uint64, P]),
        "bv_search_rows": (C.c_int, [P, C.POINTER(BvSearchArgs), P, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != BV_OK:
        msg = load().bv_last_error().decode("utf-8", "replace")
        raise BvError(rc, msg)
