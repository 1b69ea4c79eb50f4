/*
 * browservec.h -- C ABI of libbvcuda, the B200 (sm_100a) quantized flat-scan
 * engine behind BrowserVec's VectorIndex seam.
 *
 * The reference (sharma-open-source/browservec, TypeScript) runs this path as
 * WebGPU dispatches inside QuantIndex (src/index/quant.ts).  A host that
 * binds this library (a Node N-API addon for the TypeScript host, ctypes for
 * the Python host in browservec_b200/) swaps `new QuantIndex(...)` in
 * buildIndex (src/index.ts:134-140) for an index object backed by these calls.
 * Each entry point names the reference interface it replaces.
 *
 * Conventions: every function returns a bv_status (0 = OK); on failure
 * bv_last_error() returns the message (thread-local), using the reference's
 * wording where the reference has one.  Pointers are plain host or device
 * addresses as documented per call; sizes are element counts.  Calls on one
 * index must not run concurrently (the reference serializes them the same
 * way: appends are awaited in order, src/index/flat.ts:32-35).
 */
#ifndef BROWSERVEC_H
#define BROWSERVEC_H

#include <stdint.h>

#if defined(__GNUC__)
#define BV_API __attribute__((visibility("default")))
#else
#define BV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum bv_status {
  BV_OK = 0,
  BV_ERR_INVALID = 1,      /* bad argument (message says which) */
  BV_ERR_UNSUPPORTED = 2,  /* valid request this build does not serve */
  BV_ERR_CUDA = 3,         /* CUDA runtime error */
  BV_ERR_DEVICE_LOST = 4,  /* sticky device error: 'GPU device lost; re-create the store' */
  BV_ERR_TIMEOUT = 5,      /* a kernel wait ran out of budget and aborted */
  BV_ERR_NOMEM = 6
} bv_status;

/* Scoring arithmetic of the quantized scan.
 *  BV_SCORE_ASYM    fp32 rotated query x integer codes, the reference's own
 *                   asymmetric kernels (distanceQ8.ts:56-66, distanceQ4.ts:44-62,
 *                   distanceQ1.ts:44-66) in a fixed canonical order;
 *  BV_SCORE_INT     int8-coded query (codec.ts:32-54 applied to the rotated
 *                   query) x codes, exact integer dot: dp4a for int8/int4,
 *                   bit-plane popc for 1-bit;
 *  BV_SCORE_HAMMING 1-bit corpus only: sign-bit query, xor + popc. */
typedef enum bv_scoring { BV_SCORE_ASYM = 0, BV_SCORE_INT = 1, BV_SCORE_HAMMING = 2 } bv_scoring;

typedef enum bv_metric { BV_METRIC_COSINE = 0, BV_METRIC_DOT = 1 } bv_metric;

/* BrowserVecConfig / QuantConfig subset that reaches the index
 * (src/types.ts:9-128; buildIndex src/index.ts:105-142). */
typedef struct bv_config {
  uint32_t dim;           /* dimension (any positive int; padded to pow2 >= 4) */
  uint32_t bits;          /* quantBits: 8, 4 or 1 */
  uint32_t metric;        /* bv_metric; l2 is rejected like index.ts:135-137 */
  uint32_t seed;          /* QuantConfig.seed, default 0x9e3779b9 (index.ts:71) */
  uint32_t rounds;        /* QuantConfig.rounds, default 2 */
  uint32_t scoring;       /* bv_scoring */
  int32_t device;         /* CUDA device ordinal */
  uint32_t row_base;      /* global row id of this shard's row 0 (row-sharded corpora) */
} bv_config;

typedef struct bv_index bv_index;

/* Replaces `new QuantIndex(ctx, dim, seed, rounds, bits)` (src/index/quant.ts:43-88). */
BV_API int bv_create(const bv_config* cfg, bv_index** out);

/* Replaces QuantIndex.destroy (src/index/quant.ts:247-257). */
BV_API int bv_destroy(bv_index* idx);

/* Thread-local message of the last failed call. */
BV_API const char* bv_last_error(void);

/* QuantIndex.append (src/index/quant.ts:129-141): `rows` are `count` host
 * fp32 vectors (count*dim floats), already prepared by Store.prepare
 * (normalized for cosine, src/store/store.ts:163-170).  The library keeps the
 * fp32 originals on the device for the exact re-rank and encodes the codes on
 * the GPU with the reference encoder's arithmetic (src/quant/encode.ts:64-78). */
BV_API int bv_append(bv_index* idx, const float* rows, uint64_t count);

/* Same with device-resident rows, stream-ordered on `stream` (cudaStream_t). */
BV_API int bv_append_device(bv_index* idx, const float* rows_dev, uint64_t count, void* stream);

/* QuantIndex.size (src/index/quant.ts:90-92). */
BV_API int bv_size(const bv_index* idx, uint64_t* rows);

/* One search request: queries, k, the candidate pool and the optional mask.
 * queries: nq*dim fp32 (normalized for cosine, src/index.ts:349).
 * fetch:   F approximate candidates per query, min(total, max(k, k*rf))
 *          (src/index.ts:414-417); 0 means k.
 * rerank:  1 = exact fp32 re-rank of the F candidates (src/index.ts:583-594)
 *          then top k; 0 = the approximate top k.
 * mask:    optional 1 bit per row, bit r of mask[r>>5] set = row r passes
 *          (src/index/scoreMask.ts:66-92); mask_words must cover the rows.
 * Results per query q: out_rows/out_scores[q*k .. q*k+out_counts[q]), sorted
 * by score descending, ties by lower row.  cand_* (optional) receive the F
 * approximate candidates with their quantized scores; cand_exact (optional,
 * needs rerank and cand_*) their exact re-rank scores in the same order, the
 * per-shard record a row-sharded search all-gathers (bv_merge_shards). */
typedef struct bv_search_args {
  const float* queries;
  uint32_t nq;
  uint32_t k;
  uint32_t fetch;
  int32_t rerank;
  const uint32_t* mask;
  uint64_t mask_words;
  uint32_t* out_rows;
  float* out_scores;
  uint32_t* out_counts;
  uint32_t* cand_rows;
  float* cand_scores;
  uint32_t* cand_counts;
  float* cand_exact;
} bv_search_args;

/* QuantIndex.query / queryMasked (src/index/quant.ts:165-245) plus the
 * re-rank BrowserVec.query applies (src/index.ts:414-419), and the batched
 * form BrowserVec.queryBatch lacks for quantized stores (src/index.ts:473-481).
 * All pointers are HOST memory; the call returns when results are written. */
BV_API int bv_search(bv_index* idx, const bv_search_args* args);

/* Same with DEVICE pointers, enqueued on `stream` (cudaStream_t, NULL = the
 * index's own stream) without a host synchronisation. */
BV_API int bv_search_async(bv_index* idx, const bv_search_args* args, void* stream);

/* n independent bv_search_async calls in one: entry i searches idx[i] with
 * args[i] (DEVICE pointers), all enqueued on `stream` in order.  The entries
 * may name different indexes (the shards or replicas one process serves);
 * stops at the first failing entry, whose status it returns.  One call
 * submits a stream of single-query scans without a host round trip each. */
BV_API int bv_search_async_n(bv_index* const* idx, const bv_search_args* args, uint32_t n, void* stream);

/* BrowserVec.queryRowsExact (src/index.ts:445-464): exact f64-accumulated dot
 * over an explicit list of rows (host pointers), top k.  Used for filters that
 * match at most FILTER_CPU_SCAN_MAX = 4096 rows (src/index.ts:76, :388). */
BV_API int bv_query_rows_exact(bv_index* idx, const float* query, const uint32_t* rows, uint32_t nrows,
                        uint32_t k, uint32_t* out_rows, float* out_scores, uint32_t* out_count);

/* Copy `count` rows of codes (count*wordsPerRow u32) and scales to host
 * memory, starting at row `row0` (for parity checks; the reference exposes
 * the same data through BatchEncoder.encode, src/quant/encode.ts:64-78). */
BV_API int bv_export_codes(const bv_index* idx, uint64_t row0, uint64_t count, uint32_t* words,
                    float* scales);

/* Copy `count` stored fp32 rows (the normalized originals the re-rank reads,
 * count*dim floats) to host memory from row `row0`: the vectors a snapshot
 * holds (the reference keeps them in its host store for
 * BrowserVec.export / save, src/index.ts:646-671). */
BV_API int bv_export_originals(const bv_index* idx, uint64_t row0, uint64_t count, float* out);

/* Stats the index contributes to BrowserVec.stats() (src/index.ts:702-750). */
typedef struct bv_stats {
  uint64_t rows;
  uint32_t dim, padded_dim, bits, words_per_row;
  uint32_t chunks;            /* chunkCount: shards held by this index (1) */
  float last_query_gpu_ms;    /* device time of the last bv_search (lastQueryGpuMs) */
  uint64_t device_bytes;      /* HBM held by codes, scales and originals */
} bv_stats;
BV_API int bv_get_stats(const bv_index* idx, bv_stats* out);

/* Per-phase device timestamps of every search (the device-side counterpart
 * of the reference's queryTrace, src/engine/profile.ts:16-29).  trace_dev is a
 * caller-owned device buffer of `capacity` u64; a search with scan grid G
 * writes globaltimer ns at trace[b*8 + {0 entry, 1 query rotated, 2 rows
 * scored, 3 CTA list written}] for scan CTA b, and the tail kernel writes
 * trace[G*8 + {5 entry, 0 merge start, 6 CTA lists in shared memory, 1 merged,
 * 3 rows gathered, 4 re-ranked, 2 done}].  Needs capacity >= (G+1)*8 (G < the
 * SM count); NULL disables. */
BV_API int bv_set_phase_trace(bv_index* idx, uint64_t* trace_dev, uint64_t capacity);

/* Kernel launches made by the last bv_search / bv_search_async /
 * bv_query_rows_exact on this index (a search launches one scan per query,
 * whose last CTA finishes the query, when fetch <= 256, else a scan and a
 * tail kernel per query; a batched search several per batch). */
BV_API int bv_launches_last_search(const bv_index* idx, uint32_t* launches);

/* Batched search on the tensor cores: the same request and results as
 * bv_search_async (DEVICE pointers; results identical to it, bit for bit) for
 * an index created with the integer scorings (BV_SCORE_INT, or
 * BV_SCORE_HAMMING with bits = 1).  The batch is scored as one int8
 * contraction (tcgen05.mma kind::i8) of the queries' int8 codes with the
 * corpus codes widened to int8; the best F per query are selected in rounds
 * and re-ranked exactly.  This is the batched query path the reference runs
 * as a per-query loop (BrowserVec.queryBatch, src/index.ts:473-517, over
 * QuantIndex.search, src/index/quant.ts:178-245).  The first batched search
 * after an append widens the new rows' codes (rows x paddedDim bytes more
 * device memory).  Synchronises `stream` before returning. */
BV_API int bv_search_batch(bv_index* idx, const bv_search_args* args, void* stream);

/* The batched search of a row-sharded corpus in two halves, so that each
 * shard re-ranks only its members of the global best F instead of its own
 * best F (the per-shard work the reference's chunk loop does not split:
 * QuantIndex.search, src/index/quant.ts:194-245, over ChunkedCorpus,
 * src/engine/buffers.ts:92-214).
 *
 * bv_batch_select: bv_search_batch's candidate rounds only.  Writes per query
 * q its best `fetch` approximate keys to keys_out[q*F .. q*F+F) (F = max(fetch,
 * k); DEVICE memory; u64 key = orderable(score) << 32 | ~global_row, larger =
 * better; unsorted, zero padded) and keeps the candidates in the index for
 * bv_batch_finish.  The rounds synchronise `stream`; the keys themselves are
 * written in stream order after the call returns. */
BV_API int bv_batch_select(bv_index* idx, const bv_search_args* args, uint64_t* keys_out, void* stream);

/* Per query, the least key of the global best F among `world` shards' key
 * lists as bv_batch_select writes them, gathered in rank order (gathered:
 * world x nq x fetch u64, DEVICE).  thr_out[q] (DEVICE) is a key such that
 * exactly min(F, keys present) gathered keys are >= it (1 when fewer than F
 * keys exist).  world x fetch <= 16384.  Enqueued on `stream`. */
BV_API int bv_keys_threshold(const uint64_t* gathered, uint32_t world, uint32_t nq, uint32_t fetch,
                             uint64_t* thr_out, void* stream);

/* The second half: the same request as the preceding bv_batch_select on this
 * index.  Candidates whose global key is below min_keys[q] (DEVICE; NULL keeps
 * all) are dropped, the rest re-ranked exactly; outputs as bv_search_batch
 * (cand_* hold the kept candidates only).  With min_keys from
 * bv_keys_threshold, the shard records merge (bv_merge_shards) to the single-
 * index answer.  Synchronises `stream`. */
BV_API int bv_batch_finish(bv_index* idx, const bv_search_args* args, const uint64_t* min_keys, void* stream);

/* The final merge of a two-phase sharded batch: each shard's bv_batch_finish
 * outputs (its best k by exact score among its members of the global best F,
 * rows global) are all-gathered in rank order as W records of
 * [rows nq*k | scores nq*k | counts nq] u32 words; writes per query the best k
 * by (score desc, row asc) -- the single-index answer, since the members of
 * all shards are exactly the global best F.  DEVICE pointers, enqueued on
 * `stream`.  world <= 64, k <= 1024. */
BV_API int bv_merge_topk(const uint32_t* gathered, uint32_t world, uint32_t nq, uint32_t k, uint32_t* out_rows,
                         float* out_scores, uint32_t* out_counts, void* stream);

/* Device time of the phases of the last batched search (events on its stream),
 * when enabled with bv_set_batch_timing (off by default).  gemm_macs: queries x
 * contracted rows x paddedDim, the algorithmic multiply-adds of the GEMM. */
typedef struct bv_batch_profile {
  float prep_ms, gemm_ms, select_ms, tail_ms, compact_ms;
  uint32_t gemm_launches, rounds, kept_rows, nq;
  double gemm_macs;
} bv_batch_profile;
BV_API int bv_set_batch_timing(bv_index* idx, int enable);
BV_API int bv_last_batch_profile(bv_index* idx, bv_batch_profile* out);

/* The IVF x quant scan in candidate-list mode (src/index/ivfquant.ts:468-490:
 * the quantized shaders with indexed: true, src/engine/wgsl/distanceQ8.ts:25-41,
 * distanceQ4.ts, distanceQ1.ts): query q is scored against only the index
 * rows cand_rows[offsets[q] - offsets[0] .. offsets[q+1] - offsets[0]) (the
 * probed lists' rows, any order; offsets: nq + 1 HOST u32, cand_rows DEVICE
 * u32), with the index's scoring, then re-ranked and written like
 * bv_search_async (DEVICE args; no mask).  Ties among equal scores keep the
 * earlier candidate, as the reference's topK over candidate slots does.  A
 * candidate outside the index is BV_ERR_INVALID.  The candidates' codes are
 * gathered into per-query segments of scratch memory first.  Synchronises
 * `stream`. */
BV_API int bv_search_rows(bv_index* idx, const bv_search_args* args, const uint32_t* offsets,
                          const uint32_t* cand_rows, void* stream);

/* Self-test of the kernels' bounded waits: one thread waits, with a budget of
 * `polls` mbarrier polls (1 .. 2^22, the budget every kernel wait uses), on a
 * barrier nothing completes, raises the index's timeout flag and returns; the
 * call then reports exactly what a search whose wait ran out reports --
 * BV_ERR_TIMEOUT, "scan kernel wait ran out of budget (flag 0x1)" -- and clears
 * the flag, so the index stays usable.  Nothing else runs.  No counterpart in
 * the reference (WebGPU has no device-side timeouts; its device-loss path is
 * src/engine/device.ts). */
BV_API int bv_check_wait_timeout(bv_index* idx, uint32_t polls);

/* Change the scoring mode of an index (BV_SCORE_*; hamming needs bits 1, the
 * exact index keeps asym).  Codes are shared by every mode, so this only
 * changes how later searches score.  No counterpart in the reference (its
 * scoring is always asym, src/index/quant.ts:187). */
BV_API int bv_set_scoring(bv_index* idx, uint32_t scoring);

/* Cross-shard merge of a row-sharded search (DEVICE pointers, enqueued on
 * `stream`).  The corpus is split into W contiguous row ranges, one per GPU;
 * each shard runs bv_search_async with cand_rows/cand_scores/cand_exact/
 * cand_counts pointing into one record of 3*nq*fetch + nq u32 words laid out
 * [rows nq*fetch | approx scores nq*fetch | exact scores nq*fetch | counts nq]
 * (rows global: the index's row_base added), and the W records are
 * all-gathered in rank order into `gathered`.  Writes per query the best k by
 * exact score among the global best `fetch` by approximate score -- what one
 * index over all rows returns.  This replaces the chunk loop and partial merge
 * of QuantIndex.search (src/index/quant.ts:194-245, mergePartials in
 * src/index/gpuTopk.ts:160-189) followed by the re-rank's topK
 * (src/index.ts:583-594).  W <= 64; W*fetch*12 + fetch*8 bytes must fit in
 * shared memory (W = 8 takes fetch up to 1024). */
BV_API int bv_merge_shards(const uint32_t* gathered, uint32_t world, uint32_t nq, uint32_t fetch, uint32_t k,
                           uint32_t* out_rows, float* out_scores, uint32_t* out_counts, void* stream);

/* ---------------------------------------------------------- metadata filter
 * The per-row metadata predicate of a filtered query (compileFilter,
 * src/store/filter.ts:18-68, applied row by row at src/index.ts:372-395),
 * evaluated on the GPU over device columns.  One column per metadata field:
 * a type tag per row, the value as a JS number (f64; booleans as 0/1), and
 * for strings a dictionary code.  A filter is an AND of terms, one per
 * (field, operator) pair, with strict JS equality: $eq/$in match when tag and
 * value both match, $ne matches everything $eq does not (missing fields
 * included), range operators match numbers only. */
typedef enum bv_tag { BV_TAG_MISSING = 0, BV_TAG_NULL = 1, BV_TAG_BOOL = 2, BV_TAG_NUMBER = 3,
                      BV_TAG_STRING = 4 } bv_tag;
typedef enum bv_op { BV_OP_EQ = 0, BV_OP_NE = 1, BV_OP_IN = 2, BV_OP_GT = 3, BV_OP_GTE = 4, BV_OP_LT = 5,
                     BV_OP_LTE = 6 } bv_op;
typedef struct bv_column {
  const uint8_t* tag;   /* rows: bv_tag */
  const double* num;    /* rows: number / bool value (read where tag is NUMBER or BOOL) */
  const int32_t* code;  /* rows: string dictionary code (read where tag is STRING); may be NULL */
} bv_column;
#define BV_FILTER_MAX_TERMS 16
#define BV_FILTER_MAX_IN 16
typedef struct bv_value {
  uint32_t tag;         /* bv_tag of the argument */
  int32_t code;         /* string argument: dictionary code (-1: absent from the column) */
  double num;           /* number / bool argument */
} bv_value;
typedef struct bv_filter_term {
  uint32_t column;      /* index into the columns */
  uint32_t op;          /* bv_op */
  uint32_t nvals;       /* 1, or the $in list length (<= BV_FILTER_MAX_IN) */
  bv_value vals[BV_FILTER_MAX_IN];
} bv_filter_term;
/* Writes ceil(rows/32) mask words (bit r of word r/32 set = row r matches),
 * ANDed with `live` (optional, same layout: tombstoned rows cleared,
 * src/index.ts:378-383).  Columns and masks are DEVICE pointers; terms are
 * host memory.  Enqueued on `stream`. */
BV_API int bv_filter_mask(const bv_column* cols, uint32_t ncols, const bv_filter_term* terms, uint32_t nterms,
                          uint64_t rows, const uint32_t* live, uint32_t* mask_out, void* stream);

/* bv_search_noalloc: bv_search_async for callers that may not allocate
 * device memory once they are running -- hosts whose device memory is all
 * reserved up front by their own pool, or that run under a memory budget where
 * a cudaMalloc (and the device-wide synchronisation a cudaFree brings) is not
 * allowed on the query path.  It has no counterpart in the reference.
 *
 * Same arguments and results as bv_search_async (DEVICE pointers, the caller
 * owns queries and outputs), but all scratch of the scan and tail kernels lives
 * in one fixed array inside this library: 160 x 256 candidate keys plus a few
 * counters, about 320 KB on every GPU that loads the library, held until the
 * process exits.  Limits: quantized indexes only (bits 1, 4 or 8; an exact
 * fp32 index, bits 0, gets BV_ERR_UNSUPPORTED), fetch = max(fetch, k) <= 256
 * (BV_ERR_INVALID above that) and a scan grid of at most 160 CTAs
 * (BV_ERR_UNSUPPORTED otherwise).
 * The first call on a device looks up the array's device address with that
 * device current; make that first call before any stream capture.  Every call
 * on a device shares the one array, so calls that overlap on the GPU (other
 * streams, other threads, other indexes on the same device) race and corrupt
 * each other's results: serialise them.  The call synchronises `stream`
 * (NULL = the index's stream) before it returns, and reports a kernel wait
 * that ran out of budget as BV_ERR_TIMEOUT. */
BV_API int bv_search_noalloc(bv_index* idx, const bv_search_args* args, void* stream);

#ifdef __cplusplus
}
#endif
#endif
