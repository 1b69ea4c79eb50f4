/*
 * bv_oracle.h -- CPU restatement of BrowserVec's quantized flat-scan path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * path in browservec_b200/.  Only tests/, __graft_entry__.smoke() and the CPU
 * baseline legs of bench.py may load it; the product path never calls it.
 *
 * Every function names the reference file:line (sharma-open-source/browservec,
 * TypeScript) whose behaviour it restates.  JavaScript arithmetic is reproduced
 * exactly: Float32Array stores round an f64 result to f32, Number math is f64,
 * Math.imul / >>> are uint32 wraparound, Math.round rounds half toward +inf.
 *
 * Canonical scoring arithmetic.  The reference scores with WGSL `dot()`, whose
 * association (and FMA use) is implementation-defined, so no reference test
 * pins a score bit pattern (the browser tests pin recall floors only).  This
 * oracle therefore DEFINES one canonical order, which the CUDA kernels follow
 * bit for bit:
 *   - a row's codes are R bytes (int8: P, int4: P/2, 1-bit: P/8); they split
 *     into C = R / min(16, R) chunks of min(16,R) bytes; L = min(32, C) lanes;
 *     lane l owns chunks l, l+L, l+2L, ... in that order;
 *   - inside a chunk the elements are taken in index order (byte order for
 *     int8, low nibble then high nibble for int4, bit 0..31 of each LE word
 *     for 1-bit);
 *   - asym mode: each lane keeps two accumulators, both starting at +0.0f;
 *     the lane's elements, counted in the order above, go alternately to the
 *     even and the odd accumulator, each acc = fmaf(v, q, acc) with v the exact
 *     integer code (int8 b in [-127,127], int4 n in [-7,7], 1-bit +-1) and q
 *     the fp32 rotated query; the lane sum is even + odd (the two chains run
 *     as one packed f32x2 FMA on the GPU);
 *   - the L lane sums reduce with an xor butterfly: for off = L/2 .. 1,
 *     s[l] = s[l] + s[l ^ off]; the result is s[0];
 *   - the row factor is applied last: int8 acc * (scale * f32(1/127)),
 *     int4 acc * (scale * f32(1/7)) (distanceQ4.ts:61), 1-bit acc * scale
 *     (distanceQ1.ts:66).
 *   - int mode (integer query, the dp4a / popc / tensor-core path): the
 *     rotated query is quantized with the reference's own int8 codec
 *     (quantizeRow, codec.ts:32-54) to bytes qb and scale qs; the integer dot
 *     idot = sum(v_i * qb_i) is exact; score = (f32(idot) * rowfac) * qfac with
 *     rowfac = scale*f32(1/127) | scale*f32(1/7) | scale and
 *     qfac = qs * f32(1/127).
 *   - hamming mode (1-bit corpus only): the query's sign bits (rq >= 0, the
 *     bit rule of quantizeRow1, codec.ts:135-154); idot = P - 2*popc(x ^ y);
 *     score = f32(idot) * scale (the query's own scale is one positive factor
 *     per query and is left out).
 * Top-k order is (score desc, row asc) for both membership and output, the
 * north_star's tie rule; the reference's heap (flat.ts:217-239) agrees on every
 * set without exact ties at the k boundary.
 */
#ifndef BV_ORACLE_H
#define BV_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { BVO_MODE_ASYM = 0, BVO_MODE_INT = 1, BVO_MODE_HAMMING = 2 };

/* prng.ts:5-14 -- one mulberry32 step; returns the uint32 the JS divides by 2^32. */
uint32_t bvo_mulberry32_next(uint32_t *state);
/* prng.ts:5-14 -- fill `out` with n successive rng() doubles from `seed`. */
void bvo_mulberry32_doubles(uint32_t seed, double *out, int64_t n);
/* prng.ts:17-22 */
void bvo_random_signs(float *out, int n, uint32_t seed);
/* rotator.ts:16-21 */
int bvo_pad_to_pow2(int n);
/* rotator.ts:46-58 (in place, n a power of two) */
void bvo_fwht(float *a, int n);
/* rotator.ts:44-58 -- rounds*P pre-scaled signs; returns P. */
int bvo_rotator_signs(int dim, uint32_t seed, int rounds, float *signs_out);
/* rotator.ts:60-70 -- rotate one row: src[dim] -> dst[P]. */
void bvo_rotate(const float *signs, int rounds, int dim, int P, const float *src, float *dst);

/* codec.ts:32-54 / :85-108 / :135-154 -- returns 0, or -1 on a bad length. */
int bvo_quantize_row8(const float *rot, int n, uint32_t *words, float *scale);
int bvo_quantize_row4(const float *rot, int n, uint32_t *words, float *scale);
int bvo_quantize_row1(const float *rot, int n, uint32_t *words, float *scale);
/* codec.ts:56-66 / :110-120 / :156-167 */
void bvo_dequant_row8(const uint32_t *words, int nwords, float scale, float *out);
void bvo_dequant_row4(const uint32_t *words, int nwords, float scale, float *out);
void bvo_dequant_row1(const uint32_t *words, int nwords, float scale, float *out);

/* encode.ts:31-78 -- words: count*wordsPerRow, scales: count; rotated optional (count*P). */
int bvo_words_per_row(int P, int bits);
int bvo_encode(const float *data, int64_t count, int dim, uint32_t seed, int rounds, int bits,
               uint32_t *words, float *scales, float *rotated_or_null);

/* Prepared query for one scoring mode: rq = rotated fp32 query (P floats);
 * qwords/qscale = its int8 (int mode) or 1-bit (hamming) code. */
void bvo_prepare_query(const float *signs, int rounds, int dim, int P, int bits, int mode,
                       const float *q, float *rq, uint32_t *qwords, float *qscale);

/* Canonical score of `nrows` consecutive rows (see header comment). */
void bvo_score_rows(int bits, int mode, int P, const uint32_t *codes, const float *scales,
                    int64_t nrows, const float *rq, const uint32_t *qwords, float qscale,
                    float *out);

/* Canonical order key: larger key = better (score desc, row asc). */
uint64_t bvo_key(float score, uint32_t row);
float bvo_key_score(uint64_t key);
uint32_t bvo_key_row(uint64_t key);

/* Canonical top-k over scores[0..n) restricted to rows whose mask bit is set
 * (mask may be NULL).  Writes up to k (row, score); returns the count. */
int bvo_topk(const float *scores, int64_t n, const uint32_t *mask, int k,
             uint32_t *rows_out, float *scores_out);

/* flat.ts:217-239 -- the reference's own heap selection, ties included. */
int bvo_topk_ref(const float *scores, int64_t n, int k, uint32_t *rows_out, float *scores_out);
/* gpuTopk.ts:160-189 -- the reference's merge of per-segment partials. */
int bvo_merge_partials_ref(const float *scores, const uint32_t *rows, int64_t count, int64_t n, int k,
                           uint32_t *rows_out, float *scores_out);

/* store.ts:114-130 -- exact dot of an fp32 row and the query, f64 lanes. */
double bvo_dot_row(const float *row, const float *q, int dim);
/* store.ts:209-217 -- normalizeInPlace. */
void bvo_normalize(float *v, int n);

/* index.ts:343-436 (quant branch) + quant.ts:178-245 + index.ts:583-594:
 * one query through rotate -> score -> (mask) -> top-F -> exact re-rank -> top-k.
 * `fetch` = F (already min(total, max(k, k*rf))); rerank=0 returns the first k
 * approximate hits.  originals: count*dim normalized fp32 rows.  Returns hits. */
int bvo_query(int bits, int mode, int dim, int P, const float *signs, int rounds,
              const uint32_t *codes, const float *scales, const float *originals, int64_t nrows,
              const uint32_t *mask, const float *q, int k, int fetch, int rerank,
              uint32_t *rows_out, float *scores_out,
              uint32_t *cand_rows_out /* F or NULL */, float *cand_scores_out /* F or NULL */);

/* index.ts:445-464 -- exact scan of an explicit row list, topK(k). */
int bvo_query_rows_exact(const float *originals, int dim, const uint32_t *rows, int64_t nrows,
                         const float *q, int k, uint32_t *rows_out, float *scores_out);

/* kernel.wat:6-43 -- the WASM-SIMD dot kernel: f32x4 lanes, separate mul and
 * add, lanes (l0+l1)+(l2+l3), then a sequential scalar tail. */
void bvo_wasm_dot(const float *data, const float *q, float *out, int64_t rows, int dim);
/* cpu.ts:66-88 -- CpuIndex.query: wasm dot + topK (reference heap). */
int bvo_cpu_index_query(const float *data, int64_t rows, int dim, const float *q, int k,
                        uint32_t *rows_out, float *scores_out);
/* Threaded CpuIndex.query over nq queries (queries split over nthreads, one
 * private scratch each, like one process per core).  Returns 0. */
int bvo_cpu_index_query_batch(const float *data, int64_t rows, int dim, const float *qs, int nq,
                              int k, int nthreads, uint32_t *rows_out, float *scores_out);
/* Threaded bvo_query over nq queries (same arguments, queries packed). */
int bvo_query_batch(int bits, int mode, int dim, int P, const float *signs, int rounds,
                    const uint32_t *codes, const float *scales, const float *originals,
                    int64_t nrows, const uint32_t *mask, const float *qs, int nq, int k, int fetch,
                    int rerank, int nthreads, uint32_t *rows_out, float *scores_out,
                    int32_t *counts_out);

/* Sharded CPU baseline: one CpuIndex per row shard (cpu.ts:66-88 + flat.ts:217-239),
 * merged with mergePartials (gpuTopk.ts:160-189); see bv_oracle.c. */
int bvo_cpu_sharded_query_batch(const float *const *data, const int64_t *rows, const int64_t *base,
                                const uint32_t *const *map, int nshards, int64_t total_rows, int dim,
                                const float *qs, int nq, int k, int nthreads, uint32_t *rows_out,
                                float *scores_out, int32_t *counts_out);

#ifdef __cplusplus
}
#endif
#endif
