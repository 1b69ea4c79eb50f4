/*
 * bv_oracle.c -- CPU restatement of BrowserVec's quantized flat-scan path.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker and the timed CPU baseline).
 * The shipped CUDA path never links or calls this file.
 *
 * Build: gcc -O2 -ffp-contract=off -fno-fast-math -msse2 -fPIC -shared -pthread
 * (see oracle/Makefile).  -ffp-contract=off matters: the canonical order uses
 * explicit fmaf() where it fuses and plain f32 mul/add everywhere else.
 */
#include "bv_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <emmintrin.h>

#define INV127 0x1.020408p-7f /* f32(1/127) */
#define INV7 0x1.24924ap-3f   /* f32(1/7), the WGSL constant of distanceQ4.ts:61 */

/* ------------------------------------------------------------------ prng */

/* prng.ts:5-14.  `a |= 0; a = (a + 0x6d2b79f5) | 0` etc. are uint32 wraps. */
uint32_t bvo_mulberry32_next(uint32_t *state) {
  uint32_t a = *state + 0x6d2b79f5u;
  *state = a;
  uint32_t t = (a ^ (a >> 15)) * (1u | a);
  t = (t + (t ^ (t >> 7)) * (61u | t)) ^ t;
  return t ^ (t >> 14);
}

void bvo_mulberry32_doubles(uint32_t seed, double *out, int64_t n) {
  uint32_t s = seed;
  for (int64_t i = 0; i < n; i++) out[i] = (double)bvo_mulberry32_next(&s) / 4294967296.0;
}

/* prng.ts:17-22: rng() < 0.5 ? -1 : 1, i.e. the uint32 draw < 2^31. */
void bvo_random_signs(float *out, int n, uint32_t seed) {
  uint32_t s = seed;
  for (int i = 0; i < n; i++) out[i] = (bvo_mulberry32_next(&s) < 0x80000000u) ? -1.0f : 1.0f;
}

/* -------------------------------------------------------------- rotation */

/* rotator.ts:16-21 */
int bvo_pad_to_pow2(int n) {
  int p = 4;
  while (p < n) p <<= 1;
  return p;
}

/* rotator.ts:46-58.  Float32Array stores of f64 sums: identical to f32 add/sub
 * (double rounding is innocuous for +,-,* since 53 >= 2*24+2). */
void bvo_fwht(float *a, int n) {
  for (int len = 1; len < n; len <<= 1)
    for (int i = 0; i < n; i += len << 1)
      for (int j = i; j < i + len; j++) {
        float x = a[j], y = a[j + len];
        a[j] = x + y;
        a[j + len] = x - y;
      }
}

/* rotator.ts:44-58.  Round seed (seed ^ (0x9e3779b9*(r+1))) >>> 0 is a uint32
 * multiply-wrap; the sign vector is Float32Array(+-1) *= f64 1/sqrt(P). */
int bvo_rotator_signs(int dim, uint32_t seed, int rounds, float *signs_out) {
  int P = bvo_pad_to_pow2(dim);
  double inv_scale = 1.0 / sqrt((double)P);
  for (int r = 0; r < rounds; r++) {
    uint32_t rs = seed ^ (0x9e3779b9u * (uint32_t)(r + 1));
    float *s = signs_out + (size_t)r * P;
    bvo_random_signs(s, P, rs);
    for (int i = 0; i < P; i++) s[i] = (float)((double)s[i] * inv_scale);
  }
  return P;
}

/* rotator.ts:60-70 */
void bvo_rotate(const float *signs, int rounds, int dim, int P, const float *src, float *dst) {
  memcpy(dst, src, sizeof(float) * (size_t)dim);
  for (int i = dim; i < P; i++) dst[i] = 0.0f;
  for (int r = 0; r < rounds; r++) {
    const float *s = signs + (size_t)r * P;
    for (int i = 0; i < P; i++) dst[i] = dst[i] * s[i];
    bvo_fwht(dst, P);
  }
}

/* ----------------------------------------------------------------- codec */

/* Math.round: nearest integer, halves toward +infinity. */
static double js_round(double x) {
  double r = floor(x);
  if (x - r >= 0.5) r += 1.0;
  return r;
}

/* codec.ts:22-30 (levels = 127) and :77-83 (levels = 7). */
static int snorm_level(double v, double levels) {
  double c = v < -1.0 ? -1.0 : (v > 1.0 ? 1.0 : v);
  double b = js_round(c * levels);
  if (b < -levels) b = -levels;
  if (b > levels) b = levels;
  return (int)b;
}

static float max_abs_scale(const float *rot, int n) {
  float m = 0.0f;
  for (int i = 0; i < n; i++) {
    float a = fabsf(rot[i]);
    if (a > m) m = a;
  }
  return m > 0.0f ? m : 1.0f;
}

/* codec.ts:32-54 */
int bvo_quantize_row8(const float *rot, int n, uint32_t *words, float *scale) {
  if (n % 4 != 0) return -1;
  float sc = max_abs_scale(rot, n);
  double inv = 1.0 / (double)sc;
  for (int g = 0; g < n / 4; g++) {
    uint32_t w = 0;
    for (int j = 0; j < 4; j++)
      w |= (uint32_t)(snorm_level((double)rot[g * 4 + j] * inv, 127.0) & 0xff) << (8 * j);
    words[g] = w;
  }
  *scale = sc;
  return 0;
}

/* codec.ts:85-108 */
int bvo_quantize_row4(const float *rot, int n, uint32_t *words, float *scale) {
  if (n % 8 != 0) return -1;
  float sc = max_abs_scale(rot, n);
  double inv = 1.0 / (double)sc;
  for (int g = 0; g < n / 8; g++) {
    uint32_t w = 0;
    for (int j = 0; j < 8; j++)
      w |= (uint32_t)(snorm_level((double)rot[g * 8 + j] * inv, 7.0) & 0xf) << (4 * j);
    words[g] = w;
  }
  *scale = sc;
  return 0;
}

/* codec.ts:135-154: scale = f32(f64 sum|x| / n), bit j of word g = x[32g+j] >= 0. */
int bvo_quantize_row1(const float *rot, int n, uint32_t *words, float *scale) {
  if (n % 32 != 0) return -1;
  double abs_sum = 0.0;
  for (int i = 0; i < n; i++) abs_sum += fabs((double)rot[i]);
  for (int g = 0; g < n / 32; g++) {
    uint32_t w = 0;
    for (int j = 0; j < 32; j++)
      if (rot[g * 32 + j] >= 0.0f) w |= 1u << j;
    words[g] = w;
  }
  *scale = abs_sum > 0.0 ? (float)(abs_sum / n) : 1.0f;
  return 0;
}

/* codec.ts:56-66 */
void bvo_dequant_row8(const uint32_t *words, int nwords, float scale, float *out) {
  for (int g = 0; g < nwords; g++)
    for (int j = 0; j < 4; j++) {
      int b = (int)((words[g] >> (8 * j)) & 0xff);
      if (b > 127) b -= 256;
      double v = (double)b / 127.0;
      if (v < -1.0) v = -1.0;
      out[g * 4 + j] = (float)(v * (double)scale);
    }
}

/* codec.ts:110-120 */
void bvo_dequant_row4(const uint32_t *words, int nwords, float scale, float *out) {
  for (int g = 0; g < nwords; g++)
    for (int j = 0; j < 8; j++) {
      int b = (int)((words[g] >> (4 * j)) & 0xf);
      if (b > 7) b -= 16;
      double v = (double)b / 7.0;
      if (v < -1.0) v = -1.0;
      out[g * 8 + j] = (float)(v * (double)scale);
    }
}

/* codec.ts:156-167 */
void bvo_dequant_row1(const uint32_t *words, int nwords, float scale, float *out) {
  for (int g = 0; g < nwords; g++)
    for (int j = 0; j < 32; j++) out[g * 32 + j] = ((words[g] >> j) & 1u) ? scale : -scale;
}

/* encode.ts:49-53 */
int bvo_words_per_row(int P, int bits) {
  int per = bits == 8 ? 4 : (bits == 4 ? 8 : 32);
  return P / per;
}

/* encode.ts:64-78: rotate each row into scratch (or `rotated`), then quantize. */
int bvo_encode(const float *data, int64_t count, int dim, uint32_t seed, int rounds, int bits,
               uint32_t *words, float *scales, float *rotated_or_null) {
  if (bits != 1 && bits != 4 && bits != 8) return -1;
  int P = bvo_pad_to_pow2(dim);
  float *signs = (float *)malloc(sizeof(float) * (size_t)P * (rounds > 0 ? rounds : 1));
  float *scratch = (float *)malloc(sizeof(float) * (size_t)P);
  bvo_rotator_signs(dim, seed, rounds, signs);
  int wpr = bvo_words_per_row(P, bits);
  int rc = 0;
  for (int64_t i = 0; i < count && rc == 0; i++) {
    float *dst = rotated_or_null ? rotated_or_null + (size_t)i * P : scratch;
    bvo_rotate(signs, rounds, dim, P, data + (size_t)i * dim, dst);
    uint32_t *w = words + (size_t)i * wpr;
    if (bits == 8) rc = bvo_quantize_row8(dst, P, w, &scales[i]);
    else if (bits == 4) rc = bvo_quantize_row4(dst, P, w, &scales[i]);
    else rc = bvo_quantize_row1(dst, P, w, &scales[i]);
  }
  free(signs);
  free(scratch);
  return rc;
}

/* --------------------------------------------------------------- scoring */

static int row_bytes(int P, int bits) { return bits == 8 ? P : (bits == 4 ? P / 2 : P / 8); }

void bvo_prepare_query(const float *signs, int rounds, int dim, int P, int bits, int mode,
                       const float *q, float *rq, uint32_t *qwords, float *qscale) {
  bvo_rotate(signs, rounds, dim, P, q, rq);
  *qscale = 1.0f;
  if (mode == BVO_MODE_INT) bvo_quantize_row8(rq, P, qwords, qscale);
  else if (mode == BVO_MODE_HAMMING && bits == 1) bvo_quantize_row1(rq, P, qwords, qscale);
}

/* Exact integer code of element e of a row (int8 byte, int4 nibble, 1-bit +-1). */
static inline int code_at(const uint8_t *row, int bits, int e) {
  if (bits == 8) return (int)(int8_t)row[e];
  if (bits == 4) {
    int n = (row[e >> 1] >> ((e & 1) * 4)) & 0xf;
    return n > 7 ? n - 16 : n;
  }
  return ((row[e >> 3] >> (e & 7)) & 1) ? 1 : -1;
}

static float row_factor(int bits, float scale) {
  if (bits == 8) return scale * INV127;
  if (bits == 4) return scale * INV7;
  return scale;
}

/* Canonical asym score of one row (lane chunks, fmaf chains, xor butterfly). */
static float score_asym(int bits, int P, const uint8_t *row, float scale, const float *rq) {
  int R = row_bytes(P, bits);
  int CB = R < 16 ? R : 16;
  int C = R / CB;
  int L = C < 32 ? C : 32;
  int epb = bits == 8 ? 1 : (bits == 4 ? 2 : 8); /* elements per byte */
  int epc = CB * epb;                             /* elements per chunk */
  float s[32] = {0};
  for (int l = 0; l < L; l++) {
    /* two sub-chains per lane: even and odd element positions in lane order */
    float acc[2] = {0.0f, 0.0f};
    int pos = 0;
    for (int c = l; c < C; c += L)
      for (int j = 0; j < epc; j++, pos++) {
        int e = c * epc + j;
        acc[pos & 1] = fmaf((float)code_at(row, bits, e), rq[e], acc[pos & 1]);
      }
    s[l] = acc[0] + acc[1];
  }
  for (int off = L / 2; off >= 1; off >>= 1) {
    float t[32];
    for (int l = 0; l < L; l++) t[l] = s[l] + s[l ^ off];
    memcpy(s, t, sizeof(float) * (size_t)L);
  }
  return s[0] * row_factor(bits, scale);
}

static float score_int(int bits, int P, const uint8_t *row, float scale, const uint32_t *qwords,
                       float qscale) {
  const uint8_t *qb = (const uint8_t *)qwords;
  int32_t idot = 0;
  for (int e = 0; e < P; e++) idot += code_at(row, bits, e) * (int)(int8_t)qb[e];
  float qfac = qscale * INV127;
  return ((float)idot * row_factor(bits, scale)) * qfac;
}

static float score_hamming(int P, const uint8_t *row, float scale, const uint32_t *qwords,
                           float qscale) {
  const uint32_t *w = (const uint32_t *)row;
  int ham = 0;
  for (int g = 0; g < P / 32; g++) ham += __builtin_popcount(w[g] ^ qwords[g]);
  int32_t idot = P - 2 * ham;
  (void)qscale; /* one positive factor per query: not part of the canonical score */
  return (float)idot * scale;
}

void bvo_score_rows(int bits, int mode, int P, const uint32_t *codes, const float *scales,
                    int64_t nrows, const float *rq, const uint32_t *qwords, float qscale,
                    float *out) {
  int R = row_bytes(P, bits);
  const uint8_t *base = (const uint8_t *)codes;
  for (int64_t r = 0; r < nrows; r++) {
    const uint8_t *row = base + (size_t)r * R;
    if (mode == BVO_MODE_ASYM) out[r] = score_asym(bits, P, row, scales[r], rq);
    else if (mode == BVO_MODE_HAMMING && bits == 1) out[r] = score_hamming(P, row, scales[r], qwords, qscale);
    else out[r] = score_int(bits, P, row, scales[r], qwords, qscale);
  }
}

/* ----------------------------------------------------------------- top-k */

uint64_t bvo_key(float score, uint32_t row) {
  if (score == 0.0f) score = 0.0f; /* -0 and +0 compare equal in JS */
  uint32_t u;
  memcpy(&u, &score, 4);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((uint64_t)u << 32) | (uint64_t)(~row);
}

float bvo_key_score(uint64_t key) {
  uint32_t u = (uint32_t)(key >> 32);
  u = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

uint32_t bvo_key_row(uint64_t key) { return ~(uint32_t)key; }

/* min-heap of keys (root = worst kept key) */
static void heap_sift_down(uint64_t *h, int n, int i) {
  for (;;) {
    int l = 2 * i + 1, r = l + 1, m = i;
    if (l < n && h[l] < h[m]) m = l;
    if (r < n && h[r] < h[m]) m = r;
    if (m == i) return;
    uint64_t t = h[i];
    h[i] = h[m];
    h[m] = t;
    i = m;
  }
}

static int cmp_key_desc(const void *a, const void *b) {
  uint64_t x = *(const uint64_t *)a, y = *(const uint64_t *)b;
  return x < y ? 1 : (x > y ? -1 : 0);
}

/* keys[0..n) -> best k keys sorted desc into out; returns count. */
static int select_keys(const uint64_t *keys, int64_t n, int k, uint64_t *out) {
  if (k <= 0) return 0;
  uint64_t *h = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)k);
  int len = 0;
  for (int64_t i = 0; i < n; i++) {
    uint64_t x = keys[i];
    if (len < k) {
      h[len++] = x;
      if (len == k)
        for (int j = k / 2 - 1; j >= 0; j--) heap_sift_down(h, k, j);
    } else if (x > h[0]) {
      h[0] = x;
      heap_sift_down(h, k, 0);
    }
  }
  qsort(h, (size_t)len, sizeof(uint64_t), cmp_key_desc);
  memcpy(out, h, sizeof(uint64_t) * (size_t)len);
  free(h);
  return len;
}

int bvo_topk(const float *scores, int64_t n, const uint32_t *mask, int k, uint32_t *rows_out,
             float *scores_out) {
  uint64_t *keys = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)(n > 0 ? n : 1));
  int64_t m = 0;
  for (int64_t r = 0; r < n; r++) {
    if (mask && !((mask[r >> 5] >> (r & 31)) & 1u)) continue;
    keys[m++] = bvo_key(scores[r], (uint32_t)r);
  }
  uint64_t *best = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)(k > 0 ? k : 1));
  int c = select_keys(keys, m, k, best);
  for (int i = 0; i < c; i++) {
    rows_out[i] = bvo_key_row(best[i]);
    scores_out[i] = scores[rows_out[i]];
  }
  free(keys);
  free(best);
  return c;
}

/* Stable insertion sort of (row, score) by score, ascending or descending. */
typedef struct {
  uint32_t row;
  float score;
} hit_t;

static void stable_sort_hits(hit_t *h, int n, int descending) {
  for (int i = 1; i < n; i++) {
    hit_t x = h[i];
    int j = i - 1;
    while (j >= 0 && (descending ? (h[j].score < x.score) : (h[j].score > x.score))) {
      h[j + 1] = h[j];
      j--;
    }
    h[j + 1] = x;
  }
}

/* flat.ts:217-239 */
int bvo_topk_ref(const float *scores, int64_t n, int k, uint32_t *rows_out, float *scores_out) {
  int64_t limit64 = k < n ? k : n;
  int limit = (int)limit64;
  if (limit <= 0) return 0;
  hit_t *heap = (hit_t *)malloc(sizeof(hit_t) * (size_t)limit);
  int len = 0;
  for (int64_t row = 0; row < n; row++) {
    float score = scores[row];
    if (len < limit) {
      heap[len].row = (uint32_t)row;
      heap[len].score = score;
      len++;
      if (len == limit) stable_sort_hits(heap, len, 0);
    } else if (score > heap[0].score) {
      heap[0].row = (uint32_t)row;
      heap[0].score = score;
      int i = 0;
      while (i + 1 < len && heap[i].score > heap[i + 1].score) {
        hit_t t = heap[i];
        heap[i] = heap[i + 1];
        heap[i + 1] = t;
        i++;
      }
    }
  }
  stable_sort_hits(heap, len, 1);
  for (int i = 0; i < len; i++) {
    rows_out[i] = heap[i].row;
    scores_out[i] = heap[i].score;
  }
  free(heap);
  return len;
}

/* gpuTopk.ts:160-189 (NEG_MAX = -3.4e38 compared as a double). */
int bvo_merge_partials_ref(const float *scores, const uint32_t *rows, int64_t count, int64_t n, int k,
                           uint32_t *rows_out, float *scores_out) {
  int64_t limit64 = k < n ? k : n;
  int limit = (int)limit64;
  if (limit <= 0) return 0;
  hit_t *heap = (hit_t *)malloc(sizeof(hit_t) * (size_t)limit);
  int len = 0;
  for (int64_t i = 0; i < count; i++) {
    float score = scores[i];
    if ((double)score <= -3.4e38) continue;
    uint32_t row = rows[i];
    if ((int64_t)row >= n) continue;
    if (len < limit) {
      heap[len].row = row;
      heap[len].score = score;
      len++;
      if (len == limit) stable_sort_hits(heap, len, 0);
    } else if (score > heap[0].score) {
      heap[0].row = row;
      heap[0].score = score;
      int j = 0;
      while (j + 1 < len && heap[j].score > heap[j + 1].score) {
        hit_t t = heap[j];
        heap[j] = heap[j + 1];
        heap[j + 1] = t;
        j++;
      }
    }
  }
  stable_sort_hits(heap, len, 1);
  for (int i = 0; i < len; i++) {
    rows_out[i] = heap[i].row;
    scores_out[i] = heap[i].score;
  }
  free(heap);
  return len;
}

/* ------------------------------------------------------ exact re-rank */

/* store.ts:114-130: four f64 lanes, ((a0+a1)+a2)+a3, then a sequential tail.
 * Each f32*f32 product is exact in f64. */
double bvo_dot_row(const float *row, const float *q, int dim) {
  int vec = dim & ~3;
  double a0 = 0, a1 = 0, a2 = 0, a3 = 0;
  int i = 0;
  for (; i < vec; i += 4) {
    a0 += (double)row[i] * (double)q[i];
    a1 += (double)row[i + 1] * (double)q[i + 1];
    a2 += (double)row[i + 2] * (double)q[i + 2];
    a3 += (double)row[i + 3] * (double)q[i + 3];
  }
  double acc = a0 + a1 + a2 + a3;
  for (; i < dim; i++) acc += (double)row[i] * (double)q[i];
  return acc;
}

/* store.ts:209-217 */
void bvo_normalize(float *v, int n) {
  double sum = 0;
  for (int i = 0; i < n; i++) sum += (double)v[i] * (double)v[i];
  double norm = sqrt(sum);
  if (norm > 0) {
    double inv = 1.0 / norm;
    for (int i = 0; i < n; i++) v[i] = (float)((double)v[i] * inv);
  }
}

/* index.ts:583-594 under the canonical tie rule. */
static int rerank_exact(const float *originals, int dim, const float *q, const uint32_t *cand,
                        int nc, int k, uint32_t *rows_out, float *scores_out) {
  uint64_t *keys = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)(nc > 0 ? nc : 1));
  float *ex = (float *)malloc(sizeof(float) * (size_t)(nc > 0 ? nc : 1));
  for (int c = 0; c < nc; c++) {
    ex[c] = (float)bvo_dot_row(originals + (size_t)cand[c] * dim, q, dim);
    keys[c] = bvo_key(ex[c], cand[c]);
  }
  uint64_t *best = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)(k > 0 ? k : 1));
  int m = select_keys(keys, nc, k, best);
  for (int i = 0; i < m; i++) {
    rows_out[i] = bvo_key_row(best[i]);
    scores_out[i] = bvo_key_score(best[i]);
  }
  free(keys);
  free(ex);
  free(best);
  return m;
}

int bvo_query(int bits, int mode, int dim, int P, const float *signs, int rounds,
              const uint32_t *codes, const float *scales, const float *originals, int64_t nrows,
              const uint32_t *mask, const float *q, int k, int fetch, int rerank,
              uint32_t *rows_out, float *scores_out, uint32_t *cand_rows_out,
              float *cand_scores_out) {
  if (nrows <= 0 || k <= 0) return 0;
  float *rq = (float *)malloc(sizeof(float) * (size_t)P);
  uint32_t *qw = (uint32_t *)calloc((size_t)P / 4 + 1, sizeof(uint32_t));
  float qscale = 1.0f;
  bvo_prepare_query(signs, rounds, dim, P, bits, mode, q, rq, qw, &qscale);
  float *sc = (float *)malloc(sizeof(float) * (size_t)nrows);
  bvo_score_rows(bits, mode, P, codes, scales, nrows, rq, qw, qscale, sc);
  int F = fetch > 0 ? fetch : k;
  uint32_t *cr = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)F);
  float *cs = (float *)malloc(sizeof(float) * (size_t)F);
  int nc = bvo_topk(sc, nrows, mask, F, cr, cs);
  if (cand_rows_out) memcpy(cand_rows_out, cr, sizeof(uint32_t) * (size_t)nc);
  if (cand_scores_out) memcpy(cand_scores_out, cs, sizeof(float) * (size_t)nc);
  int out;
  if (rerank) {
    out = rerank_exact(originals, dim, q, cr, nc, k, rows_out, scores_out);
  } else {
    out = nc < k ? nc : k;
    memcpy(rows_out, cr, sizeof(uint32_t) * (size_t)out);
    memcpy(scores_out, cs, sizeof(float) * (size_t)out);
  }
  free(rq);
  free(qw);
  free(sc);
  free(cr);
  free(cs);
  return out;
}

int bvo_query_rows_exact(const float *originals, int dim, const uint32_t *rows, int64_t nrows,
                         const float *q, int k, uint32_t *rows_out, float *scores_out) {
  return rerank_exact(originals, dim, q, rows, (int)nrows, k, rows_out, scores_out);
}

/* ------------------------------------------------ CPU fallback (baseline) */

/* kernel.wat:6-43: f32x4.mul then f32x4.add per 4 floats (no FMA), lanes
 * (l0+l1)+(l2+l3), then the scalar tail in order. */
void bvo_wasm_dot(const float *data, const float *q, float *out, int64_t rows, int dim) {
  int tail = dim & ~3;
  for (int64_t r = 0; r < rows; r++) {
    const float *base = data + (size_t)r * dim;
    __m128 acc = _mm_setzero_ps();
    int i = 0;
    for (; i < tail; i += 4) acc = _mm_add_ps(acc, _mm_mul_ps(_mm_loadu_ps(base + i), _mm_loadu_ps(q + i)));
    float l[4];
    _mm_storeu_ps(l, acc);
    float sum = (l[0] + l[1]) + (l[2] + l[3]);
    for (; i < dim; i++) sum = sum + base[i] * q[i];
    out[r] = sum;
  }
}

int bvo_cpu_index_query(const float *data, int64_t rows, int dim, const float *q, int k,
                        uint32_t *rows_out, float *scores_out) {
  if (rows <= 0) return 0;
  float *sc = (float *)malloc(sizeof(float) * (size_t)rows);
  bvo_wasm_dot(data, q, sc, rows, dim);
  int n = bvo_topk_ref(sc, rows, k, rows_out, scores_out);
  free(sc);
  return n;
}

typedef struct {
  int kind; /* 0 = cpu index, 1 = quant query */
  int bits, mode, dim, P, rounds, k, fetch, rerank;
  const float *signs, *scales, *originals, *data, *qs;
  const uint32_t *codes, *mask;
  int64_t nrows;
  int q0, q1;
  uint32_t *rows_out;
  float *scores_out;
  int32_t *counts_out;
} job_t;

static void *run_job(void *arg) {
  job_t *j = (job_t *)arg;
  for (int i = j->q0; i < j->q1; i++) {
    const float *q = j->qs + (size_t)i * j->dim;
    uint32_t *ro = j->rows_out + (size_t)i * j->k;
    float *so = j->scores_out + (size_t)i * j->k;
    int n;
    if (j->kind == 0) n = bvo_cpu_index_query(j->data, j->nrows, j->dim, q, j->k, ro, so);
    else
      n = bvo_query(j->bits, j->mode, j->dim, j->P, j->signs, j->rounds, j->codes, j->scales,
                    j->originals, j->nrows, j->mask, q, j->k, j->fetch, j->rerank, ro, so, NULL, NULL);
    if (j->counts_out) j->counts_out[i] = n;
  }
  return NULL;
}

static int run_threads(job_t proto, int nq, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > nq) nthreads = nq > 0 ? nq : 1;
  pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)nthreads);
  job_t *jobs = (job_t *)malloc(sizeof(job_t) * (size_t)nthreads);
  for (int t = 0; t < nthreads; t++) {
    jobs[t] = proto;
    jobs[t].q0 = (int)((int64_t)nq * t / nthreads);
    jobs[t].q1 = (int)((int64_t)nq * (t + 1) / nthreads);
    pthread_create(&th[t], NULL, run_job, &jobs[t]);
  }
  for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
  free(th);
  free(jobs);
  return 0;
}

int bvo_cpu_index_query_batch(const float *data, int64_t rows, int dim, const float *qs, int nq,
                              int k, int nthreads, uint32_t *rows_out, float *scores_out) {
  job_t p;
  memset(&p, 0, sizeof(p));
  p.kind = 0;
  p.data = data;
  p.nrows = rows;
  p.dim = dim;
  p.qs = qs;
  p.k = k;
  p.rows_out = rows_out;
  p.scores_out = scores_out;
  return run_threads(p, nq, nthreads);
}

int bvo_query_batch(int bits, int mode, int dim, int P, const float *signs, int rounds,
                    const uint32_t *codes, const float *scales, const float *originals,
                    int64_t nrows, const uint32_t *mask, const float *qs, int nq, int k, int fetch,
                    int rerank, int nthreads, uint32_t *rows_out, float *scores_out,
                    int32_t *counts_out) {
  job_t p;
  memset(&p, 0, sizeof(p));
  p.kind = 1;
  p.bits = bits;
  p.mode = mode;
  p.dim = dim;
  p.P = P;
  p.signs = signs;
  p.rounds = rounds;
  p.codes = codes;
  p.scales = scales;
  p.originals = originals;
  p.nrows = nrows;
  p.mask = mask;
  p.qs = qs;
  p.k = k;
  p.fetch = fetch;
  p.rerank = rerank;
  p.rows_out = rows_out;
  p.scores_out = scores_out;
  p.counts_out = counts_out;
  return run_threads(p, nq, nthreads);
}

/* ------------------------------------------ sharded CPU baseline (bench) */

/* The reference CPU path over a corpus split into row shards, as one
 * CpuIndex per shard (cpu.ts:66-88: WASM-SIMD dot, then topK of flat.ts:217-239
 * over the shard's rows) and the final merge of every shard's k hits with
 * mergePartials (gpuTopk.ts:160-189).  A wasm32 CpuIndex holds at most ~4 GiB
 * of corpus (cpu.ts:97-104), so a large corpus needs several.  Thread t owns
 * shards t, t + T, ... and runs the queries in order over them (one process
 * per shard in the reference's terms); the merge follows a join.  Shard s
 * holds global rows base[s] .. base[s] + rows[s] (or the rows listed in
 * map[s] when given: a filtered shard compacted to its kept rows). */
typedef struct {
  const float *const *data;
  const int64_t *rows, *base;
  const uint32_t *const *map;
  int nshards, dim, nq, k, t, nthreads;
  const float *qs;
  float *part_scores; /* nq x nshards x k */
  uint32_t *part_rows;
} shard_job_t;

static void *run_shard_job(void *arg) {
  shard_job_t *j = (shard_job_t *)arg;
  int64_t most = 0;
  for (int s = j->t; s < j->nshards; s += j->nthreads) most = j->rows[s] > most ? j->rows[s] : most;
  float *sc = (float *)malloc(sizeof(float) * (size_t)(most > 0 ? most : 1));
  uint32_t *ro = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)j->k);
  float *so = (float *)malloc(sizeof(float) * (size_t)j->k);
  for (int i = 0; i < j->nq; i++) {
    const float *q = j->qs + (size_t)i * j->dim;
    for (int s = j->t; s < j->nshards; s += j->nthreads) {
      float *ps = j->part_scores + ((size_t)i * j->nshards + s) * j->k;
      uint32_t *pr = j->part_rows + ((size_t)i * j->nshards + s) * j->k;
      int n = 0;
      if (j->rows[s] > 0) {
        bvo_wasm_dot(j->data[s], q, sc, j->rows[s], j->dim);
        n = bvo_topk_ref(sc, j->rows[s], j->k, ro, so);
      }
      for (int h = 0; h < j->k; h++) {
        if (h < n) {
          ps[h] = so[h];
          pr[h] = j->map && j->map[s] ? j->map[s][ro[h]] : (uint32_t)(j->base[s] + ro[h]);
        } else {
          ps[h] = -3.4028234663852886e38f; /* filler, dropped by the merge */
          pr[h] = 0xFFFFFFFFu;
        }
      }
    }
  }
  free(sc);
  free(ro);
  free(so);
  return NULL;
}

int bvo_cpu_sharded_query_batch(const float *const *data, const int64_t *rows, const int64_t *base,
                                const uint32_t *const *map, int nshards, int64_t total_rows, int dim,
                                const float *qs, int nq, int k, int nthreads, uint32_t *rows_out,
                                float *scores_out, int32_t *counts_out) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > nshards) nthreads = nshards;
  float *ps = (float *)malloc(sizeof(float) * (size_t)nq * nshards * k);
  uint32_t *pr = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)nq * nshards * k);
  pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)nthreads);
  shard_job_t *jobs = (shard_job_t *)malloc(sizeof(shard_job_t) * (size_t)nthreads);
  for (int t = 0; t < nthreads; t++) {
    shard_job_t j = {data, rows, base, map, nshards, dim, nq, k, t, nthreads, qs, ps, pr};
    jobs[t] = j;
    pthread_create(&th[t], NULL, run_shard_job, &jobs[t]);
  }
  for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
  for (int i = 0; i < nq; i++) {
    const size_t o = (size_t)i * nshards * k;
    counts_out[i] = bvo_merge_partials_ref(ps + o, pr + o, (int64_t)nshards * k, total_rows, k,
                                           rows_out + (size_t)i * k, scores_out + (size_t)i * k);
  }
  free(ps);
  free(pr);
  free(th);
  free(jobs);
  return 0;
}
