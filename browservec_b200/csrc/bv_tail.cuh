// bv_tail.cuh -- parameters and shared-memory layout of the per-query tail
// kernel (merge of the scan's CTA lists + exact re-rank), see bv_tail.cu.
#pragma once

#include <cstdint>

namespace bv {

struct TailParams {
  const uint64_t* partials;  // G x Fp keys written by the scan (sorted per CTA if Fp <= 256)
  uint32_t G, F, Fp, capc, k;
  int rerank;
  const float* query;        // dim fp32, normalized
  const float* originals;    // rows x dim fp32
  uint32_t dim, row_base;
  uint32_t rows_bytes;       // shared-memory staging for gathered rows
  uint32_t* err;
  uint32_t* out_rows;
  float* out_scores;
  uint32_t* out_count;
  uint32_t* cand_rows;       // optional
  float* cand_scores;
  uint32_t* cand_count;
  float* cand_exact;         // optional: exact scores of the candidates, candidate order
  uint64_t* trace;           // optional: trace[kTrTail*]
  // grid of queries (batched search): CTA b serves query b, its partials at
  // partials + b * partials_stride; 0 for the one-CTA launch of a scan
  uint32_t partials_stride;
  const uint32_t* rowmap;    // optional: row of each key position (candidate-list search)
};

// Tail timestamps (globaltimer ns) in the trace record given to the tail.
enum : int { kTrTailStart = 0, kTrTailMerged = 1, kTrTailDone = 2, kTrTailGathered = 3,
             kTrTailDotted = 4, kTrTailEntry = 5, kTrTailStaged = 6 };

struct TailSmem {
  uint32_t cand_off, hist_off, misc_off, q_off, qd_off, rows_off, bar_off, total;
};

__host__ __device__ inline TailSmem tail_smem_layout(uint32_t dim, uint32_t capc, uint32_t rows_bytes) {
  auto up = [](uint32_t x, uint32_t a) { return (x + a - 1) / a * a; };
  TailSmem s;
  uint32_t o = 0;
  s.rows_off = o;
  o = up(o + rows_bytes, 128);
  s.cand_off = o;
  o = up(o + capc * 8, 16);
  s.hist_off = o;
  o = up(o + 2048 * 4, 16);
  s.misc_off = o;
  o = up(o + 128 * 4, 16);
  s.q_off = o;
  o = up(o + dim * 4 + 16, 16);
  s.qd_off = o;  // the query widened to double (batches with wide F)
  o = up(o + dim * 8, 16);
  s.bar_off = o;
  o = up(o + 16, 16);
  s.total = o;
  return s;
}

}  // namespace bv
