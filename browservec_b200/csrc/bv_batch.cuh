// bv_batch.cuh -- the batched search path: many queries against one shard on
// the tensor cores (tcgen05.mma kind::i8), for the integer scorings.
//
// A batch of B queries is scored as one int8 contraction S = Q x C^T with
// exact int32 accumulators: Q holds the queries' int8 codes (int mode: the
// corpus int8 codec applied to the rotated query; hamming: +-1 from the
// rotated query's signs), C the corpus codes widened to int8 (int4 nibbles
// sign-extended, 1-bit codes as +-1).  Every integer dot is exact, so the
// scores ((f32(idot) * rowfac) * qfac) are bit-identical to the single-query
// integer scans.
//
// Both operands live in HBM pre-arranged as the shared-memory image of a
// 128-byte-swizzled, K-major UMMA operand: a tile of T rows x 128 bytes of K
// is T*128 contiguous bytes, row r at r*128, its 16-byte chunk c stored at
// chunk c ^ (r & 7).  One 1-D bulk copy moves a tile into shared memory
// unchanged (the swizzle is a function of the shared-memory address, so the
// destination is 1024-byte aligned).
//
// Top-F selection runs in rounds over growing row ranges: the GEMM epilogue
// appends the keys that beat each query's current F-th best key to a
// per-query buffer, then a per-query select keeps the best F and raises the
// threshold for the next round.  A buffer that would overflow is flagged and
// the host repeats the batch with rounds small enough that it cannot.
//
// Per query the buffer is [kept: Fp slots | slices]: the select leaves the
// best F (sorted for Fp <= 256) in the kept region; the GEMM appends behind it
// either densely (one slice; a global atomic counter per query, used by the
// first round, whose rows all qualify) or, in later rounds, into one slice per
// GEMM CTA that handles the query, counted by shared-memory atomics and
// published at the CTA's end (no global atomic on the epilogue's hit path).
#pragma once

#include <cstdint>

namespace bv {

constexpr uint32_t kBRowTile = 256;  // corpus rows per MMA tile (UMMA N)
constexpr uint32_t kBQTile = 128;    // queries per MMA tile (UMMA M)
constexpr uint32_t kKBlock = 128;    // bytes of K per stage: one swizzle atom row
constexpr uint32_t kBRowTileBytes = kBRowTile * kKBlock;  // 32 KB
constexpr uint32_t kBQTileBytes = kBQTile * kKBlock;      // 16 KB

// Byte offset of (row r, byte k) inside one swizzled tile of 128-byte rows.
__host__ __device__ inline uint32_t sw128_offset(uint32_t r, uint32_t k) {
  return r * 128u + ((((k >> 4) ^ (r & 7u)) & 7u) << 4) + (k & 15u);
}

// Tile positions hold rows in ascending order of their score factor, so the
// rows of one tile have nearly equal factors and the tile's maximum factor
// gives a tight integer prefilter.  posrow keeps each position's row for the
// candidate keys (the tie rule orders by row, not position).
struct ExpandParams {
  const uint8_t* codes;  // rows x R packed codes
  const float* scales;   // rows
  uint32_t R, P, KB, bits;
  const uint32_t* rows;  // position pos0 + i holds row rows[i]
  uint32_t pos0, count;  // positions written
  uint32_t total;        // positions in use; positions past it are zeroed
  int8_t* tiles;         // [tile][KB] swizzled 256 x 128 int8 tiles
  float* posfac;         // per position: score factor
  uint32_t* posrow;      // per position: row
  float* tmax;           // per tile: maximum factor
};

struct PrepParams {
  const float* queries;  // nq x dim (normalized for cosine)
  const float* signs;    // rounds x P
  uint32_t nq, dim, P, KB, rounds;
  int hamming;           // 1: +-1 query from signs; 0: int8 codec
  int8_t* qtiles;        // [query tile][KB] swizzled 128 x 128 int8 tiles
  float* qfac;           // per-query factor (qscale / 127, or 1)
  uint64_t* thr;         // per-query threshold key (0 = none yet)
  uint32_t* cnt;         // per-query candidate count
};

struct GemmParams {
  const int8_t* ctiles;
  const int8_t* qtiles;
  const float* posfac;
  const uint32_t* posrow;
  const float* tmax;
  const uint32_t* mask;  // optional, 1 bit per row (not position)
  uint32_t npos, nq, KB, nqt;
  uint32_t rt0, rt1;     // row tiles of this round
  const uint64_t* thr;
  const float* qfac;
  uint64_t* cand;        // nq x cap keys: [kept Fp | slices]
  uint32_t cap, Fp;
  uint32_t sbase;        // first slot of the slices: Fp, or 0 while nothing is kept (first round)
  uint32_t* scnt;        // per slice, per query: keys appended (slice s of query q at s * nq + q)
  uint32_t max_slices;
  uint32_t slice_g;      // 0: one dense slice, global counters; else CTA c owns slice c / slice_g
                         //    of the queries of query tiles qt = c mod slice_g (mod slice_g)
  uint32_t slice_cap;    // slots per slice
  uint32_t cnt_words;    // shared-memory counter words (two 16-bit counters each), slice_g != 0
  uint32_t* overflow;    // set when a buffer would overflow
  uint32_t* err;
  uint32_t direct;       // first round without a mask: every position is a candidate and
                         // writes its key at slot (position - rt0 x 256); scnt counts them
};

struct SelectParams {
  uint64_t* cand;        // nq x cap
  uint32_t cap, F, Fp, nq;
  uint32_t* cnt;         // per query: keys in the kept region
  uint64_t* thr;
  uint32_t* scnt;        // per slice, per query: keys appended by the last GEMM (zeroed here)
  uint32_t max_slices, nslices, slice_cap, sbase;
};

}  // namespace bv
