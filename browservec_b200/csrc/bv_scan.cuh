// bv_scan.cuh -- the fused single-query quantized flat scan for sm_100a.
//
// One launch scores one query against one corpus shard:
//   1. the producer warp's first 1-D bulk copies (TMA engine) bring the query
//      and the rotation signs into shared memory, then it streams code tiles
//      into a 2..4-stage ring;
//   2. meanwhile the 16 consumer warps rotate the query (random-sign diagonal
//      + FWHT in the operation order of rotator.ts:60-70: warp-shuffle stages
//      for len < 32, shared-memory stages above) and, for the integer modes,
//      code it with the reference int8 codec (codec.ts:32-54);
//   3. the consumers score every row of every tile in the canonical lane order
//      (asym: exact integer codes x fp32 query in fmaf chains, two rows per
//      f32x2 instruction -- the restatement of distanceQ8.ts:56-66,
//      distanceQ4.ts:44-62, distanceQ1.ts:44-66; int: dp4a / bit-plane popc;
//      hamming: xor + popc), drop rows whose mask bit is clear (a masked row
//      can never win a slot, scoreMask.ts:66-92 + mask.ts:20-35) and append
//      the (score,row) keys above the CTA threshold to a shared candidate
//      buffer, compacted by block radix select when it fills;
//   4. each CTA writes its best F keys (sorted when F <= 256) to global
//      scratch; the tail kernel (bv_tail.cu) merges them and re-ranks.
// Launches chain with programmatic dependent launch: a CTA lets the next
// kernel start once its rows are scored, and waits for the previous kernel
// (the previous query's tail) to finish before it writes the shared scratch.
// Every wait is bounded; a timeout raises a flag in `err` instead of hanging.
#pragma once

#include <cstdint>
#include <type_traits>

#include "bv_device.cuh"

namespace bv {

enum ScoreMode : int { kAsym = 0, kInt = 1, kHamming = 2 };

constexpr int kConsumerWarps = 16;
constexpr int kScanThreads = (kConsumerWarps + 1) * 32;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr uint32_t kBarConsumers = 1;  // named barrier id of the consumer warps
constexpr uint32_t kBarRotate = 2;     // named barrier id of the warps rotating the query
constexpr int kSelMax = 8;             // keys per consumer thread in a CTA selection
constexpr int kMergeMax = 24;          // keys per consumer thread in the last-CTA merge

struct ScanParams {
  const uint8_t* codes;      // rows x R bytes (capacity padded to whole tiles)
  const float* scales;       // one per row (padded like codes)
  const float* signs;        // rounds x P, pre-scaled (rotator.ts:44-58)
  const float* query;        // dim fp32, normalized by the host (store.ts:209-217)
  const uint32_t* mask;      // optional: bit r of mask[r>>5] = row r passes
  uint64_t nrows;
  uint32_t dim, P, rounds;
  uint32_t R;                // code bytes per row
  uint32_t tile_rows;        // rows per pipeline tile
  uint32_t tile_bytes;       // tile_rows * R
  uint32_t ntiles;
  uint32_t stages;           // 2..4
  uint32_t F, Fp;            // fetch, pow2 >= max(F, 32)
  uint32_t capc;             // CTA candidate buffer slots (pow2, <= kSelMax * 512, >= 2*Fp)
  uint32_t check_tiles;      // tiles between candidate-buffer checks
  uint64_t* partials;        // gridDim.x x Fp keys (this query's slot of the partials ring)
  unsigned long long* tile_ctr;  // dynamic tile counter slot: (epoch << 32) | next tile
  uint32_t epoch;            // launch number owning tile_ctr
  uint32_t serial;           // 1: the partials are shared with the previous query (wait for its tail)
  uint32_t seed;             // rotator seed (rotator.ts:44-58): signs computed on the fly
  float sign_scale;          // f32(1 / sqrt(P) in f64), the signs' magnitude
  // The query's finish by its last CTA (fold = 1, Fp <= 256): merge of the CTA
  // lists, exact re-rank and outputs, as the tail kernel does.
  uint32_t fold;
  unsigned int* done;        // CTAs of this query finished (its ring slot); reset by the last one
  uint32_t k;
  int rerank;
  const float* originals;    // rows x dim fp32
  uint32_t row_base;
  uint32_t* out_rows;
  float* out_scores;
  uint32_t* out_count;
  uint32_t* cand_rows;       // optional
  float* cand_scores;
  uint32_t* cand_count;
  float* cand_exact;
  uint32_t* err;             // error flags
  uint64_t* trace;           // optional: per-CTA phase timestamps (globaltimer ns)
  const uint32_t* rowmap;    // optional: row of each scanned position (candidate-list search)
};

// Next tile of this launch from the shared counter.  The slot still holds an
// older launch's epoch until the first grab of this launch installs its own
// (CAS), claiming tile 0; later grabs are plain atomic adds.
__device__ __forceinline__ uint32_t grab_tile(unsigned long long* ctr, uint32_t epoch, uint32_t* err) {
  unsigned long long prev = atomicAdd(ctr, 1ull);
  if (static_cast<uint32_t>(prev >> 32) == epoch) return static_cast<uint32_t>(prev);
  unsigned long long cur = prev + 1ull;
  for (int i = 0; i < 4096; ++i) {
    if (static_cast<uint32_t>(cur >> 32) == epoch) {
      prev = atomicAdd(ctr, 1ull);
      if (static_cast<uint32_t>(prev >> 32) == epoch) return static_cast<uint32_t>(prev);
      cur = prev + 1ull;
      continue;
    }
    const unsigned long long want = (static_cast<unsigned long long>(epoch) << 32) | 1ull;
    const unsigned long long got = atomicCAS(ctr, cur, want);
    if (got == cur) return 0u;
    cur = got;
  }
  atomicOr(err, kErrBadLaunch);
  return 0xFFFFFFFFu;
}

// Phase timestamps: CTA b writes trace[b*8 + phase].
enum : int { kTrEntry = 0, kTrRotated = 1, kTrScanned = 2, kTrCtaMerged = 3, kTrQueryIn = 4, kTrFirstTile = 5 };

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// The rotation of 32 <= P <= 1024 runs in registers (rotate_query_fast) on a
// padded buffer of P/32 rows of 33 floats, with the signs computed on the fly.
__host__ __device__ inline bool fast_rotation(uint32_t P) { return P >= 32 && P <= 1024; }
__host__ __device__ inline uint32_t rotation_pad_floats(uint32_t P) { return (P / 32) * 33; }

// Shared-memory carve-up (host and device agree on it).
struct ScanSmem {
  uint32_t codes_off, scales_off, bars_off, q_off, signs_off, qb_off, cand_off, hist_off, misc_off,
      total;
};

__host__ __device__ inline uint32_t align_up(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }

__host__ __device__ inline ScanSmem scan_smem_layout(uint32_t tile_bytes, uint32_t tile_rows,
                                                     uint32_t stages, uint32_t P, uint32_t rounds,
                                                     uint32_t capc) {
  ScanSmem s;
  uint32_t o = 0;
  s.codes_off = o;
  o = align_up(o + stages * tile_bytes, 128);
  s.scales_off = o;
  o = align_up(o + stages * tile_rows * 4, 128);
  s.bars_off = o;
  o = align_up(o + (2 * stages + 1) * 8 + stages * 4, 16);
  s.q_off = o;
  o = align_up(o + P * 4, 16);
  s.signs_off = o;  // the signs (P > 1024), or the padded rotation buffer (P <= 1024)
  o = align_up(o + (fast_rotation(P) ? rotation_pad_floats(P) * 4 : rounds * P * 4), 16);
  s.qb_off = o;
  o = align_up(o + P, 16);
  s.cand_off = o;
  o = align_up(o + capc * 8, 16);
  s.hist_off = o;
  o = align_up(o + kSelBins * 4, 16);
  s.misc_off = o;
  o = align_up(o + 128 * 4, 16);
  s.total = o;
  return s;
}

// Shared memory of the exact flat scan (bv_flat.cu), from a 1024-byte aligned
// base: stages of 128 rows x 32 f32 (16 KB each, swizzled), the query, the
// barriers, each stage's block and column step, then the candidate buffer,
// histogram and misc words as in the quantized scan.  `total` includes 1 KB
// of alignment slack.
struct FlatSmem {
  uint32_t rows_off, q_off, bars_off, ids_off, cand_off, hist_off, misc_off, total;
};

__host__ __device__ inline FlatSmem flat_smem_layout(uint32_t dim, uint32_t stages, uint32_t capc) {
  FlatSmem s;
  uint32_t o = 0;
  s.rows_off = o;
  o += stages * 16384u;
  s.q_off = o;
  o = align_up(o + dim * 4, 16);
  s.bars_off = o;
  o = align_up(o + (2 * stages + 1) * 8, 16);
  s.ids_off = o;
  o = align_up(o + 2 * stages * 4, 16);
  s.cand_off = o;
  o = align_up(o + capc * 8, 16);
  s.hist_off = o;
  o = align_up(o + kSelBins * 4, 16);
  s.misc_off = o;
  o = align_up(o + 128 * 4, 16);
  s.total = o + 1024;
  return s;
}

// misc word slots
enum : int { kMiscCount = 0, kMiscNc = 5, kMiscTicket = 6, kMiscQScale = 7, kMiscRed = 16, kMiscSel = 64 };

// ------------------------------------------------------------ code -> value
// int8 byte of word xb (= x ^ 0x80808080) as a biased float 2^23 + (b + 128):
// PRMT places the byte in the low mantissa; subtracting 2^23 + 128 gives b.
__device__ __forceinline__ float s8_biased(uint32_t xb, int byte) {
  return __uint_as_float(__byte_perm(xb, 0x4B00u, 0x5440u | static_cast<uint32_t>(byte)));
}
// int4 nibble of word xn (= x ^ 0x88888888) as a biased float 2^23 + (n + 8).
__device__ __forceinline__ float s4_biased(uint32_t xn, int nib) {
  return __uint_as_float(((xn >> (4 * nib)) & 0xFu) | 0x4B000000u);
}
constexpr float kBias8 = 8388736.0f;  // 2^23 + 128
constexpr float kBias4 = 8388616.0f;  // 2^23 + 8

// Butterfly sums of N = 2 or 4 rows over the L lanes of a row group with one
// shuffle per row per level while a lane still carries several rows: at
// offset L/2 the lanes of the lower half keep the first half of the rows and
// send the second (the upper half the reverse), at L/4 (N = 4) the same within
// each half, so from then on each lane carries one row.  Every level adds the
// same two values as the per-row butterfly (t[l] = s[l] + s[l ^ off]; the add
// is commutative), so each sum is bitwise the per-row butterfly's.  `own`
// receives the row this lane holds; lanes whose low log2(L/N) bits are zero
// hold one each.
__device__ __forceinline__ float lane_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ int lane_add(int a, int b) { return a + b; }
template <int N>
__device__ __forceinline__ uint32_t pick_row(const uint32_t (&rho)[N], uint32_t own) {
  if constexpr (N == 2) return own ? rho[1] : rho[0];
  else return own < 2u ? (own ? rho[1] : rho[0]) : (own == 3u ? rho[3] : rho[2]);
}
template <int L, int N, typename T>
__device__ __forceinline__ T group_sum(const T (&v)[N], int sl, uint32_t& own) {
  static_assert(N == 2 || N == 4, "two or four rows");
  static_assert(L >= N, "a lane per row at least");
  T a[N / 2];
  const bool up1 = (sl & (L / 2)) != 0;
#pragma unroll
  for (int i = 0; i < N / 2; ++i) {
    const T keep = up1 ? v[N / 2 + i] : v[i];
    const T send = up1 ? v[i] : v[N / 2 + i];
    a[i] = lane_add(keep, __shfl_xor_sync(0xffffffffu, send, L / 2));
  }
  T t;
  int next;
  if constexpr (N == 4) {
    const bool up2 = (sl & (L / 4)) != 0;
    own = (up1 ? 2u : 0u) + (up2 ? 1u : 0u);
    const T keep = up2 ? a[1] : a[0];
    const T send = up2 ? a[0] : a[1];
    t = lane_add(keep, __shfl_xor_sync(0xffffffffu, send, L / 4));
    next = L / 8;
  } else {
    own = up1 ? 1u : 0u;
    t = a[0];
    next = L / 4;
  }
#pragma unroll
  for (int off = next; off >= 1; off >>= 1) t = lane_add(t, __shfl_xor_sync(0xffffffffu, t, off));
  return t;
}

__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_us(uint32_t a_unsigned, uint32_t b_signed, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_unsigned), "r"(b_signed), "r"(c));
  return d;
}

template <int W>
struct Chunk {
  uint32_t w[W];
};

template <int W>
__device__ __forceinline__ Chunk<W> lds_chunk(const uint8_t* p) {
  Chunk<W> c;
  if constexpr (W == 4) {
    uint4 v = *reinterpret_cast<const uint4*>(p);
    c.w[0] = v.x, c.w[1] = v.y, c.w[2] = v.z, c.w[3] = v.w;
  } else if constexpr (W == 2) {
    uint2 v = *reinterpret_cast<const uint2*>(p);
    c.w[0] = v.x, c.w[1] = v.y;
  } else {
    c.w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
  return c;
}

// ----------------------------------------------------------- query prologue
// Rotate q[0..P) in place (rotator.ts:60-70): per round a sign multiply and
// the FWHT stages len = 1, 2, ..., P/2 in order.  Consumer-collective.
__device__ __forceinline__ void rotate_query(float* q, const float* signs, uint32_t P,
                                             uint32_t rounds, int ctid) {
  const int lane = ctid & 31, warp = ctid >> 5;
  for (uint32_t r = 0; r < rounds; ++r) {
    const float* s = signs + static_cast<size_t>(r) * P;
    if (P >= 32) {
      for (uint32_t blk = warp; blk < P / 32; blk += kConsumerWarps) {
        const uint32_t i = blk * 32 + lane;
        float x = __fmul_rn(q[i], s[i]);
#pragma unroll
        for (int len = 1; len < 32; len <<= 1) {
          const float y = __shfl_xor_sync(0xffffffffu, x, len);
          x = (lane & len) ? __fsub_rn(y, x) : __fadd_rn(x, y);
        }
        q[i] = x;
      }
      named_bar_sync(kBarConsumers, kConsumerThreads);
      for (uint32_t lg = 5; (1u << lg) < P; ++lg) {
        const uint32_t len = 1u << lg;
        for (uint32_t b = ctid; b < P / 2; b += kConsumerThreads) {
          const uint32_t j = ((b >> lg) << (lg + 1)) | (b & (len - 1));
          const float x = q[j], y = q[j + len];
          q[j] = __fadd_rn(x, y);
          q[j + len] = __fsub_rn(x, y);
        }
        named_bar_sync(kBarConsumers, kConsumerThreads);
      }
    } else {
      for (uint32_t i = ctid; i < P; i += kConsumerThreads) q[i] = __fmul_rn(q[i], s[i]);
      named_bar_sync(kBarConsumers, kConsumerThreads);
      for (uint32_t lg = 0; (1u << lg) < P; ++lg) {
        const uint32_t len = 1u << lg;
        for (uint32_t b = ctid; b < P / 2; b += kConsumerThreads) {
          const uint32_t j = ((b >> lg) << (lg + 1)) | (b & (len - 1));
          const float x = q[j], y = q[j + len];
          q[j] = __fadd_rn(x, y);
          q[j + len] = __fsub_rn(x, y);
        }
        named_bar_sync(kBarConsumers, kConsumerThreads);
      }
    }
  }
}

// Sign i of one rotation round: randomSigns (prng.ts:5-22) draws
// mulberry32 values in sequence, and mulberry32's state after i + 1 draws is
// seed + (i + 1) * 0x6d2b79f5, so draw i is computed directly.  Value
// u < 2^31 gives -1, scaled by f32(1/sqrt(P)) (rotator.ts:44-58).
__device__ __forceinline__ float rot_sign(uint32_t round_seed, uint32_t i, float scale) {
  const uint32_t a = round_seed + (i + 1u) * 0x6d2b79f5u;
  uint32_t t = (a ^ (a >> 15)) * (1u | a);
  t = (t + (t ^ (t >> 7)) * (61u | t)) ^ t;
  return ((t ^ (t >> 14)) < 0x80000000u) ? -scale : scale;
}

// Math.round (halves toward +inf) of an f64.
__device__ __forceinline__ double js_round(double x);

// The whole query prologue of 32 <= P <= 1024 in ONE warp, no barrier: lane c
// holds elements i = 32 r + c (r < NR = P / 32) in registers.  Per round the
// sign multiply, the FWHT stages of bits 0..4 by shuffles and of bits 5.. by
// register butterflies -- the reference's stage order (rotator.ts:60-70), the
// same f32 operations as rotate_query.  Then, by mode, the rotated query to
// q (asym), its int8 codes to qb with the codec of quantize_query8 (int,
// returns qscale), or its sign bits to qb as words (hamming).
template <int NR, int MODE>
__device__ __forceinline__ float prologue_warp(float* q, int8_t* qb, uint32_t seed, float scale, uint32_t rounds,
                                               int lane) {
  float x[NR];
#pragma unroll
  for (int r = 0; r < NR; ++r) x[r] = q[r * 32 + lane];
  for (uint32_t rd = 0; rd < rounds; ++rd) {
    const uint32_t rs = seed ^ (0x9e3779b9u * (rd + 1u));
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      float v = __fmul_rn(x[r], rot_sign(rs, static_cast<uint32_t>(r * 32 + lane), scale));
#pragma unroll
      for (int len = 1; len < 32; len <<= 1) {
        const float y = __shfl_xor_sync(0xffffffffu, v, len);
        v = (lane & len) ? __fsub_rn(y, v) : __fadd_rn(v, y);
      }
      x[r] = v;
    }
#pragma unroll
    for (int len = 1; len < NR; len <<= 1)
#pragma unroll
      for (int r = 0; r < NR; ++r)
        if ((r & len) == 0) {
          const float a = x[r], b = x[r + len];
          x[r] = __fadd_rn(a, b);
          x[r + len] = __fsub_rn(a, b);
        }
  }
  float qscale = 1.0f;
  if constexpr (MODE == 0) {  // asym: the rotated query itself
#pragma unroll
    for (int r = 0; r < NR; ++r) q[r * 32 + lane] = x[r];
  } else if constexpr (MODE == 1) {  // int: the corpus int8 codec (codec.ts:32-54)
    float m = 0.0f;
#pragma unroll
    for (int r = 0; r < NR; ++r) m = fmaxf(m, fabsf(x[r]));
#pragma unroll
    for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    qscale = m > 0.0f ? m : 1.0f;
    const double inv = __ddiv_rn(1.0, static_cast<double>(qscale));
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      double v = __dmul_rn(static_cast<double>(x[r]), inv);
      v = v < -1.0 ? -1.0 : (v > 1.0 ? 1.0 : v);
      double b = js_round(__dmul_rn(v, 127.0));
      b = b < -127.0 ? -127.0 : (b > 127.0 ? 127.0 : b);
      qb[r * 32 + lane] = static_cast<int8_t>(static_cast<int>(b));
      q[r * 32 + lane] = x[r];
    }
  } else {  // hamming: bit i of the query = rotated element i >= 0
    uint32_t* qbits = reinterpret_cast<uint32_t*>(qb);
#pragma unroll
    for (int r = 0; r < NR; ++r) {
      const uint32_t w = __ballot_sync(0xffffffffu, x[r] >= 0.0f);
      if (lane == 0) qbits[r] = w;
      q[r * 32 + lane] = x[r];
    }
  }
  return qscale;
}

// Not inlined: its register arrays get their own allocation instead of
// pressing on the scan loop's under the two-CTAs-per-SM register cap.
template <int MODE>
static __device__ __noinline__ float prologue_warp_dispatch(uint32_t P, float* q, int8_t* qb, uint32_t seed, float scale,
                                                        uint32_t rounds, int lane) {
  switch (P) {
    case 32: return prologue_warp<1, MODE>(q, qb, seed, scale, rounds, lane);
    case 64: return prologue_warp<2, MODE>(q, qb, seed, scale, rounds, lane);
    case 128: return prologue_warp<4, MODE>(q, qb, seed, scale, rounds, lane);
    case 256: return prologue_warp<8, MODE>(q, qb, seed, scale, rounds, lane);
    case 512: return prologue_warp<16, MODE>(q, qb, seed, scale, rounds, lane);
    default: return prologue_warp<32, MODE>(q, qb, seed, scale, rounds, lane);
  }
}

// The query prologue of P = 2^(6 + HB) (512 or 1024) over W = 2^HB warps,
// two elements per lane, with the arithmetic of prologue_warp.  Layout A:
// warp w, lane l, register r hold element 64 w + 32 r + l, so the FWHT stages
// of bits 0..5 are five shuffles and one register butterfly.  Layout B: the
// element ((l & (W-1)) << 6) | (w << (6-HB)) | ((l >> HB) << 1) | r, so the
// stages of bits 6.. are shuffles over lane bits 0..HB-1.  The layouts meet
// in `xs` (element i at i + i / 32, conflict-free for layout A): three
// exchanges for two rounds.  Writes the query codes like prologue_warp and
// returns qscale (int mode) to every participating thread; warps >= W do not
// take part.
template <int HB, int MODE>
static __device__ __noinline__ float prologue_multi(float* q, int8_t* qb, float* xs, float* red, uint32_t seed,
                                                    float scale, uint32_t rounds, int warp, int lane) {
  constexpr int W = 1 << HB;
  constexpr uint32_t kThreads = W * 32;
  const uint32_t ia = static_cast<uint32_t>(warp) * 64u + static_cast<uint32_t>(lane);
  const uint32_t ib = ((static_cast<uint32_t>(lane) & (W - 1u)) << 6) | (static_cast<uint32_t>(warp) << (6 - HB)) |
                      ((static_cast<uint32_t>(lane) >> HB) << 1);
  const auto pad = [](uint32_t i) { return i + (i >> 5); };
  float x0 = q[ia], x1 = q[ia + 32u];
  for (uint32_t rd = 0; rd < rounds; ++rd) {
    if (rd > 0) {  // layout B -> A
      xs[pad(ib)] = x0;
      xs[pad(ib + 1u)] = x1;
      named_bar_sync(kBarRotate, kThreads);
      x0 = xs[pad(ia)];
      x1 = xs[pad(ia + 32u)];
    }
    const uint32_t rs = seed ^ (0x9e3779b9u * (rd + 1u));
    x0 = __fmul_rn(x0, rot_sign(rs, ia, scale));
    x1 = __fmul_rn(x1, rot_sign(rs, ia + 32u, scale));
#pragma unroll
    for (int len = 1; len < 32; len <<= 1) {
      const float y0 = __shfl_xor_sync(0xffffffffu, x0, len);
      const float y1 = __shfl_xor_sync(0xffffffffu, x1, len);
      x0 = (lane & len) ? __fsub_rn(y0, x0) : __fadd_rn(x0, y0);
      x1 = (lane & len) ? __fsub_rn(y1, x1) : __fadd_rn(x1, y1);
    }
    {
      const float a = x0, b = x1;  // bit 5: the register pair
      x0 = __fadd_rn(a, b);
      x1 = __fsub_rn(a, b);
    }
    xs[pad(ia)] = x0;  // layout A -> B
    xs[pad(ia + 32u)] = x1;
    named_bar_sync(kBarRotate, kThreads);
    x0 = xs[pad(ib)];
    x1 = xs[pad(ib + 1u)];
#pragma unroll
    for (int len = 1; len < W; len <<= 1) {  // bits 6.. in stage order
      const float y0 = __shfl_xor_sync(0xffffffffu, x0, len);
      const float y1 = __shfl_xor_sync(0xffffffffu, x1, len);
      x0 = (lane & len) ? __fsub_rn(y0, x0) : __fadd_rn(x0, y0);
      x1 = (lane & len) ? __fsub_rn(y1, x1) : __fadd_rn(x1, y1);
    }
  }
  q[ib] = x0;
  q[ib + 1u] = x1;
  float qscale = 1.0f;
  if constexpr (MODE == 1) {  // int: the corpus int8 codec (codec.ts:32-54)
    float m = fmaxf(fabsf(x0), fabsf(x1));
#pragma unroll
    for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) red[warp] = m;
    named_bar_sync(kBarRotate, kThreads);
    m = 0.0f;
#pragma unroll
    for (int w = 0; w < W; ++w) m = fmaxf(m, red[w]);
    qscale = m > 0.0f ? m : 1.0f;
    const double inv = __ddiv_rn(1.0, static_cast<double>(qscale));
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      double v = __dmul_rn(static_cast<double>(r ? x1 : x0), inv);
      v = v < -1.0 ? -1.0 : (v > 1.0 ? 1.0 : v);
      double b = js_round(__dmul_rn(v, 127.0));
      b = b < -127.0 ? -127.0 : (b > 127.0 ? 127.0 : b);
      qb[ib + static_cast<uint32_t>(r)] = static_cast<int8_t>(static_cast<int>(b));
    }
  } else if constexpr (MODE == 2) {  // hamming: sign bits of 32 consecutive elements per word
    named_bar_sync(kBarRotate, kThreads);
    uint32_t* qbits = reinterpret_cast<uint32_t*>(qb);
    for (uint32_t blk = static_cast<uint32_t>(warp); blk < (64u << HB) / 32u; blk += W) {
      const uint32_t wd = __ballot_sync(0xffffffffu, q[blk * 32u + static_cast<uint32_t>(lane)] >= 0.0f);
      if (lane == 0) qbits[blk] = wd;
    }
  }
  return qscale;
}

__device__ __forceinline__ double js_round(double x) {
  double r = floor(x);
  if (__dadd_rn(x, -r) >= 0.5) r = __dadd_rn(r, 1.0);
  return r;
}

// int8 code of the rotated query with the corpus codec (codec.ts:32-54):
// qb[i] in [-127,127]; returns the f32 scale (max |rq|, or 1).
__device__ __forceinline__ float quantize_query8(const float* rq, int8_t* qb, uint32_t P, int ctid,
                                                 float* red /* >= 16 floats */) {
  float m = 0.0f;
  for (uint32_t i = ctid; i < P; i += kConsumerThreads) m = fmaxf(m, fabsf(rq[i]));
#pragma unroll
  for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((ctid & 31) == 0) red[ctid >> 5] = m;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  m = 0.0f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) m = fmaxf(m, red[w]);
  const float scale = m > 0.0f ? m : 1.0f;
  const double inv = __ddiv_rn(1.0, static_cast<double>(scale));
  for (uint32_t i = ctid; i < P; i += kConsumerThreads) {
    double v = __dmul_rn(static_cast<double>(rq[i]), inv);
    v = v < -1.0 ? -1.0 : (v > 1.0 ? 1.0 : v);
    double b = js_round(__dmul_rn(v, 127.0));
    b = b < -127.0 ? -127.0 : (b > 127.0 ? 127.0 : b);
    qb[i] = static_cast<int8_t>(static_cast<int>(b));
  }
  return scale;
}

// ------------------------------------------------------------- selection
// Append the keys of lanes with `want` to cand (warp-aggregated reservation).
__device__ __forceinline__ void append_keys(uint64_t* cand, uint32_t* count, uint64_t key, bool want,
                                            int lane) {
  const unsigned m = __ballot_sync(0xffffffffu, want);
  if (m) {
    const int leader = __ffs(m) - 1;
    uint32_t pos = 0;
    if (lane == leader) pos = atomicAdd(count, static_cast<uint32_t>(__popc(m)));
    pos = __shfl_sync(0xffffffffu, pos, leader);
    if (want) cand[pos + __popc(m & ((1u << lane) - 1u))] = key;
  }
}

// Keep the best F of the keys held in v[] (zero = empty slot; `total` nonzero
// keys across the consumers): radix select, then the survivors are written to
// cand[0..min(total,F)).  Returns the kept count.  Consumer-collective; ends
// with a barrier.  The caller must have finished reading cand into v[].
template <int MAXK>
__device__ __forceinline__ uint32_t keep_best(const uint64_t (&v)[MAXK], uint32_t total, uint32_t F,
                                              uint64_t* cand, uint32_t* hist, uint32_t* misc,
                                              int ctid) {
  const uint64_t thr = block_select_threshold<MAXK, kConsumerThreads>(
      v, MAXK, F, total, hist, misc + kMiscSel, ctid, kBarConsumers);
  if (ctid == 0) misc[kMiscCount] = 0;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  const int lane = ctid & 31;
#pragma unroll
  for (int i = 0; i < MAXK; ++i) append_keys(cand, &misc[kMiscCount], v[i], v[i] != 0ull && v[i] >= thr, lane);
  named_bar_sync(kBarConsumers, kConsumerThreads);
  return total < F ? total : F;
}

// Bitonic sort (descending) of n = 2^m keys in shared memory, consumer-collective.
__device__ __forceinline__ void cta_sort_desc(uint64_t* a, uint32_t n, int ctid) {
  for (uint32_t size = 2; size <= n; size <<= 1)
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (uint32_t i = ctid; i < n; i += kConsumerThreads) {
        const uint32_t j = i ^ stride;
        if (j > i) {
          const uint64_t x = a[i], y = a[j];
          const bool desc = (i & size) == 0;
          if (desc ? (x < y) : (x > y)) {
            a[i] = y;
            a[j] = x;
          }
        }
      }
      named_bar_sync(kBarConsumers, kConsumerThreads);
    }
}

// ------------------------------------------------- fast top-F (F <= 256)
// Warp-register sorts and merges: shuffles and register swaps, barriers only
// between the levels of the cross-warp tree.

// The CTA's best Fp keys, sorted descending, into cand[0..Fp): every warp
// sorts a slice of Fp candidates in registers, then a 4-level tree of register
// merges through shared memory.  Requires n <= 16 * Fp <= capc.
template <int E>
__device__ __forceinline__ void cta_best_sorted(uint64_t* cand, uint32_t n, int ctid) {
  constexpr int Fp = 32 * E;
  const int lane = ctid & 31, warp = ctid >> 5;
  uint64_t v[E];
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const uint32_t idx = static_cast<uint32_t>(warp * Fp + lane + 32 * r);
    v[r] = idx < n ? cand[idx] : 0ull;
  }
  wreg_sort_desc<E>(v, lane);
  named_bar_sync(kBarConsumers, kConsumerThreads);  // every slice is in registers
#pragma unroll 1
  for (int step = 1; step < kConsumerWarps; step <<= 1) {
    if ((warp % (2 * step)) == step) {
#pragma unroll
      for (int r = 0; r < E; ++r) cand[warp * Fp + lane + 32 * r] = v[r];
    }
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if ((warp % (2 * step)) == 0) {
      uint64_t b[E];
#pragma unroll
      for (int r = 0; r < E; ++r) b[r] = cand[(warp + step) * Fp + lane + 32 * r];
      wreg_merge_top<E>(v, b, lane);
    }
  }
  if (warp == 0) {
#pragma unroll
    for (int r = 0; r < E; ++r) cand[lane + 32 * r] = v[r];
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);
}

// Last CTA: merge the G sorted CTA lists (partials, Fp keys each) into
// out[0..Fp), descending.  Warps merge strided lists in registers (the next
// list loads while the current one merges), then the same 4-level tree
// through `stage` (16 * Fp keys); out may alias stage.
// A key of a CTA list: from shared memory, or from global memory past L1
// (the lists were written by another kernel).
template <bool kSmemSrc>
__device__ __forceinline__ uint64_t load_key(const uint64_t* p) {
  if constexpr (kSmemSrc) return *p;
  else return __ldcg(p);
}

template <int E, bool kSmemSrc = false>
__device__ __forceinline__ void merge_cta_lists(const uint64_t* partials, uint32_t G, uint64_t* stage,
                                             int ctid) {
  constexpr int Fp = 32 * E;
  const int lane = ctid & 31, warp = ctid >> 5;
  uint64_t v[E], nx[E];
#pragma unroll
  for (int r = 0; r < E; ++r) {
    v[r] = 0ull;
    nx[r] = static_cast<uint32_t>(warp) < G ? load_key<kSmemSrc>(partials + static_cast<size_t>(warp) * Fp + lane + 32 * r) : 0ull;
  }
#pragma unroll 1
  for (uint32_t l = warp; l < G; l += kConsumerWarps) {
    uint64_t cur[E];
#pragma unroll
    for (int r = 0; r < E; ++r) cur[r] = nx[r];
    const uint32_t ln = l + kConsumerWarps;
#pragma unroll
    for (int r = 0; r < E; ++r) nx[r] = ln < G ? load_key<kSmemSrc>(partials + static_cast<size_t>(ln) * Fp + lane + 32 * r) : 0ull;
    wreg_merge_top<E>(v, cur, lane);
  }
#pragma unroll 1
  for (int step = 1; step < kConsumerWarps; step <<= 1) {
    if ((warp % (2 * step)) == step) {
#pragma unroll
      for (int r = 0; r < E; ++r) stage[warp * Fp + lane + 32 * r] = v[r];
    }
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if ((warp % (2 * step)) == 0) {
      uint64_t b[E];
#pragma unroll
      for (int r = 0; r < E; ++r) b[r] = stage[(warp + step) * Fp + lane + 32 * r];
      wreg_merge_top<E>(v, b, lane);
    }
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);  // tree reads of stage are done
  if (warp == 0) {
#pragma unroll
    for (int r = 0; r < E; ++r) stage[lane + 32 * r] = v[r];
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);
}

// Warp 0 sorts a[0..32E) descending in place (the other warps return).
template <int E>
__device__ __forceinline__ void warp0_sort_smem(uint64_t* a, int ctid) {
  if ((ctid >> 5) != 0) return;
  const int lane = ctid & 31;
  uint64_t v[E];
#pragma unroll
  for (int r = 0; r < E; ++r) v[r] = a[lane + 32 * r];
  wreg_sort_desc<E>(v, lane);
#pragma unroll
  for (int r = 0; r < E; ++r) a[lane + 32 * r] = v[r];
}

__device__ __forceinline__ void cta_best_sorted_dispatch(uint32_t Fp, uint64_t* cand, uint32_t n, int ctid) {
  if (Fp == 32) cta_best_sorted<1>(cand, n, ctid);
  else if (Fp == 64) cta_best_sorted<2>(cand, n, ctid);
  else if (Fp == 128) cta_best_sorted<4>(cand, n, ctid);
  else cta_best_sorted<8>(cand, n, ctid);
}
template <bool kSmemSrc = false>
__device__ __forceinline__ void merge_cta_lists_dispatch(uint32_t Fp, const uint64_t* partials, uint32_t G,
                                                         uint64_t* stage, int ctid) {
  if (Fp == 32) merge_cta_lists<1, kSmemSrc>(partials, G, stage, ctid);
  else if (Fp == 64) merge_cta_lists<2, kSmemSrc>(partials, G, stage, ctid);
  else if (Fp == 128) merge_cta_lists<4, kSmemSrc>(partials, G, stage, ctid);
  else merge_cta_lists<8, kSmemSrc>(partials, G, stage, ctid);
}
__device__ __forceinline__ void warp0_sort_dispatch(uint32_t Fp, uint64_t* a, int ctid) {
  if (Fp == 32) warp0_sort_smem<1>(a, ctid);
  else if (Fp == 64) warp0_sort_smem<2>(a, ctid);
  else if (Fp == 128) warp0_sort_smem<4>(a, ctid);
  else warp0_sort_smem<8>(a, ctid);
}

// The best Fp keys of G sorted lists (descending, Fp keys each, zero padded)
// (in shared memory, or in global memory read past L1), sorted into cand[0..Fp).  Only the list heads are
// touched: the first m = ceil(F / G) keys of every list are a set of at least
// F keys, so their F-th largest, L, is no greater than the F-th best key
// overall, and every key of the best F is >= L.  Each list's keys >= L (a
// binary search) are gathered and the few of them sorted.  Returns false,
// having written nothing, when more than 16 * Fp keys qualify (the caller then
// merges the whole lists).
template <bool kSmemSrc>
__device__ __forceinline__ bool select_list_heads(const uint64_t* lists, uint32_t G, uint32_t F, uint32_t Fp, uint64_t* cand,
                                  uint32_t* misc, int ctid) {
  const int lane = ctid & 31, warp = ctid >> 5;
  if (G > static_cast<uint32_t>(kConsumerThreads)) return false;
  uint64_t* lsh = reinterpret_cast<uint64_t*>(misc + kMiscSel);
  const uint32_t m = (F + G - 1) / G;                 // head keys per list
  const uint32_t H = G * (m < Fp ? m : Fp);           // head set size (>= F unless the lists are short)
  // (head key h is key h / G of list h % G)
  if (ctid == 0) *lsh = 0ull;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  // L: the head key whose rank among the heads (keys are unique) is F - 1
  const uint32_t mh = m < Fp ? m : Fp;
  for (uint32_t h = ctid; h < H; h += kConsumerThreads) {
    const uint64_t key = load_key<kSmemSrc>(lists + static_cast<size_t>(h % G) * Fp + h / G);
    uint32_t rank = 0;
    for (uint32_t pos = 0; pos < mh; ++pos) {  // every thread reads the same key: broadcasts
      const uint64_t* col = lists + pos;
#pragma unroll 4
      for (uint32_t l = 0; l < G; ++l) rank += load_key<kSmemSrc>(col + static_cast<size_t>(l) * Fp) > key ? 1u : 0u;
    }
    if (rank == F - 1) *lsh = key;
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);
  const uint64_t L = *lsh;
  const uint64_t lo = L ? L : 1ull;  // zero keys are empty slots
  // keys >= lo in this thread's list: its first position below lo
  uint32_t c = 0;
  if (static_cast<uint32_t>(ctid) < G) {
    const uint64_t* li = lists + static_cast<size_t>(ctid) * Fp;
    uint32_t a = 0, b = Fp;
    while (a < b) {
      const uint32_t mid = (a + b) >> 1;
      if (load_key<kSmemSrc>(li + mid) >= lo) a = mid + 1;
      else b = mid;
    }
    c = a;
  }
  uint32_t inc = c;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, inc, off);
    if (lane >= off) inc += y;
  }
  if (lane == 31) misc[kMiscRed + warp] = inc;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  uint32_t before = 0, S = 0;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) {
    const uint32_t t = misc[kMiscRed + w];
    before += w < warp ? t : 0u;
    S += t;
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);  // misc is reused by the sorts
  if (S > 16u * Fp) return false;
  const uint32_t off = before + inc - c;
  for (uint32_t j = 0; j < c; ++j) cand[off + j] = load_key<kSmemSrc>(lists + static_cast<size_t>(ctid) * Fp + j);
  const uint32_t span = S <= Fp ? Fp : 16u * Fp;
  for (uint32_t i = S + ctid; i < span; i += kConsumerThreads) cand[i] = 0ull;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  if (S <= Fp) {
    warp0_sort_dispatch(Fp, cand, ctid);
    named_bar_sync(kBarConsumers, kConsumerThreads);
  } else {
    cta_best_sorted_dispatch(Fp, cand, S, ctid);
  }
  return true;
}


// select_list_heads for lists in global memory (written by other CTAs of the
// same grid, read past L1), with the same result: the head keys are staged in
// shared memory (`heads`, >= G * min(ceil(F / G), Fp) keys) by one round of
// loads, ranked there, and every list's count of keys >= L is found by
// probing four keys at a time from its start (the count is a prefix: the
// lists are sorted), the first four kept in registers for the gather.  Two
// rounds of memory latency instead of one per head key and per bisection step.
__device__ __forceinline__ bool select_list_heads_global(const uint64_t* lists, uint32_t G, uint32_t F, uint32_t Fp,
                                                         uint64_t* cand, uint32_t* misc, uint64_t* heads,
                                                         int ctid, uint64_t* tr = nullptr) {
  const int lane = ctid & 31, warp = ctid >> 5;
  if (G > static_cast<uint32_t>(kConsumerThreads)) return false;
  uint64_t* lsh = reinterpret_cast<uint64_t*>(misc + kMiscSel);
  const uint32_t m = (F + G - 1) / G;
  const uint32_t mh = m < Fp ? m : Fp;
  const uint32_t H = G * mh;  // head key h is key h / G of list h % G
  for (uint32_t h = ctid; h < H; h += kConsumerThreads)
    heads[h] = __ldcg(lists + static_cast<size_t>(h % G) * Fp + h / G);
  if (ctid == 0) *lsh = 0ull;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  for (uint32_t h = ctid; h < H; h += kConsumerThreads) {
    const uint64_t key = heads[h];
    uint32_t rank = 0;
#pragma unroll 4
    for (uint32_t i = 0; i < H; ++i) rank += heads[i] > key ? 1u : 0u;  // broadcasts
    if (rank == F - 1) *lsh = key;
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);
  if (tr) tr[5] = globaltimer();
  const uint64_t L = *lsh;
  const uint64_t lo = L ? L : 1ull;  // zero keys are empty slots
  uint32_t c = 0;
  uint64_t k0 = 0ull, k1 = 0ull, k2 = 0ull, k3 = 0ull;
  const uint64_t* li = lists + static_cast<size_t>(ctid) * Fp;
  if (static_cast<uint32_t>(ctid) < G) {
    k0 = __ldcg(li);
    k1 = __ldcg(li + 1);
    k2 = __ldcg(li + 2);
    k3 = __ldcg(li + 3);
    c = (k0 >= lo) + (k1 >= lo) + (k2 >= lo) + (k3 >= lo);
    if (c == 4u) {
      for (uint32_t a = 4; a < Fp; a += 4) {  // Fp is a multiple of 32
        const uint32_t n = (__ldcg(li + a) >= lo) + (__ldcg(li + a + 1) >= lo) + (__ldcg(li + a + 2) >= lo) +
                           (__ldcg(li + a + 3) >= lo);
        c += n;
        if (n < 4u) break;
      }
    }
  }
  uint32_t inc = c;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, inc, off);
    if (lane >= off) inc += y;
  }
  if (lane == 31) misc[kMiscRed + warp] = inc;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  uint32_t before = 0, S = 0;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) {
    const uint32_t t = misc[kMiscRed + w];
    before += w < warp ? t : 0u;
    S += t;
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);  // misc is reused by the sorts
  if (S > 16u * Fp) return false;
  const uint32_t off = before + inc - c;
  if (c > 0u) cand[off] = k0;
  if (c > 1u) cand[off + 1] = k1;
  if (c > 2u) cand[off + 2] = k2;
  if (c > 3u) cand[off + 3] = k3;
  for (uint32_t j = 4; j < c; ++j) cand[off + j] = __ldcg(li + j);
  const uint32_t span = S <= Fp ? Fp : 16u * Fp;
  for (uint32_t i = S + ctid; i < span; i += kConsumerThreads) cand[i] = 0ull;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  if (tr) tr[6] = globaltimer();
  if (tr) tr[7] = S;
  if (S <= Fp) {
    warp0_sort_dispatch(Fp, cand, ctid);
    named_bar_sync(kBarConsumers, kConsumerThreads);
  } else {
    cta_best_sorted_dispatch(Fp, cand, S, ctid);
  }
  return true;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// The last CTA of a query finishes it (ScanParams::fold): the best F of every
// CTA's list (list-head selection, else the full merge), the candidate
// outputs, the exact f64 re-rank of Store.dotRow (src/store/store.ts:114-130:
// four lanes j accumulating elements j, j+4, ..., summed ((a0+a1)+a2)+a3, then
// the tail), and the best k (src/index.ts:583-594).  The candidates' rows are
// staged in shared memory by 1-D bulk copies (rows of a multiple of 4 floats;
// otherwise they are read from global memory), in batches that fit.
// Consumer-collective; `scratch` is `scratch_bytes` (>= 16 KB, 16-byte
// aligned) of free shared memory, `bar` an mbarrier whose phase 0 has
// completed and that nothing else uses now; cand holds >= 16 * Fp keys.
static __device__ __noinline__ void finish_query(const ScanParams& p, uint64_t* cand, uint32_t* misc,
                                                 uint8_t* scratch, uint32_t scratch_bytes, uint64_t* bar,
                                                 int ctid) {
  const int warp = ctid >> 5, lane = ctid & 31;
  const uint32_t G = gridDim.x;
  // phase trace of the finishing CTA: the tail kernel's slots after the grid's
  uint64_t* tr = p.trace && ctid == 0 ? p.trace + static_cast<size_t>(G) * 8 : nullptr;
  if (tr) tr[0] = globaltimer();
  // scratch: [query: dim floats][work: the list heads, then the staged rows]
  float* qx = reinterpret_cast<float*>(scratch);
  const uint32_t qbytes = align_up(p.dim * 4u, 16);
  uint8_t* work = scratch + qbytes;
  const uint32_t work_bytes = scratch_bytes > qbytes ? scratch_bytes - qbytes : 0u;
  // the query's copy starts now and lands while the lists merge (phase 1 of bar)
  const bool q_async = p.rerank && (p.dim & 3u) == 0u && (reinterpret_cast<uintptr_t>(p.query) & 15u) == 0u &&
                       qbytes <= scratch_bytes;
  if (q_async && ctid == 0) {
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar, p.dim * 4u);
    bulk_g2s(qx, p.query, p.dim * 4u, bar);
  }
  const uint32_t mh0 = (p.F + G - 1) / G;
  const size_t H0 = static_cast<size_t>(G) * (mh0 < p.Fp ? mh0 : p.Fp);
  const bool heads_fit = H0 * 8 <= work_bytes;
  if (!(heads_fit && select_list_heads_global(p.partials, G, p.F, p.Fp, cand, misc,
                                              reinterpret_cast<uint64_t*>(work), ctid, tr)))
    merge_cta_lists_dispatch(p.Fp, p.partials, G, cand, ctid);
  if (tr) tr[1] = globaltimer();
  if (warp == 0) {
    uint32_t c = 0;
    for (uint32_t i = lane; i < p.Fp; i += 32) {
      if (i >= p.F) cand[i] = 0ull;
      c += __popc(__ballot_sync(0xffffffffu, i < p.F && cand[i] != 0ull));
    }
    if (lane == 0) misc[kMiscNc] = c;
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);
  const uint32_t nc = misc[kMiscNc];
  if (p.cand_rows) {
    for (uint32_t i = ctid; i < nc; i += kConsumerThreads) {
      p.cand_rows[i] = map_row(p.rowmap, key_row(cand[i])) + p.row_base;
      p.cand_scores[i] = key_score(cand[i]);
    }
    if (ctid == 0) *p.cand_count = nc;
  }
  const uint32_t n = nc < p.k ? nc : p.k;
  if (p.rerank) {
    // staged rows (dim floats each) in the work area; a warp scores two rows
    // at a time (dot_rows2_exact_warp)
    float* rows_s = reinterpret_cast<float*>(work);
    const uint32_t cap = work_bytes / (p.dim * 4u);
    const bool staged = (p.dim & 3u) == 0u && (reinterpret_cast<uintptr_t>(p.originals) & 15u) == 0u && cap > 0u;
    const uint32_t batch = staged ? cap : (nc > 0u ? nc : 1u);
    // rows past the first batch are asked of L2 now, so the later batches'
    // copies do not wait on HBM one batch after another
    if (staged && nc > batch && warp == 1)
      for (uint32_t r = batch + static_cast<uint32_t>(lane); r < nc; r += 32)
        bulk_prefetch_l2(p.originals + static_cast<size_t>(map_row(p.rowmap, key_row(cand[r]))) * p.dim,
                         p.dim * 4u);
    // the head staging above wrote the work area through the generic proxy;
    // the bulk copies below write it through the async proxy
    fence_proxy_async_smem();
    uint32_t parity = 1;  // the barrier's phase 0 (the scan's query copy) has completed
    if (q_async) {
      mbar_wait_bounded(bar, parity, p.err);
      parity ^= 1u;
    } else {
      for (uint32_t i = ctid; i < p.dim; i += kConsumerThreads) qx[i] = p.query[i];
    }
    uint64_t* ex = cand + p.Fp;
    named_bar_sync(kBarConsumers, kConsumerThreads);
    for (uint32_t c0 = 0; c0 < nc; c0 += batch) {
      const uint32_t nb = nc - c0 < batch ? nc - c0 : batch;
      if (staged) {
        if (warp == 0) {
          if (lane == 0) mbar_arrive_expect_tx(bar, nb * p.dim * 4u);
          __syncwarp();
          for (uint32_t r = lane; r < nb; r += 32)
            bulk_g2s(rows_s + static_cast<size_t>(r) * p.dim,
                     p.originals + static_cast<size_t>(map_row(p.rowmap, key_row(cand[c0 + r]))) * p.dim,
                     p.dim * 4u, bar);
        }
        mbar_wait_bounded(bar, parity, p.err);
        if (tr && c0 == 0) tr[3] = globaltimer();
        parity ^= 1u;
      }
      for (uint32_t r = static_cast<uint32_t>(warp); r < nb; r += 2u * kConsumerWarps) {
        const uint32_t r2 = r + kConsumerWarps;
        const uint32_t row = key_row(cand[c0 + r]);
        const float* xa = staged ? rows_s + static_cast<size_t>(r) * p.dim
                                 : p.originals + static_cast<size_t>(map_row(p.rowmap, row)) * p.dim;
        if (r2 < nb) {
          const uint32_t row2 = key_row(cand[c0 + r2]);
          const float* xb = staged ? rows_s + static_cast<size_t>(r2) * p.dim
                                   : p.originals + static_cast<size_t>(map_row(p.rowmap, row2)) * p.dim;
          float sa, sb;
          if (staged) dot_rows2_exact_warp<false>(xa, xb, qx, p.dim, lane, sa, sb);
          else dot_rows2_exact_warp<true>(xa, xb, qx, p.dim, lane, sa, sb);
          if (lane == 0) {
            ex[c0 + r] = make_key(sa, row);
            ex[c0 + r2] = make_key(sb, row2);
          }
        } else {
          const float sc = staged ? dot_row_exact_warp<false>(xa, qx, p.dim, lane)
                                  : dot_row_exact_warp<true>(xa, qx, p.dim, lane);
          if (lane == 0) ex[c0 + r] = make_key(sc, row);
        }
      }
      if (staged) {  // this batch's rows are read before the next batch's copies land
        fence_proxy_async_smem();
        named_bar_sync(kBarConsumers, kConsumerThreads);
      }
    }
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if (tr) tr[4] = globaltimer();
    if (p.cand_exact)
      for (uint32_t i = ctid; i < nc; i += kConsumerThreads) p.cand_exact[i] = key_score(ex[i]);
    for (uint32_t i = nc + static_cast<uint32_t>(ctid); i < p.Fp; i += kConsumerThreads) ex[i] = 0ull;
    named_bar_sync(kBarConsumers, kConsumerThreads);
    warp0_sort_dispatch(p.Fp, ex, ctid);
    if (warp == 0) {
      __syncwarp();
      for (uint32_t i = lane; i < n; i += 32) {
        p.out_rows[i] = map_row(p.rowmap, key_row(ex[i])) + p.row_base;
        p.out_scores[i] = key_score(ex[i]);
      }
    }
  } else {
    for (uint32_t i = ctid; i < n; i += kConsumerThreads) {
      p.out_rows[i] = map_row(p.rowmap, key_row(cand[i])) + p.row_base;
      p.out_scores[i] = key_score(cand[i]);
    }
  }
  if (ctid == 0) {
    *p.out_count = n;
    *p.done = 0u;  // the slot's counter starts from zero at its next use
  }
  if (tr) tr[2] = globaltimer();
}

// Consumer-collective, at the same point in every consumer: when more than
// `high` keys wait in cand, keep the best F and raise the admission threshold
// `thr` to just below the F-th best, so the next stretch of rows cannot
// overflow the buffer and no dropped key is re-admitted.
__device__ __forceinline__ void raise_threshold(uint64_t* cand, uint32_t* hist, uint32_t* misc, uint32_t F,
                                                uint32_t high, uint64_t& thr, int ctid) {
  const int warp = ctid >> 5, lane = ctid & 31;
  float* miscf = reinterpret_cast<float*>(misc);
  named_bar_sync(kBarConsumers, kConsumerThreads);
  const uint32_t n = misc[kMiscCount];
  if (n > high) {  // uniform: every consumer read the same count after the barrier
    uint64_t v[kSelMax];
#pragma unroll
    for (int i = 0; i < kSelMax; ++i) {
      const uint32_t idx = static_cast<uint32_t>(ctid) + static_cast<uint32_t>(i) * kConsumerThreads;
      v[i] = idx < n ? cand[idx] : 0ull;
    }
    named_bar_sync(kBarConsumers, kConsumerThreads);
    keep_best<kSelMax>(v, n, F, cand, hist, misc, ctid);
    // the F-th best key is the smallest kept one; admit only keys above it
    uint64_t lo = ~0ull;
    for (uint32_t i = ctid; i < F; i += kConsumerThreads) lo = cand[i] < lo ? cand[i] : lo;
#pragma unroll
    for (int off = 16; off; off >>= 1) {
      const uint64_t o = __shfl_xor_sync(0xffffffffu, lo, off);
      lo = o < lo ? o : lo;
    }
    if (lane == 0) reinterpret_cast<uint64_t*>(miscf + kMiscRed)[warp] = lo;
    named_bar_sync(kBarConsumers, kConsumerThreads);
    uint64_t t2 = ~0ull;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const uint64_t o = reinterpret_cast<const uint64_t*>(miscf + kMiscRed)[w];
      t2 = o < t2 ? o : t2;
    }
    thr = t2 - 1;  // keys > F-th best - 1, i.e. >= it (never re-admits the dropped ones)
    named_bar_sync(kBarConsumers, kConsumerThreads);
  }
}

// Consumer-collective end of a CTA's scan: its best F keys (sorted for
// Fp <= 256) into its row of p.partials; with p.fold, the CTA that finishes
// last takes every list and finishes the query (finish_query, with `scratch`
// and `bar` as described there).
__device__ __forceinline__ void cta_publish(const ScanParams& p, uint64_t* cand, uint32_t* hist, uint32_t* misc,
                                            uint8_t* scratch, uint32_t scratch_bytes, uint64_t* bar, int ctid) {
  // ---------------------------------------------- best F of this CTA
  uint32_t n = misc[kMiscCount];
  if (n > (p.Fp <= 256u ? 16u * p.Fp : p.F)) {  // radix-compact to F first
    uint64_t v[kSelMax];
#pragma unroll
    for (int i = 0; i < kSelMax; ++i) {
      const uint32_t idx = static_cast<uint32_t>(ctid) + static_cast<uint32_t>(i) * kConsumerThreads;
      v[i] = idx < n ? cand[idx] : 0ull;
    }
    named_bar_sync(kBarConsumers, kConsumerThreads);
    n = keep_best<kSelMax>(v, n, p.F, cand, hist, misc, ctid);
  }
  if (p.Fp <= 256u) {
    cta_best_sorted_dispatch(p.Fp, cand, n, ctid);
    if (p.serial) pdl_wait();  // the previous query's tail has read the shared partials
    for (uint32_t i = ctid; i < p.Fp; i += kConsumerThreads)
      p.partials[static_cast<size_t>(blockIdx.x) * p.Fp + i] = i < p.F ? cand[i] : 0ull;
  } else {
    // wide F: unsorted best F (the last CTA re-selects them)
    const uint32_t m = n < p.F ? n : p.F;
    if (p.serial) pdl_wait();
    for (uint32_t i = ctid; i < p.Fp; i += kConsumerThreads)
      p.partials[static_cast<size_t>(blockIdx.x) * p.Fp + i] = i < m ? cand[i] : 0ull;
  }
  __threadfence();
  if (p.trace && threadIdx.x == 0) p.trace[blockIdx.x * 8 + kTrCtaMerged] = globaltimer();
  if (p.fold) {
    // every thread's list writes are fenced; the CTA that finishes last
    // sees all lists and finishes the query
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if (ctid == 0) misc[kMiscTicket] = atomicAdd(p.done, 1u);
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if (misc[kMiscTicket] == gridDim.x - 1u) {
      __threadfence();
      finish_query(p, cand, misc, scratch, scratch_bytes, bar, ctid);
    }
  }
}

// ------------------------------------------------------------------ kernel
// BITS 8/4/1; MODE asym/int/hamming; CB chunk bytes (4, 8 or 16); L lanes per
// row; CPL chunks per lane; U rows in flight per row-group (asym: even, two
// rows per f32x2 accumulator).
// Largest per-lane query slice (elements) the asym scan keeps in registers;
// longer slices are read from shared memory.
#ifndef BV_ASYM_QREG_MAX
#define BV_ASYM_QREG_MAX 64
#endif

template <int BITS, int MODE, int CB, int L, int CPL, int U>
struct ScanCfg {
  static constexpr int W = CB / 4;                                     // words per chunk
  static constexpr int EPW = BITS == 8 ? 4 : (BITS == 4 ? 8 : 32);    // elements per word
  static constexpr int EPC = W * EPW;                                  // elements per chunk
  static constexpr int G = 32 / L;                                     // rows per warp step
  static constexpr int RPI = kConsumerWarps * G * U;                   // rows per iteration
  static constexpr bool kQReg = (MODE == kAsym) && (CPL * EPC <= BV_ASYM_QREG_MAX);  // fp32 query in registers
  // per-chunk integer query words: int8 W, int4 2W (even/odd), 1-bit 8W planes, hamming W
  static constexpr int QW = MODE == kInt ? (BITS == 8 ? W : (BITS == 4 ? 2 * W : 8 * W))
                                         : (MODE == kHamming ? W : 1);
};

// Two CTAs per SM (consecutive queries overlap on an SM: one streams while
// the other starts or finishes): at most 56 registers a thread.
template <int BITS, int MODE, int CB, int L, int CPL, int U>
__global__ void __launch_bounds__(kScanThreads, 2) scan_kernel(const ScanParams p) {
  using C = ScanCfg<BITS, MODE, CB, L, CPL, U>;
  extern __shared__ __align__(128) uint8_t smem[];
  const ScanSmem lay = scan_smem_layout(p.tile_bytes, p.tile_rows, p.stages, p.P, p.rounds, p.capc);
  uint8_t* s_codes = smem + lay.codes_off;
  float* s_scales = reinterpret_cast<float*>(smem + lay.scales_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + lay.bars_off);
  uint64_t* empty = full + p.stages;
  uint64_t* qbar = empty + p.stages;  // query + signs landed
  volatile uint32_t* tile_ids = reinterpret_cast<volatile uint32_t*>(qbar + 1);  // tile in each stage
  float* q = reinterpret_cast<float*>(smem + lay.q_off);  // query, rotated in place
  float* s_signs = reinterpret_cast<float*>(smem + lay.signs_off);
  int8_t* qb = reinterpret_cast<int8_t*>(smem + lay.qb_off);
  uint64_t* cand = reinterpret_cast<uint64_t*>(smem + lay.cand_off);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + lay.hist_off);
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + lay.misc_off);
  float* miscf = reinterpret_cast<float*>(misc);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (p.trace && threadIdx.x == 0) p.trace[blockIdx.x * 8 + kTrEntry] = globaltimer();
  constexpr uint32_t kNoTile = 0xFFFFFFFFu;  // end-of-work marker in tile_ids
  // bulk part of the query copy: whole 16-byte blocks of a 16-byte aligned query
  const uint32_t q_bulk =
      (reinterpret_cast<uintptr_t>(p.query) & 15u) == 0 ? (p.dim * 4u) & ~15u : 0u;

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    mbar_init(qbar, 1);
    misc[kMiscCount] = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // Programmatic dependent launch, triggered at once: the next kernel in the
  // stream (this query's tail, which then lets the next query's scan launch)
  // may be scheduled now, so an SM this scan's CTA leaves is taken by the next
  // query's CTA without waiting for the slowest CTA of this one.  Nothing the
  // next kernels write is read here, and the shared scratch is written only
  // after griddepcontrol.wait below.
  pdl_trigger();

  if (warp == kConsumerWarps) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      const uint32_t sbytes = fast_rotation(p.P) ? 0u : p.rounds * p.P * 4u;  // fast: signs on the fly
      mbar_arrive_expect_tx(qbar, q_bulk + sbytes);
      if (q_bulk) bulk_g2s(q, p.query, q_bulk, qbar);
      if (sbytes) bulk_g2s(s_signs, p.signs, sbytes, qbar);
      const uint32_t bytes = p.tile_bytes + p.tile_rows * 4;
      const uint64_t stream_policy = l2_policy_evict_first();  // codes are read once per query
      // tiles come from a shared counter, so faster SMs take more of them
      uint32_t t = grab_tile(p.tile_ctr, p.epoch, p.err);
      // stage s and its phase ph advance with the loop (no division by the
      // runtime stage count)
      uint32_t s = 0, ph = 0;
      for (uint32_t it = 0;; ++it, s = s + 1u == p.stages ? 0u : s + 1u, ph ^= s == 0u ? 1u : 0u) {
        if (it >= p.stages && !mbar_wait_bounded(&empty[s], ph ^ 1u, p.err)) break;
        if (t >= p.ntiles) {  // no more work: an empty stage tells the consumers
          tile_ids[s] = kNoTile;
          mbar_arrive(&full[s]);
          break;
        }
        tile_ids[s] = t;
        mbar_arrive_expect_tx(&full[s], bytes);
        bulk_g2s_hint(s_codes + static_cast<size_t>(s) * p.tile_bytes,
                      p.codes + static_cast<size_t>(t) * p.tile_bytes, p.tile_bytes, &full[s], stream_policy);
        bulk_g2s_hint(s_scales + static_cast<size_t>(s) * p.tile_rows,
                      p.scales + static_cast<size_t>(t) * p.tile_rows, p.tile_rows * 4, &full[s], stream_policy);
        t = grab_tile(p.tile_ctr, p.epoch, p.err);
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- consumers
    const int ctid = threadIdx.x;
    mbar_wait_bounded(qbar, 0, p.err);
    if (p.trace && ctid == 0) p.trace[blockIdx.x * 8 + kTrQueryIn] = globaltimer();
    for (uint32_t i = q_bulk / 4 + ctid; i < p.P; i += kConsumerThreads)
      q[i] = i < p.dim ? p.query[i] : 0.0f;
    named_bar_sync(kBarConsumers, kConsumerThreads);
    float qfac = 1.0f;
    if (fast_rotation(p.P)) {
      // P <= 256: one warp rotates and codes the query; P = 512, 1024: 8 or
      // 16 warps with three exchanges.  The others wait at one barrier.
      constexpr int M = MODE == kAsym ? 0 : (MODE == kInt ? 1 : 2);
      float qscale = 0.0f;
      bool lead = false;
      if (p.P == 1024u) {
        qscale = prologue_multi<4, M>(q, qb, s_signs, miscf + kMiscRed, p.seed, p.sign_scale, p.rounds, warp, lane);
        lead = ctid == 0;
      } else if (p.P == 512u) {
        if (warp < 8)
          qscale = prologue_multi<3, M>(q, qb, s_signs, miscf + kMiscRed, p.seed, p.sign_scale, p.rounds, warp, lane);
        lead = ctid == 0;
      } else if (warp == 0) {
        qscale = prologue_warp_dispatch<M>(p.P, q, qb, p.seed, p.sign_scale, p.rounds, lane);
        lead = lane == 0;
      }
      if (lead) miscf[kMiscQScale] = qscale;
      named_bar_sync(kBarConsumers, kConsumerThreads);
      if constexpr (MODE == kInt) qfac = __fmul_rn(miscf[kMiscQScale], kInv127);
    } else {
      rotate_query(q, s_signs, p.P, p.rounds, ctid);
      if constexpr (MODE == kInt) {
        const float qscale = quantize_query8(q, qb, p.P, ctid, miscf + kMiscRed);
        qfac = __fmul_rn(qscale, kInv127);
      } else if constexpr (MODE == kHamming) {
        uint32_t* qbits = reinterpret_cast<uint32_t*>(qb);
        for (uint32_t blk = warp; blk < p.P / 32; blk += kConsumerWarps)
          qbits[blk] = __ballot_sync(0xffffffffu, q[blk * 32 + lane] >= 0.0f);
      }
    }
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if (p.trace && threadIdx.x == 0) p.trace[blockIdx.x * 8 + kTrRotated] = globaltimer();

    const int g = lane / L, sl = lane % L;
    // lane-resident query slices
    uint64_t qf2[C::kQReg ? CPL : 1][C::kQReg ? C::EPC / 2 : 1];  // fp32 query pairs
    uint32_t qw[MODE == kAsym ? 1 : CPL][C::QW];
    int qsum = 0;
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const uint32_t e0 = static_cast<uint32_t>(sl + j * L) * C::EPC;  // first element of chunk
      if constexpr (C::kQReg) {
#pragma unroll
        for (int e = 0; e < C::EPC / 2; ++e) qf2[j][e] = reinterpret_cast<const uint64_t*>(q + e0)[e];
      } else if constexpr (MODE == kInt && BITS == 8) {
#pragma unroll
        for (int w = 0; w < C::W; ++w) qw[j][w] = reinterpret_cast<const uint32_t*>(qb + e0)[w];
      } else if constexpr (MODE == kInt && BITS == 4) {
#pragma unroll
        for (int w = 0; w < C::W; ++w) {
          const uint8_t* b = reinterpret_cast<const uint8_t*>(qb + e0 + 8 * w);
          qw[j][2 * w] = b[0] | (b[2] << 8) | (b[4] << 16) | (static_cast<uint32_t>(b[6]) << 24);
          qw[j][2 * w + 1] = b[1] | (b[3] << 8) | (b[5] << 16) | (static_cast<uint32_t>(b[7]) << 24);
#pragma unroll
          for (int t = 0; t < 8; ++t) qsum += qb[e0 + 8 * w + t];
        }
      } else if constexpr (MODE == kInt && BITS == 1) {
#pragma unroll
        for (int w = 0; w < C::W; ++w) {
          uint32_t planes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
          for (int t = 0; t < 32; ++t) {
            const uint32_t v = static_cast<uint8_t>(qb[e0 + 32 * w + t]);
            qsum += qb[e0 + 32 * w + t];
#pragma unroll
            for (int b = 0; b < 8; ++b) planes[b] |= ((v >> b) & 1u) << t;
          }
#pragma unroll
          for (int b = 0; b < 8; ++b) qw[j][8 * w + b] = planes[b];
        }
      } else if constexpr (MODE == kHamming) {
#pragma unroll
        for (int w = 0; w < C::W; ++w) qw[j][w] = reinterpret_cast<const uint32_t*>(qb)[e0 / 32 + w];
      }
    }
    (void)qf2;
    (void)qw;
    (void)qsum;

    // candidate buffer: keys above thr are appended; checked every check_tiles
    const uint32_t high = p.capc - p.check_tiles * p.tile_rows;
    uint64_t thr = 0;
    uint32_t s = 0, ph = 0, until_check = p.check_tiles;
    for (uint32_t it = 0;; ++it, s = s + 1u == p.stages ? 0u : s + 1u, ph ^= s == 0u ? 1u : 0u) {
      const bool landed = mbar_wait_bounded(&full[s], ph, p.err);
      const uint32_t t = landed ? tile_ids[s] : kNoTile;
      if (it == 0 && p.trace && threadIdx.x == 0) p.trace[blockIdx.x * 8 + kTrFirstTile] = globaltimer();
      if (t == kNoTile) break;
      const uint8_t* cb = s_codes + static_cast<size_t>(s) * p.tile_bytes;
      const float* sc = s_scales + static_cast<size_t>(s) * p.tile_rows;
      const uint64_t base = static_cast<uint64_t>(t) * p.tile_rows;
      const uint32_t nvalid =
          p.nrows - base < p.tile_rows ? static_cast<uint32_t>(p.nrows - base) : p.tile_rows;

      for (uint32_t rb = 0; rb < p.tile_rows; rb += C::RPI) {
        uint32_t rho[U];
        Chunk<C::W> x[U][CPL];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          rho[u] = rb + static_cast<uint32_t>(warp * (C::G * U) + u * C::G + g);
          // a tile may hold fewer rows than one iteration covers (very wide rows):
          // surplus lanes read row 0 and never offer a key
          const uint32_t rr = rho[u] < p.tile_rows ? rho[u] : 0u;
#pragma unroll
          for (int j = 0; j < CPL; ++j)
            x[u][j] = lds_chunk<C::W>(cb + static_cast<size_t>(rr) * p.R + (sl + j * L) * CB);
        }
        // kTr: the U (2 or 4) rows of a lane group share one butterfly
        // (group_sum); the lane then holds one of them (`own`) and offers its
        // key alone.
        constexpr bool kTr = ((U == 2 || U == 4) && L >= U);
        float score[kTr ? 1 : U];
        uint32_t own = 0;
        if constexpr (MODE == kAsym) {
          float lsum[U];  // the lane's two chains added, per row
          // per row one f32x2 accumulator {even, odd}: the lane's elements
          // alternate between the two chains (canonical order), so one packed
          // FMA takes an element pair of one row and a register pair of q.
          uint64_t acc[U];
#pragma unroll
          for (int u = 0; u < U; ++u) acc[u] = 0ull;
#pragma unroll
          for (int j = 0; j < CPL; ++j) {
            const uint32_t e0 = static_cast<uint32_t>(sl + j * L) * C::EPC;
#pragma unroll
            for (int w = 0; w < C::W; ++w) {
              if constexpr (BITS == 8) {
#pragma unroll
                for (int bp = 0; bp < 4; bp += 2) {
                  const uint64_t q2 = C::kQReg ? qf2[C::kQReg ? j : 0][C::kQReg ? (w * 4 + bp) / 2 : 0]
                                               : *reinterpret_cast<const uint64_t*>(q + e0 + w * 4 + bp);
#pragma unroll
                  for (int u = 0; u < U; ++u) {
                    const uint32_t xb = x[u][j].w[w] ^ 0x80808080u;
                    const uint64_t val = f2_add(f2_pack(s8_biased(xb, bp), s8_biased(xb, bp + 1)),
                                                f2_pack(-kBias8, -kBias8));
                    acc[u] = f2_fma(val, q2, acc[u]);
                  }
                }
              } else if constexpr (BITS == 4) {
#pragma unroll
                for (int np = 0; np < 8; np += 2) {
                  const uint64_t q2 = C::kQReg ? qf2[C::kQReg ? j : 0][C::kQReg ? (w * 8 + np) / 2 : 0]
                                               : *reinterpret_cast<const uint64_t*>(q + e0 + w * 8 + np);
#pragma unroll
                  for (int u = 0; u < U; ++u) {
                    const uint32_t xn = x[u][j].w[w] ^ 0x88888888u;
                    const uint64_t val = f2_add(f2_pack(s4_biased(xn, np), s4_biased(xn, np + 1)),
                                                f2_pack(-kBias4, -kBias4));
                    acc[u] = f2_fma(val, q2, acc[u]);
                  }
                }
              } else {
#pragma unroll
                for (int b4 = 0; b4 < 8; ++b4) {
                  const uint4 q4 = *reinterpret_cast<const uint4*>(q + e0 + w * 32 + b4 * 4);
#pragma unroll
                  for (int hp = 0; hp < 2; ++hp) {
                    const int b = b4 * 4 + hp * 2;  // element pair (b, b+1) of word w
                    const uint32_t qlo = hp ? q4.z : q4.x, qhi = hp ? q4.w : q4.y;
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                      // fmaf(+-1, q, acc) == acc + (+-q) exactly: flip q's sign where the bit is 0
                      const uint32_t xw = x[u][j].w[w];
                      const uint32_t f0 = (~(xw << (31 - b))) & 0x80000000u;
                      const uint32_t f1 = (~(xw << (30 - b))) & 0x80000000u;
                      acc[u] = f2_add(acc[u], f2_pack(__uint_as_float(qlo ^ f0), __uint_as_float(qhi ^ f1)));
                    }
                  }
                }
              }
            }
          }
#pragma unroll
          for (int u = 0; u < U; ++u) {
            float ev, od;
            f2_unpack(acc[u], ev, od);
            lsum[u] = __fadd_rn(ev, od);
          }
          if constexpr (kTr) {
            const float a = group_sum<L, U>(lsum, sl, own);
            const uint32_t r = pick_row<U>(rho, own);
            const float sv = sc[r < p.tile_rows ? r : 0u];
            const float f = BITS == 8 ? __fmul_rn(sv, kInv127) : (BITS == 4 ? __fmul_rn(sv, kInv7) : sv);
            score[0] = __fmul_rn(a, f);
          } else {
#pragma unroll
            for (int u = 0; u < U; ++u) {
              float a = lsum[u];
#pragma unroll
              for (int off = L / 2; off >= 1; off >>= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, off));
              const float sv = sc[rho[u] < p.tile_rows ? rho[u] : 0u];
              const float f = BITS == 8 ? __fmul_rn(sv, kInv127) : (BITS == 4 ? __fmul_rn(sv, kInv7) : sv);
              score[u] = __fmul_rn(a, f);
            }
          }
        } else {
          int iacc[U];
#pragma unroll
          for (int u = 0; u < U; ++u) iacc[u] = 0;
#pragma unroll
          for (int j = 0; j < CPL; ++j) {
#pragma unroll
            for (int w = 0; w < C::W; ++w) {
#pragma unroll
              for (int u = 0; u < U; ++u) {
                const uint32_t xw = x[u][j].w[w];
                if constexpr (MODE == kHamming) {
                  iacc[u] += __popc(xw ^ qw[j][w]);
                } else if constexpr (BITS == 8) {
                  iacc[u] = dp4a_ss(xw, qw[j][w], iacc[u]);
                } else if constexpr (BITS == 4) {
                  const uint32_t xn = xw ^ 0x88888888u;
                  iacc[u] = dp4a_us(xn & 0x0F0F0F0Fu, qw[j][2 * w], iacc[u]);
                  iacc[u] = dp4a_us((xn >> 4) & 0x0F0F0F0Fu, qw[j][2 * w + 1], iacc[u]);
                } else {
#pragma unroll
                  for (int b = 0; b < 7; ++b) iacc[u] += __popc(xw & qw[j][8 * w + b]) << b;
                  iacc[u] -= __popc(xw & qw[j][8 * w + 7]) << 7;
                }
              }
            }
          }
          int vs[U];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            int v = iacc[u];
            if constexpr (MODE == kInt && BITS == 4) v -= 8 * qsum;
            if constexpr (MODE == kInt && BITS == 1) v = 2 * v - qsum;
            vs[u] = v;
          }
#pragma unroll
          for (int u = 0; u < (kTr ? 1 : U); ++u) {
            int v;
            uint32_t r;
            if constexpr (kTr) {
              v = group_sum<L, U>(vs, sl, own);
              r = pick_row<U>(rho, own);
            } else {
              v = vs[u];
#pragma unroll
              for (int off = L / 2; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
              r = rho[u];
            }
            const float scale = sc[r < p.tile_rows ? r : 0u];
            if constexpr (MODE == kHamming) {
              score[u] = __fmul_rn(__int2float_rn(static_cast<int>(p.P) - 2 * v), scale);
            } else {
              const float rowfac = BITS == 8 ? __fmul_rn(scale, kInv127)
                                             : (BITS == 4 ? __fmul_rn(scale, kInv7) : scale);
              score[u] = __fmul_rn(__fmul_rn(__int2float_rn(v), rowfac), qfac);
            }
          }
        }
        if constexpr (kTr) {
          // one lane per row offers it: lanes 0 and L/2 (U = 2); 0, L/4, L/2, 3L/4 (U = 4)
          const uint32_t r = pick_row<U>(rho, own);
          const uint64_t row = base + r;
          bool valid = (sl & (L / U - 1)) == 0 && r < nvalid;
          if (valid && p.mask) valid = (p.mask[row >> 5] >> (row & 31)) & 1u;
          const uint64_t key = make_key(score[0], static_cast<uint32_t>(row));
          append_keys(cand, &misc[kMiscCount], key, valid && key > thr, lane);
        } else {
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const uint64_t row = base + rho[u];
            bool valid = (sl == 0) && rho[u] < nvalid;
            if (valid && p.mask) valid = (p.mask[row >> 5] >> (row & 31)) & 1u;
            const uint64_t key = make_key(score[u], static_cast<uint32_t>(row));
            append_keys(cand, &misc[kMiscCount], key, valid && key > thr, lane);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (--until_check == 0) {
        until_check = p.check_tiles;
        raise_threshold(cand, hist, misc, p.F, high, thr, ctid);
      }
    }
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if (p.trace && threadIdx.x == 0) p.trace[blockIdx.x * 8 + kTrScanned] = globaltimer();

    cta_publish(p, cand, hist, misc, s_codes, p.stages * p.tile_bytes, qbar, ctid);
  }

}

}  // namespace bv
