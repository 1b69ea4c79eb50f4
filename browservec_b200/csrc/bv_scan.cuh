// bv_scan.cuh -- the fused single-query quantized flat scan for sm_100a.
//
// One launch answers one query against one corpus shard:
//   1. every CTA rotates the query itself (random-sign diagonal + FWHT, the
//      operation order of rotator.ts:83-92; warp-shuffle stages for len < 32,
//      shared-memory stages above) while its producer warp already streams
//      code tiles with 1-D bulk copies (TMA engine) into a 2..4-stage ring;
//   2. 8 consumer warps score the rows of each tile in the canonical lane
//      order (asym: fmaf chains over exact integer codes, the restatement of
//      distanceQ8.ts:56-66 / distanceQ4.ts:44-62 / distanceQ1.ts:44-66; int:
//      dp4a / bit-plane popc over an int8-coded query; hamming: xor+popc),
//      drop rows whose mask bit is clear (scoreMask.ts:66-92 and mask.ts:20-35:
//      a masked row can never win a slot) and offer (score,row) keys to a
//      per-warp top-F buffer;
//   3. the warps' lists merge into one sorted CTA list in global scratch; the
//      last CTA to finish (atomic ticket) merges all CTA lists (the device form
//      of gpuTopk.ts:160-189), re-ranks the F candidates with the exact f64 dot
//      of store.ts:114-130 over the fp32 originals and keeps the best k
//      (index.ts:583-594), under the (score desc, row asc) order.
// Every wait is bounded; a timeout raises a flag in `err` instead of hanging.
#pragma once

#include <cstdint>

#include "bv_device.cuh"

namespace bv {

enum ScoreMode : int { kAsym = 0, kInt = 1, kHamming = 2 };

constexpr int kConsumerWarps = 8;
constexpr int kScanThreads = (kConsumerWarps + 1) * 32;
constexpr uint32_t kConsumerThreads = kConsumerWarps * 32;
constexpr uint32_t kBarConsumers = 1;  // named barrier id for the consumer warps

struct ScanParams {
  const uint8_t* codes;      // rows x R bytes (capacity padded to whole tiles)
  const float* scales;       // one per row (padded like codes)
  const float* originals;    // rows x dim fp32 (normalized, store.ts:163-170)
  const float* signs;        // rounds x P, pre-scaled (rotator.ts:66-80)
  const float* query;        // dim fp32, normalized by the host (store.ts:209-217)
  const uint32_t* mask;      // optional: bit r of mask[r>>5] = row r passes
  uint64_t nrows;
  uint32_t dim, P, rounds;
  uint32_t R;                // code bytes per row
  uint32_t tile_rows;        // rows per pipeline tile
  uint32_t tile_bytes;       // tile_rows * R
  uint32_t ntiles;
  uint32_t stages;           // 2..4
  uint32_t F, Fp, cap;       // fetch, pow2 pad (>= 32), per-warp buffer slots (2*Fp)
  uint32_t k;
  int rerank;
  uint32_t row_base;         // global row of this shard's row 0
  uint64_t* partials;        // gridDim.x x Fp keys
  uint32_t* ticket;          // last-CTA ticket (self-resetting)
  uint32_t* err;             // error flags
  uint32_t* out_rows;        // k
  float* out_scores;         // k
  uint32_t* out_count;       // 1
  uint32_t* cand_rows;       // optional: F approximate candidates
  float* cand_scores;
  uint32_t* cand_count;
};

// Shared-memory carve-up (host and device agree on it).
struct ScanSmem {
  uint32_t codes_off, scales_off, bars_off, rq_off, qb_off, bufs_off, misc_off, total;
};

__host__ __device__ inline uint32_t align_up(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }

__host__ __device__ inline ScanSmem scan_smem_layout(uint32_t tile_bytes, uint32_t tile_rows,
                                                     uint32_t stages, uint32_t P, uint32_t cap) {
  ScanSmem s;
  uint32_t o = 0;
  s.codes_off = o;
  o = align_up(o + stages * tile_bytes, 128);
  s.scales_off = o;
  o = align_up(o + stages * tile_rows * 4, 128);
  s.bars_off = o;
  o = align_up(o + 2 * stages * 8, 16);
  s.rq_off = o;
  o = align_up(o + P * 4, 16);
  s.qb_off = o;
  o = align_up(o + P, 16);
  s.bufs_off = o;
  o = align_up(o + kConsumerWarps * cap * 8, 16);
  s.misc_off = o;
  o = align_up(o + 64, 16);
  s.total = o;
  return s;
}

// ------------------------------------------------------------ code -> value
// int8 byte of word xb (= x ^ 0x80808080) as an exact float: the biased byte
// u = b + 128 goes into a float's low mantissa (2^23 + u); subtract 2^23 + 128.
__device__ __forceinline__ float s8_to_f32(uint32_t xb, int byte) {
  uint32_t v = __byte_perm(xb, 0x4B00u, 0x5440u | static_cast<uint32_t>(byte));
  return __fsub_rn(__uint_as_float(v), 8388736.0f);
}
// int4 nibble of word xn (= x ^ 0x88888888) as an exact float.
__device__ __forceinline__ float s4_to_f32(uint32_t xn, int nib) {
  uint32_t v = ((xn >> (4 * nib)) & 0xFu) | 0x4B000000u;
  return __fsub_rn(__uint_as_float(v), 8388616.0f);
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
// Rotate the query into rq[0..P) (rotator.ts:83-92) with the 256 consumer
// threads: pad, then per round a sign multiply and the FWHT stages in order
// len = 1, 2, ..., P/2 (stages below 32 by warp shuffles).
__device__ __forceinline__ void rotate_query(const ScanParams& p, float* rq, int ctid) {
  const uint32_t P = p.P;
  const int lane = ctid & 31, warp = ctid >> 5;
  for (uint32_t i = ctid; i < P; i += kConsumerThreads) rq[i] = i < p.dim ? p.query[i] : 0.0f;
  named_bar_sync(kBarConsumers, kConsumerThreads);
  for (uint32_t r = 0; r < p.rounds; ++r) {
    const float* s = p.signs + static_cast<size_t>(r) * P;
    if (P >= 32) {
      // sign multiply fused into the shuffle stages: each warp owns 32-element blocks
      for (uint32_t blk = warp; blk < P / 32; blk += kConsumerWarps) {
        uint32_t i = blk * 32 + lane;
        float x = __fmul_rn(rq[i], s[i]);
#pragma unroll
        for (int len = 1; len < 32; len <<= 1) {
          float y = __shfl_xor_sync(0xffffffffu, x, len);
          x = (lane & len) ? __fsub_rn(y, x) : __fadd_rn(x, y);
        }
        rq[i] = x;
      }
      named_bar_sync(kBarConsumers, kConsumerThreads);
      for (uint32_t len = 32; len < P; len <<= 1) {
        for (uint32_t b = ctid; b < P / 2; b += kConsumerThreads) {
          uint32_t j = (b / len) * 2 * len + (b % len);
          float x = rq[j], y = rq[j + len];
          rq[j] = __fadd_rn(x, y);
          rq[j + len] = __fsub_rn(x, y);
        }
        named_bar_sync(kBarConsumers, kConsumerThreads);
      }
    } else {
      for (uint32_t i = ctid; i < P; i += kConsumerThreads) rq[i] = __fmul_rn(rq[i], s[i]);
      named_bar_sync(kBarConsumers, kConsumerThreads);
      for (uint32_t len = 1; len < P; len <<= 1) {
        for (uint32_t b = ctid; b < P / 2; b += kConsumerThreads) {
          uint32_t j = (b / len) * 2 * len + (b % len);
          float x = rq[j], y = rq[j + len];
          rq[j] = __fadd_rn(x, y);
          rq[j + len] = __fsub_rn(x, y);
        }
        named_bar_sync(kBarConsumers, kConsumerThreads);
      }
    }
  }
}

// Math.round (halves toward +inf) of an f64.
__device__ __forceinline__ double js_round(double x) {
  double r = floor(x);
  if (__dadd_rn(x, -r) >= 0.5) r = __dadd_rn(r, 1.0);
  return r;
}

// int8 code of the rotated query with the corpus codec (codec.ts:132-154):
// qb[i] in [-127,127]; returns the f32 scale (max |rq|, or 1).
__device__ __forceinline__ float quantize_query8(const float* rq, int8_t* qb, uint32_t P, int ctid,
                                                 float* red /* >= 8 floats */) {
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

// ------------------------------------------------------------------ kernel
// BITS 8/4/1; MODE asym/int/hamming; CB chunk bytes (4, 8 or 16); L lanes per
// row; CPL chunks per lane; U rows in flight per row-group.
template <int BITS, int MODE, int CB, int L, int CPL, int U>
struct ScanCfg {
  static constexpr int W = CB / 4;                                     // words per chunk
  static constexpr int EPW = BITS == 8 ? 4 : (BITS == 4 ? 8 : 32);    // elements per word
  static constexpr int EPC = W * EPW;                                  // elements per chunk
  static constexpr int G = 32 / L;                                     // rows per warp step
  static constexpr int RPI = kConsumerWarps * G * U;                   // rows per iteration
  static constexpr bool kQReg = (MODE == kAsym) && (CPL * EPC <= 64);  // fp32 query in registers
  // per-chunk integer query words: int8 W, int4 2W (even/odd), 1-bit 8W planes, hamming W
  static constexpr int QW = MODE == kInt ? (BITS == 8 ? W : (BITS == 4 ? 2 * W : 8 * W))
                                         : (MODE == kHamming ? W : 1);
};

template <int BITS, int MODE, int CB, int L, int CPL, int U>
__global__ void __launch_bounds__(kScanThreads, 1) scan_kernel(const ScanParams p) {
  using C = ScanCfg<BITS, MODE, CB, L, CPL, U>;
  extern __shared__ __align__(128) uint8_t smem[];
  const ScanSmem lay = scan_smem_layout(p.tile_bytes, p.tile_rows, p.stages, p.P, p.cap);
  uint8_t* s_codes = smem + lay.codes_off;
  float* s_scales = reinterpret_cast<float*>(smem + lay.scales_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + lay.bars_off);
  uint64_t* empty = full + p.stages;
  float* rq = reinterpret_cast<float*>(smem + lay.rq_off);
  int8_t* qb = reinterpret_cast<int8_t*>(smem + lay.qb_off);
  uint64_t* bufs = reinterpret_cast<uint64_t*>(smem + lay.bufs_off);
  float* miscf = reinterpret_cast<float*>(smem + lay.misc_off);
  uint32_t* miscu = reinterpret_cast<uint32_t*>(smem + lay.misc_off);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t t0 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x) * p.ntiles / gridDim.x);
  const uint32_t t1 =
      static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x + 1) * p.ntiles / gridDim.x);

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      const uint32_t bytes = p.tile_bytes + p.tile_rows * 4;
      for (uint32_t t = t0, it = 0; t < t1; ++t, ++it) {
        const uint32_t s = it % p.stages, ph = (it / p.stages) & 1u;
        if (it >= p.stages && !mbar_wait_bounded(&empty[s], ph ^ 1u, p.err)) break;
        mbar_arrive_expect_tx(&full[s], bytes);
        bulk_g2s(s_codes + static_cast<size_t>(s) * p.tile_bytes,
                 p.codes + static_cast<size_t>(t) * p.tile_bytes, p.tile_bytes, &full[s]);
        bulk_g2s(s_scales + static_cast<size_t>(s) * p.tile_rows,
                 p.scales + static_cast<size_t>(t) * p.tile_rows, p.tile_rows * 4, &full[s]);
      }
    }
  } else {
    // ---------------------------------------------------------- consumers
    const int ctid = threadIdx.x;
    rotate_query(p, rq, ctid);
    float qfac = 1.0f;
    if constexpr (MODE == kInt) {
      float qscale = quantize_query8(rq, qb, p.P, ctid, miscf);
      qfac = __fmul_rn(qscale, kInv127);
    } else if constexpr (MODE == kHamming) {
      uint32_t* qbits = reinterpret_cast<uint32_t*>(qb);
      for (uint32_t blk = warp; blk < p.P / 32; blk += kConsumerWarps)
        qbits[blk] = __ballot_sync(0xffffffffu, rq[blk * 32 + lane] >= 0.0f);
    }
    named_bar_sync(kBarConsumers, kConsumerThreads);

    const int g = lane / L, sl = lane % L;
    // lane-resident query slices
    float qf[C::kQReg ? CPL : 1][C::kQReg ? C::EPC : 1];
    uint32_t qw[MODE == kAsym ? 1 : CPL][C::QW];
    int qsum = 0;
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
      const uint32_t e0 = static_cast<uint32_t>(sl + j * L) * C::EPC;  // first element of chunk
      if constexpr (C::kQReg) {
#pragma unroll
        for (int e = 0; e < C::EPC; ++e) qf[j][e] = rq[e0 + e];
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
    (void)qf;
    (void)qw;
    (void)qsum;

    WarpTopF tf;
    tf.init(bufs + static_cast<size_t>(warp) * p.cap, static_cast<int>(p.cap), static_cast<int>(p.F),
            lane);

    bool ok = true;
    for (uint32_t t = t0, it = 0; t < t1; ++t, ++it) {
      const uint32_t s = it % p.stages, ph = (it / p.stages) & 1u;
      if (!mbar_wait_bounded(&full[s], ph, p.err)) {
        ok = false;
        break;
      }
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
#pragma unroll
          for (int j = 0; j < CPL; ++j)
            x[u][j] = lds_chunk<C::W>(cb + static_cast<size_t>(rho[u]) * p.R + (sl + j * L) * CB);
        }
        float score[U];
        if constexpr (MODE == kAsym) {
          float acc[U];
#pragma unroll
          for (int u = 0; u < U; ++u) acc[u] = 0.0f;
#pragma unroll
          for (int j = 0; j < CPL; ++j) {
            const uint32_t e0 = static_cast<uint32_t>(sl + j * L) * C::EPC;
#pragma unroll
            for (int w = 0; w < C::W; ++w) {
              if constexpr (BITS == 8) {
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                  const float q = C::kQReg ? qf[C::kQReg ? j : 0][C::kQReg ? w * 4 + b : 0]
                                           : rq[e0 + w * 4 + b];
#pragma unroll
                  for (int u = 0; u < U; ++u)
                    acc[u] = __fmaf_rn(s8_to_f32(x[u][j].w[w] ^ 0x80808080u, b), q, acc[u]);
                }
              } else if constexpr (BITS == 4) {
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                  const float q = C::kQReg ? qf[C::kQReg ? j : 0][C::kQReg ? w * 8 + n : 0]
                                           : rq[e0 + w * 8 + n];
#pragma unroll
                  for (int u = 0; u < U; ++u)
                    acc[u] = __fmaf_rn(s4_to_f32(x[u][j].w[w] ^ 0x88888888u, n), q, acc[u]);
                }
              } else {
#pragma unroll
                for (int b4 = 0; b4 < 8; ++b4) {
                  const float4 q4 = *reinterpret_cast<const float4*>(rq + e0 + w * 32 + b4 * 4);
                  const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
                  for (int bb = 0; bb < 4; ++bb) {
                    const int b = b4 * 4 + bb;
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                      const uint32_t flip = (~(x[u][j].w[w] << (31 - b))) & 0x80000000u;
                      acc[u] = __fadd_rn(acc[u], __uint_as_float(__float_as_uint(qv[bb]) ^ flip));
                    }
                  }
                }
              }
            }
          }
#pragma unroll
          for (int u = 0; u < U; ++u) {
#pragma unroll
            for (int off = L / 2; off >= 1; off >>= 1)
              acc[u] = __fadd_rn(acc[u], __shfl_xor_sync(0xffffffffu, acc[u], off));
            const float scale = sc[rho[u]];
            const float rowfac =
                BITS == 8 ? __fmul_rn(scale, kInv127) : (BITS == 4 ? __fmul_rn(scale, kInv7) : scale);
            score[u] = __fmul_rn(acc[u], rowfac);
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
#pragma unroll
          for (int u = 0; u < U; ++u) {
            int v = iacc[u];
            if constexpr (MODE == kInt && BITS == 4) v -= 8 * qsum;
            if constexpr (MODE == kInt && BITS == 1) v = 2 * v - qsum;
#pragma unroll
            for (int off = L / 2; off >= 1; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            const float scale = sc[rho[u]];
            if constexpr (MODE == kHamming) {
              const int idot = static_cast<int>(p.P) - 2 * v;
              score[u] = __fmul_rn(__int2float_rn(idot), scale);
            } else {
              const float rowfac = BITS == 8 ? __fmul_rn(scale, kInv127)
                                             : (BITS == 4 ? __fmul_rn(scale, kInv7) : scale);
              score[u] = __fmul_rn(__fmul_rn(__int2float_rn(v), rowfac), qfac);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const uint64_t row = base + rho[u];
          bool valid = (sl == 0) && rho[u] < nvalid;
          if (valid && p.mask) valid = (p.mask[row >> 5] >> (row & 31)) & 1u;
          tf.offer(make_key(score[u], static_cast<uint32_t>(row)), valid, lane);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    (void)ok;
    tf.finish(lane);

    // ------------------------------------------------ CTA merge of warp lists
    named_bar_sync(kBarConsumers, kConsumerThreads);
    for (int step = 1; step < kConsumerWarps; step <<= 1) {
      if ((warp % (2 * step)) == 0)
        warp_merge_top(bufs + static_cast<size_t>(warp) * p.cap,
                       bufs + static_cast<size_t>(warp + step) * p.cap, static_cast<int>(p.Fp), lane);
      named_bar_sync(kBarConsumers, kConsumerThreads);
    }
    if (warp == 0) {
      for (uint32_t i = lane; i < p.Fp; i += 32)
        p.partials[static_cast<size_t>(blockIdx.x) * p.Fp + i] = i < p.F ? bufs[i] : 0ull;
      __threadfence();
    }
  }

  // ------------------------------------------------------ last-CTA ticket
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t ticket = atomicAdd(p.ticket, 1u);
    miscu[8] = (ticket == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (miscu[8] == 0u) return;
  __threadfence();
  if (warp == kConsumerWarps) return;  // the producer warp sits out the merge

  // ------------------------------------------------ global merge (last CTA)
  {
    WarpTopF tf;
    tf.init(bufs + static_cast<size_t>(warp) * p.cap, static_cast<int>(p.cap), static_cast<int>(p.F),
            lane);
    const uint32_t nlists = gridDim.x;
    for (uint32_t lb = 0; lb < nlists; lb += 32 * kConsumerWarps) {
      const uint32_t li = lb + static_cast<uint32_t>(lane) * kConsumerWarps + warp;
      bool active = li < nlists;
      for (uint32_t r = 0; r < p.F; ++r) {
        if (!__any_sync(0xffffffffu, active)) break;
        uint64_t key = 0;
        if (active) {
          key = __ldcg(p.partials + static_cast<size_t>(li) * p.Fp + r);
          if (key == 0 || key <= tf.thr) active = false;
        }
        tf.offer(key, active, lane);
      }
    }
    tf.finish(lane);
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);
  for (int step = 1; step < kConsumerWarps; step <<= 1) {
    if ((warp % (2 * step)) == 0)
      warp_merge_top(bufs + static_cast<size_t>(warp) * p.cap,
                     bufs + static_cast<size_t>(warp + step) * p.cap, static_cast<int>(p.Fp), lane);
    named_bar_sync(kBarConsumers, kConsumerThreads);
  }
  uint64_t* top = bufs;  // best Fp keys of the shard, sorted descending
  if (warp == 0) {
    uint32_t nc = 0;
    for (uint32_t i = lane; i < p.F; i += 32) nc += top[i] != 0ull ? 1u : 0u;
#pragma unroll
    for (int off = 16; off; off >>= 1) nc += __shfl_xor_sync(0xffffffffu, nc, off);
    if (lane == 0) miscu[9] = nc;
    if (p.cand_rows) {
      for (uint32_t i = lane; i < nc; i += 32) {
        p.cand_rows[i] = key_row(top[i]) + p.row_base;
        p.cand_scores[i] = key_score(top[i]);
      }
      if (lane == 0) *p.cand_count = nc;
    }
  }
  named_bar_sync(kBarConsumers, kConsumerThreads);
  const uint32_t nc = miscu[9];
  const int ctid = threadIdx.x;

  if (p.rerank) {
    // exact f64 dot (store.ts:114-130): 4 lanes per candidate hold a0..a3
    uint64_t* ex = bufs + p.cap;  // second warp buffer: Fp exact keys
    const uint32_t vec = p.dim & ~3u;
    const uint32_t groups = kConsumerThreads / 4;
    for (uint32_t c0 = 0; c0 < p.Fp; c0 += groups) {
      const uint32_t c = c0 + static_cast<uint32_t>(ctid) / 4u;
      const uint32_t j = static_cast<uint32_t>(ctid) & 3u;
      const bool act = c < nc;
      double a = 0.0;
      uint32_t row = 0;
      if (act) {
        row = key_row(top[c]);
        const float* xr = p.originals + static_cast<size_t>(row) * p.dim;
#pragma unroll 8
        for (uint32_t i = j; i < vec; i += 4)
          a = __fma_rn(static_cast<double>(__ldg(xr + i)), static_cast<double>(__ldg(p.query + i)), a);
      }
      const int gl = lane & ~3;
      const double a0 = __shfl_sync(0xffffffffu, a, gl + 0);
      const double a1 = __shfl_sync(0xffffffffu, a, gl + 1);
      const double a2 = __shfl_sync(0xffffffffu, a, gl + 2);
      const double a3 = __shfl_sync(0xffffffffu, a, gl + 3);
      if (c < p.Fp && j == 0) {
        uint64_t kx = 0;
        if (act) {
          double sacc = __dadd_rn(__dadd_rn(__dadd_rn(a0, a1), a2), a3);
          const float* xr = p.originals + static_cast<size_t>(row) * p.dim;
          for (uint32_t i = vec; i < p.dim; ++i)
            sacc = __fma_rn(static_cast<double>(xr[i]), static_cast<double>(p.query[i]), sacc);
          kx = make_key(__double2float_rn(sacc), row);
        }
        ex[c] = kx;
      }
    }
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if (warp == 0) {
      warp_sort_desc(ex, static_cast<int>(p.Fp), lane);
      const uint32_t n = nc < p.k ? nc : p.k;
      for (uint32_t i = lane; i < n; i += 32) {
        p.out_rows[i] = key_row(ex[i]) + p.row_base;
        p.out_scores[i] = key_score(ex[i]);
      }
      if (lane == 0) *p.out_count = n;
    }
  } else if (warp == 0) {
    const uint32_t n = nc < p.k ? nc : p.k;
    for (uint32_t i = lane; i < n; i += 32) {
      p.out_rows[i] = key_row(top[i]) + p.row_base;
      p.out_scores[i] = key_score(top[i]);
    }
    if (lane == 0) *p.out_count = n;
  }
  if (ctid == 0) *p.ticket = 0u;  // ready for the next launch (stream-ordered)
}

}  // namespace bv
