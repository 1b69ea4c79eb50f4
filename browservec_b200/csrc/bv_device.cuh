// bv_device.cuh -- device-side building blocks shared by the sm_100a kernels:
// candidate keys, bounded mbarrier waits, 1-D bulk (TMA engine) copies, and
// warp-level bitonic sort/merge used by the fused top-F selection.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace bv {

// f32(1/127) and f32(1/7): the row factors of the int8 and int4 scorers
// (distanceQ4.ts:61 folds 1/7 the same way).
__device__ __constant__ static const float kInv127 = 0x1.020408p-7f;
__device__ __constant__ static const float kInv7 = 0x1.24924ap-3f;

// Error flags a kernel may raise instead of hanging (read back by the host).
enum : uint32_t {
  kErrNone = 0,
  kErrWaitTimeout = 1u,      // an mbarrier wait ran past its iteration budget
  kErrBadLaunch = 2u,        // launch geometry the kernel cannot serve
};

// ------------------------------------------------------------ order keys
// A candidate is one 64-bit key: orderable(score) << 32 | ~row.  A larger key
// is a better candidate: higher score, then lower row -- the tie rule.  0 is
// below every real key and marks an empty slot.
__device__ __forceinline__ uint64_t make_key(float score, uint32_t row) {
  uint32_t u = __float_as_uint(score == 0.0f ? 0.0f : score);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<uint64_t>(u) << 32) | static_cast<uint64_t>(~row);
}
__device__ __forceinline__ float key_score(uint64_t key) {
  uint32_t u = static_cast<uint32_t>(key >> 32);
  u = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
  return __uint_as_float(u);
}
// Row of a key's position: a candidate-list search scores gathered rows, and
// its keys carry the position in the list (rowmap maps it back); else the
// position is the row.
__device__ __forceinline__ uint32_t map_row(const uint32_t* rowmap, uint32_t pos) {
  return rowmap ? __ldg(rowmap + pos) : pos;
}
__device__ __forceinline__ uint32_t key_row(uint64_t key) {
  return ~static_cast<uint32_t>(key);
}

// ------------------------------------------------------------- mbarrier
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(
                   smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_addr(bar)),
      "r"(bytes)
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after `budget` polls (each poll is a hardware
// try_wait that may itself suspend briefly), raising kErrWaitTimeout.
constexpr uint32_t kWaitBudget = 1u << 22;
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t* err_flag,
                                                  uint32_t budget = kWaitBudget) {
  for (uint32_t i = 0; i < budget; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (err_flag) atomicOr(err_flag, kErrWaitTimeout);
  return false;
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes % 16 == 0,
// both addresses 16-byte aligned).  No cluster multicast.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Bulk prefetch of [src, src + bytes) into L2 (16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src_gmem, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src_gmem), "r"(bytes) : "memory");
}

// Same with an L2 cache policy (createpolicy), e.g. evict-first for data read
// once, so a streamed corpus does not flush the L2 (kernel code, scratch).
__device__ __forceinline__ void bulk_g2s_hint(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, "
      "[%3], %4;" ::"r"(smem_addr(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start, and
// wait until the previous one has completed with its memory visible.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Packed fp32 pairs (sm_100 f32x2 arithmetic): two independent lanes per op.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// ------------------------------------------- block-wide radix select
constexpr int kSelBins = 2048;  // 11-bit digits
constexpr int kSelScratch = 64;  // words of `sh` the select needs

// Among `total` unique nonzero keys held in registers (v[0..nv) per thread,
// zero slots ignored) by the NT threads of named barrier `bar`, find thr such
// that exactly min(F, total) keys are >= thr.  The bits all keys share are
// skipped (block max/min), then 11-bit digits MSB-first with plain
// shared-memory histograms; usually one or two passes.  hist: kSelBins words;
// sh: kSelScratch words.  Block-collective; all threads return the same thr.
template <int MAXK, int NT>
__device__ __forceinline__ uint64_t block_select_threshold(const uint64_t (&v)[MAXK], int nv,
                                                           uint32_t F, uint32_t total,
                                                           uint32_t* hist, uint32_t* sh, int tid,
                                                           uint32_t bar) {
  static_assert(NT % 32 == 0 && NT / 32 <= 16 && kSelBins == 4 * NT, "4 bins per thread");
  if (total <= F) return 1ull;
  const int lane = tid & 31, warp = tid >> 5;
  // common leading bits: max and min of the nonzero keys
  uint64_t mx = 0ull, mn = ~0ull;
#pragma unroll
  for (int i = 0; i < MAXK; ++i)
    if (i < nv && v[i] != 0ull) {
      mx = v[i] > mx ? v[i] : mx;
      mn = v[i] < mn ? v[i] : mn;
    }
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    const uint64_t a = __shfl_xor_sync(0xffffffffu, mx, off);
    const uint64_t b = __shfl_xor_sync(0xffffffffu, mn, off);
    mx = a > mx ? a : mx;
    mn = b < mn ? b : mn;
  }
  uint64_t* sh64 = reinterpret_cast<uint64_t*>(sh);
  if (lane == 0) {
    sh64[2 * warp] = mx;
    sh64[2 * warp + 1] = mn;
  }
  named_bar_sync(bar, NT);
  mx = 0ull;
  mn = ~0ull;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) {
    mx = sh64[2 * w] > mx ? sh64[2 * w] : mx;
    mn = sh64[2 * w + 1] < mn ? sh64[2 * w + 1] : mn;
  }
  named_bar_sync(bar, NT);  // sh is reused below
  int top = 63 - __clzll(static_cast<long long>(mx ^ mn));  // highest differing bit (mx != mn)
  uint64_t pmask = top >= 63 ? 0ull : ~((2ull << top) - 1ull);
  uint64_t prefix = mx & pmask;
  uint32_t need = F;
  for (;;) {
    const int width = top + 1 < 11 ? top + 1 : 11;
    const int shift = top + 1 - width;
    const uint32_t nb = 1u << width, dmask = nb - 1u;
    for (int i = tid; i < kSelBins; i += NT) hist[i] = 0u;
    named_bar_sync(bar, NT);
    // plain shared atomics: warp aggregation with match_any costs ~1000 cycles
    // per call on sm_100a, far more than the contention it saves
#pragma unroll
    for (int i = 0; i < MAXK; ++i) {
      const bool act = i < nv && v[i] != 0ull && (v[i] & pmask) == prefix;
      if (act) atomicAdd(&hist[static_cast<uint32_t>(v[i] >> shift) & dmask], 1u);
    }
    named_bar_sync(bar, NT);
    // thread t owns bins nb-1-4t .. nb-4-4t (highest first)
    uint32_t hb[4], s = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int b = static_cast<int>(nb) - 1 - 4 * tid - j;
      hb[j] = b >= 0 ? hist[b] : 0u;
      s += hb[j];
    }
    uint32_t x = s;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += y;
    }
    if (lane == 31) sh[warp] = x;
    named_bar_sync(bar, NT);
    uint32_t run = x - s;
    for (int w = 0; w < warp; ++w) run += sh[w];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (run < need && run + hb[j] >= need) {
        sh[32] = static_cast<uint32_t>(static_cast<int>(nb) - 1 - 4 * tid - j);
        sh[33] = run;
        sh[34] = hb[j];
      }
      run += hb[j];
    }
    named_bar_sync(bar, NT);
    const uint32_t d = sh[32], above = sh[33], hd = sh[34];
    prefix |= static_cast<uint64_t>(d) << shift;
    pmask |= static_cast<uint64_t>(dmask) << shift;
    need -= above;
    named_bar_sync(bar, NT);  // sh and hist are rewritten by the next pass
    if (hd == need || shift == 0) break;
    top = shift - 1;
  }
  return prefix;
}

// ------------------------------------------ warp register sort / merge
// A warp list of n = 32*E keys lives in registers, striped: element i is
// register i/32 of lane i%32.  Bitonic networks run on shuffles (cross-lane
// strides) and register swaps (strides >= 32): no shared memory, no barrier.
__device__ __forceinline__ uint64_t shfl_xor64(uint64_t v, int m) {
  return __shfl_xor_sync(0xffffffffu, v, m);
}

// One compare-exchange stage of stride j inside bitonic blocks of `size`
// (final order descending: the lower index keeps the max in a descending block).
template <int E>
__device__ __forceinline__ void wreg_stage(uint64_t (&v)[E], int size, int j, int lane) {
  if (j >= 32) {
    const int rj = j >> 5;
#pragma unroll
    for (int r = 0; r < E; ++r) {
      const int r2 = r ^ rj;
      if (r2 > r) {
        const int i = lane + 32 * r;
        const bool desc = (i & size) == 0;
        const uint64_t x = v[r], y = v[r2];
        const uint64_t hi = x > y ? x : y, lo = x > y ? y : x;
        v[r] = desc ? hi : lo;
        v[r2] = desc ? lo : hi;
      }
    }
  } else {
#pragma unroll
    for (int r = 0; r < E; ++r) {
      const int i = lane + 32 * r;
      const uint64_t x = v[r], y = shfl_xor64(x, j);
      const bool lower = (lane & j) == 0;
      const bool desc = (i & size) == 0;
      const uint64_t hi = x > y ? x : y, lo = x > y ? y : x;
      v[r] = (lower == desc) ? hi : lo;
    }
  }
}

// Sort the warp list descending (fully unrolled: the stage indices must be
// compile-time so the register array never spills to local memory).
template <int E>
__device__ __forceinline__ void wreg_sort_desc(uint64_t (&v)[E], int lane) {
#pragma unroll
  for (int size = 2; size <= 32 * E; size <<= 1)
#pragma unroll
    for (int j = size >> 1; j > 0; j >>= 1) wreg_stage<E>(v, size, j, lane);
}

// a, b: descending warp lists.  a becomes the best 32*E keys of a U b, descending.
template <int E>
__device__ __forceinline__ void wreg_merge_top(uint64_t (&a)[E], const uint64_t (&b)[E], int lane) {
  // c[i] = max(a[i], b[n-1-i]) is bitonic and holds the top n
#pragma unroll
  for (int r = 0; r < E; ++r) {
    const uint64_t y = __shfl_sync(0xffffffffu, b[E - 1 - r], 31 - lane);
    a[r] = a[r] > y ? a[r] : y;
  }
  constexpr int n = 32 * E;
#pragma unroll
  for (int j = n >> 1; j > 0; j >>= 1) wreg_stage<E>(a, 2 * n, j, lane);  // size 2n: all descending
}

// --------------------------------------------------- warp sort / merge
// Bitonic sort, descending, of n (power of two, >= 2) keys in shared memory by
// one warp.
__device__ __forceinline__ void warp_sort_desc(uint64_t* a, int n, int lane) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = lane; i < n; i += 32) {
        int j = i ^ stride;
        if (j > i) {
          uint64_t x = a[i], y = a[j];
          bool desc = (i & size) == 0;
          if (desc ? (x < y) : (x > y)) {
            a[i] = y;
            a[j] = x;
          }
        }
      }
      __syncwarp();
    }
  }
}

// Sort a bitonic sequence of n keys into descending order (one warp).
__device__ __forceinline__ void warp_bitonic_merge_desc(uint64_t* a, int n, int lane) {
  for (int stride = n >> 1; stride > 0; stride >>= 1) {
    for (int i = lane; i < n; i += 32) {
      int j = i ^ stride;
      if (j > i) {
        uint64_t x = a[i], y = a[j];
        if (x < y) {
          a[i] = y;
          a[j] = x;
        }
      }
    }
    __syncwarp();
  }
}

// a, b: n keys each, sorted descending.  Leaves the best n of the union in a,
// sorted descending.  (max(a[i], b[n-1-i]) is bitonic and holds the top n.)
__device__ __forceinline__ void warp_merge_top(uint64_t* a, const uint64_t* b, int n, int lane) {
  for (int i = lane; i < n; i += 32) {
    uint64_t x = a[i], y = b[n - 1 - i];
    a[i] = x > y ? x : y;
  }
  __syncwarp();
  warp_bitonic_merge_desc(a, n, lane);
}

// Per-warp candidate buffer: keeps the best F keys seen by this warp.  `cap`
// slots (power of two >= 2*Fp, Fp = pow2 >= F, >= 32) live in shared memory;
// `thr` is the F-th best key once F keys have been kept (0 before), so only
// keys above it can matter.
struct WarpTopF {
  uint64_t* buf;
  int cap;
  int F;
  int cnt;
  uint64_t thr;

  __device__ __forceinline__ void init(uint64_t* b, int c, int f, int lane) {
    buf = b;
    cap = c;
    F = f;
    cnt = 0;
    thr = 0;
    for (int i = lane; i < cap; i += 32) buf[i] = 0;
    __syncwarp();
  }

  // Sort, keep the best F, refresh the threshold.  Warp-collective.
  __device__ __forceinline__ void compact(int lane) {
    __syncwarp();
    warp_sort_desc(buf, cap, lane);
    if (cnt > F) {
      for (int i = F + lane; i < cap; i += 32) buf[i] = 0;
      cnt = F;
    }
    if (cnt == F) thr = buf[F - 1];
    __syncwarp();
  }

  // Offer one key per lane (valid lanes only).  Warp-collective.
  __device__ __forceinline__ void offer(uint64_t key, bool valid, int lane) {
    bool want = valid && key > thr;
    unsigned m = __ballot_sync(0xffffffffu, want);
    if (m == 0) return;
    int n = __popc(m);
    if (cnt + n > cap) {
      compact(lane);
      want = want && key > thr;
      m = __ballot_sync(0xffffffffu, want);
      n = __popc(m);
    }
    if (want) buf[cnt + __popc(m & ((1u << lane) - 1u))] = key;
    cnt += n;
  }

  // Final: buffer sorted descending, best min(cnt, F) first, zeros after.
  __device__ __forceinline__ void finish(int lane) { compact(lane); }
};

// ------------------------------------------- exact f64 row dot, one warp
// Store.dotRow (src/store/store.ts:114-130): four f64 accumulators, lane j
// adding x[i] * q[i] for i = j, j+4, ... below vec = dim & ~3 in order, the
// sum ((a0 + a1) + a2) + a3, then the dim % 4 tail in order, and the f32 of
// that (Math.fround, round to nearest even).  Every product of two f32 is
// exact in f64, so the only roundings are the additions.
//
// Fast path: the warp adds the same exact products in another order (lane l
// takes i = l + 32t into four interleaved partial sums, then a butterfly of
// commutative adds, which leaves every lane with the same value) together
// with A = sum |x[i] q[i]|.  With K the most additions any product goes
// through in either order (K <= dim / 4 + 12) and u = 2^-53, each order is
// within gamma_K * A of the exact sum (the bound for summation in any order:
// N. J. Higham, Accuracy and Stability of Numerical Algorithms, 2nd ed.,
// sec. 4.2), so the two are within 2 gamma_K A <= B = 4 (K + 1) u A' of one
// another (A' the computed A).  Rounding to f32 is monotone: when both ends
// of [s' - B, s' + B] (outward-rounded) round to the same f32 bits, that is
// the reference's result.  Otherwise (an f32 rounding boundary inside the
// interval -- about one row in 10^5 at unit norms -- or a NaN/Inf) the warp
// computes the reference's own sequence.  Either way the result is
// bit-identical to the sequential chain, and the common case costs a
// dim / 128-step chain per lane instead of dim / 4.
template <bool kGlobal>
__device__ __forceinline__ float ld_row_f32(const float* p) {
  if constexpr (kGlobal) return __ldg(p);
  else return *p;
}

template <bool kGlobal, typename QT = float>
__device__ __noinline__ float dot_row_exact_warp(const float* x, const QT* q, uint32_t dim, int lane) {
  double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0, a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
  uint32_t i = static_cast<uint32_t>(lane);
  for (; i + 96u < dim; i += 128u) {
    const double p0 = __dmul_rn(static_cast<double>(ld_row_f32<kGlobal>(x + i)), static_cast<double>(q[i]));
    const double p1 =
        __dmul_rn(static_cast<double>(ld_row_f32<kGlobal>(x + i + 32u)), static_cast<double>(q[i + 32u]));
    const double p2 =
        __dmul_rn(static_cast<double>(ld_row_f32<kGlobal>(x + i + 64u)), static_cast<double>(q[i + 64u]));
    const double p3 =
        __dmul_rn(static_cast<double>(ld_row_f32<kGlobal>(x + i + 96u)), static_cast<double>(q[i + 96u]));
    s0 = __dadd_rn(s0, p0);
    s1 = __dadd_rn(s1, p1);
    s2 = __dadd_rn(s2, p2);
    s3 = __dadd_rn(s3, p3);
    a0 = __dadd_rn(a0, fabs(p0));
    a1 = __dadd_rn(a1, fabs(p1));
    a2 = __dadd_rn(a2, fabs(p2));
    a3 = __dadd_rn(a3, fabs(p3));
  }
  for (; i < dim; i += 32u) {
    const double p0 = __dmul_rn(static_cast<double>(ld_row_f32<kGlobal>(x + i)), static_cast<double>(q[i]));
    s0 = __dadd_rn(s0, p0);
    a0 = __dadd_rn(a0, fabs(p0));
  }
  double s = __dadd_rn(__dadd_rn(s0, s1), __dadd_rn(s2, s3));
  double a = __dadd_rn(__dadd_rn(a0, a1), __dadd_rn(a2, a3));
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
    a = __dadd_rn(a, __shfl_xor_sync(0xffffffffu, a, off));
  }
  const double K1 = static_cast<double>(dim / 4u + 13u);  // K + 1
  const double B = __dmul_ru(__dmul_ru(a, K1), 0x1p-51);  // 4 (K + 1) u A'
  const float lo = __double2float_rn(__dsub_rd(s, B));
  const float hi = __double2float_rn(__dadd_ru(s, B));
  if (lo == lo && __float_as_uint(lo) == __float_as_uint(hi)) return lo;  // warp-uniform
  // the reference's sequence: lanes 0..3 are its accumulators
  const uint32_t vec = dim & ~3u;
  double c = 0.0;
  if (lane < 4)
    for (uint32_t k = static_cast<uint32_t>(lane); k < vec; k += 4u)
      c = __fma_rn(static_cast<double>(ld_row_f32<kGlobal>(x + k)), static_cast<double>(q[k]), c);
  const double c0 = __shfl_sync(0xffffffffu, c, 0), c1 = __shfl_sync(0xffffffffu, c, 1);
  const double c2 = __shfl_sync(0xffffffffu, c, 2), c3 = __shfl_sync(0xffffffffu, c, 3);
  double r = __dadd_rn(__dadd_rn(__dadd_rn(c0, c1), c2), c3);
  for (uint32_t k = vec; k < dim; ++k)
    r = __fma_rn(static_cast<double>(ld_row_f32<kGlobal>(x + k)), static_cast<double>(q[k]), r);
  return __double2float_rn(r);
}


// Two rows at once (their latency chains interleave): the same check and
// fallback per row, with two partial sums per lane and row (lane l takes
// i = l + 32t; at most dim / 64 + 8 additions per product, within the bound
// dot_row_exact_warp uses).
template <bool kGlobal, typename QT = float>
__device__ __forceinline__ float dot_row_check(double s, double a, const float* x, const QT* q, uint32_t dim,
                                               int lane) {
  const double K1 = static_cast<double>(dim / 4u + 13u);
  const double B = __dmul_ru(__dmul_ru(a, K1), 0x1p-51);
  const float lo = __double2float_rn(__dsub_rd(s, B));
  const float hi = __double2float_rn(__dadd_ru(s, B));
  if (lo == lo && __float_as_uint(lo) == __float_as_uint(hi)) return lo;  // warp-uniform
  const uint32_t vec = dim & ~3u;
  double c = 0.0;
  if (lane < 4)
    for (uint32_t k = static_cast<uint32_t>(lane); k < vec; k += 4u)
      c = __fma_rn(static_cast<double>(ld_row_f32<kGlobal>(x + k)), static_cast<double>(q[k]), c);
  const double c0 = __shfl_sync(0xffffffffu, c, 0), c1 = __shfl_sync(0xffffffffu, c, 1);
  const double c2 = __shfl_sync(0xffffffffu, c, 2), c3 = __shfl_sync(0xffffffffu, c, 3);
  double r = __dadd_rn(__dadd_rn(__dadd_rn(c0, c1), c2), c3);
  for (uint32_t k = vec; k < dim; ++k)
    r = __fma_rn(static_cast<double>(ld_row_f32<kGlobal>(x + k)), static_cast<double>(q[k]), r);
  return __double2float_rn(r);
}

// QT: the query as float, or already widened to double (one conversion fewer
// per product; the same values, since every float is a double exactly).
template <bool kGlobal, typename QT = float>
__device__ __noinline__ void dot_rows2_exact_warp(const float* xa, const float* xb, const QT* q, uint32_t dim,
                                                     int lane, float& ra, float& rb) {
  double sa0 = 0.0, sa1 = 0.0, aa0 = 0.0, aa1 = 0.0, sb0 = 0.0, sb1 = 0.0, ab0 = 0.0, ab1 = 0.0;
  uint32_t i = static_cast<uint32_t>(lane);
  for (; i + 32u < dim; i += 64u) {
    const double q0 = static_cast<double>(q[i]), q1 = static_cast<double>(q[i + 32u]);
    const double pa0 = __dmul_rn(static_cast<double>(ld_row_f32<kGlobal>(xa + i)), q0);
    const double pa1 = __dmul_rn(static_cast<double>(ld_row_f32<kGlobal>(xa + i + 32u)), q1);
    const double pb0 = __dmul_rn(static_cast<double>(ld_row_f32<kGlobal>(xb + i)), q0);
    const double pb1 = __dmul_rn(static_cast<double>(ld_row_f32<kGlobal>(xb + i + 32u)), q1);
    sa0 = __dadd_rn(sa0, pa0);
    sa1 = __dadd_rn(sa1, pa1);
    sb0 = __dadd_rn(sb0, pb0);
    sb1 = __dadd_rn(sb1, pb1);
    aa0 = __dadd_rn(aa0, fabs(pa0));
    aa1 = __dadd_rn(aa1, fabs(pa1));
    ab0 = __dadd_rn(ab0, fabs(pb0));
    ab1 = __dadd_rn(ab1, fabs(pb1));
  }
  if (i < dim) {
    const double q0 = static_cast<double>(q[i]);
    const double pa0 = __dmul_rn(static_cast<double>(ld_row_f32<kGlobal>(xa + i)), q0);
    const double pb0 = __dmul_rn(static_cast<double>(ld_row_f32<kGlobal>(xb + i)), q0);
    sa0 = __dadd_rn(sa0, pa0);
    sb0 = __dadd_rn(sb0, pb0);
    aa0 = __dadd_rn(aa0, fabs(pa0));
    ab0 = __dadd_rn(ab0, fabs(pb0));
  }
  double sa = __dadd_rn(sa0, sa1), aa = __dadd_rn(aa0, aa1);
  double sb = __dadd_rn(sb0, sb1), ab = __dadd_rn(ab0, ab1);
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    sa = __dadd_rn(sa, __shfl_xor_sync(0xffffffffu, sa, off));
    sb = __dadd_rn(sb, __shfl_xor_sync(0xffffffffu, sb, off));
    aa = __dadd_rn(aa, __shfl_xor_sync(0xffffffffu, aa, off));
    ab = __dadd_rn(ab, __shfl_xor_sync(0xffffffffu, ab, off));
  }
  ra = dot_row_check<kGlobal, QT>(sa, aa, xa, q, dim, lane);
  rb = dot_row_check<kGlobal, QT>(sb, ab, xb, q, dim, lane);
}

}  // namespace bv
