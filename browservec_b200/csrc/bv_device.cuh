// bv_device.cuh -- device-side building blocks shared by the sm_100a kernels:
// candidate keys, bounded mbarrier waits, 1-D bulk (TMA engine) copies, and
// warp-level bitonic sort/merge used by the fused top-F selection.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace bv {

// f32(1/127) and f32(1/7): the row factors of the int8 and int4 scorers
// (distanceQ4.ts:145 folds 1/7 the same way).
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
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint32_t* err_flag) {
  constexpr uint32_t kBudget = 1u << 22;
  for (uint32_t i = 0; i < kBudget; ++i)
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

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
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

}  // namespace bv
