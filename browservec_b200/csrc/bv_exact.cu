// bv_exact.cu -- exact scan over an explicit row list (BrowserVec.queryRowsExact,
// src/index.ts:445-464): f64-accumulated dot per row in the lane order of
// Store.dotRow (src/store/store.ts:114-130), then the best k by
// (score desc, row asc).  One CTA; used for filters matching <= 4096 rows.
#include <cstdint>

#include "bv_device.cuh"
#include "bv_internal.h"

namespace bv {

constexpr int kExactThreads = 256;
constexpr uint32_t kExactMaxRows = 4096;

__global__ void __launch_bounds__(kExactThreads) exact_rows_kernel(
    const float* __restrict__ originals, uint32_t dim, const float* __restrict__ query,
    const uint32_t* __restrict__ rows, uint32_t nrows, uint32_t npow2, uint32_t k, uint32_t row_base,
    uint32_t* out_rows, float* out_scores, uint32_t* out_count) {
  extern __shared__ uint64_t keys[];  // npow2
  const int tid = threadIdx.x, lane = tid & 31;
  const uint32_t vec = dim & ~3u;
  for (uint32_t c0 = 0; c0 < npow2; c0 += kExactThreads / 4) {
    const uint32_t c = c0 + static_cast<uint32_t>(tid) / 4u;
    const uint32_t j = static_cast<uint32_t>(tid) & 3u;
    const bool act = c < nrows;
    double a = 0.0;
    uint32_t row = 0;
    if (act) {
      row = rows[c];
      const float* xr = originals + static_cast<size_t>(row) * dim;
      for (uint32_t i = j; i < vec; i += 4)
        a = __fma_rn(static_cast<double>(xr[i]), static_cast<double>(query[i]), a);
    }
    const int gl = lane & ~3;
    const double a0 = __shfl_sync(0xffffffffu, a, gl + 0);
    const double a1 = __shfl_sync(0xffffffffu, a, gl + 1);
    const double a2 = __shfl_sync(0xffffffffu, a, gl + 2);
    const double a3 = __shfl_sync(0xffffffffu, a, gl + 3);
    if (c < npow2 && j == 0) {
      uint64_t kx = 0;
      if (act) {
        double s = __dadd_rn(__dadd_rn(__dadd_rn(a0, a1), a2), a3);
        const float* xr = originals + static_cast<size_t>(row) * dim;
        for (uint32_t i = vec; i < dim; ++i)
          s = __fma_rn(static_cast<double>(xr[i]), static_cast<double>(query[i]), s);
        kx = make_key(__double2float_rn(s), row);
      }
      keys[c] = kx;
    }
  }
  __syncthreads();
  // block bitonic sort, descending
  for (uint32_t size = 2; size <= npow2; size <<= 1) {
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (uint32_t i = tid; i < npow2; i += kExactThreads) {
        const uint32_t jx = i ^ stride;
        if (jx > i) {
          const uint64_t x = keys[i], y = keys[jx];
          const bool desc = (i & size) == 0;
          if (desc ? (x < y) : (x > y)) {
            keys[i] = y;
            keys[jx] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  const uint32_t n = nrows < k ? nrows : k;
  for (uint32_t i = tid; i < n; i += kExactThreads) {
    out_rows[i] = key_row(keys[i]) + row_base;
    out_scores[i] = key_score(keys[i]);
  }
  if (tid == 0) *out_count = n;
}

cudaError_t launch_exact_rows(const float* originals, uint32_t dim, const float* query,
                              const uint32_t* rows, uint32_t nrows, uint32_t k, uint32_t row_base,
                              uint32_t* out_rows, float* out_scores, uint32_t* out_count,
                              cudaStream_t stream) {
  if (nrows > kExactMaxRows) return cudaErrorInvalidValue;
  uint32_t np = 2;
  while (np < nrows) np <<= 1;
  const size_t smem = static_cast<size_t>(np) * 8;
  exact_rows_kernel<<<1, kExactThreads, smem, stream>>>(originals, dim, query, rows, nrows, np, k,
                                                        row_base, out_rows, out_scores, out_count);
  return cudaGetLastError();
}

}  // namespace bv
