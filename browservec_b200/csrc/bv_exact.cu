// bv_exact.cu -- exact scan over an explicit row list (BrowserVec.queryRowsExact,
// src/index.ts:445-464): the f64-accumulated dot of Store.dotRow
// (src/store/store.ts:114-130) per row, two rows a warp (dot_rows2_exact_warp:
// bit-identical to the lane-ordered sequence), then the best k by
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
  const int warp = tid >> 5;
  constexpr uint32_t W = kExactThreads / 32;
  for (uint32_t c = static_cast<uint32_t>(warp); c < npow2; c += 2u * W) {  // two rows a warp
    const uint32_t c2 = c + W;
    uint64_t ka = 0, kb = 0;
    if (c2 < nrows) {
      const uint32_t ra = rows[c], rb = rows[c2];
      float sa, sb;
      dot_rows2_exact_warp<true>(originals + static_cast<size_t>(ra) * dim, originals + static_cast<size_t>(rb) * dim,
                                 query, dim, lane, sa, sb);
      ka = make_key(sa, ra);
      kb = make_key(sb, rb);
    } else if (c < nrows) {
      const uint32_t ra = rows[c];
      ka = make_key(dot_row_exact_warp<true>(originals + static_cast<size_t>(ra) * dim, query, dim, lane), ra);
    }
    if (lane == 0) {
      if (c < npow2) keys[c] = ka;
      if (c2 < npow2) keys[c2] = kb;
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
