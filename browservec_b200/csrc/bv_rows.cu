// bv_rows.cu -- the candidate-list (IVF x quant "indexed") search: gather the
// candidate rows' codes and scales into contiguous per-query segments, which
// the ordinary scan then streams; keys carry the position in the candidate
// list and the finish maps positions back to rows (src/index/ivfquant.ts:
// 468-490 and the indexed shaders, src/engine/wgsl/distanceQ8.ts:25-41).
#include <cstdint>

#include "bv_device.cuh"
#include "bv_internal.h"

namespace bv {

namespace {

constexpr int kGatherThreads = 256;

// Block (x, q): candidates of query q, one warp per candidate row; its code
// words are copied 4 bytes a lane (a row is a whole number of words), the
// scale and the row id by lane 0.  A candidate outside the index raises
// bad_row and gathers row 0 instead, so every read stays in bounds.
__global__ void __launch_bounds__(kGatherThreads) gather_rows_kernel(const uint32_t* __restrict__ codes,
                                                                    const float* __restrict__ scales, uint32_t R4,
                                                                    uint64_t rows, const uint32_t* __restrict__ cand,
                                                                    const uint32_t* __restrict__ offs,
                                                                    const uint32_t* __restrict__ seg,
                                                                    uint32_t* __restrict__ gcodes,
                                                                    float* __restrict__ gscales,
                                                                    uint32_t* __restrict__ growmap,
                                                                    uint32_t* bad_row) {
  const uint32_t q = blockIdx.y;
  const uint32_t c0 = offs[q] - offs[0], n = offs[q + 1] - offs[q], dst0 = seg[q];
  const int lane = threadIdx.x & 31;
  const uint32_t warps = kGatherThreads / 32;
  for (uint32_t i = blockIdx.x * warps + (threadIdx.x >> 5); i < n; i += gridDim.x * warps) {
    uint32_t r = cand[c0 + i];
    if (r >= rows) {
      if (lane == 0) atomicOr(bad_row, 1u);
      r = 0;
    }
    const uint32_t* src = codes + static_cast<size_t>(r) * R4;
    uint32_t* dst = gcodes + static_cast<size_t>(dst0 + i) * R4;
    for (uint32_t w = lane; w < R4; w += 32) dst[w] = __ldg(src + w);
    if (lane == 0) {
      gscales[dst0 + i] = __ldg(scales + r);
      growmap[dst0 + i] = r;
    }
  }
}

}  // namespace

cudaError_t launch_gather_rows(const uint8_t* codes, const float* scales, uint32_t R, uint64_t rows,
                               const uint32_t* cand, const uint32_t* offs, const uint32_t* seg, uint32_t nq,
                               uint32_t max_n, uint8_t* gcodes, float* gscales, uint32_t* growmap,
                               uint32_t* bad_row, cudaStream_t s) {
  if (nq == 0 || max_n == 0) return cudaSuccess;
  const uint32_t warps = kGatherThreads / 32;
  uint32_t bx = (max_n + warps - 1) / warps;
  if (bx > 1024) bx = 1024;
  gather_rows_kernel<<<dim3(bx, nq), kGatherThreads, 0, s>>>(
      reinterpret_cast<const uint32_t*>(codes), scales, R / 4, rows, cand, offs, seg,
      reinterpret_cast<uint32_t*>(gcodes), gscales, growmap, bad_row);
  return cudaGetLastError();
}

}  // namespace bv
