// bv_flat.cu -- the exact fp32 flat scan (no quantization).
//
// The reference's exact flat search scores every row with an f32 dot; its CPU
// path (src/fallback/kernel.wat:6-43, CpuIndex.query, src/index/cpu.ts:66-88)
// runs it as WASM SIMD: four f32 lanes, lane j accumulating
// x[i+j] * q[i+j] for i = 0, 4, 8, ... with a separate multiply and add, the
// lanes summed as (l0 + l1) + (l2 + l3), then the dim % 4 tail added in order.
// This kernel computes exactly that sum, so its scores equal the reference
// CPU path's bit for bit: four threads per row, thread j owning lane j's
// chain, combined by two shuffles in the same order.
//
// One CTA scores 128 rows and writes its best Fp keys (score desc, row asc),
// sorted, to the per-query partials; the tail kernel (re-rank off: the scores
// are exact) merges them into the top k, chained by programmatic dependent
// launch like the quantized scan; each query writes its own slot of the
// partials ring, so nothing here waits for an earlier query's tail.
#include <cstdint>

#include "bv_device.cuh"
#include "bv_internal.h"
#include "bv_scan.cuh"

namespace bv {

namespace {

constexpr uint32_t kFlatRows = kConsumerThreads / 4;  // rows per CTA

struct FlatParams {
  const float* rows;   // nrows x dim fp32
  const float* query;  // dim fp32
  const uint32_t* mask;
  uint32_t nrows, dim, Fp;
  uint64_t* partials;  // gridDim.x x Fp keys
};

__global__ void __launch_bounds__(kConsumerThreads, 1) flat_kernel(const FlatParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint64_t* cand = reinterpret_cast<uint64_t*>(smem);            // max(16 * Fp, 128) keys
  float* q = reinterpret_cast<float*>(cand + (p.Fp <= 256u ? 16u * p.Fp : p.Fp));
  const int ctid = threadIdx.x;
  pdl_trigger();  // the tail (then the next query's scan) may be scheduled now
  for (uint32_t i = ctid; i < p.dim; i += kConsumerThreads) q[i] = p.query[i];
  for (uint32_t i = ctid; i < (p.Fp <= 256u ? 16u * p.Fp : p.Fp); i += kConsumerThreads) cand[i] = 0ull;
  __syncthreads();

  const uint32_t local = static_cast<uint32_t>(ctid) >> 2, j = static_cast<uint32_t>(ctid) & 3u;
  const uint32_t row = blockIdx.x * kFlatRows + local;
  const bool live = row < p.nrows;
  const uint32_t vec = p.dim & ~3u;
  const float* x = p.rows + static_cast<size_t>(live ? row : 0) * p.dim;
  float acc = 0.0f;  // lane j of the f32x4 accumulator
  if (live) {
#pragma unroll 8
    for (uint32_t i = j; i < vec; i += 4) acc = __fadd_rn(acc, __fmul_rn(__ldg(x + i), q[i]));
  }
  // (l0 + l1) + (l2 + l3): lanes 0/2 add their odd neighbour, lane 0 adds lane 2's pair
  const float pair = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
  float sum = __fadd_rn(pair, __shfl_xor_sync(0xffffffffu, pair, 2));
  if (j == 0) {
    for (uint32_t i = vec; i < p.dim; ++i) sum = __fadd_rn(sum, __fmul_rn(x[i], q[i]));
    bool keep = live;
    if (keep && p.mask) keep = (p.mask[row >> 5] >> (row & 31u)) & 1u;
    cand[local] = keep ? make_key(sum, row) : 0ull;
  }
  __syncthreads();
  if (p.Fp <= 256u) {
    cta_best_sorted_dispatch(p.Fp, cand, kFlatRows, ctid);
  } else {
    cta_sort_desc(cand, kFlatRows, ctid);  // 128 keys sorted; slots up to Fp stay zero
  }
  uint64_t* out = p.partials + static_cast<size_t>(blockIdx.x) * p.Fp;
  for (uint32_t i = ctid; i < p.Fp; i += kConsumerThreads) out[i] = cand[i];
}

}  // namespace

uint32_t flat_rows_per_cta() { return kFlatRows; }

cudaError_t launch_flat(const float* rows, const float* query, const uint32_t* mask, uint32_t nrows, uint32_t dim,
                        uint32_t Fp, uint64_t* partials, cudaStream_t stream) {
  FlatParams p;
  p.rows = rows;
  p.query = query;
  p.mask = mask;
  p.nrows = nrows;
  p.dim = dim;
  p.Fp = Fp;
  p.partials = partials;
  const size_t smem = static_cast<size_t>(Fp <= 256u ? 16u * Fp : Fp) * 8 + static_cast<size_t>(dim) * 4 + 16;
  static int opted[kMaxDevices] = {};
  cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(flat_kernel), smem, opted);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((nrows + kFlatRows - 1) / kFlatRows);
  cfg.blockDim = dim3(kConsumerThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, flat_kernel, p);
}

}  // namespace bv
