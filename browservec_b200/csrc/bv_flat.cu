// bv_flat.cu -- the exact fp32 flat scan (no quantization).
//
// The reference's exact flat search scores every row with an f32 dot; its CPU
// path (src/fallback/kernel.wat:6-43, CpuIndex.query, src/index/cpu.ts:66-88)
// runs it as WASM SIMD: four f32 lanes, lane j accumulating
// x[i+j] * q[i+j] for i = 0, 4, 8, ... with a separate multiply and add, the
// lanes summed as (l0 + l1) + (l2 + l3), then the dim % 4 tail added in order.
// Both kernels here compute exactly that sum, so their scores equal the
// reference CPU path's bit for bit: four threads per row, thread j owning
// lane j's chain, combined by two shuffles in the same order.
//
// flat_scan_kernel (rows of a multiple of 4 floats): the quantized scan's
// structure.  A producer warp streams blocks of 128 rows, 32 columns per
// stage, with one 2-D TMA copy each (128-byte swizzle, so the eight rows a
// warp reads sit in distinct banks; rows and columns past the end read as
// zero); 16 consumer warps run the lane chains across a block's column
// stages, offer the finished scores to the CTA's candidate buffer above its
// admission threshold, and the last CTA of the query finishes it (merge of
// the CTA lists, top k) -- no tail kernel.  Blocks come from a shared counter.
//
// flat_kernel (any dim): one CTA scores 128 rows and writes its best Fp keys
// (score desc, row asc), sorted, to the per-query partials; the tail kernel
// (re-rank off: the scores are exact) merges them into the top k, chained by
// programmatic dependent launch like the quantized scan; each query writes its
// own slot of the partials ring, so nothing here waits for an earlier query's
// tail.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstring>

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

// ------------------------------------------------------- flat_scan_kernel
constexpr uint32_t kFsRows = 128;                    // rows per block (16 warps x 8 rows)
constexpr uint32_t kFsCols = 32;                     // columns per stage: one 128-byte swizzle row
constexpr uint32_t kFsStageBytes = kFsRows * kFsCols * 4;  // 16 KB, one TMA box

// 2-D tiled TMA load of box {32 columns, 128 rows} at (col, row) into dst
// (1024-byte aligned), completing on bar.  No cluster multicast.
__device__ __forceinline__ void tma_load_rows(void* dst, const CUtensorMap* map, uint32_t col, uint32_t row,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(col), "r"(row), "r"(smem_addr(bar))
      : "memory");
}

__global__ void __launch_bounds__(kScanThreads, 2)
    flat_scan_kernel(const __grid_constant__ CUtensorMap rows_map, const ScanParams p, const uint32_t nblocks,
                     const uint32_t nks, const uint32_t check_blocks) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);  // the swizzle pattern repeats every 1 KB
  const FlatSmem lay = flat_smem_layout(p.dim, p.stages, p.capc);
  float* xs = reinterpret_cast<float*>(smem + lay.rows_off);
  float* q = reinterpret_cast<float*>(smem + lay.q_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + lay.bars_off);
  uint64_t* empty = full + p.stages;
  uint64_t* qbar = empty + p.stages;
  volatile uint32_t* stage_blk = reinterpret_cast<volatile uint32_t*>(smem + lay.ids_off);
  volatile uint32_t* stage_ks = stage_blk + p.stages;
  uint64_t* cand = reinterpret_cast<uint64_t*>(smem + lay.cand_off);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + lay.hist_off);
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + lay.misc_off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (p.trace && threadIdx.x == 0) p.trace[blockIdx.x * 8 + kTrEntry] = globaltimer();
  constexpr uint32_t kNoTile = 0xFFFFFFFFu;
  const uint32_t q_bulk = (reinterpret_cast<uintptr_t>(p.query) & 15u) == 0 ? (p.dim * 4u) & ~15u : 0u;
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
  pdl_trigger();  // the next query's kernel may launch once every CTA of this one has started

  if (warp == kConsumerWarps) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      mbar_arrive_expect_tx(qbar, q_bulk);
      if (q_bulk) bulk_g2s(q, p.query, q_bulk, qbar);
      uint32_t b = grab_tile(p.tile_ctr, p.epoch, p.err);
      uint32_t it = 0, s = 0, ph = 0;  // stage and phase advance with it
      bool more = true;
      while (more) {
        for (uint32_t ks = 0; ks < nks; ++ks, ++it, s = s + 1u == p.stages ? 0u : s + 1u, ph ^= s == 0u ? 1u : 0u) {
          if (it >= p.stages && !mbar_wait_bounded(&empty[s], ph ^ 1u, p.err)) {
            more = false;
            break;
          }
          if (b >= nblocks) {  // no more work: an empty stage tells the consumers
            stage_blk[s] = kNoTile;
            mbar_arrive(&full[s]);
            more = false;
            break;
          }
          stage_blk[s] = b;
          stage_ks[s] = ks;
          mbar_arrive_expect_tx(&full[s], kFsStageBytes);
          tma_load_rows(xs + static_cast<size_t>(s) * (kFsStageBytes / 4), &rows_map, ks * kFsCols, b * kFsRows,
                        &full[s]);
        }
        if (more) b = grab_tile(p.tile_ctr, p.epoch, p.err);
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- consumers
    const int ctid = threadIdx.x;
    mbar_wait_bounded(qbar, 0, p.err);
    for (uint32_t i = q_bulk / 4 + ctid; i < p.dim; i += kConsumerThreads) q[i] = p.query[i];
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if (p.trace && ctid == 0) p.trace[blockIdx.x * 8 + kTrRotated] = globaltimer();
    const uint32_t high = p.capc - check_blocks * kFsRows;
    uint64_t thr = 0;
    const uint32_t r = static_cast<uint32_t>(warp) * 8u + (static_cast<uint32_t>(lane) >> 2);  // row in block
    const uint32_t j = static_cast<uint32_t>(lane) & 3u;                                       // WASM lane
    const uint32_t sw = r & 7u;  // 16-byte chunk c of row r sits at chunk c ^ sw
    float acc = 0.0f;
    uint32_t blocks_done = 0;
    uint32_t s = 0, ph = 0;
    for (uint32_t it = 0;; ++it, s = s + 1u == p.stages ? 0u : s + 1u, ph ^= s == 0u ? 1u : 0u) {
      const bool landed = mbar_wait_bounded(&full[s], ph, p.err);
      const uint32_t b = landed ? stage_blk[s] : kNoTile;
      if (it == 0 && p.trace && ctid == 0) p.trace[blockIdx.x * 8 + kTrFirstTile] = globaltimer();
      if (b == kNoTile) break;
      const uint32_t ks = stage_ks[s];
      if (ks == 0) acc = 0.0f;
      const float* xr = xs + static_cast<size_t>(s) * (kFsStageBytes / 4) + r * kFsCols + j;
      const float* qk = q + ks * kFsCols + j;
      const uint32_t left = p.dim - ks * kFsCols;
      if (left >= kFsCols) {
#pragma unroll
        for (uint32_t t = 0; t < kFsCols / 4; ++t) acc = __fadd_rn(acc, __fmul_rn(xr[(t ^ sw) * 4u], qk[t * 4u]));
      } else {
        for (uint32_t t = 0; t < left / 4u; ++t) acc = __fadd_rn(acc, __fmul_rn(xr[(t ^ sw) * 4u], qk[t * 4u]));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (ks == nks - 1u) {
        // (l0 + l1) + (l2 + l3): lanes 0/2 add their odd neighbour, lane 0 adds lane 2's pair
        const float pair = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
        const float sum = __fadd_rn(pair, __shfl_xor_sync(0xffffffffu, pair, 2));
        const uint64_t row = static_cast<uint64_t>(b) * kFsRows + r;
        bool valid = j == 0u && row < p.nrows;
        if (valid && p.mask) valid = (p.mask[row >> 5] >> (row & 31u)) & 1u;
        const uint64_t key = make_key(sum, static_cast<uint32_t>(row));
        append_keys(cand, &misc[kMiscCount], key, valid && key > thr, lane);
        if (++blocks_done % check_blocks == 0) raise_threshold(cand, hist, misc, p.F, high, thr, ctid);
      }
    }
    named_bar_sync(kBarConsumers, kConsumerThreads);
    if (p.trace && ctid == 0) p.trace[blockIdx.x * 8 + kTrScanned] = globaltimer();
    cta_publish(p, cand, hist, misc, smem + lay.rows_off, p.stages * kFsStageBytes, qbar, ctid);
  }
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

namespace {
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}
}  // namespace

bool flat_scan_supported(const float* rows, uint32_t dim) {
  return (dim & 3u) == 0u && (reinterpret_cast<uintptr_t>(rows) & 15u) == 0u && dim <= (1u << 20);
}

uint32_t flat_scan_block_rows() { return kFsRows; }
uint32_t flat_scan_stage_bytes() { return kFsStageBytes; }

// A tensor map over an array of 128-byte rows (the batched search's MMA
// tiles, already in their shared-memory image): boxes of box_rows whole
// rows, copied byte for byte (no swizzle: the tiles are pre-swizzled).
cudaError_t encode_tile_rows_map(void* map128, const void* base, uint64_t nrows, uint32_t box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {128, nrows};
  const cuuint64_t strides[1] = {128};
  const cuuint32_t box[2] = {128, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(static_cast<CUtensorMap*>(map128), CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base),
                         dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t encode_flat_rows_map(void* map128, const float* rows, uint32_t dim, uint64_t nrows) {
  static_assert(sizeof(CUtensorMap) == 128, "tensor map size");
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {dim, nrows};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(dim) * 4u};
  const cuuint32_t box[2] = {kFsCols, kFsRows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(static_cast<CUtensorMap*>(map128), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                         const_cast<float*>(rows), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_flat_scan(const void* map128, const ScanParams& p, uint32_t nblocks, uint32_t nks,
                             uint32_t check_blocks, unsigned grid, size_t smem, cudaStream_t stream) {
  static int opted[kMaxDevices] = {};
  cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(flat_scan_kernel), smem, opted);
  if (e != cudaSuccess) return e;
  CUtensorMap map;
  memcpy(&map, map128, sizeof(map));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kScanThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, flat_scan_kernel, map, p, nblocks, nks, check_blocks);
}

}  // namespace bv
