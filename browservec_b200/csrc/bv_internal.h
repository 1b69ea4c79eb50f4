// bv_internal.h -- declarations shared by the library's translation units.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/browservec.h"

namespace bv {

struct ScanParams;

// Template shape of one scan kernel (see ScanCfg in bv_scan.cuh).
struct ScanShape {
  int CB, L, CPL, U;
  uint32_t R;          // code bytes per row
  uint32_t rows_per_iter;
};

// Row bytes of the code layout (encode.ts:49-53: P/4, P/8, P/32 words).
inline uint32_t code_row_bytes(int bits, uint32_t P) {
  return bits == 8 ? P : (bits == 4 ? P / 2 : P / 8);
}

// Lane layout of one scan: the asym mode uses the canonical layout (L = min(32,
// C) lanes per row, the order the oracle defines); the integer modes, whose
// sums are exact in any order, use 8 lanes per row up to 32 chunks, 16 lanes at
// 64 chunks (so one iteration's rows stay within a 32 KB tile and two CTAs fit
// an SM), and up to 8 chunks per lane beyond.
inline bool scan_shape(int bits, int mode, uint32_t P, ScanShape* s) {
  const uint32_t R = code_row_bytes(bits, P);
  if (R < 4 || R > 4096) return false;
  s->R = R;
  s->CB = R < 16 ? static_cast<int>(R) : 16;
  const uint32_t C = R / static_cast<uint32_t>(s->CB);
  uint32_t L;
  if (mode == 0) {
    L = C < 32 ? C : 32;
  } else {
    L = C <= 8 ? C : (C <= 32 ? 8 : (C <= 64 ? 16 : C / 8));
  }
  s->L = static_cast<int>(L);
  s->CPL = static_cast<int>(C / L);
  s->U = (mode == 0 || s->CPL < 4) ? 2 : 1;
  s->rows_per_iter = 16u * (32u / L) * static_cast<uint32_t>(s->U);
  return true;
}

cudaError_t launch_encode(int bits, const float* rows, uint64_t count, uint32_t dim, uint32_t P,
                          const float* signs, uint32_t rounds, uint8_t* codes, float* scales,
                          uint32_t R, cudaStream_t stream);

cudaError_t launch_scan8_asym(const ScanShape& sh, const ScanParams& p, unsigned grid, size_t smem,
                              cudaStream_t stream);
cudaError_t launch_scan8_int(const ScanShape& sh, const ScanParams& p, unsigned grid, size_t smem,
                             cudaStream_t stream);
cudaError_t launch_scan4_asym(const ScanShape& sh, const ScanParams& p, unsigned grid, size_t smem,
                              cudaStream_t stream);
cudaError_t launch_scan4_int(const ScanShape& sh, const ScanParams& p, unsigned grid, size_t smem,
                             cudaStream_t stream);
cudaError_t launch_scan1_asym(const ScanShape& sh, const ScanParams& p, unsigned grid, size_t smem,
                              cudaStream_t stream);
cudaError_t launch_scan1_int(const ScanShape& sh, const ScanParams& p, unsigned grid, size_t smem,
                             cudaStream_t stream);
cudaError_t launch_scan1_hamming(const ScanShape& sh, const ScanParams& p, unsigned grid, size_t smem,
                                 cudaStream_t stream);

struct TailParams;
cudaError_t launch_tail(const TailParams& p, size_t smem, cudaStream_t stream);

cudaError_t launch_exact_rows(const float* originals, uint32_t dim, const float* query,
                              const uint32_t* rows, uint32_t nrows, uint32_t k, uint32_t row_base,
                              uint32_t* out_rows, float* out_scores, uint32_t* out_count,
                              cudaStream_t stream);

// Raise `func`'s dynamic shared-memory limit on the CURRENT device to the
// device's opt-in maximum (minus the kernel's static shared memory), once per
// device: function attributes belong to a device's context.  `opted` is the
// caller's per-kernel table of limits already set; cudaErrorInvalidValue when
// `need` cannot fit.
constexpr int kMaxDevices = 64;
inline cudaError_t opt_in_smem(const void* func, size_t need, int* opted) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (opted[dev] >= static_cast<int>(need)) return cudaSuccess;
  cudaFuncAttributes fa;
  if ((e = cudaFuncGetAttributes(&fa, func)) != cudaSuccess) return e;
  int maxs = 0;
  if ((e = cudaDeviceGetAttribute(&maxs, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) return e;
  const int lim = maxs - static_cast<int>(fa.sharedSizeBytes);
  if (static_cast<int>(need) > lim) return cudaErrorInvalidValue;
  if ((e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, lim)) != cudaSuccess) return e;
  opted[dev] = lim;
  return cudaSuccess;
}

// bv_flat.cu: exact fp32 flat scan (bits = 0).  The TMA-fed scan needs rows
// of a multiple of 4 floats at a 16-byte aligned base; flat_kernel takes any.
bool flat_scan_supported(const float* rows, uint32_t dim);
uint32_t flat_scan_block_rows();
uint32_t flat_scan_stage_bytes();
cudaError_t encode_flat_rows_map(void* map128, const float* rows, uint32_t dim, uint64_t nrows);
cudaError_t encode_tile_rows_map(void* map128, const void* base, uint64_t nrows, uint32_t box_rows);
cudaError_t launch_flat_scan(const void* map128, const ScanParams& p, uint32_t nblocks, uint32_t nks,
                             uint32_t check_blocks, unsigned grid, size_t smem, cudaStream_t stream);
uint32_t flat_rows_per_cta();
cudaError_t launch_flat(const float* rows, const float* query, const uint32_t* mask, uint32_t nrows, uint32_t dim,
                        uint32_t Fp, uint64_t* partials, cudaStream_t stream);

// bv_tail.cu: one tail CTA per query of a batch
struct TailParams;
cudaError_t launch_tail_grid(const TailParams& p, uint32_t nq, size_t smem, cudaStream_t stream);

// bv_batch.cu: batched tensor-core search
struct ExpandParams;
struct PrepParams;
struct GemmParams;
struct SelectParams;
uint32_t batch_gemm_smem(uint32_t cnt_words);
cudaError_t launch_expand(const ExpandParams& p, cudaStream_t s);
cudaError_t launch_prep(const PrepParams& p, cudaStream_t s);
cudaError_t launch_gemm(const GemmParams& p, uint32_t grid, cudaStream_t s);
uint32_t batch_gemm_pair_smem();
cudaError_t launch_gemm_pair(const GemmParams& p, const void* amap, const void* bmap, uint32_t npairs,
                             cudaStream_t s);
cudaError_t launch_select(const SelectParams& p, cudaStream_t s);
cudaError_t launch_export_keys(const uint64_t* cand, uint32_t cap, const uint32_t* cnt, uint32_t nq, uint32_t F,
                               uint32_t base, uint64_t* keys, cudaStream_t s);
cudaError_t launch_trim_keys(uint64_t* cand, uint32_t cap, uint32_t Fp, uint32_t nq, uint32_t base,
                             const uint64_t* thr, cudaStream_t s);
uint32_t keys_threshold_max();
cudaError_t launch_keys_threshold(const uint64_t* gathered, uint32_t world, uint32_t nq, uint32_t F, uint64_t* thr,
                                  cudaStream_t s);
uint32_t compact_block_words();
cudaError_t launch_mask_count(const uint32_t* mask, uint64_t rows, uint32_t* word_off, uint32_t* block_sum,
                              uint32_t* count, cudaStream_t s);
cudaError_t launch_row_map(const uint32_t* mask, uint64_t rows, const uint32_t* word_off, const uint32_t* block_sum,
                           uint32_t* map, cudaStream_t s);
cudaError_t launch_factor(uint32_t bits, const float* scales, const uint32_t* rows, uint32_t row0, uint32_t n,
                          float* fac, uint32_t* ids, cudaStream_t s);
cudaError_t launch_scatter_tiles(const uint32_t* in, uint32_t* out, uint32_t count, uint32_t head, uint32_t K,
                                 uint32_t ginv, cudaStream_t s);
cudaError_t launch_sort_rows(void* tmp, size_t* tmp_bytes, const float* fac_in, float* fac_out,
                             const uint32_t* ids_in, uint32_t* ids_out, uint32_t n, cudaStream_t s);
// bv_filter.cu
cudaError_t launch_filter(const bv_column* cols, uint32_t ncols, const bv_filter_term* terms, uint32_t nterms,
                          uint64_t rows, const uint32_t* live, uint32_t* mask, cudaStream_t s);

// bv_merge.cu: cross-shard merge of all-gathered shard records
size_t merge_smem_bytes(uint32_t world, uint32_t F);
uint32_t merge_max_world();
cudaError_t launch_wait_probe(uint32_t* err, uint32_t polls, cudaStream_t s);
cudaError_t launch_gather_rows(const uint8_t* codes, const float* scales, uint32_t R, uint64_t rows,
                               const uint32_t* cand, const uint32_t* offs, const uint32_t* seg, uint32_t nq,
                               uint32_t max_n, uint8_t* gcodes, float* gscales, uint32_t* growmap,
                               uint32_t* bad_row, cudaStream_t s);
cudaError_t launch_merge_topk(const uint32_t* gathered, uint32_t world, uint32_t nq, uint32_t k,
                              uint32_t* out_rows, float* out_scores, uint32_t* out_counts, cudaStream_t stream);
cudaError_t launch_merge_shards(const uint32_t* gathered, uint32_t world, uint32_t nq, uint32_t F, uint32_t k,
                                uint32_t* out_rows, float* out_scores, uint32_t* out_counts,
                                cudaStream_t stream);

}  // namespace bv
