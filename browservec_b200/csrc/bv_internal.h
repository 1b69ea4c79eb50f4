// bv_internal.h -- declarations shared by the library's translation units.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

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
// sums are exact in any order, use at most 8 lanes per row and up to 8 chunks
// per lane so fewer shuffles reduce each row.
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
    L = C <= 8 ? C : (C <= 64 ? 8 : C / 8);
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

}  // namespace bv
