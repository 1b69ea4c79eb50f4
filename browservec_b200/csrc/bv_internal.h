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

inline bool scan_shape(int bits, uint32_t P, ScanShape* s) {
  const uint32_t R = code_row_bytes(bits, P);
  if (R < 4 || R > 8192) return false;
  s->R = R;
  s->CB = R < 16 ? static_cast<int>(R) : 16;
  const uint32_t C = R / static_cast<uint32_t>(s->CB);
  s->L = C < 32 ? static_cast<int>(C) : 32;
  s->CPL = static_cast<int>(C / static_cast<uint32_t>(s->L));
  s->U = s->CPL == 1 ? 4 : (s->CPL == 2 ? 2 : 1);
  s->rows_per_iter = 8u * (32u / static_cast<uint32_t>(s->L)) * static_cast<uint32_t>(s->U);
  return true;
}

cudaError_t launch_encode(int bits, const float* rows, uint64_t count, uint32_t dim, uint32_t P,
                          const float* signs, uint32_t rounds, uint8_t* codes, float* scales,
                          uint32_t R, cudaStream_t stream);

cudaError_t launch_scan8(int mode, const ScanShape& sh, const ScanParams& p, unsigned grid,
                         size_t smem, cudaStream_t stream);
cudaError_t launch_scan4(int mode, const ScanShape& sh, const ScanParams& p, unsigned grid,
                         size_t smem, cudaStream_t stream);
cudaError_t launch_scan1(int mode, const ScanShape& sh, const ScanParams& p, unsigned grid,
                         size_t smem, cudaStream_t stream);

cudaError_t launch_exact_rows(const float* originals, uint32_t dim, const float* query,
                              const uint32_t* rows, uint32_t nrows, uint32_t k, uint32_t row_base,
                              uint32_t* out_rows, float* out_scores, uint32_t* out_count,
                              cudaStream_t stream);

}  // namespace bv
