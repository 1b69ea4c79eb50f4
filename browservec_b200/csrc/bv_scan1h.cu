// 1-bit hamming scan instantiations.
#include "bv_scan_launch.cuh"

namespace bv {
cudaError_t launch_scan1_hamming(const ScanShape& sh, const ScanParams& p, unsigned grid,
                                  size_t smem, cudaStream_t stream) {
  BV_SHAPES_SMALL(1, kHamming)
  BV_SHAPES_INT(1, kHamming)
  return cudaErrorNotSupported;
}
}  // namespace bv
