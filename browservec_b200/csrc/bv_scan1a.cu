// 1-bit asym scan instantiations.
#include "bv_scan_launch.cuh"

namespace bv {
cudaError_t launch_scan1_asym(const ScanShape& sh, const ScanParams& p, unsigned grid,
                                  size_t smem, cudaStream_t stream) {
  BV_SHAPES_SMALL(1, kAsym)
  BV_SHAPES_ASYM(1)
  return cudaErrorNotSupported;
}
}  // namespace bv
