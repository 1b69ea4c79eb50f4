// 4-bit asym scan instantiations.
#include "bv_scan_launch.cuh"

namespace bv {
cudaError_t launch_scan4_asym(const ScanShape& sh, const ScanParams& p, unsigned grid,
                                  size_t smem, cudaStream_t stream) {
  BV_SHAPES_SMALL(4, kAsym)
  BV_SHAPES_ASYM(4)
  BV_TRY_SHAPE(4, kAsym, 16, 32, 4, 2)
  return cudaErrorNotSupported;
}
}  // namespace bv
