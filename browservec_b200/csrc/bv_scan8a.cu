// 8-bit asym scan instantiations.
#include "bv_scan_launch.cuh"

namespace bv {
cudaError_t launch_scan8_asym(const ScanShape& sh, const ScanParams& p, unsigned grid,
                                  size_t smem, cudaStream_t stream) {
  BV_SHAPES_SMALL(8, kAsym)
  BV_SHAPES_ASYM(8)
  BV_SHAPES_ASYM_WIDE(8)
  return cudaErrorNotSupported;
}
}  // namespace bv
