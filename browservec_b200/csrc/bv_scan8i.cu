// 8-bit int scan instantiations.
#include "bv_scan_launch.cuh"

namespace bv {
cudaError_t launch_scan8_int(const ScanShape& sh, const ScanParams& p, unsigned grid,
                                  size_t smem, cudaStream_t stream) {
  BV_SHAPES_SMALL(8, kInt)
  BV_SHAPES_INT(8, kInt)
  BV_SHAPES_INT_WIDE(8, kInt)
  return cudaErrorNotSupported;
}
}  // namespace bv
