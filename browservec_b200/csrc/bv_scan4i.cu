// 4-bit int scan instantiations.
#include "bv_scan_launch.cuh"

namespace bv {
cudaError_t launch_scan4_int(const ScanShape& sh, const ScanParams& p, unsigned grid,
                                  size_t smem, cudaStream_t stream) {
  BV_SHAPES_SMALL(4, kInt)
  BV_SHAPES_INT(4, kInt)
  BV_TRY_SHAPE(4, kInt, 16, 16, 8, 1)
  return cudaErrorNotSupported;
}
}  // namespace bv
