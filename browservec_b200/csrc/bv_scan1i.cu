// 1-bit int scan instantiations.
#include "bv_scan_launch.cuh"

namespace bv {
cudaError_t launch_scan1_int(const ScanShape& sh, const ScanParams& p, unsigned grid,
                                  size_t smem, cudaStream_t stream) {
  BV_SHAPES_SMALL(1, kInt)
  BV_SHAPES_INT(1, kInt)
  return cudaErrorNotSupported;
}
}  // namespace bv
