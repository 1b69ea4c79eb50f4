// int8 scan instantiations (P = 4 .. 8192).
#include "bv_scan_launch.cuh"

namespace bv {
cudaError_t launch_scan8(int mode, const ScanShape& sh, const ScanParams& p, unsigned grid,
                         size_t smem, cudaStream_t stream) {
  if (mode == kAsym) {
    BV_SHAPES_SMALL(8, kAsym)
    BV_SHAPES_LARGE(8, kAsym)
    BV_TRY_SHAPE(8, kAsym, 16, 32, 16, 1)
  } else if (mode == kInt) {
    BV_SHAPES_SMALL(8, kInt)
    BV_SHAPES_LARGE(8, kInt)
    BV_TRY_SHAPE(8, kInt, 16, 32, 16, 1)
  }
  return cudaErrorNotSupported;
}
}  // namespace bv
