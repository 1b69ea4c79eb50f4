// int4 scan instantiations (P = 8 .. 8192).
#include "bv_scan_launch.cuh"

namespace bv {
cudaError_t launch_scan4(int mode, const ScanShape& sh, const ScanParams& p, unsigned grid,
                         size_t smem, cudaStream_t stream) {
  if (mode == kAsym) {
    BV_SHAPES_SMALL(4, kAsym)
    BV_SHAPES_LARGE(4, kAsym)
  } else if (mode == kInt) {
    BV_SHAPES_SMALL(4, kInt)
    BV_SHAPES_LARGE(4, kInt)
  }
  return cudaErrorNotSupported;
}
}  // namespace bv
