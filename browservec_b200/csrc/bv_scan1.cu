// 1-bit scan instantiations (P = 32 .. 8192).
#include "bv_scan_launch.cuh"

namespace bv {
cudaError_t launch_scan1(int mode, const ScanShape& sh, const ScanParams& p, unsigned grid,
                         size_t smem, cudaStream_t stream) {
  if (mode == kAsym) {
    BV_SHAPES_SMALL(1, kAsym)
  } else if (mode == kInt) {
    BV_SHAPES_SMALL(1, kInt)
  } else if (mode == kHamming) {
    BV_SHAPES_SMALL(1, kHamming)
  }
  return cudaErrorNotSupported;
}
}  // namespace bv
