// bv_scan_launch.cuh -- shape dispatch for one bit width (included once per
// bv_scan{8,4,1}.cu so the instantiations compile in parallel).
#pragma once

#include "bv_internal.h"
#include "bv_scan.cuh"

namespace bv {

template <int BITS, int MODE, int CB, int L, int CPL, int U>
cudaError_t launch_one(const ScanParams& p, unsigned grid, size_t smem, cudaStream_t stream) {
  auto kern = scan_kernel<BITS, MODE, CB, L, CPL, U>;
  // Opt in to the device's full dynamic shared memory once per kernel.
  static int opted = 0;
  if (opted < static_cast<int>(smem)) {
    int dev = 0, maxs = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&maxs, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, maxs);
    if (e != cudaSuccess) return e;
    opted = maxs;
  }
  kern<<<grid, kScanThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

#define BV_TRY_SHAPE(BITS, MODE, CB_, L_, CPL_, U_)                                   \
  if (sh.CB == CB_ && sh.L == L_ && sh.CPL == CPL_ && sh.U == U_)                     \
    return launch_one<BITS, MODE, CB_, L_, CPL_, U_>(p, grid, smem, stream);

#define BV_SHAPES_SMALL(BITS, MODE)                                                   \
  BV_TRY_SHAPE(BITS, MODE, 4, 1, 1, 4)                                                \
  BV_TRY_SHAPE(BITS, MODE, 8, 1, 1, 4)                                                \
  BV_TRY_SHAPE(BITS, MODE, 16, 1, 1, 4)                                               \
  BV_TRY_SHAPE(BITS, MODE, 16, 2, 1, 4)                                               \
  BV_TRY_SHAPE(BITS, MODE, 16, 4, 1, 4)                                               \
  BV_TRY_SHAPE(BITS, MODE, 16, 8, 1, 4)                                               \
  BV_TRY_SHAPE(BITS, MODE, 16, 16, 1, 4)                                              \
  BV_TRY_SHAPE(BITS, MODE, 16, 32, 1, 4)                                              \
  BV_TRY_SHAPE(BITS, MODE, 16, 32, 2, 2)

#define BV_SHAPES_LARGE(BITS, MODE)                                                   \
  BV_TRY_SHAPE(BITS, MODE, 16, 32, 4, 1)                                              \
  BV_TRY_SHAPE(BITS, MODE, 16, 32, 8, 1)

}  // namespace bv
