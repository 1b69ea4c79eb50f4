// bv_scan_launch.cuh -- shape dispatch for one bit width (included once per
// bv_scan{8,4,1}.cu so the instantiations compile in parallel).
#pragma once

#include "bv_internal.h"
#include "bv_scan.cuh"

namespace bv {

template <int BITS, int MODE, int CB, int L, int CPL, int U>
cudaError_t launch_one(const ScanParams& p, unsigned grid, size_t smem, cudaStream_t stream) {
  auto kern = scan_kernel<BITS, MODE, CB, L, CPL, U>;
  // Opt in to the device's full dynamic shared memory once per kernel and device.
  static int opted[kMaxDevices] = {};
  const cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(kern), smem, opted);
  if (e != cudaSuccess) return e;
  // Programmatic dependent launch: the kernel may start while the previous
  // scan in the stream finishes its merge; it waits (griddepcontrol.wait)
  // before touching the shared scratch.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kScanThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

#define BV_TRY_SHAPE(BITS, MODE, CB_, L_, CPL_, U_)                                   \
  if (sh.CB == CB_ && sh.L == L_ && sh.CPL == CPL_ && sh.U == U_)                     \
    return launch_one<BITS, MODE, CB_, L_, CPL_, U_>(p, grid, smem, stream);

// Shapes of small rows (R < 512 bytes): shared by every mode.
#define BV_SHAPES_SMALL(BITS, MODE)                                                   \
  BV_TRY_SHAPE(BITS, MODE, 4, 1, 1, 2)                                                \
  BV_TRY_SHAPE(BITS, MODE, 8, 1, 1, 2)                                                \
  BV_TRY_SHAPE(BITS, MODE, 16, 1, 1, 2)                                               \
  BV_TRY_SHAPE(BITS, MODE, 16, 2, 1, 2)                                               \
  BV_TRY_SHAPE(BITS, MODE, 16, 4, 1, 2)                                               \
  BV_TRY_SHAPE(BITS, MODE, 16, 8, 1, 2)

// Canonical asym layouts of wider rows.
#define BV_SHAPES_ASYM(BITS)                                                          \
  BV_TRY_SHAPE(BITS, kAsym, 16, 16, 1, 2)                                             \
  BV_TRY_SHAPE(BITS, kAsym, 16, 32, 1, 2)                                             \
  BV_TRY_SHAPE(BITS, kAsym, 16, 32, 2, 2)

#define BV_SHAPES_ASYM_WIDE(BITS)                                                     \
  BV_TRY_SHAPE(BITS, kAsym, 16, 32, 4, 2)                                             \
  BV_TRY_SHAPE(BITS, kAsym, 16, 32, 8, 2)

// Integer-mode layouts of wider rows (8 lanes per row up to 32 chunks, 16 at 64).
#define BV_SHAPES_INT(BITS, MODE)                                                     \
  BV_TRY_SHAPE(BITS, MODE, 16, 8, 2, 2)                                               \
  BV_TRY_SHAPE(BITS, MODE, 16, 8, 4, 1)                                               \
  BV_TRY_SHAPE(BITS, MODE, 16, 16, 4, 1)

#define BV_SHAPES_INT_WIDE(BITS, MODE)                                                \
  BV_TRY_SHAPE(BITS, MODE, 16, 16, 8, 1)                                              \
  BV_TRY_SHAPE(BITS, MODE, 16, 32, 8, 1)

}  // namespace bv
