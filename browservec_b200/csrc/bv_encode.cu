// bv_encode.cu -- on-device corpus encoder: rotate + quantize each appended row
// with the exact arithmetic of the reference's ingest path
// (encode.ts:64-78 -> rotator.ts:60-70 -> codec.ts:32-54 / :85-108 / :135-154),
// so the codes are bit-identical to the CPU encoder's.  One warp per row.
#include <cstdint>

#include "bv_device.cuh"
#include "bv_internal.h"

namespace bv {

__device__ __forceinline__ double js_round_d(double x) {
  double r = floor(x);
  if (__dadd_rn(x, -r) >= 0.5) r = __dadd_rn(r, 1.0);
  return r;
}

// codec.ts:22-30 / :77-83: clamp to [-1,1], Math.round(c*levels), clamp.
__device__ __forceinline__ int snorm_level(double v, double levels) {
  double c = v < -1.0 ? -1.0 : (v > 1.0 ? 1.0 : v);
  double b = js_round_d(__dmul_rn(c, levels));
  b = b < -levels ? -levels : (b > levels ? levels : b);
  return static_cast<int>(b);
}

template <int BITS>
__global__ void encode_kernel(const float* __restrict__ rows, uint64_t count, uint32_t dim,
                              uint32_t P, const float* __restrict__ signs, uint32_t rounds,
                              uint8_t* __restrict__ codes, float* __restrict__ scales, uint32_t R,
                              uint32_t warps_per_block) {
  extern __shared__ float enc_smem[];
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t row = static_cast<uint64_t>(blockIdx.x) * warps_per_block + warp;
  if (row >= count) return;
  float* a = enc_smem + static_cast<size_t>(warp) * P;
  const float* src = rows + row * dim;
  for (uint32_t i = lane; i < P; i += 32) a[i] = i < dim ? src[i] : 0.0f;
  __syncwarp();
  for (uint32_t r = 0; r < rounds; ++r) {
    const float* s = signs + static_cast<size_t>(r) * P;
    if (P >= 32) {
      for (uint32_t blk = 0; blk < P / 32; ++blk) {
        const uint32_t i = blk * 32 + lane;
        float x = __fmul_rn(a[i], s[i]);
#pragma unroll
        for (int len = 1; len < 32; len <<= 1) {
          float y = __shfl_xor_sync(0xffffffffu, x, len);
          x = (lane & len) ? __fsub_rn(y, x) : __fadd_rn(x, y);
        }
        a[i] = x;
      }
      __syncwarp();
      for (uint32_t len = 32; len < P; len <<= 1) {
        for (uint32_t b = lane; b < P / 2; b += 32) {
          const uint32_t j = (b / len) * 2 * len + (b % len);
          const float x = a[j], y = a[j + len];
          a[j] = __fadd_rn(x, y);
          a[j + len] = __fsub_rn(x, y);
        }
        __syncwarp();
      }
    } else {
      for (uint32_t i = lane; i < P; i += 32) a[i] = __fmul_rn(a[i], s[i]);
      __syncwarp();
      for (uint32_t len = 1; len < P; len <<= 1) {
        for (uint32_t b = lane; b < P / 2; b += 32) {
          const uint32_t j = (b / len) * 2 * len + (b % len);
          const float x = a[j], y = a[j + len];
          a[j] = __fadd_rn(x, y);
          a[j + len] = __fsub_rn(x, y);
        }
        __syncwarp();
      }
    }
  }
  uint32_t* out = reinterpret_cast<uint32_t*>(codes + row * R);
  if constexpr (BITS == 8 || BITS == 4) {
    float m = 0.0f;
    for (uint32_t i = lane; i < P; i += 32) m = fmaxf(m, fabsf(a[i]));
#pragma unroll
    for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    const float scale = m > 0.0f ? m : 1.0f;
    const double inv = __ddiv_rn(1.0, static_cast<double>(scale));
    constexpr uint32_t per = BITS == 8 ? 4 : 8;
    for (uint32_t g = lane; g < P / per; g += 32) {
      uint32_t w = 0;
#pragma unroll
      for (uint32_t j = 0; j < per; ++j) {
        const int b = snorm_level(__dmul_rn(static_cast<double>(a[g * per + j]), inv),
                                  BITS == 8 ? 127.0 : 7.0);
        w |= static_cast<uint32_t>(b & (BITS == 8 ? 0xff : 0xf)) << ((BITS == 8 ? 8 : 4) * j);
      }
      out[g] = w;
    }
    if (lane == 0) scales[row] = scale;
  } else {
    for (uint32_t blk = 0; blk < P / 32; ++blk) {
      const uint32_t w = __ballot_sync(0xffffffffu, a[blk * 32 + lane] >= 0.0f);
      if (lane == 0) out[blk] = w;
    }
    if (lane == 0) {
      double abs_sum = 0.0;  // sequential, as codec.ts:140-141
      for (uint32_t i = 0; i < P; ++i) abs_sum = __dadd_rn(abs_sum, fabs(static_cast<double>(a[i])));
      scales[row] = abs_sum > 0.0 ? __double2float_rn(__ddiv_rn(abs_sum, static_cast<double>(P))) : 1.0f;
    }
  }
}

cudaError_t launch_encode(int bits, const float* rows, uint64_t count, uint32_t dim, uint32_t P,
                          const float* signs, uint32_t rounds, uint8_t* codes, float* scales,
                          uint32_t R, cudaStream_t stream) {
  if (count == 0) return cudaSuccess;
  uint32_t wpb = (160u * 1024u) / (P * 4u);
  wpb = wpb < 1 ? 1 : (wpb > 8 ? 8 : wpb);
  const size_t smem = static_cast<size_t>(wpb) * P * 4;
  const uint64_t blocks = (count + wpb - 1) / wpb;
  if (blocks > 0x7fffffffull) return cudaErrorInvalidValue;
  auto launch = [&](auto kern) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    kern<<<static_cast<unsigned>(blocks), wpb * 32, smem, stream>>>(rows, count, dim, P, signs,
                                                                    rounds, codes, scales, R, wpb);
    return cudaGetLastError();
  };
  if (bits == 8) return launch(encode_kernel<8>);
  if (bits == 4) return launch(encode_kernel<4>);
  return launch(encode_kernel<1>);
}

}  // namespace bv
