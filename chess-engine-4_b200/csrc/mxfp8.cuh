// MXFP8 (E4M3 values, E8M0 per-32-element scales) quantisation helpers shared by the
// standalone quantiser and the fused GEMM epilogues.
//
// Recipe of the reference's custom MXFP8 path (ThunderKittens mxfp8_quantize,
// third_party/ThunderKittens/kernels/gemm/mxfp8_b200/mxfp8_b200_gemm.cu:380-426):
//   s = max(amax * 0.002232142857f, 1e-12f); S = E8M0(s) rounded toward +inf, satfinite;
//   q = E4M3(x * (1 / 2^(S - 127))) round-to-nearest-even, satfinite.
// Scale bytes of a 128x128 tile sit at (r % 32) * 16 + (r / 32) * 4 + kb (tile row r,
// 32-column block kb), the layout tcgen05 block-scaled MMAs read after a 32x128b.warpx4
// copy into tensor memory.
#pragma once

#include <cuda_fp8.h>

#include "ptx.cuh"

namespace ce4b {

__device__ __forceinline__ uint8_t mx_scale_code(float amax) {
  const float s = fmaxf(amax * 0.002232142857f, 1e-12f);
  return static_cast<uint8_t>(__nv_cvt_float_to_e8m0(s, __NV_SATFINITE, cudaRoundPosInf));
}

// 1 / 2^(S - 127) = 2^(127 - S), exact.
__device__ __forceinline__ float mx_scale_inverse(uint8_t code) {
  const uint32_t biased = 254u - code;  // biased FP32 exponent of 2^(127 - S)
  return biased >= 1u ? __uint_as_float(biased << 23) : __uint_as_float(0x00400000u);
}

// Quantise 32 values (one scale block) to packed E4M3 codes; returns the scale code.
__device__ __forceinline__ uint8_t mx_quantize32(const float (&v)[32], uint32_t (&codes)[8]) {
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
  const uint8_t sc = mx_scale_code(amax);
  const float inv = mx_scale_inverse(sc);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(v[4 * j] * inv, v[4 * j + 1] * inv),
                                                 __NV_SATFINITE, __NV_E4M3);
    const uint32_t hi = __nv_cvt_float2_to_fp8x2(
        make_float2(v[4 * j + 2] * inv, v[4 * j + 3] * inv), __NV_SATFINITE, __NV_E4M3);
    codes[j] = lo | (hi << 16);
  }
  return sc;
}

// Byte offset of the scale of (row, 32-column block) in the [rows/128][cols/128][512] layout.
__host__ __device__ __forceinline__ size_t mx_scale_offset(int row, int block, int col_tiles) {
  const int tile = (row / 128) * col_tiles + block / 4;
  const int tr = row % 128;
  return static_cast<size_t>(tile) * 512 + (tr % 32) * 16 + (tr / 32) * 4 + (block % 4);
}

}  // namespace ce4b
