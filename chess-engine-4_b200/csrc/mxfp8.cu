// Standalone MXFP8 quantiser (kernel-op API quantize_mxfp8).
#include <algorithm>

#include "gemm.cuh"
#include "internal.h"
#include "mxfp8.cuh"

namespace ce4b {

namespace {

// One thread per (row, 32-column block): 64 bytes in, 32 code bytes + 1 scale byte out.
__global__ void mx_quantize_kernel(const bf16* __restrict__ x, uint8_t* __restrict__ codes,
                                   uint8_t* __restrict__ scales, int rows, int cols) {
  const int blocks_per_row = cols / 32;
  const int64_t total = static_cast<int64_t>(rows) * blocks_per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i / blocks_per_row);
    const int blk = static_cast<int>(i - static_cast<int64_t>(row) * blocks_per_row);
    float v[32];
    load_bf16<32>(x + static_cast<size_t>(row) * cols + blk * 32, v);
    uint32_t q[8];
    const uint8_t sc = mx_quantize32(v, q);
    uint4* dst = reinterpret_cast<uint4*>(codes + static_cast<size_t>(row) * cols + blk * 32);
    dst[0] = make_uint4(q[0], q[1], q[2], q[3]);
    dst[1] = make_uint4(q[4], q[5], q[6], q[7]);
    scales[mx_scale_offset(row, blk, cols / 128)] = sc;
  }
}

// Quantisation of the transpose: codes [cols, rows], scale blocks of 32 input rows. A CTA
// stages 32 input rows x 256 input columns in shared memory (coalesced 16-byte loads), then
// each thread quantises one input column (an output row segment of 32) and stores its 32
// codes and one scale.
__global__ void mx_quantize_transpose_kernel(const bf16* __restrict__ x, uint8_t* __restrict__ codes,
                                             uint8_t* __restrict__ scales, int rows, int cols) {
  __shared__ __align__(16) bf16 tile[32][256];
  const int r0 = static_cast<int>(blockIdx.y) * 32, c0 = static_cast<int>(blockIdx.x) * 256;
  for (int i = static_cast<int>(threadIdx.x); i < 32 * 32; i += static_cast<int>(blockDim.x)) {
    const int r = i / 32, ch = i % 32, c = c0 + ch * 8;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (c < cols) v = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(r0 + r) * cols + c);
    *reinterpret_cast<uint4*>(&tile[r][ch * 8]) = v;
  }
  __syncthreads();
  const int c = c0 + static_cast<int>(threadIdx.x);
  if (c >= cols) return;
  float v[32];
#pragma unroll
  for (int r = 0; r < 32; ++r) v[r] = __bfloat162float(tile[r][threadIdx.x]);
  uint32_t q[8];
  const uint8_t sc = mx_quantize32(v, q);
  uint4* dst = reinterpret_cast<uint4*>(codes + static_cast<size_t>(c) * rows + r0);
  dst[0] = make_uint4(q[0], q[1], q[2], q[3]);
  dst[1] = make_uint4(q[4], q[5], q[6], q[7]);
  scales[mx_scale_offset(c, r0 / 32, rows / 128)] = sc;
}

}  // namespace

void mx_quantize_transpose(const bf16* x, uint8_t* codes, uint8_t* scales, int rows, int cols,
                           cudaStream_t s) {
  require(rows % 128 == 0 && cols % 128 == 0, "MXFP8 tensors need dimensions divisible by 128");
  const dim3 grid(static_cast<unsigned>((cols + 255) / 256), static_cast<unsigned>(rows / 32));
  mx_quantize_transpose_kernel<<<grid, 256, 0, s>>>(x, codes, scales, rows, cols);
  check_cuda(cudaGetLastError(), "mx_quantize_transpose launch");
}

void mx_quantize(const bf16* x, uint8_t* codes, uint8_t* scales, int rows, int cols,
                 cudaStream_t s) {
  require(rows % 128 == 0 && cols % 128 == 0, "MXFP8 tensors need dimensions divisible by 128");
  const int64_t work = static_cast<int64_t>(rows) * (cols / 32);
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((work + threads - 1) / threads, sm_count() * 16);
  mx_quantize_kernel<<<static_cast<int>(blocks), threads, 0, s>>>(x, codes, scales, rows, cols);
  check_cuda(cudaGetLastError(), "mx_quantize launch");
}

}  // namespace ce4b
