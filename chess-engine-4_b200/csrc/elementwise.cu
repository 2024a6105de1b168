// Memory-bound kernels around the GEMMs: input-plane expansion (three input layouts),
// standalone RMSNorm / SwiGLU / residual add for the kernel-op API.
#include <algorithm>
#include "internal.h"
#include "mxfp8.cuh"
#include "ptx.cuh"

namespace ce4b {

namespace {

// Source plane of selected plane `p` under history selection
// (src/chess_engine_4/model/dense.py:45-51; kernels/src/inference/runtime.cu:197-200).
__device__ __forceinline__ int source_plane(int p, int history_planes) {
  return p < history_planes ? p : kHistoryPlanes + (p - history_planes);
}

// Blocks take positions; a thread writes 8 squares (one 16-byte BF16 chunk) of one selected
// plane, for up to kExpandPer chunks of the position, blockDim apart (consecutive threads
// write consecutive chunks). All of a thread's record loads are issued before its stores,
// so that each thread keeps several independent loads in flight (32-bit in-position
// indexing).
constexpr int kExpandPer = 4;

__global__ void expand_lc0_kernel(const ce4b_input_plane* __restrict__ planes, bf16* __restrict__ out,
                                  int batch, int history) {
  static_assert(sizeof(ce4b_input_plane) == 16, "InputPlane is 16 bytes");
  // The forward kernel after it may start its prologue now; it waits for this grid's
  // completion before reading the planes.
  grid_launch_dependents();
  const int sel = selected_planes(history);
  const int hp = history * kPlanesPerHistory;
  const int nchunk = sel * 8;
  for (int64_t b = blockIdx.x; b < batch; b += gridDim.x) {
    const uint4* rec = reinterpret_cast<const uint4*>(planes + b * kInputPlanes);
    uint4* dst = reinterpret_cast<uint4*>(out) + b * nchunk;
    for (int c0 = 0; c0 < nchunk; c0 += kExpandPer * blockDim.x) {
      uint4 pl[kExpandPer];
#pragma unroll
      for (int u = 0; u < kExpandPer; ++u) {
        const int c = c0 + u * blockDim.x + threadIdx.x;
        if (c < nchunk) pl[u] = __ldg(rec + source_plane(c >> 3, hp));
      }
#pragma unroll
      for (int u = 0; u < kExpandPer; ++u) {
        const int c = c0 + u * blockDim.x + threadIdx.x;
        if (c >= nchunk) continue;
        const int chunk = c & 7;
        const int p = c >> 3;
        const uint64_t mask = static_cast<uint64_t>(pl[u].x) | (static_cast<uint64_t>(pl[u].y) << 32);
        float v = __uint_as_float(pl[u].z);
        if (p == hp + 5) v = v / 99.0f;
        const uint32_t bits = static_cast<uint32_t>(mask >> (chunk * 8)) & 0xFFu;
        float f[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = ((bits >> j) & 1u) ? v : 0.0f;
        uint4 o;
        o.x = pack_bf16x2(f[0], f[1]);
        o.y = pack_bf16x2(f[2], f[3]);
        o.z = pack_bf16x2(f[4], f[5]);
        o.w = pack_bf16x2(f[6], f[7]);
        dst[c] = o;
      }
    }
  }
}

// Dense planes [B, 112, 64] (f32 or bf16) -> BF16 [B, sel*64]; rule-50 plane / 99.
template <typename T>
__global__ void expand_dense_kernel(T* __restrict__ planes, bf16* __restrict__ out, int batch,
                                    int history, int write_back) {
  grid_launch_dependents();
  const int sel = selected_planes(history);
  const int hp = history * kPlanesPerHistory;
  for (int64_t b = blockIdx.x; b < batch; b += gridDim.x)
  for (int c = threadIdx.x; c < sel * 8; c += blockDim.x) {
    const int chunk = c & 7;
    const int p = c >> 3;
    const int64_t i = b * sel * 8 + c;
    const int src = source_plane(p, hp);
    T* in = planes + (b * kInputPlanes + src) * 64 + chunk * 8;
    float f[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if constexpr (sizeof(T) == 4) {
        f[j] = in[j];
      } else {
        f[j] = __bfloat162float(in[j]);
      }
    }
    if (p == hp + 5) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if constexpr (sizeof(T) == 4) {
          f[j] = f[j] / 99.0f;
          if (write_back) in[j] = f[j];
        } else {
          // BF16 input: the in-place division happens in BF16, as div_ on a BF16 tensor.
          const T q = __float2bfloat16(f[j] / 99.0f);
          f[j] = __bfloat162float(q);
          if (write_back) in[j] = q;
        }
      }
    }
    uint4 o;
    o.x = pack_bf16x2(f[0], f[1]);
    o.y = pack_bf16x2(f[2], f[3]);
    o.z = pack_bf16x2(f[4], f[5]);
    o.w = pack_bf16x2(f[6], f[7]);
    reinterpret_cast<uint4*>(out)[i] = o;
  }
}

// Packed training layout: u8 [B, 104, 8] (bit j of byte r, MSB first, is square r*8+j)
// plus [B, 8] aux-plane scalars (src/chess_engine_4/training/packed_input.py:24-47).
template <typename S>
__global__ void expand_packed_kernel(const uint8_t* __restrict__ packed, const S* __restrict__ scalars,
                                     bf16* __restrict__ out, int batch, int history) {
  grid_launch_dependents();
  const int sel = selected_planes(history);
  const int hp = history * kPlanesPerHistory;
  for (int64_t b = blockIdx.x; b < batch; b += gridDim.x)
  for (int c = threadIdx.x; c < sel * 8; c += blockDim.x) {
    const int chunk = c & 7;
    const int p = c >> 3;
    const int64_t i = b * sel * 8 + c;
    const int src = source_plane(p, hp);
    float f[8];
    if (src < kHistoryPlanes) {
      const uint32_t byte = packed[(b * kHistoryPlanes + src) * 8 + chunk];
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = ((byte >> (7 - j)) & 1u) ? 1.0f : 0.0f;
    } else {
      float v;
      if constexpr (sizeof(S) == 4) {
        v = scalars[b * 8 + (src - kHistoryPlanes)];
      } else {
        v = __bfloat162float(scalars[b * 8 + (src - kHistoryPlanes)]);
      }
      if (p == hp + 5) {
        if constexpr (sizeof(S) == 4) {
          v = v / 99.0f;
        } else {
          v = bf16_round(v / 99.0f);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = v;
    }
    uint4 o;
    o.x = pack_bf16x2(f[0], f[1]);
    o.y = pack_bf16x2(f[2], f[3]);
    o.z = pack_bf16x2(f[4], f[5]);
    o.w = pack_bf16x2(f[6], f[7]);
    reinterpret_cast<uint4*>(out)[i] = o;
  }
}

// MXFP8 operand of the input projection straight from any input layout: one thread = one
// 32-square half of one selected plane of one position (= one MX scale block). The values
// are formed exactly as in the BF16 path (rule-50 / 99, BF16 rounding), then quantised.
__global__ void expand_mx_kernel(int layout, const void* __restrict__ input,
                                 const void* __restrict__ scalars, uint8_t* __restrict__ codes,
                                 uint8_t* __restrict__ scales, int batch, int history,
                                 int write_back) {
  const int sel = selected_planes(history);
  const int hp = history * kPlanesPerHistory;
  const int in_dim = sel * 64;
  const int64_t blocks = static_cast<int64_t>(batch) * sel * 2;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < blocks;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int half = static_cast<int>(i % 2);
    const int p = static_cast<int>((i / 2) % sel);
    const int64_t b = i / (2 * sel);
    const int src = source_plane(p, hp);
    const bool rule50 = p == hp + 5;
    float f[32];
    if (layout == CE4B_INPUT_LC0) {
      const ce4b_input_plane pl = static_cast<const ce4b_input_plane*>(input)[b * kInputPlanes + src];
      const float v = rule50 ? pl.value / 99.0f : pl.value;
      const uint32_t bits = static_cast<uint32_t>(pl.mask >> (32 * half));
#pragma unroll
      for (int j = 0; j < 32; ++j) f[j] = ((bits >> j) & 1u) ? v : 0.0f;
    } else if (layout == CE4B_INPUT_F32_PLANES) {
      float* in = static_cast<float*>(const_cast<void*>(input)) + (b * kInputPlanes + src) * 64 + half * 32;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        f[j] = rule50 ? in[j] / 99.0f : in[j];
        if (rule50 && write_back) in[j] = f[j];
      }
    } else if (layout == CE4B_INPUT_BF16_PLANES) {
      bf16* in = static_cast<bf16*>(const_cast<void*>(input)) + (b * kInputPlanes + src) * 64 + half * 32;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        f[j] = __bfloat162float(in[j]);
        if (rule50) {
          const bf16 q = __float2bfloat16(f[j] / 99.0f);
          f[j] = __bfloat162float(q);
          if (write_back) in[j] = q;
        }
      }
    } else {
      if (src < kHistoryPlanes) {
        const uint8_t* bytes = static_cast<const uint8_t*>(input) + (b * kHistoryPlanes + src) * 8 + half * 4;
#pragma unroll
        for (int jb = 0; jb < 4; ++jb) {
          const uint32_t byte = bytes[jb];
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) f[jb * 8 + jj] = ((byte >> (7 - jj)) & 1u) ? 1.0f : 0.0f;
        }
      } else {
        float v;
        if (layout == CE4B_INPUT_PACKED_F32) {
          v = static_cast<const float*>(scalars)[b * 8 + (src - kHistoryPlanes)];
          if (rule50) v = v / 99.0f;
        } else {
          v = __bfloat162float(static_cast<const bf16*>(scalars)[b * 8 + (src - kHistoryPlanes)]);
          if (rule50) v = bf16_round(v / 99.0f);
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) f[j] = v;
      }
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) f[j] = bf16_round(f[j]);
    uint32_t q[8];
    const uint8_t sc = mx_quantize32(f, q);
    uint4* dst = reinterpret_cast<uint4*>(codes + b * in_dim + p * 64 + half * 32);
    dst[0] = make_uint4(q[0], q[1], q[2], q[3]);
    dst[1] = make_uint4(q[4], q[5], q[6], q[7]);
    scales[mx_scale_offset(static_cast<int>(b), p * 2 + half, in_dim / 128)] = sc;
  }
}

// One warp per row.
__global__ void rmsnorm_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w,
                               bf16* __restrict__ out, int rows, int width, float eps) {
  const int warps = blockDim.x / 32;
  const int row = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const bf16* xr = x + static_cast<int64_t>(row) * width;
  float ss = 0.0f;
  for (int c = lane; c < width; c += 32) {
    const float v = __bfloat162float(xr[c]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(width) + eps);
  bf16* orow = out + static_cast<int64_t>(row) * width;
  for (int c = lane; c < width; c += 32) {
    orow[c] = __float2bfloat16((__bfloat162float(xr[c]) * inv) * __bfloat162float(w[c]));
  }
}

__global__ void swiglu_kernel(const bf16* __restrict__ gate_up, bf16* __restrict__ hidden, int rows,
                              int hidden_dim) {
  const int64_t n = static_cast<int64_t>(rows) * hidden_dim;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / hidden_dim;
    const int64_t c = i - r * hidden_dim;
    const float g = __bfloat162float(gate_up[r * 2 * hidden_dim + c]);
    const float u = __bfloat162float(gate_up[r * 2 * hidden_dim + hidden_dim + c]);
    hidden[i] = __float2bfloat16(g / (1.0f + expf(-g)) * u);
  }
}

__global__ void residual_add_kernel(bf16* __restrict__ out, const bf16* __restrict__ residual,
                                    int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    out[i] = __float2bfloat16(__bfloat162float(out[i]) + __bfloat162float(residual[i]));
  }
}

int grid_for(int64_t work, int threads) {
  const int64_t blocks = (work + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  return static_cast<int>(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

}  // namespace

void expand_input(int layout, const void* input, const void* scalars, int batch, int history,
                  bf16* out, int write_back_rule50, cudaStream_t s) {
  const int threads = 256;
  const int grid = std::max(1, std::min(batch, sm_count() * 16));
  switch (layout) {
    case CE4B_INPUT_LC0:
      expand_lc0_kernel<<<std::max(1, std::min(batch, sm_count() * 8)), threads, 0, s>>>(
          static_cast<const ce4b_input_plane*>(input), out, batch, history);
      break;
    case CE4B_INPUT_F32_PLANES:
      expand_dense_kernel<float><<<grid, threads, 0, s>>>(
          static_cast<float*>(const_cast<void*>(input)), out, batch, history, write_back_rule50);
      break;
    case CE4B_INPUT_BF16_PLANES:
      expand_dense_kernel<bf16><<<grid, threads, 0, s>>>(
          static_cast<bf16*>(const_cast<void*>(input)), out, batch, history, write_back_rule50);
      break;
    case CE4B_INPUT_PACKED_F32:
      require(scalars != nullptr, "packed input needs scalars");
      expand_packed_kernel<float><<<grid, threads, 0, s>>>(
          static_cast<const uint8_t*>(input), static_cast<const float*>(scalars), out, batch,
          history);
      break;
    case CE4B_INPUT_PACKED_BF16:
      require(scalars != nullptr, "packed input needs scalars");
      expand_packed_kernel<bf16><<<grid, threads, 0, s>>>(static_cast<const uint8_t*>(input),
                                                          static_cast<const bf16*>(scalars), out,
                                                          batch, history);
      break;
    default:
      fail(CE4B_ERR_INVALID_ARGUMENT, "unknown input layout " + std::to_string(layout));
  }
  check_cuda(cudaGetLastError(), "expand_input launch");
}

void expand_input_mx(int layout, const void* input, const void* scalars, int batch, int history,
                     uint8_t* codes, uint8_t* scales, int write_back_rule50, cudaStream_t s) {
  require(layout >= CE4B_INPUT_F32_PLANES && layout <= CE4B_INPUT_PACKED_BF16,
          "unknown input layout " + std::to_string(layout));
  require((layout != CE4B_INPUT_PACKED_F32 && layout != CE4B_INPUT_PACKED_BF16) || scalars != nullptr,
          "packed input needs scalars");
  require(selected_planes(history) % 2 == 0, "MXFP8 input needs an even number of planes");
  const int64_t blocks = static_cast<int64_t>(batch) * selected_planes(history) * 2;
  const int threads = 256;
  expand_mx_kernel<<<grid_for(blocks, threads), threads, 0, s>>>(
      layout, input, scalars, codes, scales, batch, history, write_back_rule50);
  check_cuda(cudaGetLastError(), "expand_input_mx launch");
}

void rmsnorm_rows(const bf16* x, const bf16* w, bf16* out, int rows, int width, float eps,
                  cudaStream_t s) {
  const int warps = 8;
  rmsnorm_kernel<<<(rows + warps - 1) / warps, warps * 32, 0, s>>>(x, w, out, rows, width, eps);
  check_cuda(cudaGetLastError(), "rmsnorm launch");
}

void swiglu_rows(const bf16* gate_up, bf16* hidden, int rows, int hidden_dim, cudaStream_t s) {
  const int64_t n = static_cast<int64_t>(rows) * hidden_dim;
  swiglu_kernel<<<grid_for(n, 256), 256, 0, s>>>(gate_up, hidden, rows, hidden_dim);
  check_cuda(cudaGetLastError(), "swiglu launch");
}

void residual_add(bf16* out, const bf16* residual, int64_t elements, cudaStream_t s) {
  residual_add_kernel<<<grid_for(elements, 256), 256, 0, s>>>(out, residual, elements);
  check_cuda(cudaGetLastError(), "residual_add launch");
}

// ------------------------------------------------------------------ weight folding
// out[r, c] = bf16(W[r, c] * w[c]): an RMSNorm weight folded into the following linear
// (the product of two BF16 values is exact in FP32, so this rounds once).
__global__ void fold_columns_kernel(const bf16* __restrict__ W, const bf16* __restrict__ w,
                                    bf16* __restrict__ out, int64_t n, int cols) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % cols);
    out[i] = __float2bfloat16_rn(__bfloat162float(W[i]) * __bfloat162float(w[c]));
  }
}

void fold_columns(const bf16* W, const bf16* w, bf16* out, int64_t rows, int cols, cudaStream_t s) {
  const int64_t n = rows * cols;
  fold_columns_kernel<<<grid_for(n, 256), 256, 0, s>>>(W, w, out, n, cols);
  check_cuda(cudaGetLastError(), "fold_columns launch");
}

}  // namespace ce4b
