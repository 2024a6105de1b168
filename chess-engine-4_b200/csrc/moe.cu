// MoE routing plumbing around the grouped tcgen05 GEMMs: deterministic scan of the
// router's per-tile expert histograms, stable-by-token dispatch (permutation) of token
// rows into 128-row-aligned expert segments, combine of the two expert outputs with the
// residual and the next layer's RMSNorm, plus the standalone routing and offset helpers
// of the kernel-op API.
//
// Placement: route r = 2*token + k (k = 0 best, 1 second expert). Within expert e, routes
// are ordered by r, as the reference's stable argsort places them
// (src/chess_engine_4/model/moe.py:36-47); expert segments start on 128-row boundaries
// (the reference's static path aligns to 128 rows, moe.py:239-251).
#include "gemm.cuh"
#include "internal.h"

namespace ce4b {

namespace {

constexpr int kExperts = 64;

// One CTA of 1024 threads. The per-tile histograms are staged in shared memory 64 tiles at
// a time by all threads (coalesced), thread e < 64 runs expert e's prefix over them there,
// and the offsets go back to global memory coalesced; the tile table follows.
constexpr int kScanThreads = 1024;
constexpr int kScanChunk = 64;  // tiles per staged chunk (16 KB)

__global__ void __launch_bounds__(kScanThreads)
    moe_scan_kernel(const int* __restrict__ block_hist, int ntiles, int* __restrict__ expert_start,
                    int* __restrict__ block_off, int4* __restrict__ m_tiles,
                    int* __restrict__ num_m_tiles, int* __restrict__ counts_out) {
  __shared__ int hist[kScanChunk * kExperts];
  __shared__ int padded[kExperts];
  __shared__ int tiles[kExperts];
  const int tid = threadIdx.x;
  const int e = tid;  // expert of the scanning threads (tid < 64)
  int run = 0;
  for (int b0 = 0; b0 < ntiles; b0 += kScanChunk) {
    const int n = min(kScanChunk, ntiles - b0) * kExperts;
    for (int i = tid; i < n; i += kScanThreads) hist[i] = block_hist[b0 * kExperts + i];
    __syncthreads();
    if (tid < kExperts) {
      for (int b = 0; b < n / kExperts; ++b) {
        const int c = hist[b * kExperts + e];
        hist[b * kExperts + e] = run;
        run += c;
      }
    }
    __syncthreads();
    for (int i = tid; i < n; i += kScanThreads) block_off[b0 * kExperts + i] = hist[i];
    __syncthreads();
  }
  const int nt = (run + kBM - 1) / kBM;
  if (tid < kExperts) {
    padded[e] = nt * kBM;
    tiles[e] = nt;
  }
  __syncthreads();
  if (tid >= kExperts) return;
  int start = 0, tstart = 0;
  for (int j = 0; j < e; ++j) {
    start += padded[j];
    tstart += tiles[j];
  }
  expert_start[e] = start;
  for (int i = 0; i < nt; ++i) {
    m_tiles[tstart + i] = make_int4(e, start + kBM * i, min(kBM, run - kBM * i), 0);
  }
  if (counts_out != nullptr) counts_out[e] = run;
  if (e == kExperts - 1) {
    *num_m_tiles = tstart + nt;
    expert_start[kExperts] = start + nt * kBM;
  }
}

// kDispatchParts CTAs per router tile (128 tokens = 256 routes), 256 threads (one per
// route). Every CTA of a tile computes the tile's 256 destinations (cheap); the first
// writes the route positions and probabilities, and each copies a quarter of the rows.
// A copy is a flat list of (row, 16-byte chunk) items, consecutive threads on
// consecutive chunks of a row, each thread issuing kDispatchBatch loads before their
// stores so that enough bytes are in flight.
constexpr int kDispatchParts = 4;
constexpr int kDispatchBatch = 8;

__global__ void __launch_bounds__(256)
    moe_dispatch_kernel(const bf16* __restrict__ n, const int2* __restrict__ route_expert,
                        const float2* __restrict__ route_prob, const int* __restrict__ expert_start,
                        const int* __restrict__ block_off, bf16* __restrict__ xperm,
                        float* __restrict__ pprob, int* __restrict__ route_pos, int tokens, int d) {
  __shared__ int warp_cnt[8][kExperts];
  __shared__ int pos_s[256];
  const int b = blockIdx.x / kDispatchParts;
  const int part = blockIdx.x - b * kDispatchParts;
  const int i = threadIdx.x;
  const int warp = i >> 5;
  const int lane = i & 31;
  for (int j = i; j < 8 * kExperts; j += 256) (&warp_cnt[0][0])[j] = 0;
  __syncthreads();
  const int token = b * kBM + (i >> 1);
  const int k = i & 1;
  const bool valid = token < tokens;
  int e = kExperts;  // sentinel: not a route
  float prob = 0.0f;
  if (valid) {
    const int2 ex = route_expert[token];
    const float2 pr = route_prob[token];
    e = k ? ex.y : ex.x;
    prob = k ? pr.y : pr.x;
  }
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(peers & ((1u << lane) - 1u));
  if (valid && rank == 0) warp_cnt[warp][e] = __popc(peers);
  __syncthreads();
  int pos = -1;
  if (valid) {
    int prefix = 0;
    for (int w = 0; w < warp; ++w) prefix += warp_cnt[w][e];
    pos = expert_start[e] + block_off[b * kExperts + e] + prefix + rank;
    if (part == 0) {
      pprob[pos] = prob;
      route_pos[2 * token + k] = pos;
    }
  }
  pos_s[i] = pos;
  __syncthreads();
  const int chunks = d / 8;  // 16-byte chunks per row
  constexpr int kRows = 256 / kDispatchParts;
  const int r0 = part * kRows;
  const int items = kRows * chunks;
  for (int base = 0; base < items; base += 256 * kDispatchBatch) {
    uint4 v[kDispatchBatch];
    int dst_off[kDispatchBatch];
#pragma unroll
    for (int u = 0; u < kDispatchBatch; ++u) {
      const int it = base + u * 256 + i;
      dst_off[u] = -1;
      if (it < items) {
        const int r = r0 + it / chunks;
        const int c = it - (it / chunks) * chunks;
        const int p = pos_s[r];
        if (p >= 0) {
          const int t = b * kBM + (r >> 1);
          v[u] = reinterpret_cast<const uint4*>(n + static_cast<size_t>(t) * d)[c];
          dst_off[u] = p * chunks + c;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kDispatchBatch; ++u) {
      if (dst_off[u] >= 0) reinterpret_cast<uint4*>(xperm)[dst_off[u]] = v[u];
    }
  }
}

// One warp per token: x = bf16(x + bf16(y0 + y1)); n = bf16((x * rsqrt(mean(x^2)+eps)) * w).
// A lane holds up to kMaxC 16-byte chunks of the row (d <= 256 * kMaxC); all of its loads
// (x, the norm weight, then both expert outputs) are issued before the arithmetic.
template <int kMaxC>
__global__ void moe_combine_norm_kernel(bf16* __restrict__ x, const bf16* __restrict__ y,
                                        const int2* __restrict__ route_pos,
                                        const bf16* __restrict__ w, bf16* __restrict__ nout,
                                        int tokens, int d, float eps) {
  const int t = static_cast<int>((blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= tokens) return;
  const int chunks = d / 8;
  bf16* xr = x + static_cast<size_t>(t) * d;
  uint4 xa[kMaxC], wa[kMaxC], ya[kMaxC], yb[kMaxC];
#pragma unroll
  for (int j = 0; j < kMaxC; ++j) {
    const int c = lane + 32 * j;
    if (c < chunks) {
      xa[j] = reinterpret_cast<const uint4*>(xr)[c];
      wa[j] = __ldg(reinterpret_cast<const uint4*>(w) + c);
    }
  }
  const int2 rp = route_pos[t];
  const uint4* y0 = reinterpret_cast<const uint4*>(y + static_cast<size_t>(rp.x) * d);
  const uint4* y1 = reinterpret_cast<const uint4*>(y + static_cast<size_t>(rp.y) * d);
#pragma unroll
  for (int j = 0; j < kMaxC; ++j) {
    const int c = lane + 32 * j;
    if (c < chunks) {
      ya[j] = y0[c];
      yb[j] = y1[c];
    }
  }
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < kMaxC; ++j) {
    const int c = lane + 32 * j;
    if (c < chunks) {
      const uint32_t xw[4] = {xa[j].x, xa[j].y, xa[j].z, xa[j].w};
      const uint32_t aw[4] = {ya[j].x, ya[j].y, ya[j].z, ya[j].w};
      const uint32_t bw[4] = {yb[j].x, yb[j].y, yb[j].z, yb[j].w};
      uint32_t ow[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 xf = unpack_bf16x2(xw[q]), af = unpack_bf16x2(aw[q]), bf = unpack_bf16x2(bw[q]);
        const float r0 = bf16_round(af.x + bf.x);
        const float r1 = bf16_round(af.y + bf.y);
        const float v0 = bf16_round(xf.x + r0);
        const float v1 = bf16_round(xf.y + r1);
        ss = fmaf(v0, v0, ss);
        ss = fmaf(v1, v1, ss);
        ow[q] = pack_bf16x2(v0, v1);
      }
      xa[j] = make_uint4(ow[0], ow[1], ow[2], ow[3]);  // the new x (BF16)
      reinterpret_cast<uint4*>(xr)[c] = xa[j];
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(d) + eps);
  uint4* nr = reinterpret_cast<uint4*>(nout + static_cast<size_t>(t) * d);
#pragma unroll
  for (int j = 0; j < kMaxC; ++j) {
    const int c = lane + 32 * j;
    if (c < chunks) {
      const uint32_t vw[4] = {xa[j].x, xa[j].y, xa[j].z, xa[j].w};
      const uint32_t ww[4] = {wa[j].x, wa[j].y, wa[j].z, wa[j].w};
      uint32_t ow[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 vf = unpack_bf16x2(vw[q]), wf = unpack_bf16x2(ww[q]);
        ow[q] = pack_bf16x2((vf.x * inv) * wf.x, (vf.y * inv) * wf.y);
      }
      nr[c] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
  }
}

// Grouped-GEMM tile table from caller-provided expert offsets [65] (kernel-op API). The
// segments must start on 128-row boundaries; a misaligned offset is reported through the
// device error word and that expert is skipped.
__global__ void moe_tiles_from_offsets_kernel(const int* __restrict__ offsets, int4* __restrict__ m_tiles,
                                              int* __restrict__ num_m_tiles, int* err) {
  __shared__ int tiles[kExperts];
  const int e = threadIdx.x;
  const int lo = offsets[e];
  const int hi = offsets[e + 1];
  const bool ok = lo % kBM == 0 && hi >= lo;
  if (!ok) record_error(err, kErrBadShape);
  const int cnt = ok ? hi - lo : 0;
  const int nt = (cnt + kBM - 1) / kBM;
  tiles[e] = nt;
  __syncthreads();
  int tstart = 0;
  for (int j = 0; j < e; ++j) tstart += tiles[j];
  for (int i = 0; i < nt; ++i) m_tiles[tstart + i] = make_int4(e, lo + kBM * i, min(kBM, cnt - kBM * i), 0);
  if (e == kExperts - 1) *num_m_tiles = tstart + nt;
}

// Routing from given BF16 logits [T, 64] (kernel-op API): one thread per token.
__global__ void moe_route_kernel(const bf16* __restrict__ logits, const float* __restrict__ beta,
                                 int2* __restrict__ experts, float2* __restrict__ probs,
                                 int* __restrict__ counts, int tokens) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= tokens) return;
  float lo[32], hi[32];
  load_bf16<32>(logits + static_cast<size_t>(t) * 64, lo);
  load_bf16<32>(logits + static_cast<size_t>(t) * 64 + 32, hi);
  int e0, e1;
  float p0, p1;
  route_top2(lo, hi, beta, e0, e1, p0, p1);
  experts[t] = make_int2(e0, e1);
  probs[t] = make_float2(p0, p1);
  if (counts != nullptr) {
    atomicAdd(counts + e0, 1);
    atomicAdd(counts + e1, 1);
  }
}

__global__ void bf16_to_f32_kernel(const bf16* __restrict__ in, float* __restrict__ out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = __bfloat162float(in[i]);
}

}  // namespace

void moe_scan(const int* block_hist, int ntiles, int* expert_start, int* block_off,
              int4* m_tiles, int* num_m_tiles, int* counts_out, cudaStream_t s) {
  moe_scan_kernel<<<1, kScanThreads, 0, s>>>(block_hist, ntiles, expert_start, block_off, m_tiles,
                                             num_m_tiles, counts_out);
  check_cuda(cudaGetLastError(), "moe_scan launch");
}

void moe_dispatch(const bf16* n, const int2* route_expert, const float2* route_prob,
                  const int* expert_start, const int* block_off, bf16* xperm, float* pprob,
                  int* route_pos, int tokens, int d, cudaStream_t s) {
  require(d % 8 == 0, "MoE width must be a multiple of 8");
  const int tiles = (tokens + kBM - 1) / kBM;
  moe_dispatch_kernel<<<tiles * kDispatchParts, 256, 0, s>>>(n, route_expert, route_prob, expert_start,
                                                             block_off, xperm, pprob, route_pos, tokens, d);
  check_cuda(cudaGetLastError(), "moe_dispatch launch");
}

void moe_combine_norm(bf16* x, const bf16* yperm, const int* route_pos, const bf16* norm_w,
                      bf16* nout, int tokens, int d, float eps, cudaStream_t s) {
  require(d % 8 == 0 && d <= 2048, "MoE width must be a multiple of 8 and at most 2048");
  const int warps_per_block = 8;
  const int blocks = (tokens + warps_per_block - 1) / warps_per_block;
  const int2* rp = reinterpret_cast<const int2*>(route_pos);
  if (d <= 1024) {
    moe_combine_norm_kernel<4><<<blocks, warps_per_block * 32, 0, s>>>(x, yperm, rp, norm_w, nout, tokens,
                                                                      d, eps);
  } else {
    moe_combine_norm_kernel<8><<<blocks, warps_per_block * 32, 0, s>>>(x, yperm, rp, norm_w, nout, tokens,
                                                                      d, eps);
  }
  check_cuda(cudaGetLastError(), "moe_combine launch");
}

void moe_tiles_from_offsets(const int* offsets, int4* m_tiles, int* num_m_tiles, cudaStream_t s) {
  moe_tiles_from_offsets_kernel<<<1, kExperts, 0, s>>>(offsets, m_tiles, num_m_tiles,
                                                       device_error_word());
  check_cuda(cudaGetLastError(), "moe_tiles launch");
}

void moe_route_logits(const bf16* logits, const float* beta, int2* experts, float2* probs,
                      int* counts, int tokens, cudaStream_t s) {
  moe_route_kernel<<<(tokens + 127) / 128, 128, 0, s>>>(logits, beta, experts, probs, counts,
                                                        tokens);
  check_cuda(cudaGetLastError(), "moe_route launch");
}

void bf16_to_f32(const bf16* in, float* out, int n, cudaStream_t s) {
  bf16_to_f32_kernel<<<(n + 255) / 256, 256, 0, s>>>(in, out, n);
  check_cuda(cudaGetLastError(), "bf16_to_f32 launch");
}

}  // namespace ce4b
