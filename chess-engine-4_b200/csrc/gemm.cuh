// Warp-specialised tcgen05 GEMM for sm_100a with fused epilogues.
//
//   C[M, N] = A[M, K] . B[N, K]^T      A, B: BF16, K-major (row-major with K contiguous)
//
// One CTA = 6 warps: warp 0 issues TMA tile loads into an NSTAGE ring of shared-memory
// stages, warp 1 issues tcgen05.mma (M=128, N=BN, K=16) into a TMEM accumulator
// (NACC buffers so the epilogue of one tile overlaps the main loop of the next), warps 2-5
// drain the accumulator with tcgen05.ld (warp w owns TMEM lanes 32*(w%4) .. +31, i.e. one
// output row per thread) and run the epilogue functor. Tiles are 128 x BN, k-blocks are
// 64 BF16 (one 128-byte swizzle span). No TMA multicast is used anywhere.
#pragma once

#include "ptx.cuh"

namespace ce4b {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kGemmThreads = 192;
constexpr int kMaxClusterN = 8;

struct TileCoord {
  int a_row;    // first row of the A box (and of the output rows for dense GEMMs)
  int b_row;    // first row of the first B box
  int b_row2;   // first row of the second B box (SwiGLU "up" rows), unused otherwise
  int out_row;  // first output row of the tile
  int rows;     // valid output rows in this tile (<= 128)
  int n_tile;   // output column tile index
  int group;    // expert index for grouped GEMMs, 0 otherwise
};

// Dense tile order: t -> (m_tile = t / n_tiles, n_tile = t % n_tiles). A cluster of
// n_tiles CTAs therefore always shares one m_tile.
struct DenseSched {
  int m;            // rows of A / C
  int n_tiles;      // output column tiles
  int num_tiles;    // m_tiles * n_tiles
  int b_tile_rows;  // B rows advanced per n_tile
  int b_up_offset;  // row offset of the second B box (SwiGLU), 0 if unused
  __device__ __forceinline__ int count() const { return num_tiles; }
  __device__ __forceinline__ TileCoord coord(int t) const {
    TileCoord c;
    const int mt = t / n_tiles;
    c.n_tile = t - mt * n_tiles;
    c.a_row = mt * kBM;
    c.out_row = c.a_row;
    c.rows = min(kBM, m - c.a_row);
    c.b_row = c.n_tile * b_tile_rows;
    c.b_row2 = c.b_row + b_up_offset;
    c.group = 0;
    return c;
  }
};

// Grouped (MoE) tile order: the m-tile table is produced on the device by the routing
// scan; entry i = {expert, first permuted row, valid rows, 0}.
struct GroupedSched {
  const int4* m_tiles;     // [max_m_tiles]
  const int* num_m_tiles;  // device scalar
  int n_tiles;
  int b_tile_rows;
  int b_group_rows;  // B rows per expert (e.g. 2*h for gate_up, d for down)
  int b_up_offset;
  __device__ __forceinline__ int count() const { return __ldg(num_m_tiles) * n_tiles; }
  __device__ __forceinline__ TileCoord coord(int t) const {
    TileCoord c;
    const int mt = t / n_tiles;
    c.n_tile = t - mt * n_tiles;
    const int4 e = m_tiles[mt];
    c.group = e.x;
    c.a_row = e.y;
    c.out_row = e.y;
    c.rows = e.z;
    c.b_row = e.x * b_group_rows + c.n_tile * b_tile_rows;
    c.b_row2 = c.b_row + b_up_offset;
    return c;
  }
};

// Shared-memory block handed to epilogues that need cross-CTA exchange.
struct EpiShared {
  float recv[kMaxClusterN * kBM];
};

template <int BN, int NSTAGE, int NACC>
struct GemmSmem {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kRingBytes = NSTAGE * kStageBytes;
  static constexpr int kBarrierBytes = (2 * NSTAGE + 2 * NACC + 2) * 8 + 8;
  static constexpr int kBytes = 1024 /*alignment slack*/ + kRingBytes + kBarrierBytes + 64 +
                                static_cast<int>(sizeof(EpiShared));
  static constexpr uint32_t kTmemCols = (NACC * BN <= 32)    ? 32
                                        : (NACC * BN <= 64)  ? 64
                                        : (NACC * BN <= 128) ? 128
                                        : (NACC * BN <= 256) ? 256
                                                             : 512;
};

// NBOX = number of TMA boxes that make up the B tile (2 for SwiGLU: gate rows, up rows).
template <int BN, int NSTAGE, int NACC, int NBOX, bool CLUSTER, class Sched, class Epi>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const Sched sched, const typename Epi::Params ep, const int kblocks, int* err) {
  using L = GemmSmem<BN, NSTAGE, NACC>;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "invalid MMA N");
  static_assert(NACC * BN <= 512, "TMEM overflow");
  constexpr int kBoxRows = BN / NBOX;

  extern __shared__ uint8_t smem_raw[];
  uint32_t base = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (base & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  base += pad;

  const uint32_t bar_base = base + L::kRingBytes;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (NSTAGE + s); };
  auto tfull_bar = [&](int a) { return bar_base + 8u * (2 * NSTAGE + a); };
  auto tempty_bar = [&](int a) { return bar_base + 8u * (2 * NSTAGE + NACC + a); };
  const uint32_t drain_bar = bar_base + 8u * (2 * NSTAGE + 2 * NACC);
  const uint32_t epi_bar = drain_bar + 8u;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kRingBytes + L::kBarrierBytes);
  EpiShared* epi_smem =
      reinterpret_cast<EpiShared*>(smem + L::kRingBytes + L::kBarrierBytes + 64);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < NACC; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 128);
    }
    mbar_init(drain_bar, 1);
    mbar_init(epi_bar, Epi::bar_count(ep));
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  if constexpr (CLUSTER) {
    cluster_sync_all();
  } else {
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued_mask = 0, issued_phase = 0;
      const int ntiles = sched.count();
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const TileCoord tc = sched.coord(t);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u)) {
            record_error(err, kErrTimeoutProducer);
            ok = false;
            break;
          }
          const uint32_t sa = base + stage * L::kStageBytes;
          const uint32_t sb = sa + L::kABytes;
          mbar_arrive_expect_tx(full_bar(stage), L::kStageBytes);
          tma_load_2d(sa, &tmA, full_bar(stage), kb * kBK, tc.a_row);
          tma_load_2d(sb, &tmB, full_bar(stage), kb * kBK, tc.b_row);
          if constexpr (NBOX == 2) {
            tma_load_2d(sb + kBoxRows * kBK * 2, &tmB, full_bar(stage), kb * kBK, tc.b_row2);
          }
          issued_mask |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == NSTAGE) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let every load already issued land before the CTA can retire.
        for (int s = 0; s < NSTAGE; ++s) {
          if (issued_mask & (1u << s)) mbar_wait(full_bar(s), (issued_phase >> s) & 1u);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      const int ntiles = sched.count();
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u)) {
          record_error(err, kErrTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(full_bar(stage), phase)) {
            record_error(err, kErrTimeoutMma);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + stage * L::kStageBytes;
          const uint64_t adesc = sdesc_k128(sa);
          const uint64_t bdesc = sdesc_k128(sa + L::kABytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // +32 bytes per K=16 step inside the 128-byte swizzle span (encoded >> 4).
            umma_bf16(d_tmem, adesc + 2u * k, bdesc + 2u * k, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(empty_bar(stage));
          if (++stage == NSTAGE) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(tfull_bar(acc));
        if (++acc == NACC) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Every MMA issued by this thread must finish before TMEM is released.
      umma_commit(drain_bar);
      if (!mbar_wait(drain_bar, 0)) record_error(err, kErrTimeoutDrain);
    }
    __syncwarp();
  } else {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    const int ntiles = sched.count();
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      const TileCoord tc = sched.coord(t);
      if (!mbar_wait(tfull_bar(acc), acc_phase)) {
        record_error(err, kErrTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(quarter * 32) << 16);
      Epi::run(ep, tc, taddr, r, epi_smem, epi_bar, err);
      tc_fence_before();
      mbar_arrive(tempty_bar(acc));
      if (++acc == NACC) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// ------------------------------------------------------------------ epilogues

// Load 16 consecutive FP32 accumulator columns of this thread's row.
__device__ __forceinline__ void load_acc16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  tmem_ld16(taddr, r);
  tmem_ld_wait();
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
}

__device__ __forceinline__ void store_bf16x16(__nv_bfloat16* dst, const float (&v)[16]) {
  uint4 lo, hi;
  lo.x = pack_bf16x2(v[0], v[1]);
  lo.y = pack_bf16x2(v[2], v[3]);
  lo.z = pack_bf16x2(v[4], v[5]);
  lo.w = pack_bf16x2(v[6], v[7]);
  hi.x = pack_bf16x2(v[8], v[9]);
  hi.y = pack_bf16x2(v[10], v[11]);
  hi.z = pack_bf16x2(v[12], v[13]);
  hi.w = pack_bf16x2(v[14], v[15]);
  reinterpret_cast<uint4*>(dst)[0] = lo;
  reinterpret_cast<uint4*>(dst)[1] = hi;
}

__device__ __forceinline__ void load_bf16x16(const __nv_bfloat16* src, float (&v)[16]) {
  const uint4 lo = reinterpret_cast<const uint4*>(src)[0];
  const uint4 hi = reinterpret_cast<const uint4*>(src)[1];
  const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float2 f = unpack_bf16x2(w[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}

// SiLU(g) * u with the reference's operation order: g / (1 + exp(-g)) * u.
__device__ __forceinline__ float swiglu_f32(float g, float u) { return g / (1.0f + expf(-g)) * u; }

// Plain BF16 store of C (N columns, row stride ldc). Requires N % 16 == 0.
template <int BN>
struct EpiStoreBF16 {
  struct Params {
    __nv_bfloat16* c;
    int ldc;
    int n;
  };
  __device__ static uint32_t bar_count(const Params&) { return 1; }
  __device__ static void run(const Params& p, const TileCoord& tc, uint32_t taddr, int r,
                             EpiShared*, uint32_t, int*) {
    const bool valid = r < tc.rows;
    const int row = tc.out_row + r;
    const int n0 = tc.n_tile * BN;
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      if (n0 + c >= p.n) break;  // uniform across the warp
      float v[16];
      load_acc16(taddr + c, v);
      if (valid) store_bf16x16(p.c + static_cast<size_t>(row) * p.ldc + n0 + c, v);
    }
  }
};

// SwiGLU epilogue: accumulator columns [0, HC) are gate, [HC, 2*HC) are up for hidden
// columns n_tile*HC + [0, HC). Gate and up are rounded to BF16 first (the reference
// materialises the gate_up GEMM output in BF16), the product is rounded once more.
template <int HC>
struct EpiSwiGLU {
  struct Params {
    __nv_bfloat16* hidden;
    int ldh;
  };
  __device__ static uint32_t bar_count(const Params&) { return 1; }
  __device__ static void run(const Params& p, const TileCoord& tc, uint32_t taddr, int r,
                             EpiShared*, uint32_t, int*) {
    const bool valid = r < tc.rows;
    __nv_bfloat16* dst =
        p.hidden + static_cast<size_t>(tc.out_row + r) * p.ldh + tc.n_tile * HC;
#pragma unroll 1
    for (int c = 0; c < HC; c += 16) {
      float g[16], u[16], h[16];
      load_acc16(taddr + c, g);
      load_acc16(taddr + HC + c, u);
#pragma unroll
      for (int j = 0; j < 16; ++j) h[j] = swiglu_f32(bf16_round(g[j]), bf16_round(u[j]));
      if (valid) store_bf16x16(dst + c, h);
    }
  }
};

// Residual / bias epilogue with an optional fused RMSNorm of the updated row.
//   mode kBias:     x = bf16(acc + bias)                (input embedding, fused bias)
//   mode kResidual: x = bf16(x + bf16(acc))             (block output + residual)
// If norm_w is set, the CTAs of one cluster (one per BN-column slice of the row) exchange
// per-row partial sums of squares through distributed shared memory, and each writes
// nout = bf16((x * rsqrt(mean(x^2) + eps)) * norm_w) for its slice.
template <int BN>
struct EpiResNorm {
  enum Mode : int { kBias = 0, kResidual = 1 };
  struct Params {
    __nv_bfloat16* x;  // [M, d] residual stream (read for kResidual, always written)
    const __nv_bfloat16* bias;
    const __nv_bfloat16* norm_w;  // nullptr: no norm output
    __nv_bfloat16* nout;
    int d;
    int mode;
    int cluster_n;  // CTAs per row = d / BN
    float eps;
  };
  __device__ static uint32_t bar_count(const Params& p) {
    return static_cast<uint32_t>(p.cluster_n * kBM);
  }

  __device__ static void run(const Params& p, const TileCoord& tc, uint32_t taddr, int r,
                             EpiShared* sh, uint32_t epi_bar, int* err) {
    const bool valid = r < tc.rows;
    const int row = tc.out_row + r;
    const int n0 = tc.n_tile * BN;
    __nv_bfloat16* xrow = p.x + static_cast<size_t>(row) * p.d + n0;
    float ss = 0.0f;
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      float v[16];
      load_acc16(taddr + c, v);
      if (p.mode == kBias) {
        float b[16];
        load_bf16x16(p.bias + n0 + c, b);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = bf16_round(v[j] + b[j]);
      } else {
        float xo[16];
        if (valid) {
          load_bf16x16(xrow + c, xo);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) xo[j] = 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = bf16_round(xo[j] + bf16_round(v[j]));
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) ss = fmaf(v[j], v[j], ss);
      if (valid) store_bf16x16(xrow + c, v);
    }
    if (p.norm_w == nullptr) return;

    // Push this slice's partial sum to every CTA of the cluster, then collect.
    const uint32_t rank = static_cast<uint32_t>(tc.n_tile);
    const uint32_t slot = smem_u32(&sh->recv[rank * kBM + r]);
    for (int k = 0; k < p.cluster_n; ++k) st_cluster_f32(mapa_shared(slot, k), ss);
    for (int k = 0; k < p.cluster_n; ++k) mbar_arrive_remote(mapa_shared(epi_bar, k));
    if (!mbar_wait_cluster(epi_bar, 0)) {
      record_error(err, kErrTimeoutCluster);
      return;
    }
    float total = 0.0f;
    for (int k = 0; k < p.cluster_n; ++k) total += sh->recv[k * kBM + r];
    const float inv = 1.0f / sqrtf(total / static_cast<float>(p.d) + p.eps);
    if (!valid) return;
    __nv_bfloat16* nrow = p.nout + static_cast<size_t>(row) * p.d + n0;
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      float v[16], w[16];
      load_bf16x16(xrow + c, v);
      load_bf16x16(p.norm_w + n0 + c, w);
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = (v[j] * inv) * w[j];
      store_bf16x16(nrow + c, v);
    }
  }
};

// Heads epilogue over the concatenated head matrix [policy (Ps) | wdl (32) | moves-left (32)]:
// logits = bf16(acc + bias) (TE Linear fuses the bias before rounding); the policy block
// is written as FP32 for columns < policy_size, WDL as logits or as an FP32 softmax of
// the three rounded logits, moves-left as FP32.
struct EpiHeads {
  struct Params {
    const __nv_bfloat16* bias;  // [n_total]
    float* policy;              // [M, policy_size]
    float* wdl;                 // [M, 3]
    float* moves_left;          // [M]
    int policy_size;            // 1858
    int policy_storage;         // 1888 (start of the wdl block)
    int n_total;                // policy_storage + 64
    int wdl_probs;
  };
  __device__ static uint32_t bar_count(const Params&) { return 1; }
  static constexpr int BN = 256;
  __device__ static void run(const Params& p, const TileCoord& tc, uint32_t taddr, int r,
                             EpiShared*, uint32_t, int*) {
    const bool valid = r < tc.rows;
    const int row = tc.out_row + r;
    const int n0 = tc.n_tile * BN;
    float* prow = p.policy + static_cast<size_t>(row) * p.policy_size;
    float wdl[3] = {0.f, 0.f, 0.f};
    bool has_wdl = false;
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      if (n0 + c >= p.n_total) break;
      float v[16];
      load_acc16(taddr + c, v);
      if (!valid) continue;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int col = n0 + c + j;
        if (col >= p.n_total) break;
        const float logit = bf16_round(v[j] + __bfloat162float(p.bias[col]));
        if (col < p.policy_size) {
          prow[col] = logit;
        } else if (col >= p.policy_storage && col < p.policy_storage + 3) {
          wdl[col - p.policy_storage] = logit;
          has_wdl = true;
        } else if (col == p.policy_storage + 32) {
          p.moves_left[row] = logit;
        }
      }
    }
    if (valid && has_wdl) {
      float* w = p.wdl + static_cast<size_t>(row) * 3;
      if (p.wdl_probs) {
        const float mx = fmaxf(fmaxf(wdl[0], wdl[1]), wdl[2]);
        const float e0 = expf(wdl[0] - mx), e1 = expf(wdl[1] - mx), e2 = expf(wdl[2] - mx);
        const float total = e0 + e1 + e2;
        w[0] = e0 / total;
        w[1] = e1 / total;
        w[2] = e2 / total;
      } else {
        w[0] = wdl[0];
        w[1] = wdl[1];
        w[2] = wdl[2];
      }
    }
  }
};

}  // namespace ce4b
