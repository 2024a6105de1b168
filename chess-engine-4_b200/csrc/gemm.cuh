// Warp-specialised tcgen05 GEMM for sm_100a with fused epilogues.
//
//   C[M, N] = A[M, K] . B[N, K]^T      A, B: BF16, K-major (row-major with K contiguous)
//
// One CTA = 2 + 4*G warps: warp 0 issues TMA tile loads into an NSTAGE ring of
// shared-memory stages, warp 1 issues tcgen05.mma (M=128, N=BN, K=16) into a TMEM
// accumulator (NACC buffers, so the epilogue of one tile overlaps the main loop of the
// next), and 4*G epilogue warps drain the accumulator with tcgen05.ld. A warp can only
// reach the TMEM lane quarter (warp id % 4), so warp w serves rows 32*(w%4) + lane and
// column group (w-2)/4 of G; each thread owns one output row of its column group.
// Epilogues stage BF16 results in 128-byte-swizzled shared memory and write them with
// TMA bulk stores. Tiles are 128 x BN; k-blocks are 64 BF16 (one swizzle span).
// No TMA multicast is used anywhere.
#pragma once


#include "mxfp8.cuh"
#include "ptx.cuh"

namespace ce4b {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kMaxClusterN = 8;
constexpr int kMaxG = 4;
constexpr uint32_t kEpiBarrierId = 1;  // named barrier of the epilogue warps

__host__ __device__ constexpr int gemm_threads(int g) { return 64 + 128 * g; }

struct TileCoord {
  int a_row;    // first row of the A box
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
// scan; entry i = {expert, first permuted row, valid rows, 0}. Expert segments start on
// 128-row boundaries, so a tile never spans two experts.
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

// Where one epilogue thread sits in the tile.
struct EpiThread {
  int r;           // row within the tile (0..127)
  int g;           // column group (0..G-1)
  int tid;         // epilogue thread index (0..128*G-1)
  uint32_t taddr;  // TMEM address of (row quarter, accumulator buffer column 0)
};

// Shared resources handed to the epilogue of one tile.
struct EpiCtx {
  uint32_t smem;        // shared address of the epilogue region (1024-aligned)
  uint8_t* smem_ptr;    // generic pointer to the same region
  uint32_t ring;        // shared address of the stage ring (free after the last MMA of a
                        // CTA's only tile)
  uint32_t epi_bar;     // cluster exchange barrier
  uint32_t x_bar;       // producer prefetch barrier
  uint32_t tempty_bar;  // accumulator release barrier of this tile
  bool tempty_remote = false;  // tempty_bar is a shared::cluster address (CTA pairs)
  int rank_base = 0;    // cluster rank of this CTA's slice 0 (row-statistics exchange)
  int rank_stride = 1;  // cluster rank step between slices (2 for CTA pairs)
  int iter;             // tile iteration of this CTA (0, 1, ...)
  const CUtensorMap* tmO1;
  const CUtensorMap* tmO2;
  int* err;
};

// Every epilogue thread calls this once per tile after its last tcgen05.ld completed.
__device__ __forceinline__ void release_accumulator(const EpiCtx& ctx) {
  tc_fence_before();
  if (ctx.tempty_remote) {
    mbar_arrive_remote(ctx.tempty_bar);
  } else {
    mbar_arrive(ctx.tempty_bar);
  }
}

template <int G>
__device__ __forceinline__ void epi_bar_sync() {
  named_bar_sync(kEpiBarrierId, 128 * G);
}

template <int BN, int NSTAGE, int NACC, class Epi>
struct GemmSmem {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kRingBytes = NSTAGE * kStageBytes;
  static constexpr int kEpiBytes = (Epi::kSmemBytes + 1023) / 1024 * 1024;
  static constexpr int kBarrierBytes = (2 * NSTAGE + 2 * NACC + 3) * 8 + 8;
  static constexpr int kBytes = 1024 /*alignment slack*/ + kRingBytes + kEpiBytes + kBarrierBytes;
  static constexpr uint32_t kTmemCols = (NACC * BN <= 32)    ? 32
                                        : (NACC * BN <= 64)  ? 64
                                        : (NACC * BN <= 128) ? 128
                                        : (NACC * BN <= 256) ? 256
                                                             : 512;
  static_assert(kBytes <= 232448, "shared memory budget exceeded");
};

// NBOX = number of TMA boxes that make up the B tile (2 for SwiGLU: gate rows, up rows).
template <int BN, int NSTAGE, int NACC, int NBOX, int G, bool CLUSTER, class Sched, class Epi>
__global__ void __launch_bounds__(gemm_threads(G), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmO1, const __grid_constant__ CUtensorMap tmO2,
                   const Sched sched, const typename Epi::Params ep, const int kblocks, int* err) {
  using L = GemmSmem<BN, NSTAGE, NACC, Epi>;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "invalid MMA N");
  static_assert(NACC * BN <= 512, "TMEM overflow");
  static_assert(G >= 1 && G <= kMaxG, "invalid epilogue width");
  constexpr int kBoxRows = BN / NBOX;
  constexpr uint32_t kEpiThreads = 128 * G;

  extern __shared__ uint8_t smem_raw[];
  uint32_t base = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (base & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  base += pad;

  const uint32_t epi_base = base + L::kRingBytes;
  const uint32_t bar_base = epi_base + L::kEpiBytes;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (NSTAGE + s); };
  auto tfull_bar = [&](int a) { return bar_base + 8u * (2 * NSTAGE + a); };
  auto tempty_bar = [&](int a) { return bar_base + 8u * (2 * NSTAGE + NACC + a); };
  const uint32_t drain_bar = bar_base + 8u * (2 * NSTAGE + 2 * NACC);
  const uint32_t epi_bar = drain_bar + 8u;
  const uint32_t x_bar = drain_bar + 16u;
  uint32_t* tmem_slot =
      reinterpret_cast<uint32_t*>(smem + L::kRingBytes + L::kEpiBytes + L::kBarrierBytes - 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < NACC; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), kEpiThreads);
    }
    mbar_init(drain_bar, 1);
    mbar_init(epi_bar, Epi::bar_count(ep, G));
    mbar_init(x_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
    tmem_relinquish();
  }
  __syncwarp();
  tc_fence_before();
  if constexpr (CLUSTER) {
    cluster_sync_all();
  } else {
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  // The prologue above (barriers, TMEM) may overlap the previous kernel of the stream; no
  // global memory is read or written before that kernel has completed.
  grid_dependency_wait();
  grid_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued_mask = 0, issued_phase = 0;
      bool x_issued = false;
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
          // Epilogue operand (e.g. the residual tile) behind the first k-block; only for
          // kernels launched with one tile per CTA.
          if (kb == 0 && !x_issued && Epi::prefetch(ep, tc, &tmO1, epi_base, x_bar)) x_issued = true;
        }
      }
      if (!ok) {
        // Let every load already issued land before the CTA can retire.
        for (int s = 0; s < NSTAGE; ++s) {
          if (issued_mask & (1u << s)) mbar_wait(full_bar(s), (issued_phase >> s) & 1u);
        }
        if (x_issued) mbar_wait(x_bar, 0);
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
          // Operands landed by TMA: the stage barrier orders the MMAs after them (no
          // tcgen05 fence; it is needed only where TMEM changes hands between threads).
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
    EpiThread et;
    et.r = quarter * 32 + lane;
    et.g = (warp - 2) >> 2;
    et.tid = threadIdx.x - 64;
    EpiCtx ctx;
    ctx.smem = epi_base;
    ctx.smem_ptr = smem + L::kRingBytes;
    ctx.ring = base;
    ctx.epi_bar = epi_bar;
    ctx.x_bar = x_bar;
    ctx.tmO1 = &tmO1;
    ctx.tmO2 = &tmO2;
    ctx.err = err;
    int acc = 0;
    uint32_t acc_phase = 0;
    int iter = 0;
    const int ntiles = sched.count();
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++iter) {
      const TileCoord tc = sched.coord(t);
      if (!mbar_wait(tfull_bar(acc), acc_phase)) {
        record_error(err, kErrTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      et.taddr =
          tmem_base + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(quarter * 32) << 16);
      ctx.iter = iter;
      ctx.tempty_bar = tempty_bar(acc);
      Epi::template run<G>(ep, tc, et, ctx);
      if (++acc == NACC) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (et.tid == 0) bulk_wait_all();  // bulk stores read shared memory until complete
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// ------------------------------------------------------------------ CTA-pair GEMM
// The same pipeline on tcgen05 CTA pairs (cta_group::2). A pair tile is 256 rows x BN
// columns: the even CTA of the pair computes rows 0..127 (in its tensor memory), the odd
// CTA rows 128..255. Each CTA loads its own 128 A rows and half of the B tile (BN/2 rows;
// for SwiGLU the even CTA loads the gate rows and the odd CTA the up rows) into its own
// shared memory, so a CTA stages 16 KB + BN*64 B per k-block for a 128 x BN result: half
// the B traffic of a single-CTA tile, which is what limits the single-CTA main loop (the
// tensor core's operand reads and TMA's writes share the SM's shared-memory bandwidth).
// Both CTAs' loads complete on the even CTA's full barrier; its single MMA thread issues
// M=256 MMAs and multicasts each commit to the empty / accumulator-full barriers of both
// CTAs; both CTAs' epilogue threads release the accumulator on the even CTA's barrier.
// CLUSTER_N > 1 groups CLUSTER_N pairs in one cluster (ranks 2j, 2j+1 = pair j = column
// slice j of the same 256 rows) for the row-statistics exchange of EpiResNorm.
struct DensePairSched {
  int m;            // rows of A / C
  int n_tiles;      // output column tiles
  int num_tiles;    // ceil(m / 256) * n_tiles
  int b_tile_rows;  // B rows advanced per n_tile
  int b_half_rows;  // B rows held by each CTA (BN / 2)
  int b_up_offset;  // SwiGLU: the odd CTA's rows start this far past the even CTA's, else 0
  __device__ __forceinline__ int count() const { return num_tiles; }
  __device__ __forceinline__ TileCoord coord(int t, int half) const {
    TileCoord c;
    const int mt = t / n_tiles;
    c.n_tile = t - mt * n_tiles;
    c.a_row = (2 * mt + half) * kBM;
    c.out_row = c.a_row;
    c.rows = min(kBM, m - c.a_row);  // <= 0 for the odd CTA of a final half-empty tile
    c.b_row = c.n_tile * b_tile_rows + half * (b_up_offset != 0 ? b_up_offset : b_half_rows);
    c.b_row2 = c.b_row;
    c.group = 0;
    return c;
  }
};

template <int BN, int NSTAGE, int NACC, class Epi>
struct GemmPairSmem {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = (BN / 2) * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kRingBytes = NSTAGE * kStageBytes;
  static constexpr int kEpiBytes = (Epi::kSmemBytes + 1023) / 1024 * 1024;
  static constexpr int kBarrierBytes = (2 * NSTAGE + 2 * NACC + 3) * 8 + 8;
  static constexpr int kBytes = 1024 + kRingBytes + kEpiBytes + kBarrierBytes;
  static constexpr uint32_t kTmemCols = (NACC * BN <= 32)    ? 32
                                        : (NACC * BN <= 64)  ? 64
                                        : (NACC * BN <= 128) ? 128
                                        : (NACC * BN <= 256) ? 256
                                                             : 512;
  static_assert(kStageBytes % 1024 == 0, "stages must stay 1024-byte aligned");
  static_assert(kBytes <= 232448, "shared memory budget exceeded");
};

// Bounded pause used where a CTA cannot observe its own in-flight loads (the odd CTA's
// loads complete on the even CTA's barrier): long enough for any issued TMA to land.
__device__ __forceinline__ void settle_inflight_loads() {
  const unsigned long long start = global_timer_ns();
  while (global_timer_ns() - start < 200000ull) {
  }
}

template <int BN, int NSTAGE, int NACC, int G, int CLUSTER_N, class Epi>
__global__ void __launch_bounds__(gemm_threads(G), 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmO1, const __grid_constant__ CUtensorMap tmO2,
                     const DensePairSched sched, const typename Epi::Params ep, const int kblocks,
                     int* err) {
  using L = GemmPairSmem<BN, NSTAGE, NACC, Epi>;
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "invalid pair MMA N");
  static_assert(NACC * BN <= 512, "TMEM overflow");
  static_assert(2 * CLUSTER_N <= 16, "cluster too large");
  constexpr uint32_t kEpiThreads = 128 * G;

  extern __shared__ uint8_t smem_raw[];
  uint32_t base = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (base & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  base += pad;

  const uint32_t epi_base = base + L::kRingBytes;
  const uint32_t bar_base = epi_base + L::kEpiBytes;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (NSTAGE + s); };
  auto tfull_bar = [&](int a) { return bar_base + 8u * (2 * NSTAGE + a); };
  auto tempty_bar = [&](int a) { return bar_base + 8u * (2 * NSTAGE + NACC + a); };
  const uint32_t drain_bar = bar_base + 8u * (2 * NSTAGE + 2 * NACC);
  const uint32_t epi_bar = drain_bar + 8u;
  const uint32_t x_bar = drain_bar + 16u;
  uint32_t* tmem_slot =
      reinterpret_cast<uint32_t*>(smem + L::kRingBytes + L::kEpiBytes + L::kBarrierBytes - 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int half = static_cast<int>(rank & 1u);
  const uint32_t even = rank & ~1u;
  const uint16_t pair_mask = static_cast<uint16_t>(3u << even);

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < NACC; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 2 * kEpiThreads);
    }
    mbar_init(drain_bar, 1);
    mbar_init(epi_bar, Epi::bar_count(ep, G));
    mbar_init(x_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), L::kTmemCols);
    tmem_relinquish_pair();
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  // The prologue above may overlap the previous kernel of the stream; no global memory is
  // read or written before that kernel has completed.
  grid_dependency_wait();
  grid_launch_dependents();

  const int first = static_cast<int>(blockIdx.x >> 1);
  const int stride = static_cast<int>(gridDim.x >> 1);

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued_mask = 0, issued_phase = 0;
      bool x_issued = false;
      const int ntiles = sched.count();
      for (int t = first; t < ntiles && ok; t += stride) {
        const TileCoord tc = sched.coord(t, half);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_cluster(empty_bar(stage), phase ^ 1u)) {
            record_error(err, kErrTimeoutProducer);
            ok = false;
            break;
          }
          const uint32_t sa = base + stage * L::kStageBytes;
          const uint32_t sb = sa + L::kABytes;
          const uint32_t full_even = mapa_shared(full_bar(stage), even);
          if (half == 0) mbar_arrive_expect_tx(full_bar(stage), 2 * L::kStageBytes);
          tma_load_2d_pair(sa, &tmA, full_even, kb * kBK, tc.a_row);
          tma_load_2d_pair(sb, &tmB, full_even, kb * kBK, tc.b_row);
          issued_mask |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == NSTAGE) {
            stage = 0;
            phase ^= 1u;
          }
          if (kb == 0 && !x_issued && Epi::prefetch(ep, tc, &tmO1, epi_base, x_bar)) x_issued = true;
        }
      }
      if (!ok) {
        // Let every load already issued land before the CTA can retire.
        if (half == 0) {
          for (int s = 0; s < NSTAGE; ++s) {
            if (issued_mask & (1u << s)) mbar_wait(full_bar(s), (issued_phase >> s) & 1u);
          }
        } else {
          settle_inflight_loads();
        }
        if (x_issued) mbar_wait(x_bar, 0);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && half == 0) {
      constexpr uint32_t idesc = idesc_bf16(2 * kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      const int ntiles = sched.count();
      for (int t = first; t < ntiles && ok; t += stride) {
        if (!mbar_wait_cluster(tempty_bar(acc), acc_phase ^ 1u)) {
          record_error(err, kErrTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_cluster(full_bar(stage), phase)) {
            record_error(err, kErrTimeoutMma);
            ok = false;
            break;
          }
          // Operands landed by TMA: the stage barrier orders the MMAs after them (no
          // tcgen05 fence; it is needed only where TMEM changes hands between threads).
          const uint32_t sa = base + stage * L::kStageBytes;
          const uint64_t adesc = sdesc_k128(sa);
          const uint64_t bdesc = sdesc_k128(sa + L::kABytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            umma_bf16_pair(d_tmem, adesc + 2u * k, bdesc + 2u * k, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair_mc(empty_bar(stage), pair_mask);
          if (++stage == NSTAGE) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair_mc(tfull_bar(acc), pair_mask);
        if (++acc == NACC) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Every MMA issued by this thread must finish before either CTA releases TMEM or
      // shared memory.
      umma_commit_pair(drain_bar);
      if (!mbar_wait(drain_bar, 0)) record_error(err, kErrTimeoutDrain);
    }
    __syncwarp();
  } else {
    const int quarter = warp & 3;
    EpiThread et;
    et.r = quarter * 32 + lane;
    et.g = (warp - 2) >> 2;
    et.tid = threadIdx.x - 64;
    EpiCtx ctx;
    ctx.smem = epi_base;
    ctx.smem_ptr = smem + L::kRingBytes;
    ctx.ring = base;
    ctx.epi_bar = epi_bar;
    ctx.x_bar = x_bar;
    ctx.tmO1 = &tmO1;
    ctx.tmO2 = &tmO2;
    ctx.err = err;
    ctx.tempty_remote = true;
    ctx.rank_base = half;
    ctx.rank_stride = 2;
    int acc = 0;
    uint32_t acc_phase = 0;
    int iter = 0;
    const int ntiles = sched.count();
    for (int t = first; t < ntiles; t += stride, ++iter) {
      const TileCoord tc = sched.coord(t, half);
      if (!mbar_wait_cluster(tfull_bar(acc), acc_phase)) {
        record_error(err, kErrTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      et.taddr =
          tmem_base + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(quarter * 32) << 16);
      ctx.iter = iter;
      ctx.tempty_bar = mapa_shared(tempty_bar(acc), even);
      Epi::template run<G>(ep, tc, et, ctx);
      if (++acc == NACC) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (et.tid == 0) bulk_wait_all();  // bulk stores read shared memory until complete
  }

  __syncthreads();
  // Both CTAs are done with the pair's shared memory and tensor memory (the even CTA's
  // MMAs drained above) before either releases them.
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, L::kTmemCols);
  }
}

// ------------------------------------------------------------------ MXFP8 GEMM
// Block-scaled variant: A, B are E4M3 codes (K-major, one k-block = 128 codes = one
// 128-byte swizzle span), with E8M0 scales per row per 32 codes stored as 512-byte
// [32][16] tiles per (128 rows, 128 codes) (the tcgen05 scale-factor layout). Each stage
// holds the A and B code tiles plus their scale tiles; the MMA thread copies the scale
// tiles into a per-stage tensor-memory region (tcgen05.cp ... 32x128b.warpx4) and issues
// four K=32 block-scaled MMAs per k-block. Every MMA is N=128; a BN=256 tile issues two
// (one per 128-row half of B, each with its own B scale tile).
struct MxScales {
  const uint8_t* sfa;  // [M/128][K/128][512]
  const uint8_t* sfb;  // [N/128][K/128][512]
  int k_tiles;         // K / 128
};

template <int BN, int NSTAGE, int NACC, class Epi>
struct GemmMxSmem {
  static constexpr int kNSub = BN / 128;
  static constexpr int kABytes = kBM * 128;
  static constexpr int kBBytes = BN * 128;
  static constexpr int kLoadBytes = kABytes + kBBytes + 512 * (1 + kNSub);  // per stage
  static constexpr int kSfBytes = (512 * (1 + kNSub) + 1023) / 1024 * 1024;
  static constexpr int kStageBytes = kABytes + kBBytes + kSfBytes;
  static constexpr int kRingBytes = NSTAGE * kStageBytes;
  static constexpr int kEpiBytes = (Epi::kSmemBytes + 1023) / 1024 * 1024;
  static constexpr int kBarrierBytes = (2 * NSTAGE + 2 * NACC + 3) * 8 + 8;
  static constexpr int kBytes = 1024 + kRingBytes + kEpiBytes + kBarrierBytes;
  static constexpr int kSfCols = 4 * (1 + kNSub);  // TMEM columns of one stage's scales
  static constexpr int kUsedCols = NACC * BN + NSTAGE * kSfCols;
  static constexpr uint32_t kTmemCols = kUsedCols <= 128 ? 128 : (kUsedCols <= 256 ? 256 : 512);
  static_assert(kUsedCols <= 512, "TMEM overflow");
  static_assert(kStageBytes % 1024 == 0, "stages must stay 1024-byte aligned");
  static_assert(kBytes <= 232448, "shared memory budget exceeded");
};

template <int BN, int NSTAGE, int NACC, int NBOX, int G, bool CLUSTER, class Sched, class Epi>
__global__ void __launch_bounds__(gemm_threads(G), 1)
    gemm_mx_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmO1, const __grid_constant__ CUtensorMap tmO2,
                   const Sched sched, const typename Epi::Params ep, const MxScales sf,
                   const int kblocks, int* err) {
  using L = GemmMxSmem<BN, NSTAGE, NACC, Epi>;
  constexpr int kNSub = L::kNSub;
  constexpr int kBoxRows = BN / NBOX;
  static_assert(BN == 128 || BN == 256, "MXFP8 tiles are 128 or 256 columns");
  constexpr uint32_t kEpiThreads = 128 * G;

  extern __shared__ uint8_t smem_raw[];
  uint32_t base = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (base & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  base += pad;

  const uint32_t epi_base = base + L::kRingBytes;
  const uint32_t bar_base = epi_base + L::kEpiBytes;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (NSTAGE + s); };
  auto tfull_bar = [&](int a) { return bar_base + 8u * (2 * NSTAGE + a); };
  auto tempty_bar = [&](int a) { return bar_base + 8u * (2 * NSTAGE + NACC + a); };
  const uint32_t drain_bar = bar_base + 8u * (2 * NSTAGE + 2 * NACC);
  const uint32_t epi_bar = drain_bar + 8u;
  const uint32_t x_bar = drain_bar + 16u;
  uint32_t* tmem_slot =
      reinterpret_cast<uint32_t*>(smem + L::kRingBytes + L::kEpiBytes + L::kBarrierBytes - 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < NACC; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), kEpiThreads);
    }
    mbar_init(drain_bar, 1);
    mbar_init(epi_bar, Epi::bar_count(ep, G));
    mbar_init(x_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
    tmem_relinquish();
  }
  __syncwarp();
  tc_fence_before();
  if constexpr (CLUSTER) {
    cluster_sync_all();
  } else {
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  // The prologue above (barriers, TMEM) may overlap the previous kernel of the stream; no
  // global memory is read or written before that kernel has completed.
  grid_dependency_wait();
  grid_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued_mask = 0, issued_phase = 0;
      bool x_issued = false;
      const int ntiles = sched.count();
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const TileCoord tc = sched.coord(t);
        const int a_tile = tc.a_row / kBM;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u)) {
            record_error(err, kErrTimeoutProducer);
            ok = false;
            break;
          }
          const uint32_t sa = base + stage * L::kStageBytes;
          const uint32_t sb = sa + L::kABytes;
          const uint32_t ssf = sb + L::kBBytes;
          mbar_arrive_expect_tx(full_bar(stage), L::kLoadBytes);
          tma_load_2d(sa, &tmA, full_bar(stage), kb * 128, tc.a_row);
          tma_load_2d(sb, &tmB, full_bar(stage), kb * 128, tc.b_row);
          if constexpr (NBOX == 2) {
            tma_load_2d(sb + kBoxRows * 128, &tmB, full_bar(stage), kb * 128, tc.b_row2);
          }
          bulk_load(ssf, sf.sfa + (static_cast<size_t>(a_tile) * sf.k_tiles + kb) * 512, 512,
                    full_bar(stage));
#pragma unroll
          for (int j = 0; j < kNSub; ++j) {
            const int brow = (NBOX == 2 && j == 1) ? tc.b_row2 : tc.b_row + 128 * j;
            bulk_load(ssf + 512u * (1 + j),
                      sf.sfb + (static_cast<size_t>(brow / 128) * sf.k_tiles + kb) * 512, 512,
                      full_bar(stage));
          }
          issued_mask |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == NSTAGE) {
            stage = 0;
            phase ^= 1u;
          }
          if (kb == 0 && !x_issued && Epi::prefetch(ep, tc, &tmO1, epi_base, x_bar)) x_issued = true;
        }
      }
      if (!ok) {
        for (int s = 0; s < NSTAGE; ++s) {
          if (issued_mask & (1u << s)) mbar_wait(full_bar(s), (issued_phase >> s) & 1u);
        }
        if (x_issued) mbar_wait(x_bar, 0);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      const int ntiles = sched.count();
      const uint32_t sf_base = tmem_base + static_cast<uint32_t>(NACC * BN);
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
          // Operands landed by TMA: the stage barrier orders the MMAs after them (no
          // tcgen05 fence; it is needed only where TMEM changes hands between threads).
          const uint32_t sa = base + stage * L::kStageBytes;
          const uint32_t sb = sa + L::kABytes;
          const uint32_t ssf = sb + L::kBBytes;
          const uint32_t sfa_t = sf_base + static_cast<uint32_t>(stage * L::kSfCols);
          tmem_cp_32x128b_x4(sfa_t, sdesc_sf32x16(ssf));
#pragma unroll
          for (int j = 0; j < kNSub; ++j) {
            tmem_cp_32x128b_x4(sfa_t + 4u * (1 + j), sdesc_sf32x16(ssf + 512u * (1 + j)));
          }
          // One MMA covers all BN columns: the B rows of the 128-row boxes are contiguous
          // 8-row swizzle atoms, and their scales sit in consecutive 4-column groups (rows
          // 32q..32q+31 of each 128-row group in column 4 * group + q), the layout the
          // block-scaled MMA reads for N > 128. (Two N = 128 MMAs per K step cost ~1.4x
          // the issue time of one N = 256 MMA on the same operands.)
          const uint64_t adesc = sdesc_k128(sa);
          const uint64_t bdesc = sdesc_k128(sb);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            umma_mxf8(d_tmem, adesc + 2u * k, bdesc + 2u * k, idesc_mxf8(kBM, BN, k), sfa_t,
                      sfa_t + 4u, (kb | k) != 0 ? 1u : 0u);
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
      umma_commit(drain_bar);
      if (!mbar_wait(drain_bar, 0)) record_error(err, kErrTimeoutDrain);
    }
    __syncwarp();
  } else {
    const int quarter = warp & 3;
    EpiThread et;
    et.r = quarter * 32 + lane;
    et.g = (warp - 2) >> 2;
    et.tid = threadIdx.x - 64;
    EpiCtx ctx;
    ctx.smem = epi_base;
    ctx.smem_ptr = smem + L::kRingBytes;
    ctx.ring = base;
    ctx.epi_bar = epi_bar;
    ctx.x_bar = x_bar;
    ctx.tmO1 = &tmO1;
    ctx.tmO2 = &tmO2;
    ctx.err = err;
    int acc = 0;
    uint32_t acc_phase = 0;
    int iter = 0;
    const int ntiles = sched.count();
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++iter) {
      const TileCoord tc = sched.coord(t);
      if (!mbar_wait(tfull_bar(acc), acc_phase)) {
        record_error(err, kErrTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      et.taddr =
          tmem_base + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(quarter * 32) << 16);
      ctx.iter = iter;
      ctx.tempty_bar = tempty_bar(acc);
      Epi::template run<G>(ep, tc, et, ctx);
      if (++acc == NACC) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (et.tid == 0) bulk_wait_all();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// Weight-stationary MXFP8 SwiGLU GEMM for short K (K <= 128 * KBMAX): every CTA keeps the
// whole B tile of one 128-column hidden chunk (gate and up rows, all k-blocks, with their
// scale tiles) in shared memory and its B scales in tensor memory, and streams only A
// (128-row code tiles + scale tiles) through the stage ring for row blocks t = blockIdx.x,
// + gridDim.x, ... The grid is a multiple of the chunk count, so a CTA's chunk never
// changes (DenseSched is chunk-fastest). Per tile that moves 64 KB of A at K = 512
// instead of A + B = 192 KB.
template <int KBMAX, int NSTAGE, class Epi>
struct GemmMxBStatSmem {
  static constexpr int BN = 256;
  static constexpr int kBBytes = BN * 128 * KBMAX;        // B codes, k-block-major
  static constexpr int kSfbBytes = 2 * 512 * KBMAX;        // B scale tiles [k-block][half]
  static constexpr int kABytes = kBM * 128;                // one A code tile
  static constexpr int kStageBytes = kABytes + 1024;       // + its scale tile (512 B, padded)
  static constexpr int kRingBytes = NSTAGE * kStageBytes;
  static constexpr int kEpiBytes = (Epi::kSmemBytes + 1023) / 1024 * 1024;
  static constexpr int kBarrierBytes = (2 * NSTAGE + 6) * 8 + 8;
  static constexpr int kBytes = 1024 + kBBytes + kSfbBytes + kRingBytes + kEpiBytes + kBarrierBytes;
  static constexpr int kSfbCol = BN;                       // TMEM: accumulator, B scales, A scales
  static constexpr int kSfaCol = BN + 8 * KBMAX;
  static_assert(kSfaCol + 4 * NSTAGE <= 512, "TMEM overflow");
  static_assert(kBytes <= 232448, "shared memory budget exceeded");
};

template <int KBMAX, int NSTAGE, int G, class Epi>
__global__ void __launch_bounds__(gemm_threads(G), 1)
    gemm_mx_bstat_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmO1, const DenseSched sched,
                         const typename Epi::Params ep, const MxScales sf, const int kblocks, int* err) {
  using L = GemmMxBStatSmem<KBMAX, NSTAGE, Epi>;
  constexpr int BN = L::BN;
  constexpr uint32_t kEpiThreads = 128 * G;

  extern __shared__ uint8_t smem_raw[];
  uint32_t base = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (base & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  base += pad;

  const uint32_t b_base = base;
  const uint32_t sfb_base = b_base + L::kBBytes;
  const uint32_t ring = sfb_base + L::kSfbBytes;
  const uint32_t epi_base = ring + L::kRingBytes;
  const uint32_t bar_base = epi_base + L::kEpiBytes;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (NSTAGE + s); };
  const uint32_t tfull_bar = bar_base + 8u * (2 * NSTAGE);
  const uint32_t tempty_bar = tfull_bar + 8u;
  const uint32_t drain_bar = tfull_bar + 16u;
  const uint32_t epi_bar = tfull_bar + 24u;
  const uint32_t x_bar = tfull_bar + 32u;
  const uint32_t b_bar = tfull_bar + 40u;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + (bar_base - base) + L::kBarrierBytes - 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(tempty_bar, kEpiThreads);
    mbar_init(drain_bar, 1);
    mbar_init(epi_bar, Epi::bar_count(ep, G));
    mbar_init(x_bar, 1);
    mbar_init(b_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  grid_dependency_wait();
  grid_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      const int ntiles = sched.count();
      bool ok = blockIdx.x < ntiles;
      bool b_issued = false;
      if (ok) {
        // This CTA's hidden chunk: gate rows b_row, up rows b_row2, every k-block.
        const TileCoord tc0 = sched.coord(blockIdx.x);
        mbar_arrive_expect_tx(b_bar, static_cast<uint32_t>(kblocks * (BN * 128 + 2 * 512)));
        for (int kb = 0; kb < kblocks; ++kb) {
          const uint32_t sb = b_base + static_cast<uint32_t>(kb * BN * 128);
          tma_load_2d(sb, &tmB, b_bar, kb * 128, tc0.b_row);
          tma_load_2d(sb + 128 * 128, &tmB, b_bar, kb * 128, tc0.b_row2);
          bulk_load(sfb_base + static_cast<uint32_t>(kb * 1024),
                    sf.sfb + (static_cast<size_t>(tc0.b_row / 128) * sf.k_tiles + kb) * 512, 512, b_bar);
          bulk_load(sfb_base + static_cast<uint32_t>(kb * 1024 + 512),
                    sf.sfb + (static_cast<size_t>(tc0.b_row2 / 128) * sf.k_tiles + kb) * 512, 512, b_bar);
        }
        b_issued = true;
      }
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_phase = 0;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        const TileCoord tc = sched.coord(t);
        const int a_tile = tc.a_row / kBM;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u)) {
            record_error(err, kErrTimeoutProducer);
            ok = false;
            break;
          }
          const uint32_t sa = ring + static_cast<uint32_t>(stage * L::kStageBytes);
          mbar_arrive_expect_tx(full_bar(stage), L::kABytes + 512);
          tma_load_2d(sa, &tmA, full_bar(stage), kb * 128, tc.a_row);
          bulk_load(sa + L::kABytes, sf.sfa + (static_cast<size_t>(a_tile) * sf.k_tiles + kb) * 512, 512,
                    full_bar(stage));
          issued_mask |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == NSTAGE) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        for (int s = 0; s < NSTAGE; ++s) {
          if (issued_mask & (1u << s)) mbar_wait(full_bar(s), (issued_phase >> s) & 1u);
        }
      }
      if (b_issued) mbar_wait(b_bar, 0);  // (normally long complete: the MMA thread waited)
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const int ntiles = sched.count();
      bool ok = blockIdx.x < ntiles;
      if (ok && !mbar_wait(b_bar, 0)) {
        record_error(err, kErrTimeoutMma);
        ok = false;
      }
      if (ok) {
        tc_fence_after();
        for (int kb = 0; kb < kblocks; ++kb) {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            tmem_cp_32x128b_x4(tmem_base + static_cast<uint32_t>(L::kSfbCol + kb * 8 + 4 * j),
                               sdesc_sf32x16(sfb_base + static_cast<uint32_t>(kb * 1024 + 512 * j)));
          }
        }
      }
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        if (!mbar_wait(tempty_bar, acc_phase ^ 1u)) {
          record_error(err, kErrTimeoutMma);
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(full_bar(stage), phase)) {
            record_error(err, kErrTimeoutMma);
            ok = false;
            break;
          }
          // Operands landed by TMA: the stage barrier orders the MMAs after them (no
          // tcgen05 fence; it is needed only where TMEM changes hands between threads).
          const uint32_t sa = ring + static_cast<uint32_t>(stage * L::kStageBytes);
          const uint32_t sfa_t = tmem_base + static_cast<uint32_t>(L::kSfaCol + stage * 4);
          tmem_cp_32x128b_x4(sfa_t, sdesc_sf32x16(sa + L::kABytes));
          const uint64_t adesc = sdesc_k128(sa);
          const uint64_t bdesc = sdesc_k128(b_base + static_cast<uint32_t>(kb * BN * 128));
          const uint32_t sfb_t = tmem_base + static_cast<uint32_t>(L::kSfbCol + kb * 8);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            umma_mxf8(tmem_base, adesc + 2u * k, bdesc + 2u * k, idesc_mxf8(kBM, BN, k), sfa_t, sfb_t,
                      (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(empty_bar(stage));
          if (++stage == NSTAGE) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(tfull_bar);
        acc_phase ^= 1u;
      }
      umma_commit(drain_bar);
      if (!mbar_wait(drain_bar, 0)) record_error(err, kErrTimeoutDrain);
    }
    __syncwarp();
  } else {
    const int quarter = warp & 3;
    EpiThread et;
    et.r = quarter * 32 + lane;
    et.g = (warp - 2) >> 2;
    et.tid = threadIdx.x - 64;
    EpiCtx ctx;
    ctx.smem = epi_base;
    ctx.smem_ptr = smem + (epi_base - base);
    ctx.ring = ring;
    ctx.epi_bar = epi_bar;
    ctx.x_bar = x_bar;
    ctx.tmO1 = &tmO1;
    ctx.tmO2 = &tmO1;
    ctx.err = err;
    uint32_t acc_phase = 0;
    int iter = 0;
    const int ntiles = sched.count();
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++iter) {
      const TileCoord tc = sched.coord(t);
      if (!mbar_wait(tfull_bar, acc_phase)) {
        record_error(err, kErrTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      et.taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
      ctx.iter = iter;
      ctx.tempty_bar = tempty_bar;
      Epi::template run<G>(ep, tc, et, ctx);
      acc_phase ^= 1u;
    }
    if (et.tid == 0) bulk_wait_all();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ------------------------------------------------------------------ epilogue helpers

// Load 32 consecutive FP32 accumulator columns of this thread's row (one wait).
__device__ __forceinline__ void load_acc32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  tmem_ld32(taddr, r);
  tmem_ld_wait();
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

// Two 32-column loads behind one wait.
__device__ __forceinline__ void load_acc32x2(uint32_t ta, uint32_t tb, float (&a)[32], float (&b)[32]) {
  uint32_t ra[32], rb[32];
  tmem_ld32(ta, ra);
  tmem_ld32(tb, rb);
  tmem_ld_wait();
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    a[j] = __uint_as_float(ra[j]);
    b[j] = __uint_as_float(rb[j]);
  }
}

// Round pairs to BF16 (one cvt per pair) and back to FP32.
__device__ __forceinline__ void round_bf16_inplace(float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    const float2 f = unpack_bf16x2(pack_bf16x2(v[j], v[j + 1]));
    v[j] = f.x;
    v[j + 1] = f.y;
  }
}

template <int N>
__device__ __forceinline__ void load_bf16(const __nv_bfloat16* src, float* v) {
  static_assert(N % 8 == 0, "16-byte chunks");
#pragma unroll
  for (int c = 0; c < N; c += 8) {
    const uint4 q = reinterpret_cast<const uint4*>(src)[c / 8];
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(w[j]);
      v[c + 2 * j] = f.x;
      v[c + 2 * j + 1] = f.y;
    }
  }
}

// Write 32 BF16 values (columns col..col+31 of row r, col % 32 == 0) into a staging
// tile made of [128 rows][64 cols] boxes with the 128-byte swizzle (the layout a TMA
// store with SWIZZLE_128B reads).
__device__ __forceinline__ void stage_bf16x32(uint32_t tile, int r, int col, const float (&v)[32]) {
  const uint32_t box = tile + static_cast<uint32_t>(col / 64) * (kBM * 128);
  const int chunk0 = (col % 64) / 8;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uint4 o;
    o.x = pack_bf16x2(v[8 * k + 0], v[8 * k + 1]);
    o.y = pack_bf16x2(v[8 * k + 2], v[8 * k + 3]);
    o.z = pack_bf16x2(v[8 * k + 4], v[8 * k + 5]);
    o.w = pack_bf16x2(v[8 * k + 6], v[8 * k + 7]);
    st_shared_v4(box + swz128(r, chunk0 + k), o);
  }
}

// Read 32 BF16 values back from the same staging layout.
__device__ __forceinline__ void unstage_bf16x32(uint32_t tile, int r, int col, float (&v)[32]) {
  const uint32_t box = tile + static_cast<uint32_t>(col / 64) * (kBM * 128);
  const int chunk0 = (col % 64) / 8;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint4 q = ld_shared_v4(box + swz128(r, chunk0 + k));
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(w[j]);
      v[8 * k + 2 * j] = f.x;
      v[8 * k + 2 * j + 1] = f.y;
    }
  }
}

// Write 32 E4M3 codes (columns col..col+31 of row r, col % 32 == 0) into a staging tile
// of [128 rows][128 codes] boxes with the 128-byte swizzle.
__device__ __forceinline__ void stage_u8x32(uint32_t tile, int r, int col, const uint32_t (&q)[8]) {
  const uint32_t box = tile + static_cast<uint32_t>(col / 128) * (kBM * 128);
  const int chunk0 = (col % 128) / 16;
  st_shared_v4(box + swz128(r, chunk0), make_uint4(q[0], q[1], q[2], q[3]));
  st_shared_v4(box + swz128(r, chunk0 + 1), make_uint4(q[4], q[5], q[6], q[7]));
}

// TMA-store a staged [128 x cols] code tile (cols / 128 boxes) at (x0, y0).
// 32 BF16 values of one row to global memory (a test tap of the MXFP8 epilogues: the
// values a quantising epilogue saw).
__device__ __forceinline__ void store_bf16x32_global(__nv_bfloat16* dst, const float (&v)[32]) {
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    d4[u] = make_uint4(pack_bf16x2(v[8 * u], v[8 * u + 1]), pack_bf16x2(v[8 * u + 2], v[8 * u + 3]),
                       pack_bf16x2(v[8 * u + 4], v[8 * u + 5]), pack_bf16x2(v[8 * u + 6], v[8 * u + 7]));
  }
}

__device__ __forceinline__ void store_staged_u8(const CUtensorMap* map, uint32_t tile, int cols,
                                                int x0, int y0) {
  for (int b = 0; b < cols / 128; ++b) {
    tma_store_2d(map, tile + static_cast<uint32_t>(b) * (kBM * 128), x0 + 128 * b, y0);
  }
  bulk_commit();
}

// TMA-store a staged [128 x cols] BF16 tile (cols / 64 boxes) at (x0, y0).
__device__ __forceinline__ void store_staged(const CUtensorMap* map, uint32_t tile, int cols, int x0,
                                             int y0) {
  for (int b = 0; b < cols / 64; ++b) {
    tma_store_2d(map, tile + static_cast<uint32_t>(b) * (kBM * 128), x0 + 64 * b, y0);
  }
  bulk_commit();
}

// SiLU(g) * u, evaluated as g / (1 + exp(-g)) * u with the special-function unit's exp2
// and reciprocal (a few FP32 ulp; the result is rounded to BF16, whose ulp is 2^16 times
// coarser, so the approximation changes the output only in rare rounding ties).
__device__ __forceinline__ float swiglu_f32(float g, float u) {
  const float e = ex2_approx(g * -1.4426950408889634f);
  return g * rcp_approx(1.0f + e) * u;
}

// ------------------------------------------------------------------ epilogues

// Plain BF16 C tile, staged and TMA-stored through tmO1 (box 64 x 128).
template <int BN>
struct EpiStoreBF16 {
  static_assert(BN % 64 == 0, "64-column boxes");
  static constexpr int kSmemBytes = kBM * BN * 2;
  struct Params {
    int n;  // logical columns (for the tail of the last tile)
  };
  __device__ static uint32_t bar_count(const Params&, int) { return 1; }
  __device__ static bool prefetch(const Params&, const TileCoord&, const CUtensorMap*, uint32_t,
                                  uint32_t) {
    return false;
  }
  template <int G>
  __device__ static void run(const Params& p, const TileCoord& tc, const EpiThread& et,
                             const EpiCtx& ctx) {
    if (ctx.iter > 0) {
      if (et.tid == 0) bulk_wait_read_all();
      epi_bar_sync<G>();
    }
    const int n0 = tc.n_tile * BN;
    for (int c = et.g * 32; c < BN; c += G * 32) {
      float v[32];
      load_acc32(et.taddr + c, v);
      stage_bf16x32(ctx.smem, et.r, c, v);
    }
    release_accumulator(ctx);
    fence_proxy_async_smem();
    epi_bar_sync<G>();
    if (et.tid == 0 && tc.rows > 0) store_staged(ctx.tmO1, ctx.smem, BN, n0, tc.out_row);
    (void)p;
  }
};

// SwiGLU epilogue: accumulator columns [0, HC) are gate, [HC, 2*HC) are up for hidden
// columns n_tile*HC + [0, HC). Gate and up are rounded to BF16 first (the reference
// materialises the gate_up GEMM output in BF16), the product is rounded once more.
// The hidden tile is TMA-stored through tmO1 (box 64 x 128 over [M, h]).
// With MX, the hidden tile is written as MXFP8 instead: the BF16-rounded values (the
// reference quantises the BF16 hidden tensor) become E4M3 codes TMA-stored through tmO1
// (a byte map over [M, h], 128-code boxes) and one E8M0 scale per row and 32 columns,
// each thread's 32-column group being exactly one scale block.
template <int HC, bool MX = false>
struct EpiSwiGLU {
  static_assert(HC % 64 == 0, "64-column boxes");
  static_assert(!MX || HC == 128, "MXFP8 output needs 128-column chunks");
  static constexpr int kSmemBytes = MX ? kBM * HC : kBM * HC * 2;
  struct Params {
    uint8_t* scales;  // MX: [M/128][h/128][512] scale tiles of the hidden codes
    int col_tiles;    // MX: h / 128
    __nv_bfloat16* tap;  // MX: [M, h] the BF16 hidden values quantised (nullptr: not stored)
  };
  __device__ static uint32_t bar_count(const Params&, int) { return 1; }
  __device__ static bool prefetch(const Params&, const TileCoord&, const CUtensorMap*, uint32_t,
                                  uint32_t) {
    return false;
  }
  template <int G>
  __device__ static void run(const Params& p, const TileCoord& tc, const EpiThread& et,
                             const EpiCtx& ctx) {
    if (ctx.iter > 0) {
      if (et.tid == 0) bulk_wait_read_all();  // previous tile's store has read the staging
      epi_bar_sync<G>();
    }
    // With one 32-column chunk per thread (HC == 32 * G) the accumulator is released right
    // after it has been read, so the next tile's MMAs overlap the SwiGLU (and the MXFP8
    // quantisation) of this one even with a single accumulator.
    constexpr bool kOneChunk = HC == 32 * G;
    for (int c = et.g * 32; c < HC; c += G * 32) {
      float g[32], u[32];
      load_acc32x2(et.taddr + c, et.taddr + HC + c, g, u);
      if constexpr (kOneChunk) release_accumulator(ctx);
      round_bf16_inplace(g);
      round_bf16_inplace(u);
#pragma unroll
      for (int j = 0; j < 32; ++j) g[j] = swiglu_f32(g[j], u[j]);
      if constexpr (MX) {
        round_bf16_inplace(g);
        uint32_t q[8];
        const uint8_t sc = mx_quantize32(g, q);
        stage_u8x32(ctx.smem, et.r, c, q);
        if (et.r < tc.rows) {
          p.scales[mx_scale_offset(tc.out_row + et.r, (tc.n_tile * HC + c) / 32, p.col_tiles)] = sc;
          if (p.tap != nullptr) {
            store_bf16x32_global(
                p.tap + static_cast<size_t>(tc.out_row + et.r) * (p.col_tiles * 128) + tc.n_tile * HC + c, g);
          }
        }
      } else {
        stage_bf16x32(ctx.smem, et.r, c, g);
      }
    }
    if constexpr (!kOneChunk) release_accumulator(ctx);
    fence_proxy_async_smem();
    epi_bar_sync<G>();
    if (et.tid == 0 && tc.rows > 0) {
      if constexpr (MX) {
        store_staged_u8(ctx.tmO1, ctx.smem, HC, tc.n_tile * HC, tc.out_row);
      } else {
        store_staged(ctx.tmO1, ctx.smem, HC, tc.n_tile * HC, tc.out_row);
      }
    }
  }
};

// Residual / bias epilogue with an optional fused RMSNorm of the updated row.
//   mode kBias:     x = bf16(acc + bias)                (input embedding, fused bias)
//   mode kResidual: x = bf16(x + bf16(acc))             (block output + residual)
// tmO1 is the x map (box 64 x 128): the producer prefetches the residual tile through it
// and the epilogue stores the updated tile through it. If norm_w is set, every
// (CTA, column group) of a cluster — one CTA per BN-column slice of the row — pushes its
// per-row partial sum of squares to all CTAs through distributed shared memory; each CTA
// then writes n = bf16((x * rsqrt(mean(x^2) + eps)) * norm_w) for its slice through tmO2.
// Partials are summed in a fixed order, so results are deterministic. Launched with
// exactly one tile per CTA (the stage ring is reused as the n staging buffer).
// With MX, n is written as MXFP8 (BF16-rounded, then E4M3 codes through tmO2 as a byte
// map with 128-code boxes, one E8M0 scale per row and 32 columns into n_scales).
// MAXC bounds the CTAs per row (cluster_n), which sizes the partial-sum receive buffer.
// LATE: the x tile lives in the stage ring, which is idle once the CTA's only tile has been
// accumulated; the residual is then loaded after the main loop instead of prefetched during
// it. This frees the tile's shared memory for another operand stage (wide models, where the
// cluster's receive buffer and a 256-column x tile would otherwise leave three stages).
template <int BN, bool MX = false, int MAXC = kMaxClusterN, bool LATE = false>
struct EpiResNorm {
  static_assert(BN % 64 == 0, "64-column boxes");
  static_assert(!MX || BN % 128 == 0, "MXFP8 output needs 128-column slices");
  static_assert(MAXC >= 1 && MAXC <= kMaxClusterN, "cluster bound");
  enum Mode : int { kBias = 0, kResidual = 1 };
  static constexpr int kXBytes = kBM * BN * 2;
  static constexpr int kRecvFloats = MAXC * kMaxG * kBM;
  static constexpr int kSmemBytes = (LATE ? 0 : kXBytes) + kRecvFloats * 4;
  struct Params {
    const __nv_bfloat16* bias;
    const __nv_bfloat16* norm_w;  // nullptr: no norm output
    int d;
    int mode;
    int cluster_n;  // CTAs per row = d / BN
    float eps;
    uint8_t* n_scales;  // MX: [M/128][d/128][512]
    __nv_bfloat16* tap;  // MX: [M, d] the BF16 values of n quantised (nullptr: not stored)
  };
  __device__ static int groups(int G) { return G < BN / 32 ? G : BN / 32; }
  __device__ static uint32_t bar_count(const Params& p, int G) {
    return static_cast<uint32_t>(p.cluster_n * groups(G) * kBM);
  }
  __device__ static void load_x(const TileCoord& tc, const CUtensorMap* tm_x, uint32_t dst, uint32_t bar) {
    mbar_arrive_expect_tx(bar, kXBytes);
    for (int b = 0; b < BN / 64; ++b) {
      tma_load_2d(dst + static_cast<uint32_t>(b) * (kBM * 128), tm_x, bar, tc.n_tile * BN + 64 * b,
                  tc.out_row);
    }
  }
  __device__ static bool prefetch(const Params& p, const TileCoord& tc, const CUtensorMap* tm_x,
                                  uint32_t dst, uint32_t bar) {
    if (LATE || p.mode != kResidual) return false;
    load_x(tc, tm_x, dst, bar);
    return true;
  }

  template <int G>
  __device__ static void run(const Params& p, const TileCoord& tc, const EpiThread& et,
                             const EpiCtx& ctx) {
    constexpr int kPer = BN / 32;  // 32-column chunks in this slice
    constexpr int kGroups = G < kPer ? G : kPer;
    constexpr int kChunks = kPer / kGroups;  // chunks per column group
    static_assert(kPer % kGroups == 0, "chunks must split evenly");
    const bool active = et.g < kGroups;
    const int n0 = tc.n_tile * BN;
    // x tile (residual, then updated x) and n staging: the tile's own shared memory and the
    // idle ring, or both in the ring (LATE).
    const uint32_t xs = LATE ? ctx.ring : ctx.smem;
    const uint32_t n_stage = LATE ? ctx.ring + kXBytes : ctx.ring;
    float* recv = reinterpret_cast<float*>(ctx.smem_ptr + (LATE ? 0 : kXBytes));
    if (LATE && p.mode == kResidual && et.tid == 0) load_x(tc, ctx.tmO1, xs, ctx.x_bar);
    bool ok = true;
    if (p.mode == kResidual && !mbar_wait(ctx.x_bar, 0)) {
      record_error(ctx.err, kErrTimeoutEpilogue);
      ok = false;
    }
    float ss = 0.0f;
    if (active) {
#pragma unroll
      for (int i = 0; i < kChunks; ++i) {
        const int c = (et.g * kChunks + i) * 32;
        float v[32];
        load_acc32(et.taddr + c, v);
        if (p.mode == kBias) {
          float b[32];
          load_bf16<32>(p.bias + n0 + c, b);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = v[j] + b[j];
          round_bf16_inplace(v);
        } else {
          float xo[32];
          unstage_bf16x32(xs, et.r, c, xo);
          round_bf16_inplace(v);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = xo[j] + v[j];
          round_bf16_inplace(v);
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) ss = fmaf(v[j], v[j], ss);
        stage_bf16x32(xs, et.r, c, v);
      }
    }
    release_accumulator(ctx);
    fence_proxy_async_smem();
    epi_bar_sync<G>();
    if (et.tid == 0 && tc.rows > 0) store_staged(ctx.tmO1, xs, BN, n0, tc.out_row);
    if (p.norm_w == nullptr || !ok) return;

    // Push this (slice, group) partial to every CTA of the cluster, then collect.
    if (active) {
      const uint32_t rank = static_cast<uint32_t>(tc.n_tile);
      const uint32_t slot = smem_u32(&recv[(rank * kGroups + et.g) * kBM + et.r]);
      for (int k = 0; k < p.cluster_n; ++k) {
        st_cluster_f32(mapa_shared(slot, ctx.rank_base + ctx.rank_stride * k), ss);
      }
      for (int k = 0; k < p.cluster_n; ++k) {
        mbar_arrive_remote(mapa_shared(ctx.epi_bar, ctx.rank_base + ctx.rank_stride * k));
      }
    }
    if (!mbar_wait_cluster(ctx.epi_bar, 0)) {
      record_error(ctx.err, kErrTimeoutCluster);
      return;
    }
    if (active) {
      float total = 0.0f;
      const int parts = p.cluster_n * kGroups;
      for (int k = 0; k < parts; ++k) total += recv[k * kBM + et.r];
      const float inv = 1.0f / sqrtf(total / static_cast<float>(p.d) + p.eps);
      // The stage ring is idle after this CTA's only tile: stage n there.
#pragma unroll
      for (int i = 0; i < kChunks; ++i) {
        const int c = (et.g * kChunks + i) * 32;
        float v[32], w[32];
        unstage_bf16x32(xs, et.r, c, v);
        load_bf16<32>(p.norm_w + n0 + c, w);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = (v[j] * inv) * w[j];
        if constexpr (MX) {
          round_bf16_inplace(v);
          uint32_t q[8];
          const uint8_t sc = mx_quantize32(v, q);
          stage_u8x32(n_stage, et.r, c, q);
          if (et.r < tc.rows) {
            p.n_scales[mx_scale_offset(tc.out_row + et.r, (n0 + c) / 32, p.d / 128)] = sc;
            if (p.tap != nullptr) {
              store_bf16x32_global(p.tap + static_cast<size_t>(tc.out_row + et.r) * p.d + n0 + c, v);
            }
          }
        } else {
          stage_bf16x32(n_stage, et.r, c, v);
        }
      }
    }
    fence_proxy_async_smem();
    epi_bar_sync<G>();
    if (et.tid == 0 && tc.rows > 0) {
      if constexpr (MX) {
        store_staged_u8(ctx.tmO2, n_stage, BN, n0, tc.out_row);
      } else {
        store_staged(ctx.tmO2, n_stage, BN, n0, tc.out_row);
      }
    }
  }
};

// Heads epilogue over the concatenated head matrix [policy (Ps) | wdl (32) | moves-left (32)]:
// logits = bf16(acc + bias) (TE Linear fuses the bias before rounding); the policy block
// is written as FP32 for columns < policy_size, WDL as logits or as an FP32 softmax of
// the three rounded logits, moves-left as FP32. Each warp transposes its 32 x 32 block
// through shared memory so that every store instruction writes 32 consecutive floats of
// one row (the 7432-byte policy row stride rules out TMA stores).
struct EpiHeads {
  static constexpr int BN = 256;
  static constexpr int kPitch = 33;  // floats per transposed row (bank-conflict free)
  static constexpr int kSmemBytes = 16 * 32 * kPitch * 4;
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
  __device__ static uint32_t bar_count(const Params&, int) { return 1; }
  __device__ static bool prefetch(const Params&, const TileCoord&, const CUtensorMap*, uint32_t,
                                  uint32_t) {
    return false;
  }
  template <int G>
  __device__ static void run(const Params& p, const TileCoord& tc, const EpiThread& et,
                             const EpiCtx& ctx) {
    static_assert(G <= 4, "transpose buffers for 16 warps");
    const int lane = et.r & 31;
    const int row0 = tc.out_row + (et.r & ~31);  // first row of this warp's 32 rows
    float* tbuf = reinterpret_cast<float*>(ctx.smem_ptr) + (et.tid >> 5) * 32 * kPitch;
    const int n0 = tc.n_tile * BN;
    for (int c = et.g * 32; c < BN; c += G * 32) {
      const int c0 = n0 + c;
      if (c0 >= p.n_total) break;  // uniform across the warp
      float v[32], b[32];
      load_acc32(et.taddr + c, v);
      load_bf16<32>(p.bias + c0, b);  // bias is padded to a multiple of 32 columns
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = v[j] + b[j];
      round_bf16_inplace(v);
      const int row = tc.out_row + et.r;
      const bool valid = et.r < tc.rows;
      if (c0 < p.policy_size) {
#pragma unroll
        for (int j = 0; j < 32; ++j) tbuf[lane * kPitch + j] = v[j];
        __syncwarp();
        const bool col_ok = c0 + lane < p.policy_size;
        for (int rr = 0; rr < 32; ++rr) {
          if (col_ok && (et.r & ~31) + rr < tc.rows) {
            p.policy[static_cast<size_t>(row0 + rr) * p.policy_size + c0 + lane] =
                tbuf[rr * kPitch + lane];
          }
        }
        __syncwarp();
      } else if (c0 == p.policy_storage && valid) {
        float* w = p.wdl + static_cast<size_t>(row) * 3;
        if (p.wdl_probs) {
          const float mx = fmaxf(fmaxf(v[0], v[1]), v[2]);
          const float e0 = expf(v[0] - mx), e1 = expf(v[1] - mx), e2 = expf(v[2] - mx);
          const float total = e0 + e1 + e2;
          w[0] = e0 / total;
          w[1] = e1 / total;
          w[2] = e2 / total;
        } else {
          w[0] = v[0];
          w[1] = v[1];
          w[2] = v[2];
        }
      } else if (c0 == p.policy_storage + 32 && valid) {
        p.moves_left[row] = v[0];
      }
    }
    release_accumulator(ctx);
  }
};

// ------------------------------------------------------------------ MoE epilogues

// Top-2 routing of one token from its 64 router logits (BF16 values held as FP32):
// experts = the two largest (logit - beta), the lower expert index winning ties;
// weights = FP32 softmax over all 64 raw logits at those experts, rounded to BF16
// (src/chess_engine_4/model/moe.py:160-177; tie rule of the reference runtime's router).
__device__ __forceinline__ void route_top2(const float (&lo)[32], const float (&hi)[32],
                                           const float* __restrict__ beta, int& e0, int& e1,
                                           float& p0, float& p1) {
  float mx = -INFINITY;
#pragma unroll
  for (int e = 0; e < 32; ++e) mx = fmaxf(mx, fmaxf(lo[e], hi[e]));
  float denom = 0.0f, s0 = -INFINITY, s1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  e0 = 0;
  e1 = 1;
#pragma unroll
  for (int e = 0; e < 64; ++e) {
    const float l = e < 32 ? lo[e] : hi[e - 32];
    const float s = l - __ldg(beta + e);
    denom += expf(l - mx);
    if (s > s0) {
      s1 = s0;
      e1 = e0;
      l1 = l0;
      s0 = s;
      e0 = e;
      l0 = l;
    } else if (s > s1) {
      s1 = s;
      e1 = e;
      l1 = l;
    }
  }
  p0 = bf16_round(expf(l0 - mx) / denom);
  p1 = bf16_round(expf(l1 - mx) / denom);
}

// Router epilogue over a [tokens, 64] logit tile (BN = 64). One thread per token routes it;
// each CTA writes the expert histogram of its 128 tokens to block_hist[tile] so that the
// scan can place every route deterministically (stable by token).
struct EpiRouter {
  static constexpr int kSmemBytes = 64 * 4;
  struct Params {
    const float* beta;   // [64]
    int2* route_expert;  // [T]
    float2* route_prob;  // [T] (BF16-rounded values)
    int* block_hist;     // [T/128 tiles][64]
    __nv_bfloat16* logits;  // [T, 64] the BF16 logits the selection used (nullptr: not stored)
  };
  __device__ static uint32_t bar_count(const Params&, int) { return 1; }
  __device__ static bool prefetch(const Params&, const TileCoord&, const CUtensorMap*, uint32_t,
                                  uint32_t) {
    return false;
  }
  template <int G>
  __device__ static void run(const Params& p, const TileCoord& tc, const EpiThread& et,
                             const EpiCtx& ctx) {
    int* hist = reinterpret_cast<int*>(ctx.smem_ptr);
    if (ctx.iter > 0) epi_bar_sync<G>();  // previous tile's histogram has been written out
    if (et.tid < 64) hist[et.tid] = 0;
    epi_bar_sync<G>();
    if (et.g == 0) {
      float lo[32], hi[32];
      load_acc32x2(et.taddr, et.taddr + 32, lo, hi);
      round_bf16_inplace(lo);
      round_bf16_inplace(hi);
      int e0, e1;
      float p0, p1;
      route_top2(lo, hi, p.beta, e0, e1, p0, p1);
      if (et.r < tc.rows) {
        const int row = tc.out_row + et.r;
        p.route_expert[row] = make_int2(e0, e1);
        p.route_prob[row] = make_float2(p0, p1);
        if (p.logits != nullptr) {
          uint4* dst = reinterpret_cast<uint4*>(p.logits + static_cast<size_t>(row) * 64);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            dst[u] = make_uint4(pack_bf16x2(lo[8 * u], lo[8 * u + 1]), pack_bf16x2(lo[8 * u + 2], lo[8 * u + 3]),
                                pack_bf16x2(lo[8 * u + 4], lo[8 * u + 5]), pack_bf16x2(lo[8 * u + 6], lo[8 * u + 7]));
            dst[4 + u] = make_uint4(pack_bf16x2(hi[8 * u], hi[8 * u + 1]), pack_bf16x2(hi[8 * u + 2], hi[8 * u + 3]),
                                    pack_bf16x2(hi[8 * u + 4], hi[8 * u + 5]), pack_bf16x2(hi[8 * u + 6], hi[8 * u + 7]));
          }
        }
        atomicAdd(&hist[e0], 1);
        atomicAdd(&hist[e1], 1);
      }
    }
    release_accumulator(ctx);
    epi_bar_sync<G>();
    if (et.tid < 64) p.block_hist[(tc.a_row / kBM) * 64 + et.tid] = hist[et.tid];
  }
};

// Expert down-projection epilogue: y = bf16(acc * prob[row]) for the permuted rows of one
// expert segment, staged and TMA-stored through tmO1 (the probability scales the FP32
// accumulator, as the reference's expert kernels do).
template <int BN>
struct EpiScaleStore {
  static_assert(BN % 64 == 0, "64-column boxes");
  // The output is staged at most 128 columns at a time (32 KB), leaving the shared memory
  // of a fourth operand stage to a 256-column tile.
  static constexpr int kPart = BN < 128 ? BN : 128;
  static constexpr int kSmemBytes = kBM * kPart * 2;
  struct Params {
    const float* row_scale;  // [rows] per permuted row
  };
  __device__ static uint32_t bar_count(const Params&, int) { return 1; }
  __device__ static bool prefetch(const Params&, const TileCoord&, const CUtensorMap*, uint32_t,
                                  uint32_t) {
    return false;
  }
  template <int G>
  __device__ static void run(const Params& p, const TileCoord& tc, const EpiThread& et,
                             const EpiCtx& ctx) {
    if (ctx.iter > 0) {
      if (et.tid == 0) bulk_wait_read_all();
      epi_bar_sync<G>();
    }
    const float scale = et.r < tc.rows ? __ldg(p.row_scale + tc.out_row + et.r) : 0.0f;
    for (int c0 = 0; c0 < BN; c0 += kPart) {
      if (c0 > 0) {
        if (et.tid == 0) bulk_wait_read_all();  // the previous part's store has read the staging
        epi_bar_sync<G>();
      }
      for (int c = et.g * 32; c < kPart; c += G * 32) {
        float v[32];
        load_acc32(et.taddr + c0 + c, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] *= scale;
        stage_bf16x32(ctx.smem, et.r, c, v);
      }
      if (c0 + kPart >= BN) release_accumulator(ctx);
      fence_proxy_async_smem();
      epi_bar_sync<G>();
      if (et.tid == 0) store_staged(ctx.tmO1, ctx.smem, kPart, tc.n_tile * BN + c0, tc.out_row);
    }
  }
};

}  // namespace ce4b
