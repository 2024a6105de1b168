// Persistent forward of the dense SwiGLU tower in one launch (sm_100a).
//
// The reference runs the tower as a chain of GEMM and element-wise launches per layer
// (kernels/src/inference/runtime.cu:578-645; src/chess_engine_4/model/dense.py:112-125,
// 188-199). At inference batch sizes every layer is only a few microseconds of tensor-core
// work, so a launch per GEMM pays its prologue, first-load latency, wave quantisation and
// last epilogue every time. Here one persistent CTA per SM takes tiles from a global task
// counter in dependency order and runs them on the same warp-specialised pipeline as the
// single-GEMM kernels (warp 0: TMA producer, warp 1: tcgen05.mma issuer, 16 epilogue
// warps; two accumulators so one tile's epilogue overlaps the next tile's MMAs):
//
//   input tile   (rb, j, s): x[rb, j] = bf16((P_0 + P_1 + ...) + b), P_s = A_in . W_in^T over
//                            K part s of kis; every part stores FP32 P_s and the part that
//                            checks in last sums them in index order (the same whichever
//                            finishes last)
//   gate_up tile (l, rb, c): hidden[rb, c] = bf16(silu(bf16(r * x W'_g^T)) * bf16(r * x W'_u^T))
//   down tile    (l, rb, j): x[rb, j] = bf16(x + bf16(hidden . W_d^T)).
//
// Tiles are 128 rows; gate_up tiles are 256 accumulator columns (128 gate + 128 up, one
// 128-column hidden chunk). Input tiles are 256 columns of x where d allows, split into two
// K halves (K = 7168 is the longest loop of the forward; halving it shortens the first
// step of every row block's chain and keeps all SMs busy at the start). Down tiles are xw
// columns of x, chosen per forward:
// 128 when a layer's down tiles fill less than two waves of SMs (the dependency chain of
// each row block bounds the forward, and narrower tiles give it more SMs), 256 otherwise
// (throughput bounds it, and a 128-column tile fed by TMA runs at half the MMA rate). The
// width changes which CTA computes which columns, not the arithmetic.
//
// RMSNorm is folded: W' = bf16(W * diag(norm weight)) is prepared once, and the row scale
// r = rsqrt(mean(x^2) + eps) multiplies the FP32 accumulator of the gate_up tile, so
// r * (x W'^T) = (x * r * w) W^T without a separate pass over x. (The reference rounds the
// normalised row n = bf16(x * r * w) before its GEMM; here the rounding sits on W' instead.
// Each x slice tile stores per-(row, column group) sums of squares of its BF16 outputs;
// r sums them in slice, group order.)
//
// Tasks are numbered input tiles first, then per layer all gate_up tiles and all down
// tiles, each row-block-major. A CTA only ever waits on tasks with smaller numbers, which
// running CTAs already hold, so the schedule cannot deadlock. Row block rb's dependencies
// are counters in global memory: slice_cnt[rb] (finished 128-column x slices) and
// hid_cnt[rb] (finished gate_up tiles). Tiles are written by TMA stores from a staging
// tile; the store warp waits for a tile's stores to complete, then issues a proxy fence, a
// GPU-scope acq_rel fence and a relaxed increment. Readers acquire the counter and issue a
// proxy fence before TMA reads the data. Every wait is bounded (a timed-out wait records an
// error code and its role stops; the epilogue warps stop together).
#pragma once

#include "forward_types.h"
#include "gemm.cuh"

namespace ce4b {

struct FwdTask {
  int type;
  int layer;
  int rb;
  int col;  // hidden chunk (gate_up), x tile of width xwi (input) or xw (down)
  int kh;   // K part (input, of kis; down, of dks)
};

__device__ __forceinline__ FwdTask fwd_decode(const FwdParams& p, int t) {
  FwdTask k{kTaskEnd, 0, 0, 0, 0};
  if (t < 0 || t >= p.total_tasks) return k;
  const int n_in = p.nb * p.xti * p.kis;
  if (t < n_in) {
    k.type = kTaskInput;
    k.rb = t / (p.xti * p.kis);
    const int rem = t - k.rb * (p.xti * p.kis);
    k.col = rem / p.kis;
    k.kh = rem - k.col * p.kis;
    return k;
  }
  t -= n_in;
  const int per_layer = p.nb * (p.nc + p.xt * p.dks);
  k.layer = t / per_layer;
  if (k.layer >= p.depth) {
    t -= p.depth * per_layer;
    k.type = kTaskHeads;
    k.layer = p.depth;
    k.rb = t / p.nht;
    k.col = t - k.rb * p.nht;
    return k;
  }
  t -= k.layer * per_layer;
  // Within a layer: the gate_up tiles of row block i, followed by the down tiles of row block
  // i - lag (lag = nb: every gate_up tile of the layer first, then every down tile).
  const int per_dn = p.xt * p.dks;
  const int lag = p.lag;
  int i, r;
  bool gu;
  if (t < lag * p.nc) {
    i = t / p.nc;
    r = t - i * p.nc;
    gu = true;
  } else if (t < lag * p.nc + (p.nb - lag) * (p.nc + per_dn)) {
    const int u = t - lag * p.nc;
    i = lag + u / (p.nc + per_dn);
    r = u - (i - lag) * (p.nc + per_dn);
    gu = r < p.nc;
    if (!gu) r -= p.nc;
  } else {
    const int u = t - lag * p.nc - (p.nb - lag) * (p.nc + per_dn);
    i = p.nb + u / per_dn;
    r = u - (i - p.nb) * per_dn;
    gu = false;
  }
  if (gu) {
    k.type = kTaskGateUp;
    k.rb = i;
    k.col = r;
  } else {
    k.type = kTaskDown;
    k.rb = i - lag;
    k.col = r / p.dks;
    k.kh = r - k.col * p.dks;
  }
  return k;
}

// ------------------------------------------------------------------ global synchronisation
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* ptr, int v) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], %2;" : "=r"(old) : "l"(ptr), "r"(v)
               : "memory");
  return old;
}

__device__ __forceinline__ void fwd_stamp(const FwdParams& p, int t, int slot) {
  if (p.trace != nullptr && t < p.trace_cap) {
    p.trace[static_cast<size_t>(t) * kFwdTraceWords + slot] = global_timer_ns();
  }
}

__device__ __forceinline__ void fwd_epi_sync() { named_bar_sync(kEpiBarrierId, kFwdEpiThreads); }

// Epilogue barrier that ORs the threads' `failed` flags (a timed-out wait): all epilogue
// threads reach the same barriers and take the same decision to stop.
__device__ __forceinline__ bool fwd_epi_sync_or(bool failed) {
  return named_bar_or(kEpiBarrierId, kFwdEpiThreads, failed);
}

// ------------------------------------------------------------------ epilogues
// Publishing: all epilogue threads store, pass the epilogue barrier, then one thread
// issues a GPU-scope acq_rel fence (which also releases the other threads' stores made
// before the barrier) and the counter update.
__device__ __forceinline__ void fence_acq_rel_gpu() {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

__device__ __forceinline__ void red_add_relaxed_gpu(int* ptr, int v) {
  asm volatile("red.relaxed.gpu.global.add.s32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

// Row scale r = rsqrt(mean(x^2) + eps) of one row from the sums of squares its x slices
// published (slice-major, column-group-minor, the order of the cluster-exchange epilogue).
__device__ __forceinline__ float fwd_row_scale(const FwdParams& p, int row) {
  const float4* ss = reinterpret_cast<const float4*>(p.ss + static_cast<size_t>(row) * p.sj * kFwdG);
  float total = 0.0f;
  for (int q = 0; q < p.sj; q += 2) {
    const float4 a = __ldcg(ss + q);
    const float4 b = q + 1 < p.sj ? __ldcg(ss + q + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
    total += a.x;
    total += a.y;
    total += a.z;
    total += a.w;
    if (q + 1 < p.sj) {
      total += b.x;
      total += b.y;
      total += b.z;
      total += b.w;
    }
  }
  return 1.0f / sqrtf(total / static_cast<float>(p.d) + p.eps);
}

// ------------------------------------------------------------------ staged tile output
// Epilogues write their BF16 tiles through a 32 KB staging tile in shared memory (two
// 64-column TMA boxes of 128 rows, 128-byte swizzle: row r's 16-byte unit u sits at
// r * 128 + ((u ^ (r & 7)) * 16)). A thread owns one row and 32 consecutive columns, so
// writing global memory directly would touch 32 lines per warp instruction; the swizzled
// staging writes are conflict-free and the TMA store is fully coalesced. Down tiles also
// load their residual into the staging tile with TMA and overwrite it in place.
//
// A store warp takes each filled staging tile (stage_full, with a job record: tensor map,
// coordinates, counter to publish), issues its TMA store, returns the buffer as soon as
// the store has read it (stage_free), then waits for the store to complete and publishes.
// The epilogue warps go on to the next tile meanwhile.
struct FwdEpi {
  uint32_t stage;      // staging tile
  uint32_t x_bar;      // mbarrier of the residual load into the staging tile
  uint32_t full_bar;   // stage_full (count 1: epilogue thread 0)
  uint32_t free_bar;   // stage_free (count 1: the store thread)
  uint32_t x_phase;    // parity of x_bar's next phase
  uint32_t uses;       // staging tiles handed over so far
  int r, g, tid;       // row in the tile, 32-column group, epilogue thread index
  bool x_pending;      // (thread 0) a residual load was issued and not yet waited for
  volatile int* job;   // job record: map, x0, y0, counter kind, row block, increment, task
};

// kStoreNone: nothing to store (the staging tile was used and read back by the epilogue
// itself); the store warp only frees the tile.
enum FwdStoreMap : int { kStoreStop = -1, kStoreHidden = 0, kStoreX = 1, kStoreNone = 2 };
enum FwdCounter : int { kCounterNone = 0, kCounterHidden = 1, kCounterSlice = 2 };

// All epilogue threads: wait until the store warp has read the staging tile of the
// previous hand-over. Returns true on a timed-out wait.
__device__ __forceinline__ bool fwd_stage_acquire(FwdEpi& e, bool failed) {
  const bool f = failed || !mbar_wait(e.free_bar, (e.uses & 1u) ^ 1u);
  return f;
}

// Epilogue thread 0, after the barrier that follows the staging writes: hand the tile to
// the store warp.
__device__ __forceinline__ void fwd_stage_post(FwdEpi& e, int map, int x0, int y0, int counter, int rb,
                                               int inc, int t) {
  e.job[0] = map;
  e.job[1] = x0;
  e.job[2] = y0;
  e.job[3] = counter;
  e.job[4] = rb;
  e.job[5] = inc;
  e.job[6] = t;
  mbar_arrive(e.full_bar);
}

__device__ __forceinline__ uint32_t fwd_stage_addr(uint32_t stage, int r, int c) {
  return stage + static_cast<uint32_t>((c >> 6) * 16384 + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4));
}

__device__ __forceinline__ void fwd_stage_write32(uint32_t stage, int r, int c, const float (&v)[32]) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    st_shared_v4(fwd_stage_addr(stage, r, c + 8 * u),
                 make_uint4(pack_bf16x2(v[8 * u], v[8 * u + 1]), pack_bf16x2(v[8 * u + 2], v[8 * u + 3]),
                            pack_bf16x2(v[8 * u + 4], v[8 * u + 5]), pack_bf16x2(v[8 * u + 6], v[8 * u + 7])));
  }
}

// Load columns [x0, x0 + 128) of rows [y0, y0 + 128) into the staging tile.
__device__ __forceinline__ void fwd_stage_load(const CUtensorMap* map, uint32_t stage, uint32_t bar, int x0,
                                               int y0) {
  mbar_arrive_expect_tx(bar, 32768);
  tma_load_2d(stage, map, bar, x0, y0);
  tma_load_2d(stage + 16384, map, bar, x0 + 64, y0);
}

// Sum of squares of 32 finished BF16 values of x, stored per (row, 128-column slice,
// 32-column group): the layout the row scale reads.
__device__ __forceinline__ void fwd_store_ss32(const FwdParams& p, int row, int col0, const float (&v)[32]) {
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; ++j) ss = fmaf(v[j], v[j], ss);
  p.ss[static_cast<size_t>(row) * (p.sj * kFwdG) + (col0 >> 7) * kFwdG + ((col0 & 127) >> 5)] = ss;
}

__device__ __forceinline__ void fwd_add_bf16x32(float (&v)[32], const uint4 (&w)[4], bool acc_first) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t wq[4] = {w[q].x, w[q].y, w[q].z, w[q].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(wq[j]);
      v[8 * q + 2 * j] = acc_first ? v[8 * q + 2 * j] + f.x : f.x + v[8 * q + 2 * j];
      v[8 * q + 2 * j + 1] = acc_first ? v[8 * q + 2 * j + 1] + f.y : f.y + v[8 * q + 2 * j + 1];
    }
  }
}

// Each epilogue returns true when some epilogue thread's wait timed out (`failed`): a
// failed thread skips the work but reaches the same barriers, and nothing is published.

// gate_up tile: accumulator columns [0, 128) gate, [128, 256) up; A was the raw x, and
// `scale` is the row's RMSNorm scale.
__device__ __forceinline__ bool fwd_epi_gate_up(const FwdParams& p, const FwdTask& k, int t, FwdEpi& e,
                                                uint32_t taddr, uint32_t tempty, float scale, bool failed) {
  const int c = e.g * 32;
  float gv[32];
  if (!failed) {
    float uv[32];
    load_acc32x2(taddr + c, taddr + 128 + c, gv, uv);
    tc_fence_before();
    mbar_arrive(tempty);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      gv[j] = __fmul_rn(gv[j], scale);
      uv[j] = __fmul_rn(uv[j], scale);
    }
    round_bf16_inplace(gv);
    round_bf16_inplace(uv);
#pragma unroll
    for (int j = 0; j < 32; ++j) gv[j] = swiglu_f32(gv[j], uv[j]);
  }
  failed = fwd_stage_acquire(e, failed);
  if (!failed) {
    fwd_stage_write32(e.stage, e.r, c, gv);
    fence_proxy_async_smem();
  }
  if (fwd_epi_sync_or(failed)) return true;
  if (e.tid == 0) {
    fwd_stamp(p, t, 7);
    fwd_stage_post(e, kStoreHidden, k.col * 128, k.rb * kBM, kCounterHidden, k.rb, 1, t);
  }
  ++e.uses;
  return false;
}

// Down tile, xw columns, in 128-column halves: x = bf16(x + bf16(acc)) on the residual the
// staging tile holds (half 0 was loaded when the task started), stored with its sums of
// squares; then the tile publishes the xw / 128 slices it covers.
__device__ __forceinline__ bool fwd_epi_down(const FwdParams& p, const FwdTask& k, int t, FwdEpi& e,
                                             uint32_t taddr, uint32_t tempty, bool failed) {
  const int row = k.rb * kBM + e.r;
  const int nh = p.xw / 128;
  for (int h = 0; h < nh; ++h) {
    const int x0 = k.col * p.xw + h * 128;
    bool f = failed;
    if (h > 0) {
      // Half 0 was handed over: wait for the buffer, then load this half's residual.
      f = fwd_stage_acquire(e, f);
      if (e.tid == 0 && !f) {
        fence_proxy_async_global();
        fwd_stage_load(&p.maps->x, e.stage, e.x_bar, x0, k.rb * kBM);
        e.x_pending = true;
      }
    }
    f = f || !mbar_wait(e.x_bar, e.x_phase);
    if (!f) e.x_pending = false;
    if (!f || !e.x_pending) e.x_phase ^= 1u;  // a load still in flight keeps its phase
    if (!f) {
      float v[32];
      load_acc32(taddr + h * 128 + e.g * 32, v);
      if (h == nh - 1) {
        tc_fence_before();
        mbar_arrive(tempty);
      }
      round_bf16_inplace(v);
      uint4 res[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) res[u] = ld_shared_v4(fwd_stage_addr(e.stage, e.r, e.g * 32 + 8 * u));
      fwd_add_bf16x32(v, res, false);  // residual + bf16(acc)
      round_bf16_inplace(v);
      fwd_store_ss32(p, row, x0 + e.g * 32, v);
      fwd_stage_write32(e.stage, e.r, e.g * 32, v);
      fence_proxy_async_smem();
    }
    if (fwd_epi_sync_or(f)) return true;
    if (e.tid == 0) {
      if (h == nh - 1) fwd_stamp(p, t, 7);
      fwd_stage_post(e, kStoreX, x0, k.rb * kBM, h == nh - 1 ? kCounterSlice : kCounterNone, k.rb, nh, t);
    }
    ++e.uses;
  }
  return false;
}

// K-part partial sums of an input or down tile (`width` columns, `tiles` tiles per row
// block, `parts` K parts) are stored in epilogue-thread order (128-column half h, float4
// index q, thread) so that every warp access covers 512 contiguous bytes; all parts use the
// same thread mapping, so each thread reads back exactly its own fragments. A row block's
// region holds part_rb_chunks = (d / 128) * max(kis, dks) chunks of 64 KB, enough for
// either tile kind; its input tiles have finished before its first down tile starts, so
// both share the buffer.
__device__ __forceinline__ float4* fwd_part_frag(const FwdParams& p, int rb, int col, int tiles, int width,
                                                 int parts, int kh, int h, int tid) {
  (void)tiles;
  const size_t chunk = static_cast<size_t>(rb) * p.part_rb_chunks +
                       ((static_cast<size_t>(col) * parts + kh) * (width / 128) + h);
  return reinterpret_cast<float4*>(p.part) + chunk * (8 * kFwdEpiThreads) + tid;
}

// Store a thread's 32 FP32 sums of K part kh.
__device__ __forceinline__ void fwd_part_store(float4* dst, const float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) dst[q * kFwdEpiThreads] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}

// Sum of all K parts of a thread's 32 columns, in part order (whichever part finished last).
__device__ __forceinline__ void fwd_part_sum(const FwdParams& p, int rb, int col, int tiles, int width,
                                             int parts, int h, int tid, float (&v)[32]) {
  const float4* src = fwd_part_frag(p, rb, col, tiles, width, parts, 0, h, tid);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 a = __ldcg(src + q * kFwdEpiThreads);
    v[4 * q] = a.x;
    v[4 * q + 1] = a.y;
    v[4 * q + 2] = a.z;
    v[4 * q + 3] = a.w;
  }
  const size_t part_stride = static_cast<size_t>(width / 128) * 8 * kFwdEpiThreads;  // float4s
#pragma unroll 1
  for (int s = 1; s < parts; ++s) {
    src += part_stride;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 a = __ldcg(src + q * kFwdEpiThreads);
      v[4 * q] += a.x;
      v[4 * q + 1] += a.y;
      v[4 * q + 2] += a.z;
      v[4 * q + 3] += a.w;
    }
  }
}

// Input tile K part: stores its FP32 sums; the part that checks in last reads all parts
// back, adds them in part order, then the bias (TE's fused bias), and finishes and
// publishes the x tile.
__device__ __forceinline__ bool fwd_epi_input(const FwdParams& p, const FwdTask& k, int t, FwdEpi& e,
                                              uint32_t taddr, uint32_t tempty, volatile int* flag,
                                              bool failed) {
  const int row = k.rb * kBM + e.r;
  const int nh = p.xwi / 128;
  for (int h = 0; h < nh && !failed; ++h) {
    float v[32];
    load_acc32(taddr + h * 128 + e.g * 32, v);
    if (h == nh - 1) {
      tc_fence_before();
      mbar_arrive(tempty);
    }
    fwd_part_store(fwd_part_frag(p, k.rb, k.col, p.xti, p.xwi, p.kis, k.kh, h, e.tid), v);
  }
  if (fwd_epi_sync_or(failed)) return true;
  if (e.tid == 0) {
    fence_acq_rel_gpu();
    const int old = atom_add_acq_rel_gpu(p.part_cnt + k.rb * p.xti + k.col, 1);
    *flag = old == p.kis - 1;
  }
  fwd_epi_sync();
  if (*flag == 0) return false;
  for (int h = 0; h < nh; ++h) {
    const int col0 = k.col * p.xwi + h * 128 + e.g * 32;
    float v[32];
    fwd_part_sum(p, k.rb, k.col, p.xti, p.xwi, p.kis, h, e.tid, v);
    uint4 bias[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) bias[q] = *reinterpret_cast<const uint4*>(p.bias + col0 + 8 * q);
    fwd_add_bf16x32(v, bias, true);
    round_bf16_inplace(v);
    fwd_store_ss32(p, row, col0, v);
    const bool f = fwd_stage_acquire(e, false);
    if (!f) {
      fwd_stage_write32(e.stage, e.r, e.g * 32, v);
      fence_proxy_async_smem();
    }
    if (fwd_epi_sync_or(f)) return true;
    if (e.tid == 0) {
      if (h == nh - 1) fwd_stamp(p, t, 7);
      fwd_stage_post(e, kStoreX, k.col * p.xwi + h * 128, k.rb * kBM,
                     h == nh - 1 ? kCounterSlice : kCounterNone, k.rb, nh, t);
    }
    ++e.uses;
  }
  return false;
}

// Down tile (128 columns) with its K split in dks parts (small batches): each part stores
// its FP32 sums; the part that checks in last adds all parts in part order and finishes
// the tile like an unsplit one. The residual was loaded into the staging tile when the
// task started (for every part, so that all parts keep the same barrier sequence).
__device__ __forceinline__ bool fwd_epi_down_split(const FwdParams& p, const FwdTask& k, int t, FwdEpi& e,
                                                   uint32_t taddr, uint32_t tempty, volatile int* flag,
                                                   bool failed) {
  const int row = k.rb * kBM + e.r;
  if (!failed) {
    float v[32];
    load_acc32(taddr + e.g * 32, v);
    tc_fence_before();
    mbar_arrive(tempty);
    fwd_part_store(fwd_part_frag(p, k.rb, k.col, p.xt, 128, p.dks, k.kh, 0, e.tid), v);
  }
  if (fwd_epi_sync_or(failed)) return true;
  if (e.tid == 0) {
    fence_acq_rel_gpu();
    const int old = atom_add_acq_rel_gpu(p.dpart_cnt + k.rb * p.xt + k.col, 1);
    *flag = old % p.dks == p.dks - 1;  // dks check-ins a layer: the last one finishes
  }
  fwd_epi_sync();
  const bool last = *flag != 0;
  // The residual load lands whichever part this is.
  bool f = !mbar_wait(e.x_bar, e.x_phase);
  if (!f) e.x_pending = false;
  if (!f || !e.x_pending) e.x_phase ^= 1u;
  if (!last) return fwd_epi_sync_or(f);
  if (!f) {
    float v[32];
    fwd_part_sum(p, k.rb, k.col, p.xt, 128, p.dks, 0, e.tid, v);
    round_bf16_inplace(v);
    uint4 res[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) res[u] = ld_shared_v4(fwd_stage_addr(e.stage, e.r, e.g * 32 + 8 * u));
    fwd_add_bf16x32(v, res, false);  // residual + bf16(acc)
    round_bf16_inplace(v);
    fwd_store_ss32(p, row, k.col * 128 + e.g * 32, v);
    fwd_stage_write32(e.stage, e.r, e.g * 32, v);
    fence_proxy_async_smem();
  }
  if (fwd_epi_sync_or(f)) return true;
  if (e.tid == 0) {
    fwd_stamp(p, t, 7);
    fwd_stage_post(e, kStoreX, k.col * 128, k.rb * kBM, kCounterSlice, k.rb, 1, t);
  }
  ++e.uses;
  return false;
}

// Heads tile: accumulator columns [0, 256) are head columns col * 256 + [0, 256) of the
// folded [policy | wdl | moves-left] matrix; thread (r, g) reads columns g * 32 and
// 128 + g * 32. Logits = bf16(acc * r + bias) with r the final RMSNorm scale (the norm
// weight is folded into the matrix), as the heads GEMM computes them
// (src/chess_engine_4/model/dense.py:167-199; kernels/src/inference/runtime.cu:630-643).
// Policy columns leave as FP32: each warp transposes its 32 rows x 32 columns through its
// own 2 KB of the staging tile, 16 rows at a time, and stores each row's 32 values with one
// coalesced instruction. The WDL (softmax or logits) and moves-left columns are written by
// the threads that hold them.
__device__ __forceinline__ bool fwd_epi_heads(const FwdParams& p, const FwdTask& k, int t, FwdEpi& e,
                                              uint32_t taddr, uint32_t tempty, float scale, bool failed) {
  const int row = k.rb * kBM + e.r;
  const int lane = e.tid & 31;
  const int row0 = k.rb * kBM + (e.r & ~31);  // first row of this warp
  const uint32_t area = e.stage + static_cast<uint32_t>((e.tid >> 5) * 2048);
  failed = fwd_stage_acquire(e, failed);
  if (!failed) {
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
      const int c = h * 128 + e.g * 32;
      const int c0 = k.col * 256 + c;  // uniform across the warp
      if (c0 >= p.head_cols) continue;
      float v[32];
      {
        float b[32];
        load_acc32(taddr + c, v);
        load_bf16<32>(p.head_bias + c0, b);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(__fmul_rn(v[j], scale), b[j]);
        round_bf16_inplace(v);
      }
      if (c0 == p.policy_storage) {
        if (row < p.batch) {
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
        }
        continue;
      }
      if (c0 == p.policy_storage + 32) {
        if (row < p.batch) p.moves_left[row] = v[0];
        continue;
      }
      if (c0 >= p.policy_size) continue;
      // 16 rows at a time: [16][32] FP32, 16-byte chunk q of row i at q ^ (i % 8).
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        if ((lane >> 4) == half) {
          const int i = lane & 15;
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            st_shared_v4(area + static_cast<uint32_t>(i * 128 + ((u ^ (i & 7)) << 4)),
                         make_uint4(__float_as_uint(v[4 * u]), __float_as_uint(v[4 * u + 1]),
                                    __float_as_uint(v[4 * u + 2]), __float_as_uint(v[4 * u + 3])));
          }
        }
        __syncwarp();
        const bool col_ok = c0 + lane < p.policy_size;
#pragma unroll 4
        for (int i = 0; i < 16; ++i) {
          const int grow = row0 + half * 16 + i;
          const float val =
              ld_shared_f32(area + static_cast<uint32_t>(i * 128 + (((lane >> 2) ^ (i & 7)) << 4) + (lane & 3) * 4));
          if (col_ok && grow < p.batch) p.policy[static_cast<size_t>(grow) * p.policy_size + c0 + lane] = val;
        }
        __syncwarp();
      }
    }
    fence_proxy_async_smem();  // these generic accesses precede the tile's next TMA write
    tc_fence_before();
    mbar_arrive(tempty);
  }
  if (fwd_epi_sync_or(failed)) return true;
  if (e.tid == 0) {
    fwd_stamp(p, t, 7);
    fwd_stage_post(e, kStoreNone, 0, 0, kCounterNone, 0, 0, t);
  }
  ++e.uses;
  return false;
}

// ------------------------------------------------------------------ the kernel
struct FwdSmem {
  static constexpr int kABytes = kBM * kBK * 2;          // 16 KB
  static constexpr int kBBytesMax = 256 * kBK * 2;       // 32 KB (gate + up boxes)
  static constexpr int kStageBytes = kABytes + kBBytesMax;
  static constexpr int kRingBytes = kFwdNStage * kStageBytes;
  static constexpr int kOutBytes = kBM * 128 * 2;         // 32 KB staging tile
  // full[s], empty[s], tfull[2], tempty[2], task_full[q], task_empty[q], drain, x_bar,
  // stage_full, stage_free
  static constexpr int kBarriers = 2 * kFwdNStage + 4 + 2 * kFwdTaskRing + 4;
  static constexpr int kJobInts = 8;  // store job record
  static constexpr int kMiscBytes = kBarriers * 8 + kFwdTaskRing * 4 + 16 + kJobInts * 4;
  static constexpr int kBytes = 1024 + kRingBytes + kOutBytes + kMiscBytes;
  static_assert(kBytes <= 232448, "shared memory budget exceeded");
  static_assert(kFwdD96B1 + 128 * (kFwdDownStep - kBK) * 2 <= kStageBytes,
                "a 96-deep down stage must fit one ring stage");
};

__global__ void __launch_bounds__(kFwdThreads, 1) dense_forward_kernel(const FwdParams p) {
  using L = FwdSmem;
  extern __shared__ uint8_t smem_raw[];
  uint32_t base = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (base & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  base += pad;

  const uint32_t stage_out = base + L::kRingBytes;
  const uint32_t bar_base = stage_out + L::kOutBytes;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (kFwdNStage + s); };
  auto tfull_bar = [&](int a) { return bar_base + 8u * (2 * kFwdNStage + a); };
  auto tempty_bar = [&](int a) { return bar_base + 8u * (2 * kFwdNStage + 2 + a); };
  auto task_full = [&](int q) { return bar_base + 8u * (2 * kFwdNStage + 4 + q); };
  auto task_empty = [&](int q) { return bar_base + 8u * (2 * kFwdNStage + 4 + kFwdTaskRing + q); };
  const uint32_t drain_bar = bar_base + 8u * (L::kBarriers - 4);
  const uint32_t x_bar = bar_base + 8u * (L::kBarriers - 3);
  const uint32_t stage_full = bar_base + 8u * (L::kBarriers - 2);
  const uint32_t stage_free = bar_base + 8u * (L::kBarriers - 1);
  volatile int* task_slot =
      reinterpret_cast<volatile int*>(smem + L::kRingBytes + L::kOutBytes + L::kBarriers * 8);
  volatile int* flag = task_slot + kFwdTaskRing;  // input-tile check-in result
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(const_cast<int*>(flag + 1));
  volatile int* job = flag + 4;                   // store job record (kJobInts)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFwdNStage; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), kFwdEpiThreads);
    }
    for (int q = 0; q < kFwdTaskRing; ++q) {
      mbar_init(task_full(q), 1);
      mbar_init(task_empty(q), 1 + kFwdEpiThreads);
    }
    mbar_init(drain_bar, 1);
    mbar_init(x_bar, 1);
    mbar_init(stage_full, 1);
    mbar_init(stage_free, 1);
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
  // The prologue may overlap the previous kernel (the plane expansion); nothing global is
  // touched before it has completed.
  grid_dependency_wait();
  grid_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      const FwdMaps* maps = p.maps;
      tma_prefetch_desc(&maps->a_in);
      tma_prefetch_desc(&maps->x);
      tma_prefetch_desc(&maps->hidden);
      tma_prefetch_desc(&maps->hidden32);
      tma_prefetch_desc(&maps->w_in);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_phase = 0;
      bool ok = true;
      for (int i = 0; ok; ++i) {
        const int q = i % kFwdTaskRing;
        if (!mbar_wait(task_empty(q), ((i / kFwdTaskRing) & 1) ^ 1u)) {
          record_error(p.err, kErrTimeoutProducer);
          ok = false;
        }
        int t = ok ? atomicAdd(p.task_counter, 1) : -1;
        if (t >= p.total_tasks) t = -1;
        FwdTask k{kTaskEnd, 0, 0, 0};
        const CUtensorMap* ma = nullptr;
        const CUtensorMap* mb = nullptr;
        const CUtensorMap* mb32 = nullptr;  // 96-deep down stages: 32-wide B box
        bool d96 = false;
        int kb0 = 0, kb1 = 0, b_row = 0, b_row2 = -1;
        const int* dep = nullptr;  // counter the task's A operand waits for
        int dep_target = 0;
        if (t >= 0) {
          fwd_stamp(p, t, 0);
          if (p.trace != nullptr && t < p.trace_cap) {
            p.trace[static_cast<size_t>(t) * kFwdTraceWords + 10] = blockIdx.x;
          }
          k = fwd_decode(p, t);
          if (k.type == kTaskInput) {
            ma = &maps->a_in;
            mb = &maps->w_in;
            kb0 = k.kh * p.kb_in / p.kis;
            kb1 = (k.kh + 1) * p.kb_in / p.kis;
            b_row = k.col * p.xwi;
            if (p.xwi == 256) b_row2 = b_row + 128;
          } else if (k.type == kTaskGateUp) {
            dep = p.slice_cnt + k.rb;
            dep_target = (k.layer + 1) * p.sj;
            ma = &maps->x;
            mb = &maps->gate_up[k.layer];
            kb1 = p.d / kBK;
            b_row = k.col * 128;
            b_row2 = p.h + k.col * 128;
          } else if (k.type == kTaskHeads) {
            dep = p.slice_cnt + k.rb;
            dep_target = (p.depth + 1) * p.sj;
            ma = &maps->x;
            mb = &maps->heads;
            kb1 = p.d / kBK;
            b_row = k.col * 256;
            b_row2 = b_row + 128;
          } else {
            dep = p.hid_cnt + k.rb;
            dep_target = (k.layer + 1) * p.nc;
            ma = &maps->hidden;
            mb = &maps->down[k.layer];
            mb32 = &maps->down32[k.layer];
            d96 = p.d96 != 0 && p.xw == 128;
            const int steps = p.h / (d96 ? kFwdDownStep : kBK);
            kb0 = k.kh * steps / p.dks;
            kb1 = (k.kh + 1) * steps / p.dks;
            b_row = k.col * p.xw;
            if (p.xw == 256) b_row2 = b_row + 128;
          }
        }
        const uint32_t bytes =
            d96 ? 2u * 128u * kFwdDownStep * 2u : L::kABytes + (b_row2 >= 0 ? 2 : 1) * 128 * kBK * 2;
        // Weight (B) and activation (A) boxes of step kb into stage address sa.
        auto load_b = [&](uint32_t sa, uint32_t bar, int kb) {
          if (d96) {
            tma_load_2d(sa + kFwdD96B0, mb, bar, kb * kFwdDownStep, b_row);
            tma_load_2d(sa + kFwdD96B1, mb32, bar, kb * kFwdDownStep + kBK, b_row);
          } else {
            tma_load_2d(sa + L::kABytes, mb, bar, kb * kBK, b_row);
            if (b_row2 >= 0) tma_load_2d(sa + L::kABytes + 128 * kBK * 2, mb, bar, kb * kBK, b_row2);
          }
        };
        auto load_a = [&](uint32_t sa, uint32_t bar, int kb) {
          if (d96) {
            tma_load_2d(sa, ma, bar, kb * kFwdDownStep, k.rb * kBM);
            tma_load_2d(sa + kFwdD96A1, &maps->hidden32, bar, kb * kFwdDownStep + kBK, k.rb * kBM);
          } else {
            tma_load_2d(sa, ma, bar, kb * kBK, k.rb * kBM);
          }
        };
        // While the task's inputs are still being produced, its first k-blocks' weight (B)
        // boxes go into the stages that are already free; their A boxes follow once the
        // inputs are complete. (The stage's full barrier expects both.)
        int pre = 0;
        const int pre_stage = stage;
        if (dep != nullptr && ld_acquire_gpu(dep) < dep_target) {
          while (pre < kb1 - kb0 && pre < kFwdNStage && mbar_test_wait(empty_bar(stage), phase ^ 1u)) {
            mbar_arrive_expect_tx(full_bar(stage), bytes);
            load_b(base + stage * L::kStageBytes, full_bar(stage), kb0 + pre);
            issued_mask |= 1u << stage;
            issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
            if (++stage == kFwdNStage) {
              stage = 0;
              phase ^= 1u;
            }
            ++pre;
          }
          if (!wait_counter(dep, dep_target)) record_error(p.err, kErrTimeoutDependency);
        }
        // The task is published once its inputs are complete (the acquire above), so the
        // MMA thread and the epilogue warps may read its inputs as soon as they see it.
        task_slot[q] = t;
        mbar_arrive(task_full(q));
        if (t < 0) break;
        // Data written by other SMs' generic stores is read below by TMA (async proxy).
        fence_proxy_async_global();
        fwd_stamp(p, t, 1);
        for (int i = 0, st = pre_stage; i < pre; ++i, st = (st + 1) % kFwdNStage) {
          load_a(base + st * L::kStageBytes, full_bar(st), kb0 + i);
        }
        for (int kb = kb0 + pre; kb < kb1; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u)) {
            record_error(p.err, kErrTimeoutProducer);
            ok = false;
            break;
          }
          const uint32_t sa = base + stage * L::kStageBytes;
          mbar_arrive_expect_tx(full_bar(stage), bytes);
          load_a(sa, full_bar(stage), kb);
          load_b(sa, full_bar(stage), kb);
          issued_mask |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == kFwdNStage) {
            stage = 0;
            phase ^= 1u;
          }
        }
        fwd_stamp(p, t, 2);
      }
      if (!ok) {
        for (int s = 0; s < kFwdNStage; ++s) {
          if (issued_mask & (1u << s)) mbar_wait(full_bar(s), (issued_phase >> s) & 1u);
        }
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
      for (int i = 0; ok; ++i) {
        const int q = i % kFwdTaskRing;
        if (!mbar_wait(task_full(q), (i / kFwdTaskRing) & 1)) {
          record_error(p.err, kErrTimeoutMma);
          break;
        }
        const int t = task_slot[q];
        mbar_arrive(task_empty(q));
        if (t < 0) break;
        const FwdTask k = fwd_decode(p, t);
        const bool d96 = k.type == kTaskDown && p.d96 != 0 && p.xw == 128;
        const int kbh = p.h / (d96 ? kFwdDownStep : kBK);
        const int nkb = k.type == kTaskInput  ? (k.kh + 1) * p.kb_in / p.kis - k.kh * p.kb_in / p.kis
                        : k.type == kTaskDown ? (k.kh + 1) * kbh / p.dks - k.kh * kbh / p.dks
                                              : p.d / kBK;
        const int n_mma = (k.type == kTaskGateUp || k.type == kTaskHeads) ? 256
                          : (k.type == kTaskInput ? p.xwi : p.xw);
        const uint32_t idesc = idesc_bf16(kBM, n_mma);
        if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u)) {
          record_error(p.err, kErrTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * 256);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(full_bar(stage), phase)) {
            record_error(p.err, kErrTimeoutMma);
            ok = false;
            break;
          }
          // Operands landed by TMA: the stage barrier orders the MMAs after them (no
          // tcgen05 fence; it is needed only where TMEM changes hands between threads).
          if (kb == 0) fwd_stamp(p, t, 3);
          const uint32_t sa = base + stage * L::kStageBytes;
          if (d96) {
            const uint64_t adesc = sdesc_k128(sa), bdesc = sdesc_k128(sa + kFwdD96B0);
            const uint64_t adesc1 = sdesc_k64(sa + kFwdD96A1), bdesc1 = sdesc_k64(sa + kFwdD96B1);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              umma_bf16(d_tmem, adesc + 2u * kk, bdesc + 2u * kk, idesc, (kb | kk) != 0 ? 1u : 0u);
            }
#pragma unroll
            for (int kk = 0; kk < (kFwdDownStep - kBK) / 16; ++kk) {
              umma_bf16(d_tmem, adesc1 + 2u * kk, bdesc1 + 2u * kk, idesc, 1u);
            }
          } else {
            const uint64_t adesc = sdesc_k128(sa);
            const uint64_t bdesc = sdesc_k128(sa + L::kABytes);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              umma_bf16(d_tmem, adesc + 2u * kk, bdesc + 2u * kk, idesc, (kb | kk) != 0 ? 1u : 0u);
            }
          }
          umma_commit(empty_bar(stage));
          if (++stage == kFwdNStage) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(tfull_bar(acc));
        fwd_stamp(p, t, 4);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      umma_commit(drain_bar);
      if (!mbar_wait(drain_bar, 0)) record_error(p.err, kErrTimeoutDrain);
    }
    __syncwarp();
  } else if (warp < kFwdStoreWarp) {
    const int quarter = warp & 3;
    FwdEpi e{stage_out, x_bar, stage_full, stage_free, 0u, 0u, quarter * 32 + lane, (warp - 2) >> 2,
             static_cast<int>(threadIdx.x) - 64, false, job};
    const FwdMaps* maps = p.maps;
    int acc = 0;
    uint32_t acc_phase = 0;
    // Every epilogue thread takes the same branches and barriers; a timed-out wait is
    // ORed into the next barrier, after which all epilogue threads stop together.
    for (int i = 0;; ++i) {
      const int q = i % kFwdTaskRing;
      bool failed = !mbar_wait(task_full(q), (i / kFwdTaskRing) & 1);
      const int t = failed ? -1 : task_slot[q];
      if (!failed) mbar_arrive(task_empty(q));
      if (fwd_epi_sync_or(failed)) {
        record_error(p.err, kErrTimeoutEpilogue);
        break;
      }
      if (t < 0) break;
      const FwdTask k = fwd_decode(p, t);
      // Global inputs of the epilogue, fetched while the MMAs run (the producer published
      // the task after its dependencies completed): the row scale, or the first 128
      // columns of the residual into the staging tile once the previous store read it.
      float scale = 1.0f;
      if (k.type == kTaskGateUp || k.type == kTaskHeads) {
        scale = fwd_row_scale(p, k.rb * kBM + e.r);
      } else if (k.type == kTaskDown) {
        failed = fwd_stage_acquire(e, false);
        if (e.tid == 0 && !failed) {
          fence_proxy_async_global();
          fwd_stage_load(&maps->x, e.stage, e.x_bar, k.col * p.xw, k.rb * kBM);
          e.x_pending = true;
        }
      }
      failed = !mbar_wait(tfull_bar(acc), acc_phase) || failed;
      tc_fence_after();
      if (e.tid == 0) fwd_stamp(p, t, 5);
      const uint32_t taddr =
          tmem_base + static_cast<uint32_t>(acc * 256) + (static_cast<uint32_t>(quarter * 32) << 16);
      bool abort;
      if (k.type == kTaskGateUp) {
        abort = fwd_epi_gate_up(p, k, t, e, taddr, tempty_bar(acc), scale, failed);
      } else if (k.type == kTaskDown) {
        abort = p.dks > 1 ? fwd_epi_down_split(p, k, t, e, taddr, tempty_bar(acc), flag, failed)
                          : fwd_epi_down(p, k, t, e, taddr, tempty_bar(acc), failed);
      } else if (k.type == kTaskHeads) {
        abort = fwd_epi_heads(p, k, t, e, taddr, tempty_bar(acc), scale, failed);
      } else {
        abort = fwd_epi_input(p, k, t, e, taddr, tempty_bar(acc), flag, failed);
      }
      if (abort) {
        record_error(p.err, kErrTimeoutEpilogue);
        break;
      }
      if (e.tid == 0) fwd_stamp(p, t, 6);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // Stop the store warp once it has taken the last tile; a residual load issued for a
    // task that then timed out lands before the shared memory is released.
    if (e.tid == 0) {
      if (mbar_wait(e.free_bar, (e.uses & 1u) ^ 1u)) fwd_stage_post(e, kStoreStop, 0, 0, 0, 0, 0, -1);
      if (e.x_pending) mbar_wait(e.x_bar, e.x_phase);
    }
  } else if (warp == kFwdStoreWarp) {
    if (lane == 0) {
      const FwdMaps* maps = p.maps;
      for (uint32_t n = 0;; ++n) {
        if (!mbar_wait(stage_full, n & 1u)) {
          record_error(p.err, kErrTimeoutEpilogue);
          break;
        }
        const int map = job[0];
        if (map == kStoreStop) break;
        const int x0 = job[1], y0 = job[2], counter = job[3], rb = job[4], inc = job[5], t = job[6];
        fwd_stamp(p, t, 9);
        if (map == kStoreNone) {
          mbar_arrive(stage_free);
          continue;
        }
        const CUtensorMap* m = map == kStoreHidden ? &maps->hidden : &maps->x;
        tma_store_2d(m, stage_out, x0, y0);
        tma_store_2d(m, stage_out + 16384, x0 + 64, y0);
        bulk_commit();
        bulk_wait_read_all();
        mbar_arrive(stage_free);
        if (counter != kCounterNone) {
          // Every store of the tile is complete before the GPU-scope release.
          bulk_wait_all();
          fwd_stamp(p, t, 11);
          fence_proxy_async_global();
          fence_acq_rel_gpu();
          red_add_relaxed_gpu((counter == kCounterHidden ? p.hid_cnt : p.slice_cnt) + rb, inc);
          fwd_stamp(p, t, 8);
        }
      }
      bulk_wait_all();
    }
    __syncwarp();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace ce4b
