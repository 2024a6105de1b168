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
//   input tile   (rb, j):    x[rb, j] = bf16(A_in . W_in^T + b)
//   gate_up tile (l, rb, c): hidden[rb, c] = bf16(silu(bf16(r * x W'_g^T)) * bf16(r * x W'_u^T))
//   down tile    (l, rb, j): x[rb, j] = bf16(x + bf16(hidden . W_d^T)).
//
// Tiles are 128 rows; gate_up tiles are 256 accumulator columns (128 gate + 128 up, one
// 128-column hidden chunk). Input and down tiles are xw columns of x, chosen per forward:
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
// are counters in global memory: slice_cnt[rb] (finished x slices) and hid_cnt[rb]
// (finished gate_up tiles). Writers publish with an epilogue barrier, then one thread's
// GPU-scope acq_rel fence (which also releases the other threads' stores) and a relaxed
// increment; readers acquire the counter, and issue a proxy fence before TMA reads the
// data. Every wait is bounded (a timed-out wait records an error code and the kernel
// runs to its end).
#pragma once

#include "forward_types.h"
#include "gemm.cuh"

namespace ce4b {

struct FwdTask {
  int type;
  int layer;
  int rb;
  int col;  // hidden chunk (gate_up) or x tile of width xw (input, down)
};

__device__ __forceinline__ FwdTask fwd_decode(const FwdParams& p, int t) {
  FwdTask k{kTaskEnd, 0, 0, 0};
  if (t < 0 || t >= p.total_tasks) return k;
  const int n_in = p.nb * p.xt;
  if (t < n_in) {
    k.type = kTaskInput;
    k.rb = t / p.xt;
    k.col = t - k.rb * p.xt;
    return k;
  }
  t -= n_in;
  const int per_layer = p.nb * (p.nc + p.xt);
  k.layer = t / per_layer;
  t -= k.layer * per_layer;
  if (t < p.nb * p.nc) {
    k.type = kTaskGateUp;
    k.rb = t / p.nc;
    k.col = t - k.rb * p.nc;
  } else {
    t -= p.nb * p.nc;
    k.type = kTaskDown;
    k.rb = t / p.xt;
    k.col = t - k.rb * p.xt;
  }
  return k;
}

// ------------------------------------------------------------------ global synchronisation
__device__ __forceinline__ int ld_acquire_gpu(const int* ptr) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Waits until *ptr >= target (bounded). Returns false after kWaitLimitNs.
__device__ __forceinline__ bool wait_counter(const int* ptr, int target) {
  if (ld_acquire_gpu(ptr) >= target) return true;
  const unsigned long long start = global_timer_ns();
  while (true) {
    __nanosleep(64);
    if (ld_acquire_gpu(ptr) >= target) return true;
    if (global_timer_ns() - start > kWaitLimitNs) return false;
  }
}

__device__ __forceinline__ uint4 ldcg_u4(const void* ptr) {
  return __ldcg(reinterpret_cast<const uint4*>(ptr));
}

__device__ __forceinline__ float4 ldcg_f4(const float* ptr) {
  return __ldcg(reinterpret_cast<const float4*>(ptr));
}

// 32 FP32 values -> 32 BF16 at dst (64 contiguous bytes, 16-byte aligned).
__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float (&v)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    d[k] = make_uint4(pack_bf16x2(v[8 * k + 0], v[8 * k + 1]), pack_bf16x2(v[8 * k + 2], v[8 * k + 3]),
                      pack_bf16x2(v[8 * k + 4], v[8 * k + 5]), pack_bf16x2(v[8 * k + 6], v[8 * k + 7]));
  }
}

// 32 BF16 at src (L2, bypassing L1: the data was written by other SMs) -> FP32.
__device__ __forceinline__ void load_bf16x32_cg(const __nv_bfloat16* src, float (&v)[32]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint4 q = ldcg_u4(src + 8 * k);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(w[j]);
      v[8 * k + 2 * j] = f.x;
      v[8 * k + 2 * j + 1] = f.y;
    }
  }
}

__device__ __forceinline__ void fwd_stamp(const FwdParams& p, int t, int slot) {
  if (p.trace != nullptr && t < p.trace_cap) {
    p.trace[static_cast<size_t>(t) * kFwdTraceWords + slot] = global_timer_ns();
  }
}

__device__ __forceinline__ void fwd_epi_sync() { named_bar_sync(kEpiBarrierId, kFwdEpiThreads); }

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

// gate_up tile: accumulator columns [0, 128) gate, [128, 256) up; A was the raw x, and
// `scale` is the row's RMSNorm scale.
__device__ __forceinline__ void fwd_epi_gate_up(const FwdParams& p, const FwdTask& k, int t, int r,
                                                int g, int tid, uint32_t taddr, uint32_t tempty,
                                                float scale) {
  const int row = k.rb * kBM + r;
  const int c = g * 32;
  float gv[32], uv[32];
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
  store_bf16x32(p.hidden + static_cast<size_t>(row) * p.h + k.col * 128 + c, gv);
  fwd_epi_sync();
  if (tid == 0) {
    fwd_stamp(p, t, 7);
    fence_acq_rel_gpu();
    fence_proxy_async_global();
    red_add_relaxed_gpu(p.hid_cnt + k.rb, 1);
    fwd_stamp(p, t, 8);
  }
}

// x tile (input or down), xw columns: thread (r, g) handles xw / 128 chunks of 32 columns,
// c = g * (xw / 4) + 32 * i. Per chunk it stores the BF16 values and their sum of squares
// in ss[row][slice * kFwdG + group] (slice = 128-column slice, group = 32-column group in
// it, the layout the row scale reads); then the tile publishes the xw / 128 slices it
// covers. `pre0` holds the thread's first chunk of the residual (down) or of the bias
// (input), loaded before the accumulator was ready; later chunks are loaded after the
// previous one is stored.
__device__ __forceinline__ void fwd_epi_slice(const FwdParams& p, const FwdTask& k, int t, int r,
                                              int g, int tid, uint32_t taddr, uint32_t tempty,
                                              const uint4 (&pre0)[4]) {
  const int row = k.rb * kBM + r;
  const int nchunk = p.xw / 128;
  for (int ci = 0; ci < nchunk; ++ci) {
    const int c = g * (p.xw / 4) + 32 * ci;  // column in the tile
    const int col0 = k.col * p.xw + c;       // column in x
    uint4 pre[4];
    if (ci == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) pre[q] = pre0[q];
    } else {
      const __nv_bfloat16* src = k.type == kTaskDown
                                     ? p.x + static_cast<size_t>(row) * p.d + col0
                                     : p.bias + col0;
#pragma unroll
      for (int q = 0; q < 4; ++q) pre[q] = ldcg_u4(src + 8 * q);
    }
    float v[32];
    load_acc32(taddr + c, v);
    if (ci == nchunk - 1) {
      tc_fence_before();
      mbar_arrive(tempty);
    }
    if (k.type != kTaskInput) round_bf16_inplace(v);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t wq[4] = {pre[q].x, pre[q].y, pre[q].z, pre[q].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(wq[j]);
        // input: acc + bias (TE's fused bias); down: residual + bf16(acc)
        v[8 * q + 2 * j] = k.type == kTaskInput ? v[8 * q + 2 * j] + f.x : f.x + v[8 * q + 2 * j];
        v[8 * q + 2 * j + 1] =
            k.type == kTaskInput ? v[8 * q + 2 * j + 1] + f.y : f.y + v[8 * q + 2 * j + 1];
      }
    }
    round_bf16_inplace(v);
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) ss = fmaf(v[j], v[j], ss);
    store_bf16x32(p.x + static_cast<size_t>(row) * p.d + col0, v);
    p.ss[static_cast<size_t>(row) * (p.sj * kFwdG) + (col0 >> 7) * kFwdG + ((col0 & 127) >> 5)] = ss;
  }
  fwd_epi_sync();
  if (tid == 0) {
    fwd_stamp(p, t, 7);
    fence_acq_rel_gpu();
    fence_proxy_async_global();
    red_add_relaxed_gpu(p.slice_cnt + k.rb, nchunk);
    fwd_stamp(p, t, 8);
  }
}

// ------------------------------------------------------------------ the kernel
struct FwdSmem {
  static constexpr int kABytes = kBM * kBK * 2;          // 16 KB
  static constexpr int kBBytesMax = 256 * kBK * 2;       // 32 KB (gate + up boxes)
  static constexpr int kStageBytes = kABytes + kBBytesMax;
  static constexpr int kRingBytes = kFwdNStage * kStageBytes;
  static constexpr int kBarriers = 2 * kFwdNStage + 4 + 2 * kFwdTaskRing + 1;
  static constexpr int kMiscBytes = kBarriers * 8 + kFwdTaskRing * 4 + 16;
  static constexpr int kBytes = 1024 + kRingBytes + kMiscBytes;
  static_assert(kBytes <= 232448, "shared memory budget exceeded");
};

__global__ void __launch_bounds__(kFwdThreads, 1) dense_forward_kernel(const FwdParams p) {
  using L = FwdSmem;
  extern __shared__ uint8_t smem_raw[];
  uint32_t base = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (base & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  base += pad;

  const uint32_t bar_base = base + L::kRingBytes;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (kFwdNStage + s); };
  auto tfull_bar = [&](int a) { return bar_base + 8u * (2 * kFwdNStage + a); };
  auto tempty_bar = [&](int a) { return bar_base + 8u * (2 * kFwdNStage + 2 + a); };
  auto task_full = [&](int q) { return bar_base + 8u * (2 * kFwdNStage + 4 + q); };
  auto task_empty = [&](int q) { return bar_base + 8u * (2 * kFwdNStage + 4 + kFwdTaskRing + q); };
  const uint32_t drain_bar = bar_base + 8u * (L::kBarriers - 1);
  volatile int* task_slot =
      reinterpret_cast<volatile int*>(smem + L::kRingBytes + L::kBarriers * 8);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(const_cast<int*>(task_slot + kFwdTaskRing + 1));

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
        int kb0 = 0, kb1 = 0, b_row = 0, b_row2 = -1;
        if (t >= 0) {
          fwd_stamp(p, t, 0);
          if (p.trace != nullptr && t < p.trace_cap) {
            p.trace[static_cast<size_t>(t) * kFwdTraceWords + 10] = blockIdx.x;
          }
          k = fwd_decode(p, t);
          if (k.type == kTaskInput) {
            ma = &maps->a_in;
            mb = &maps->w_in;
            kb1 = p.kb_in;
            b_row = k.col * p.xw;
            if (p.xw == 256) b_row2 = b_row + 128;
          } else if (k.type == kTaskGateUp) {
            if (!wait_counter(p.slice_cnt + k.rb, (k.layer + 1) * p.sj)) {
              record_error(p.err, kErrTimeoutDependency);
            }
            ma = &maps->x;
            mb = &maps->gate_up[k.layer];
            kb1 = p.d / kBK;
            b_row = k.col * 128;
            b_row2 = p.h + k.col * 128;
          } else {
            if (!wait_counter(p.hid_cnt + k.rb, (k.layer + 1) * p.nc)) {
              record_error(p.err, kErrTimeoutDependency);
            }
            ma = &maps->hidden;
            mb = &maps->down[k.layer];
            kb1 = p.h / kBK;
            b_row = k.col * p.xw;
            if (p.xw == 256) b_row2 = b_row + 128;
          }
        }
        // The task is published once its inputs are complete (the acquire above), so the
        // MMA thread and the epilogue warps may read its inputs as soon as they see it.
        task_slot[q] = t;
        mbar_arrive(task_full(q));
        if (t < 0) break;
        // Data written by other SMs' generic stores is read below by TMA (async proxy).
        fence_proxy_async_global();
        fwd_stamp(p, t, 1);
        const uint32_t bytes = L::kABytes + (b_row2 >= 0 ? 2 : 1) * 128 * kBK * 2;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u)) {
            record_error(p.err, kErrTimeoutProducer);
            ok = false;
            break;
          }
          const uint32_t sa = base + stage * L::kStageBytes;
          const uint32_t sb = sa + L::kABytes;
          mbar_arrive_expect_tx(full_bar(stage), bytes);
          tma_load_2d(sa, ma, full_bar(stage), kb * kBK, k.rb * kBM);
          tma_load_2d(sb, mb, full_bar(stage), kb * kBK, b_row);
          if (b_row2 >= 0) tma_load_2d(sb + 128 * kBK * 2, mb, full_bar(stage), kb * kBK, b_row2);
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
        const int nkb = k.type == kTaskInput ? p.kb_in : (k.type == kTaskGateUp ? p.d : p.h) / kBK;
        const uint32_t idesc = idesc_bf16(kBM, k.type == kTaskGateUp ? 256 : p.xw);
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
          tc_fence_after();
          if (kb == 0) fwd_stamp(p, t, 3);
          const uint32_t sa = base + stage * L::kStageBytes;
          const uint64_t adesc = sdesc_k128(sa);
          const uint64_t bdesc = sdesc_k128(sa + L::kABytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            umma_bf16(d_tmem, adesc + 2u * kk, bdesc + 2u * kk, idesc, (kb | kk) != 0 ? 1u : 0u);
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
  } else {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int g = (warp - 2) >> 2;
    const int tid = threadIdx.x - 64;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int i = 0;; ++i) {
      const int q = i % kFwdTaskRing;
      if (!mbar_wait(task_full(q), (i / kFwdTaskRing) & 1)) {
        record_error(p.err, kErrTimeoutEpilogue);
        break;
      }
      const int t = task_slot[q];
      mbar_arrive(task_empty(q));
      if (t < 0) break;
      const FwdTask k = fwd_decode(p, t);
      // Global inputs of the epilogue, fetched while the MMAs run (the producer published
      // the task after its dependencies completed).
      float scale = 1.0f;
      uint4 pre[4];
      if (k.type == kTaskGateUp) {
        scale = fwd_row_scale(p, k.rb * kBM + r);
      } else {
        const int col0 = k.col * p.xw + g * (p.xw / 4);
        const __nv_bfloat16* src = k.type == kTaskDown
                                       ? p.x + static_cast<size_t>(k.rb * kBM + r) * p.d + col0
                                       : p.bias + col0;
#pragma unroll
        for (int q = 0; q < 4; ++q) pre[q] = ldcg_u4(src + 8 * q);
      }
      if (!mbar_wait(tfull_bar(acc), acc_phase)) {
        record_error(p.err, kErrTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      if (tid == 0) fwd_stamp(p, t, 5);
      const uint32_t taddr =
          tmem_base + static_cast<uint32_t>(acc * 256) + (static_cast<uint32_t>(quarter * 32) << 16);
      if (k.type == kTaskGateUp) {
        fwd_epi_gate_up(p, k, t, r, g, tid, taddr, tempty_bar(acc), scale);
      } else {
        fwd_epi_slice(p, k, t, r, g, tid, taddr, tempty_bar(acc), pre);
      }
      if (tid == 0) fwd_stamp(p, t, 6);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace ce4b
