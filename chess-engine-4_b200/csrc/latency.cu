// Small-batch dense forward (sm_100a): the whole tower in one cooperative launch for
// batches of at most 64 positions, laid out for latency instead of throughput.
//
// The reference evaluates a batch as a chain of GEMM and element-wise launches per layer
// (kernels/src/inference/runtime.cu:578-645; src/chess_engine_4/model/dense.py:112-125,
// 188-199). At the batch sizes of a search (the lc0 backend sends up to a few dozen
// positions, third_party/lc0/src/neural/backends/ce4/backend.cc:163-168) a layer is a few
// MFLOP and the time is all dependency latency. Here every GEMM is computed transposed,
// D^T = W . X^T: the weights are the 128-row M side of tcgen05.mma and the positions the
// N side (batch rounded up to 16), so a 64-position batch pads nothing to 128 rows. Each
// layer is spread over ~100 SMs as short tiles:
//
//   input   (m, k): partial x^T[m*128.., :] over K part k of the 7168 input columns
//   gate_up (l, j): hidden[:, 64j..64j+63] = bf16(silu(bf16(n W_g^T)) * bf16(n W_u^T)) with
//                   n = bf16((x * rsqrt(mean(x^2) + eps)) * w_norm) computed by the CTA
//                   itself from x (the reference's RMSNorm rounding point)
//   down    (l, m, k): partial of (hidden . W_d^T)[:, m*128..] over K part k
//   heads   (t): head columns t*128.. of bf16(n_final . H^T + b), FP32 policy, WDL, moves-left
//
// K-split partial sums go to global memory; once all parts of a 128-row block are in
// (a counter), every part's CTA sums its share of the block in part order (the result does
// not depend on which part finished last), adds bias or residual, rounds to BF16 and
// stores x. Layer l + 1's gate_up tiles wait for all x stores of layer l (a counter), the
// down tiles for all gate_up tiles of their layer.
//
// Every CTA has a fixed list of tasks, planned on the host (gate_up tiles of even and odd
// layers on two CTA sets, down tiles of every layer on a third, heads on a fourth), so
// each CTA's weights for its next task are TMA-loaded into one of two 64 KB shared-memory
// slots while it waits for that task's inputs. The launch is cooperative: all CTAs are
// resident at once, which the cross-CTA waits need. Every wait is bounded (1 s); a CTA that
// gives up records an error code, lets its own copies and MMAs land, frees its tensor
// memory and returns, and the CTAs waiting on it then time out the same way.
#include <mutex>
#include <set>

#include "gemm.cuh"
#include "internal.h"
#include "latency_types.h"

namespace ce4b {

namespace {

constexpr uint32_t kLatKbBytes = 128 * 64 * 2;  // one 128-row x 64-column weight k-block
constexpr uint32_t kLatActKb = 64 * 64 * 2;     // one 64-row x 64-column activation k-block
constexpr uint32_t kOffW = 0;
constexpr uint32_t kOffAct = 2 * kLatWSlotBytes;
constexpr uint32_t kOffXch = kOffAct + kLatMaxRows * kLatMaxD * 2;
constexpr uint32_t kOffBar = kOffXch + kLatMaxRows * 64 * 4;
constexpr uint32_t kOffNorm = kOffBar + 64;  // norm weights of the current task [d] BF16
constexpr int kLatSmemBytes = 1024 + kOffNorm + kLatMaxD * 2;
static_assert(kLatSmemBytes <= 232448, "shared memory budget exceeded");

__device__ __forceinline__ void lat_stamp(const LatParams& p, int idx, int slot) {
  if (p.trace != nullptr && idx < p.trace_cap) {
    p.trace[static_cast<size_t>(idx) * kLatTraceWords + slot] = global_timer_ns();
  }
}

// K extent of a task in 64-column k-blocks (weights and activations alike).
__device__ __forceinline__ int lat_kb(const LatParams& p, const int4& t) {
  switch (t.x) {
    case kLatInput: return p.kb_in / p.kp_in;
    case kLatDown: return (p.h / 64) / p.kp_dn;
    default: return p.d / 64;
  }
}

// First k-block of the task's K range.
__device__ __forceinline__ int lat_kb0(const LatParams& p, const int4& t) {
  switch (t.x) {
    case kLatInput: return t.w * (p.kb_in / p.kp_in);
    case kLatDown: return t.w * ((p.h / 64) / p.kp_dn);
    default: return 0;
  }
}

// Weights of task t into the slots from `first` on (k-block kb at slot byte kb * 16 KB).
__device__ __forceinline__ void lat_issue_weights(const LatParams& p, const int4& t, uint32_t w_base,
                                                  uint32_t wbar0, uint32_t wbar1, int first, int nkb) {
  const LatMaps* maps = p.maps;
  const int lo = first * kLatMaxKbSlot, hi = lo + nkb;
  const int in0 = max(0, min(hi, kLatMaxKbSlot) - lo), in1 = max(0, hi - max(lo, kLatMaxKbSlot));
  if (in0 > 0) mbar_arrive_expect_tx(wbar0, static_cast<uint32_t>(in0) * kLatKbBytes);
  if (in1 > 0) mbar_arrive_expect_tx(wbar1, static_cast<uint32_t>(in1) * kLatKbBytes);
  const int kb0 = lat_kb0(p, t);
  for (int kb = 0; kb < nkb; ++kb) {
    const int pos = lo + kb;
    const uint32_t dst = w_base + static_cast<uint32_t>(kb) * kLatKbBytes;
    const uint32_t bar = pos < kLatMaxKbSlot ? wbar0 : wbar1;
    switch (t.x) {
      case kLatInput:
        tma_load_2d(dst, &maps->w_in, bar, (kb0 + kb) * 64, t.z * 128);
        break;
      case kLatGateUp:
        tma_load_2d(dst, &maps->gate_up[t.y], bar, kb * 64, t.z * 64);
        tma_load_2d(dst + kLatKbBytes / 2, &maps->gate_up[t.y], bar, kb * 64, p.h + t.z * 64);
        break;
      case kLatDown:
        tma_load_2d(dst, &maps->down[t.y], bar, (kb0 + kb) * 64, t.z * 128);
        break;
      default:
        tma_load_2d(dst, &maps->heads, bar, kb * 64, t.z * 128);
        break;
    }
  }
}

// In place: the 64 x d BF16 tile at `act` (d / 64 boxes of [64 rows][128 B] with the 128-byte
// swizzle) becomes n = bf16((x * rsqrt(mean(x^2) + eps)) * w), row by row (four threads a
// row, eight columns a chunk).
__device__ __forceinline__ void lat_normalize(uint8_t* act, const uint4* __restrict__ wq, int d, float eps) {
  const int r = threadIdx.x >> 2, q = threadIdx.x & 3;
  const int nch = d / 32;
  uint4 v[kLatMaxD / 32];
  float ss[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int k = 0; k < kLatMaxD / 32; ++k) {
    if (k < nch) {
      const int c = q + 4 * k;
      v[k] = *reinterpret_cast<const uint4*>(act + (c >> 3) * kLatActKb + swz128(r, c & 7));
      const uint32_t wd[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(wd[j]);
        ss[j] = fmaf(f.x, f.x, ss[j]);
        ss[j] = fmaf(f.y, f.y, ss[j]);
      }
    }
  }
  float sum = (ss[0] + ss[1]) + (ss[2] + ss[3]);
  sum += __shfl_xor_sync(0xffffffffu, sum, 1);
  sum += __shfl_xor_sync(0xffffffffu, sum, 2);
  const float rs = rsqrtf(__fdiv_rn(sum, static_cast<float>(d)) + eps);
#pragma unroll
  for (int k = 0; k < kLatMaxD / 32; ++k) {
    if (k < nch) {
      const int c = q + 4 * k;
      const uint32_t xs[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
      const uint4 wc = wq[c];
      const uint32_t ws[4] = {wc.x, wc.y, wc.z, wc.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 xf = unpack_bf16x2(xs[j]);
        const float2 wf = unpack_bf16x2(ws[j]);
        o[j] = pack_bf16x2(__fmul_rn(__fmul_rn(xf.x, rs), wf.x), __fmul_rn(__fmul_rn(xf.y, rs), wf.y));
      }
      *reinterpret_cast<uint4*>(act + (c >> 3) * kLatActKb + swz128(r, c & 7)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

__device__ __forceinline__ void lat_fence_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ __forceinline__ void lat_red_add(int* ptr, int v) {
  asm volatile("red.relaxed.gpu.global.add.s32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

// All threads' global stores of this task, then one increment of `counter` (release).
// `tma_readers`: the stores are read by TMA (async proxy) in other CTAs.
__device__ __forceinline__ void lat_publish(int* counter, bool tma_readers) {
  if (tma_readers) fence_proxy_async_global();
  __syncthreads();
  if (threadIdx.x == 0) {
    lat_fence_gpu();
    lat_red_add(counter, 1);
  }
}

// Sum of the part tiles of 128-row block m, this CTA's share (part kp of kpn), in part
// order; then x = bf16(sum + bias) (input) or x = bf16(x + bf16(sum)) (down).
__device__ __forceinline__ void lat_reduce(const LatParams& p, const float* part, int m, int kp, int kpn,
                                           bool input) {
  const int e4 = p.n * 32;  // float4 elements of one [n][128] part tile
  const int lo = static_cast<int>(static_cast<long long>(kp) * e4 / kpn);
  const int hi = static_cast<int>(static_cast<long long>(kp + 1) * e4 / kpn);
  const float4* src = reinterpret_cast<const float4*>(part) + static_cast<size_t>(m) * kpn * e4;
  for (int e = lo + static_cast<int>(threadIdx.x); e < hi; e += kLatThreads) {
    const int b = e >> 5, col = m * 128 + (e & 31) * 4;
    bf16* xp = p.x + static_cast<size_t>(b) * p.d + col;
    // Bias or residual, loaded together with the parts.
    const uint2 addq =
        input ? *reinterpret_cast<const uint2*>(p.in_bias + col) : __ldcg(reinterpret_cast<const uint2*>(xp));
    float4 s = __ldcg(src + e);
    // Up to 12 parts' loads in flight at once, then added in part order.
    for (int q0 = 1; q0 < kpn; q0 += 12) {
      float4 t[12];
#pragma unroll
      for (int j = 0; j < 12; ++j) {
        if (q0 + j < kpn) t[j] = __ldcg(src + static_cast<size_t>(q0 + j) * e4 + e);
      }
#pragma unroll
      for (int j = 0; j < 12; ++j) {
        if (q0 + j < kpn) {
          s.x += t[j].x;
          s.y += t[j].y;
          s.z += t[j].z;
          s.w += t[j].w;
        }
      }
    }
    float o[4];
    if (input) {
      const float2 b01 = unpack_bf16x2(addq.x), b23 = unpack_bf16x2(addq.y);
      o[0] = __fadd_rn(s.x, b01.x);
      o[1] = __fadd_rn(s.y, b01.y);
      o[2] = __fadd_rn(s.z, b23.x);
      o[3] = __fadd_rn(s.w, b23.y);
    } else {
      const float2 x01 = unpack_bf16x2(addq.x), x23 = unpack_bf16x2(addq.y);
      o[0] = __fadd_rn(x01.x, bf16_round(s.x));
      o[1] = __fadd_rn(x01.y, bf16_round(s.y));
      o[2] = __fadd_rn(x23.x, bf16_round(s.z));
      o[3] = __fadd_rn(x23.y, bf16_round(s.w));
    }
    *reinterpret_cast<uint2*>(xp) = make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
  }
}

__global__ void __launch_bounds__(kLatThreads, 1) latency_forward_kernel(const __grid_constant__ LatParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint32_t base = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (base & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  base += pad;
  const uint32_t w_base = base + kOffW;
  const uint32_t act = base + kOffAct;
  float* xch = reinterpret_cast<float*>(smem + kOffXch);  // [row][64 up units]
  const uint32_t wbar0 = base + kOffBar, wbar1 = wbar0 + 8, abar = wbar0 + 16, mbar = wbar0 + 24;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + 32);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    mbar_init(wbar0, 1);
    mbar_init(wbar1, 1);
    mbar_init(abar, 1);
    mbar_init(mbar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 64);
    tmem_relinquish();
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  const int4* list = p.tasks + static_cast<size_t>(blockIdx.x) * p.max_tasks;
  int ntask = 0;
  while (ntask < p.max_tasks && list[ntask].x != kLatEnd) ++ntask;
  const int n_in = p.mt * p.kp_in, n_dn = p.mt * p.kp_dn;

  // Thread 0's bookkeeping of the two weight slots: loads are issued in task order into the
  // slot(s) that are free (a task of more than 4 k-blocks takes both, others alternate),
  // and consumed in the same order, so the two walks agree on every task's slots.
  int next_w = 0, alt_issue = 0, alt_use = 0;
  uint32_t busy = 0, cur_mask = 0;
  uint32_t issued0 = 0, issued1 = 0, landed0 = 0, landed1 = 0;
  bool act_pending = false, mma_pending = false;
  uint32_t act_phase = 0, mma_phase = 0;

  auto prefetch = [&]() {
    while (next_w < ntask) {
      const int4 t = list[next_w];
      const int nkb = lat_kb(p, t);
      const bool both = nkb > kLatMaxKbSlot;
      const int first = both ? 0 : alt_issue;
      const uint32_t mask = both ? 3u : (1u << first);
      if (busy & mask) break;
      if (!both) alt_issue ^= 1;
      busy |= mask;
      lat_issue_weights(p, t, w_base + static_cast<uint32_t>(first) * kLatWSlotBytes, wbar0, wbar1, first, nkb);
      if (mask & 1u) ++issued0;
      if (mask & 2u) ++issued1;
      ++next_w;
    }
  };

  if (tid == 0) {
    const LatMaps* maps = p.maps;
    tma_prefetch_desc(&maps->a_in);
    tma_prefetch_desc(&maps->x);
    tma_prefetch_desc(&maps->hidden);
    prefetch();
  }

  const int q4 = warp & 3;     // TMEM lane quarter of this warp
  const int half = warp >> 2;  // accumulator columns [32 * half, +32)
  const bool has_cols = 32 * half < p.n;
  bool failed = false;

#pragma unroll 1
  for (int i = 0; i < ntask; ++i) {
    const int4 t = list[i];
    const int type = t.x, layer = t.y, tile = t.z, part = t.w;
    const int nkb = lat_kb(p, t);
    const int kb0 = lat_kb0(p, t);
    const int tr = static_cast<int>(blockIdx.x) * p.max_tasks + i;
    // 1. Inputs ready, then their activation boxes.
    if (tid == 0) {
      lat_stamp(p, tr, 0);
      if (p.trace != nullptr && tr < p.trace_cap) {
        p.trace[static_cast<size_t>(tr) * kLatTraceWords + 10] = blockIdx.x;
        p.trace[static_cast<size_t>(tr) * kLatTraceWords + 11] =
            (static_cast<unsigned long long>(type) << 48) | (static_cast<unsigned long long>(layer) << 32) |
            (static_cast<unsigned long long>(tile) << 16) | static_cast<unsigned long long>(part);
      }
      const int* dep = nullptr;
      int target = 0;
      if (type == kLatGateUp) {
        dep = p.cnt;
        target = n_in + layer * n_dn;
      } else if (type == kLatHeads) {
        dep = p.cnt;
        target = n_in + p.depth * n_dn;
      } else if (type == kLatDown) {
        dep = p.cnt + 1;
        target = (layer + 1) * p.gt;
      }
      if (dep != nullptr && !wait_counter(dep, target)) {
        record_error(p.err, kErrTimeoutDependency);
        failed = true;
      } else {
        fence_proxy_async_global();
        lat_stamp(p, tr, 1);
        const LatMaps* maps = p.maps;
        const CUtensorMap* ma = type == kLatInput ? &maps->a_in : (type == kLatDown ? &maps->hidden : &maps->x);
        mbar_arrive_expect_tx(abar, static_cast<uint32_t>(nkb) * kLatActKb);
        act_pending = true;
        for (int kb = 0; kb < nkb; ++kb) {
          tma_load_2d(act + static_cast<uint32_t>(kb) * kLatActKb, ma, abar, (kb0 + kb) * 64, 0);
        }
      }
    }
    if (__syncthreads_or(failed)) break;
    // 2. gate_up and heads normalise their x rows in shared memory.
    const bool norm = type == kLatGateUp || type == kLatHeads;
    if (norm) {
      // The norm weights go to shared memory while the x tile lands.
      const bf16* nw = type == kLatHeads ? p.final_norm : p.norm[layer];
      if (tid < p.d / 2) {
        reinterpret_cast<uint32_t*>(smem + kOffNorm)[tid] = __ldg(reinterpret_cast<const uint32_t*>(nw) + tid);
      }
      if (!mbar_wait(abar, act_phase)) failed = true;
      if (__syncthreads_or(failed)) {
        if (tid == 0) record_error(p.err, kErrTimeoutProducer);
        break;
      }
      if (tid == 0) {
        act_pending = false;
        lat_stamp(p, tr, 2);
      }
      lat_normalize(smem + kOffAct, reinterpret_cast<const uint4*>(smem + kOffNorm), p.d, p.eps);
      fence_proxy_async_smem();
      __syncthreads();
      if (tid == 0) lat_stamp(p, tr, 8);
    }
    // 3. MMAs (one thread): D^T[128 x n] over the task's K range.
    if (tid == 0) {
      bool ok = true;
      if (!norm) {
        ok = mbar_wait(abar, act_phase);
        if (ok) {
          act_pending = false;
          lat_stamp(p, tr, 2);
        }
      }
      const bool both = nkb > kLatMaxKbSlot;
      const int first = both ? 0 : alt_use;
      if (!both) alt_use ^= 1;
      cur_mask = both ? 3u : (1u << first);
      if (ok && (cur_mask & 1u)) {
        ok = mbar_wait(wbar0, landed0 & 1u);
        if (ok) ++landed0;
      }
      if (ok && (cur_mask & 2u)) {
        ok = mbar_wait(wbar1, landed1 & 1u);
        if (ok) ++landed1;
      }
      if (ok) {
        lat_stamp(p, tr, 9);
        tc_fence_after();
        const uint32_t idesc = idesc_bf16(128, p.n);
        const uint32_t wa = w_base + static_cast<uint32_t>(first) * kLatWSlotBytes;
        for (int kb = 0; kb < nkb; ++kb) {
          const uint32_t a = wa + static_cast<uint32_t>(kb) * kLatKbBytes;
          const uint32_t b = act + static_cast<uint32_t>(kb) * kLatActKb;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            umma_bf16(tmem, sdesc_k128(a + 32u * k), sdesc_k128(b + 32u * k), idesc, (kb | k) != 0 ? 1u : 0u);
          }
        }
        umma_commit(mbar);
        mma_pending = true;
        lat_stamp(p, tr, 3);
      } else {
        record_error(p.err, kErrTimeoutMma);
        failed = true;
      }
    }
    if (__syncthreads_or(failed)) break;
    if (!mbar_wait(mbar, mma_phase)) failed = true;
    if (__syncthreads_or(failed)) {
      if (tid == 0) record_error(p.err, kErrTimeoutEpilogue);
      break;
    }
    tc_fence_after();
    mma_phase ^= 1u;
    act_phase ^= 1u;
    if (tid == 0) {
      mma_pending = false;
      busy &= ~cur_mask;  // the slots this task read are free again (refilled after the epilogue)
      lat_stamp(p, tr, 4);
    }
    // 4. Epilogue. Warp w reads TMEM lanes 32 * (w % 4).. (output features) and accumulator
    // columns 32 * (w / 4).. (positions).
    if (type == kLatInput || type == kLatDown) {
      const bool input = type == kLatInput;
      const int kpn = input ? p.kp_in : p.kp_dn;
      float* part_base = input ? p.part_in : p.part_dn;
      if (has_cols) {
        float v[32];
        load_acc32(tmem + (static_cast<uint32_t>(32 * q4) << 16) + static_cast<uint32_t>(32 * half), v);
        float* dst = part_base + (static_cast<size_t>(tile) * kpn + part) * p.n * 128 + 32 * q4 + lane;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int b = 32 * half + c;
          if (b < p.n) __stcg(dst + static_cast<size_t>(b) * 128, v[c]);
        }
      }
      tc_fence_before();
      int* pc = p.cnt + 2 + (input ? 0 : p.mt) + tile;
      lat_publish(pc, false);
      // 5. Once every K part of this 128-row block is in, this CTA's share of the sum.
      if (tid == 0) {
        lat_stamp(p, tr, 5);
        prefetch();
        if (!wait_counter(pc, input ? kpn : (layer + 1) * kpn)) {
          record_error(p.err, kErrTimeoutDependency);
          failed = true;
        } else {
          lat_stamp(p, tr, 6);
        }
      }
      if (__syncthreads_or(failed)) break;
      lat_reduce(p, part_base, tile, part, kpn, input);
      lat_publish(p.cnt, true);
      if (tid == 0) lat_stamp(p, tr, 7);
    } else if (type == kLatGateUp) {
      // Lanes 0..63: gate units 64 * tile + lane; lanes 64..127: the matching up units.
      // Every warp reads its accumulator columns first; the up warps then hand theirs over.
      float v[32];
      if (has_cols) {
        load_acc32(tmem + (static_cast<uint32_t>(32 * q4) << 16) + static_cast<uint32_t>(32 * half), v);
        round_bf16_inplace(v);
      }
      if (q4 >= 2 && has_cols) {
        const int u = 32 * (q4 - 2) + lane;
#pragma unroll
        for (int c = 0; c < 32; ++c) xch[(32 * half + c) * 64 + u] = v[c];
      }
      __syncthreads();
      if (q4 < 2 && has_cols) {
        const int u = 32 * q4 + lane;
        float up[32];  // read every up value before the first global store
#pragma unroll
        for (int c = 0; c < 32; ++c) up[c] = xch[(32 * half + c) * 64 + u];
        bf16* dst = p.hidden + tile * 64 + u;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int b = 32 * half + c;
          if (b < p.n) dst[static_cast<size_t>(b) * p.h] = __float2bfloat16(swiglu_f32(v[c], up[c]));
        }
      }
      if (tid == 0) lat_stamp(p, tr, 6);
      tc_fence_before();
      lat_publish(p.cnt + 1, true);
      if (tid == 0) {
        lat_stamp(p, tr, 5);
        prefetch();
      }
    } else {
      // Heads: lane = head column tile * 128 + 32 * (w % 4) + lane.
      if (has_cols) {
        float v[32];
        load_acc32(tmem + (static_cast<uint32_t>(32 * q4) << 16) + static_cast<uint32_t>(32 * half), v);
        const int c0 = tile * 128 + 32 * q4;  // first head column of this warp
        const int c = c0 + lane;
        const float bias = c < p.head_cols ? __bfloat162float(p.head_bias[c]) : 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], bias);
        round_bf16_inplace(v);
        if (c0 == p.policy_storage) {
          // Lanes 0..2 hold the three WDL logits of 32 positions: transpose them through the
          // exchange area so that lane j takes position 32 * half + j.
          float* tw = xch + half * 96;
          if (lane < 3) {
#pragma unroll
            for (int j = 0; j < 32; ++j) tw[lane * 32 + j] = v[j];
          }
          __syncwarp();
          const int b = 32 * half + lane;
          const float a0 = tw[lane], a1 = tw[32 + lane], a2 = tw[64 + lane];
          if (b < p.batch) {
            float* w = p.wdl + static_cast<size_t>(b) * 3;
            if (p.wdl_probs) {
              const float mx = fmaxf(fmaxf(a0, a1), a2);
              const float e0 = expf(a0 - mx), e1 = expf(a1 - mx), e2 = expf(a2 - mx);
              const float total = e0 + e1 + e2;
              w[0] = e0 / total;
              w[1] = e1 / total;
              w[2] = e2 / total;
            } else {
              w[0] = a0;
              w[1] = a1;
              w[2] = a2;
            }
          }
        } else if (c0 == p.policy_storage + 32) {
          float* tm = xch + 192 + half * 32;
          if (lane == 0) {
#pragma unroll
            for (int j = 0; j < 32; ++j) tm[j] = v[j];
          }
          __syncwarp();
          if (32 * half + lane < p.batch) p.moves_left[32 * half + lane] = tm[lane];
        } else if (c < p.policy_size) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int b = 32 * half + j;
            if (b < p.batch) p.policy[static_cast<size_t>(b) * p.policy_size + c] = v[j];
          }
        }
      }
      tc_fence_before();
      __syncthreads();
      if (tid == 0) lat_stamp(p, tr, 5);
    }
  }

  // Teardown: let this CTA's own loads and MMAs land (bounded) before its shared and
  // tensor memory are released.
  if (tid == 0) {
    while (landed0 < issued0 && mbar_wait(wbar0, landed0 & 1u)) ++landed0;
    while (landed1 < issued1 && mbar_wait(wbar1, landed1 & 1u)) ++landed1;
    if (act_pending) mbar_wait(abar, act_phase);
    if (mma_pending) mbar_wait(mbar, mma_phase);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 64);
}

}  // namespace

void latency_forward(const LatParams& p, int grid, cudaStream_t s) {
  require(p.maps != nullptr && p.tasks != nullptr && p.max_tasks >= 1 && grid >= 1 && grid <= sm_count() &&
              p.batch >= 1 && p.batch <= kLatMaxRows && p.n % 16 == 0 && p.n >= p.batch && p.n <= kLatMaxRows &&
              p.d % 128 == 0 && p.d <= kLatMaxD && p.mt == p.d / 128 && p.h % 64 == 0 && p.gt == p.h / 64 &&
              p.depth >= 1 && p.depth <= kFwdMaxDepth && p.kp_in >= 1 && p.kb_in % p.kp_in == 0 &&
              p.kb_in / p.kp_in <= kLatMaxKbSlot && p.kp_dn >= 1 && (p.h / 64) % p.kp_dn == 0 &&
              (p.h / 64) / p.kp_dn <= kLatMaxKbSlot && p.policy_size <= p.policy_storage &&
              p.policy_storage % 32 == 0 && p.head_cols == p.policy_storage + 64 &&
              p.ht == (p.head_cols + 127) / 128 && p.x != nullptr && p.hidden != nullptr &&
              p.part_in != nullptr && p.part_dn != nullptr && p.cnt != nullptr && p.policy != nullptr &&
              p.wdl != nullptr && p.moves_left != nullptr,
          "small-batch forward: unsupported shape");
  {
    static std::mutex mu;
    static std::set<int> done;
    int dev = 0;
    check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lock(mu);
    if (!done.count(dev)) {
      check_cuda(cudaFuncSetAttribute(latency_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      kLatSmemBytes),
                 "cudaFuncSetAttribute(small-batch forward smem)");
      done.insert(dev);
    }
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kLatThreads, 1, 1);
  cfg.dynamicSmemBytes = kLatSmemBytes;
  cfg.stream = s;
  // Cooperative: every CTA is resident at once (CTAs wait on counters other CTAs publish).
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  check_cuda(cudaLaunchKernelEx(&cfg, latency_forward_kernel, p), "small-batch forward launch");
}

}  // namespace ce4b
