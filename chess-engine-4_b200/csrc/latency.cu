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
//   gate_up (l, j): hidden[:, 64j..64j+63] = bf16(silu(bf16(r * x W'_g^T)) * bf16(r * x W'_u^T))
//                   with the RMSNorm folded as in the persistent forward: W' = bf16(W * diag(w)),
//                   r = rsqrt(mean(x^2) + eps) per position, computed by four warps of the CTA
//                   from its x tile while the MMAs run (so no normalisation pass precedes them)
//   down    (l, m, k): partial of (hidden . W_d^T)[:, m*128..] over K part k
//   heads   (t): head columns t*128.. of bf16(r * x H'^T + b), FP32 policy, WDL, moves-left
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
// gate_up tiles are M = 64 (32 gate + 32 up rows): an N = 64 MMA reads its operands from
// shared memory, so a 64-row weight tile makes each of its 32 MMAs a third cheaper.
constexpr int kLatGuRows = 2 * kLatGuUnits;
constexpr uint32_t kLatActKb = 64 * 64 * 2;     // one 64-row x 64-column activation k-block
constexpr uint32_t kOffW = 0;
constexpr uint32_t kOffAct = 2 * kLatWSlotBytes;
constexpr uint32_t kOffXch = kOffAct + kLatMaxRows * kLatMaxD * 2;
constexpr uint32_t kOffBar = kOffXch + kLatMaxRows * 64 * 4;
constexpr uint32_t kOffRow = kOffBar + 128;  // row scales of the current gate_up / heads task [64]
constexpr int kLatSmemBytes = 1024 + kOffRow + kLatMaxRows * 4;
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

// Bytes of one weight k-block of a task (M rows x 64 columns).
__device__ __forceinline__ uint32_t lat_kb_bytes(int type) {
  return type == kLatGateUp ? kLatGuRows * 64 * 2 : kLatKbBytes;
}

// Weights of task t into the slots from `first` on (k-block kb at byte kb * lat_kb_bytes).
__device__ __forceinline__ void lat_issue_weights(const LatParams& p, const int4& t, uint32_t w_base,
                                                  uint32_t wbar0, uint32_t wbar1, int first, int nkb) {
  const LatMaps* maps = p.maps;
  const uint32_t kbb = lat_kb_bytes(t.x);
  const uint32_t lo = static_cast<uint32_t>(first) * kLatWSlotBytes, hi = lo + static_cast<uint32_t>(nkb) * kbb;
  const uint32_t slot = kLatWSlotBytes;
  const uint32_t in0 = hi > lo && lo < slot ? min(hi, slot) - lo : 0u;
  const uint32_t in1 = hi > slot ? hi - max(lo, slot) : 0u;
  if (in0 > 0) mbar_arrive_expect_tx(wbar0, in0);
  if (in1 > 0) mbar_arrive_expect_tx(wbar1, in1);
  const int kb0 = lat_kb0(p, t);
  for (int kb = 0; kb < nkb; ++kb) {
    const uint32_t pos = lo + static_cast<uint32_t>(kb) * kbb;
    const uint32_t dst = w_base + static_cast<uint32_t>(kb) * kbb;
    const uint32_t bar = pos < slot ? wbar0 : wbar1;
    switch (t.x) {
      case kLatInput:
        tma_load_2d(dst, &maps->w_in, bar, (kb0 + kb) * 64, t.z * 128);
        break;
      case kLatGateUp:
        tma_load_2d(dst, &maps->gate_up[t.y], bar, kb * 64, t.z * kLatGuUnits);
        tma_load_2d(dst + kbb / 2, &maps->gate_up[t.y], bar, kb * 64, p.h + t.z * kLatGuUnits);
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

// r[row] = rsqrt(mean(x^2) + eps) for the 64 rows of the x tile at `act` (d / 64 boxes of
// [64 rows][128 B] with the 128-byte swizzle), by threads 0..127, two a row.
__device__ __forceinline__ void lat_row_scale(const uint8_t* act, float* rsm, int d, float eps) {
  const int r = threadIdx.x >> 1, q = threadIdx.x & 1;
  float ss[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 8
  for (int k = 0; k < d / 16; ++k) {
    const int c = q + 2 * k;
    const uint4 v = *reinterpret_cast<const uint4*>(act + (c >> 3) * kLatActKb + swz128(r, c & 7));
    const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(wd[j]);
      ss[j] = fmaf(f.x, f.x, ss[j]);
      ss[j] = fmaf(f.y, f.y, ss[j]);
    }
  }
  float sum = (ss[0] + ss[1]) + (ss[2] + ss[3]);
  sum += __shfl_xor_sync(0xffffffffu, sum, 1);
  if (q == 0) rsm[r] = rsqrtf(__fdiv_rn(sum, static_cast<float>(d)) + eps);
}

// This thread's 32 accumulator columns [32 * half, +32) of TMEM lane quarter q: the sum of
// the two issuers' accumulators (columns 0.. and 64..; the second only when the task had at
// least two k-blocks, `two`).
__device__ __forceinline__ void lat_load_acc(uint32_t tmem, int q, int half, bool two, float (&v)[32]) {
  const uint32_t t = tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(32 * half);
  if (!two) {
    load_acc32(t, v);
    return;
  }
  float a[32], b[32];
  load_acc32x2(t, t + 64, a, b);
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = a[j] + b[j];
}

__device__ __forceinline__ void lat_fence_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ __forceinline__ void lat_red_add(int* ptr, int v) {
  asm volatile("red.relaxed.gpu.global.add.s32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

__device__ __forceinline__ int lat_atom_add(int* ptr, int v) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], %2;" : "=r"(old) : "l"(ptr), "r"(v) : "memory");
  return old;
}

// All threads' global stores of this task, then one increment of `counter` (release). The
// stores are generic; a reader that loads them with TMA issues fence.proxy.async.global
// after acquiring the counter, which orders them before its async-proxy reads.
__device__ __forceinline__ void lat_publish(int* counter) {
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
  // Barriers: two weight slots, MMA completion, then one per group of 4 activation k-blocks
  // (MMAs start on the first group while the second lands; a wait costs ~250 ns, so finer
  // groups lose).
  const uint32_t wbar0 = base + kOffBar, wbar1 = wbar0 + 8, mbar = wbar0 + 16, abar0 = wbar0 + 32;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffBar + 24);
  auto abar = [&](int kb) { return abar0 + 8u * static_cast<uint32_t>(kb >> 2); };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // The leader (lane 0 of the last warp) issues every TMA load and MMA and polls the
  // counters; warps 0..3 compute row scales while it issues a task's MMAs.
  constexpr int kLead = kLatThreads - 32;
  constexpr int kIssueWarp = kLatThreads / 32 - 2;  // warps 6, 7 issue the MMAs
  constexpr uint32_t kIssueBarrier = 2;             // named barrier of those two warps
  float* rsm = reinterpret_cast<float*>(smem + kOffRow);
  if (tid == 0) {
    mbar_init(wbar0, 1);
    mbar_init(wbar1, 1);
    for (int g = 0; g < kLatMaxD / 256; ++g) mbar_init(abar0 + 8u * g, 1);
    mbar_init(mbar, 2);  // one arrival per MMA issuer
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), 128);
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
  uint32_t act_par = 0, mma_phase = 0;  // act_par bit kb: parity of k-block kb's next phase
  int act_nkb = 0;

  auto prefetch = [&]() {
    while (next_w < ntask) {
      const int4 t = list[next_w];
      const int nkb = lat_kb(p, t);
      const bool both = static_cast<uint32_t>(nkb) * lat_kb_bytes(t.x) > kLatWSlotBytes;
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

  if (tid == kLead) {
    const LatMaps* maps = p.maps;
    tma_prefetch_desc(&maps->a_in);
    tma_prefetch_desc(&maps->x);
    tma_prefetch_desc(&maps->hidden);
    prefetch();
  }
  // Everything above reads only what finalize wrote (weights, maps, task lists), so with a
  // programmatic launch it overlaps the plane expansion; the tasks read its output.
  grid_dependency_wait();

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
    if (tid == kLead) {
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
        act_pending = true;
        act_nkb = nkb;
        for (int kb = 0; kb < nkb; ++kb) {
          if ((kb & 3) == 0) mbar_arrive_expect_tx(abar(kb), static_cast<uint32_t>(min(4, nkb - kb)) * kLatActKb);
          tma_load_2d(act + static_cast<uint32_t>(kb) * kLatActKb, ma, abar(kb), (kb0 + kb) * 64, 0);
        }
      }
    }
    if (__syncthreads_or(failed)) break;
    // 2. gate_up and heads normalise their x rows in shared memory.
    const bool norm = type == kLatGateUp || type == kLatHeads;
    if (norm && warp < 4) {
      // Row scales of the folded RMSNorm (warps 0..3) while the leader issues the MMAs.
      for (int kb = 0; kb < nkb && !failed; kb += 4) {
        if (!mbar_wait(abar(kb), (act_par >> (kb >> 2)) & 1u)) {
          record_error(p.err, kErrTimeoutProducer);
          failed = true;
        }
      }
      if (!failed) lat_row_scale(smem + kOffAct, rsm, p.d, p.eps);
      if (tid == 0) lat_stamp(p, tr, 8);
    }
    // 3. MMAs: D^T[M x n] over the task's K range, issued by two threads (the leader and lane 0
    // of warp 6), each over half of the k-blocks into its own 64-column accumulator (a
    // tcgen05.mma of these shapes costs ~60 ns to issue; the epilogue adds the halves).
    if (warp >= kIssueWarp) {
      volatile int* mma_go = reinterpret_cast<volatile int*>(smem + kOffBar + 28);
      if (tid == kLead) {
        bool ok = true;
        const bool both = static_cast<uint32_t>(nkb) * lat_kb_bytes(type) > kLatWSlotBytes;
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
        if (ok) lat_stamp(p, tr, 9);
        *mma_go = ok ? first : -1;
        if (!ok) {
          record_error(p.err, kErrTimeoutMma);
          failed = true;
        }
      }
      named_bar_sync(kIssueBarrier, 64);
      const int first = *mma_go;
      if (lane == 0) {
        const bool leader = tid == kLead;
        const int mid = (nkb + 1) / 2;  // the leader takes k-blocks [0, mid), the other [mid, nkb)
        const int kb_lo = leader ? 0 : mid, kb_hi = leader ? mid : nkb;
        bool ok = first >= 0, issued = false;
        if (ok && kb_lo < kb_hi) {
          tc_fence_after();
          const uint32_t idesc = idesc_bf16(type == kLatGateUp ? kLatGuRows : 128, p.n);
          const uint32_t kbb = lat_kb_bytes(type);
          // Descriptors advance by address / 16 in their low field (every operand lies in the
          // first 256 KB of shared memory, so the field does not carry).
          const uint64_t da = sdesc_k128(w_base + static_cast<uint32_t>(first) * kLatWSlotBytes);
          const uint64_t db = sdesc_k128(act);
          const uint32_t acc = tmem + (leader ? 0u : 64u);
          int waited = -1;
          for (int kb = kb_lo; kb < kb_hi && ok; ++kb) {
            if ((kb >> 2) != waited) {
              waited = kb >> 2;
              ok = mbar_wait(abar(kb), (act_par >> waited) & 1u);
              if (!ok) break;
              if (leader && kb == 0) lat_stamp(p, tr, 2);
            }
            issued = true;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              umma_bf16(acc, da + ((kb * kbb + 32u * k) >> 4), db + ((kb * kLatActKb + 32u * k) >> 4), idesc,
                        (kb != kb_lo || k != 0) ? 1u : 0u);
            }
          }
        }
        // Each issuer arrives once on the MMA barrier: through a commit when it issued (also
        // after a later wait timed out, so that the MMAs in flight are waited for), else directly.
        if (issued) {
          umma_commit(mbar);
        } else {
          mbar_arrive(mbar);
        }
        if (leader) {
          mma_pending = true;
          lat_stamp(p, tr, 3);
        }
        if (first >= 0 && !ok) {
          record_error(p.err, kErrTimeoutMma);
          failed = true;
        }
      }
    }
    if (__syncthreads_or(failed)) break;
    if (!mbar_wait(mbar, mma_phase)) failed = true;
    if (__syncthreads_or(failed)) {
      if (tid == kLead) record_error(p.err, kErrTimeoutEpilogue);
      break;
    }
    tc_fence_after();
    mma_phase ^= 1u;
    act_par ^= (1u << ((nkb + 3) >> 2)) - 1u;
    if (tid == kLead) {
      mma_pending = false;
      act_pending = false;  // both issuers waited for every activation group
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
        lat_load_acc(tmem, q4, half, nkb >= 2, v);
        float* dst = part_base + (static_cast<size_t>(tile) * kpn + part) * p.n * 128 + 32 * q4 + lane;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int b = 32 * half + c;
          if (b < p.n) __stcg(dst + static_cast<size_t>(b) * 128, v[c]);
        }
      }
      tc_fence_before();
      int* pc = p.cnt + 2 + (input ? 0 : p.mt) + tile;
      lat_publish(pc);
      // 5. Once every K part of this 128-row block is in, this CTA's share of the sum.
      if (tid == kLead) {
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
      lat_publish(p.cnt);
      if (tid == kLead) lat_stamp(p, tr, 7);
    } else if (type == kLatGateUp) {
      // M = 64 accumulator: rows 16q..16q+15 sit in lanes 32q..32q+15 of TMEM (lane quarter
      // q), so quarters 0, 1 hold the 32 gate rows and quarters 2, 3 the 32 matching up rows.
      // Every warp stages its scaled, rounded columns in the (consumed) activation area as
      // G[position][unit] and U[position][unit]; then all 256 threads take 8 units of one
      // position each, so the SiLU runs on every SM sub-partition and a thread stores 16 B.
      constexpr int kStride = kLatGuUnits + 4;  // floats a staged row (16-byte aligned)
      float* gsm = reinterpret_cast<float*>(smem + kOffAct);
      float* usm = gsm + kLatMaxRows * kStride;
      if (has_cols) {
        float v[32];
        lat_load_acc(tmem, q4, half, nkb >= 2, v);
#pragma unroll
        for (int c = 0; c < 32; ++c) v[c] = __fmul_rn(rsm[32 * half + c], v[c]);  // folded RMSNorm
        round_bf16_inplace(v);
        if (lane < 16) {
          float* dst = (q4 < 2 ? gsm : usm) + 16 * (q4 & 1) + lane;
#pragma unroll
          for (int c = 0; c < 32; ++c) dst[(32 * half + c) * kStride] = v[c];
        }
      }
      __syncthreads();
      {
        const int b = tid >> 2, u0 = (tid & 3) * 8;
        if (b < p.n) {
          const float4* g4 = reinterpret_cast<const float4*>(gsm + b * kStride + u0);
          const float4* u4 = reinterpret_cast<const float4*>(usm + b * kStride + u0);
          uint32_t o[4];
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const float4 g = g4[k], u = u4[k];
            o[2 * k] = pack_bf16x2(swiglu_f32(g.x, u.x), swiglu_f32(g.y, u.y));
            o[2 * k + 1] = pack_bf16x2(swiglu_f32(g.z, u.z), swiglu_f32(g.w, u.w));
          }
          *reinterpret_cast<uint4*>(p.hidden + static_cast<size_t>(b) * p.h + tile * kLatGuUnits + u0) =
              make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      fence_proxy_async_smem();  // these generic accesses precede the next TMA into the area
      if (tid == kLead) lat_stamp(p, tr, 6);
      tc_fence_before();
      lat_publish(p.cnt + 1);
      if (tid == kLead) {
        lat_stamp(p, tr, 5);
        prefetch();
      }
    } else {
      // Heads: lane = head column tile * 128 + 32 * (w % 4) + lane.
      if (has_cols) {
        float v[32];
        lat_load_acc(tmem, q4, half, nkb >= 2, v);
        const int c0 = tile * 128 + 32 * q4;  // first head column of this warp
        const int c = c0 + lane;
        const float bias = c < p.head_cols ? __bfloat162float(p.head_bias[c]) : 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(__fmul_rn(v[j], rsm[32 * half + j]), bias);
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
      if (tid == kLead) lat_stamp(p, tr, 5);
    }
  }

  // Teardown: let this CTA's own loads and MMAs land (bounded) before its shared and
  // tensor memory are released.
  if (tid == kLead) {
    while (landed0 < issued0 && mbar_wait(wbar0, landed0 & 1u)) ++landed0;
    while (landed1 < issued1 && mbar_wait(wbar1, landed1 & 1u)) ++landed1;
    for (int kb = 0; act_pending && kb < act_nkb; kb += 4) mbar_wait(abar(kb), (act_par >> (kb >> 2)) & 1u);
    if (mma_pending) mbar_wait(mbar, mma_phase);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 128);
  // The last CTA out zeroes the counters for the next launch (every CTA's counter accesses
  // precede its arrival here), so no reset runs before the kernel.
  if (tid == 0) {
    const int exit_idx = 2 + 2 * p.mt;
    lat_fence_gpu();
    if (lat_atom_add(p.cnt + exit_idx, 1) == static_cast<int>(gridDim.x) - 1) {
      for (int i = 0; i <= exit_idx; ++i) reinterpret_cast<volatile int*>(p.cnt)[i] = 0;
    }
  }
}

}  // namespace

void latency_forward(const LatParams& p, int grid, cudaStream_t s) {
  require(p.maps != nullptr && p.tasks != nullptr && p.max_tasks >= 1 && grid >= 1 && grid <= sm_count() &&
              p.batch >= 1 && p.batch <= kLatMaxRows && p.n % 16 == 0 && p.n >= p.batch && p.n <= kLatMaxRows &&
              p.d % 128 == 0 && p.d <= kLatMaxD && p.mt == p.d / 128 && p.h % 64 == 0 && p.gt == p.h / kLatGuUnits &&
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
  // Programmatic: the prologue and the first weight loads may run under the expansion
  // kernel before it (the kernel waits for it before its tasks). If the driver refuses the
  // pair of attributes, the launch is repeated cooperative only, and remembered per device.
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  static std::mutex pdl_mu;
  static std::set<int> pdl_refused;
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  bool pdl = false;
  {
    std::lock_guard<std::mutex> lock(pdl_mu);
    pdl = !pdl_refused.count(dev);
  }
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  check_cuda(cudaStreamIsCapturing(s, &capture), "query stream capture");
  if (pdl) {
    cfg.numAttrs = 2;
    const cudaError_t st = cudaLaunchKernelEx(&cfg, latency_forward_kernel, p);
    if (st == cudaSuccess) return;
    // A refusal under stream capture invalidates the capture: report it as it is.
    if (capture != cudaStreamCaptureStatusNone) check_cuda(st, "small-batch forward launch");
    (void)cudaGetLastError();
    std::lock_guard<std::mutex> lock(pdl_mu);
    pdl_refused.insert(dev);
  }
  cfg.numAttrs = 1;
  check_cuda(cudaLaunchKernelEx(&cfg, latency_forward_kernel, p), "small-batch forward launch");
}

}  // namespace ce4b
