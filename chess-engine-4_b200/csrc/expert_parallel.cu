// Expert parallelism for moe64a2 over NVLink peer memory: the 64 experts are split over
// `world` ranks (64 / world consecutive experts each, and only those are held), every rank
// routes its own tokens, and the routed rows travel to the rank that owns their expert and
// back through the ranks' shared EP buffers. No host synchronisation: every size is a
// device value, and the forward can be captured in a CUDA graph.
//
// One MoE layer on rank q (the reference's static dispatch path, moe.py:226-287, with an
// exchange of the routed rows between the ranks that own the experts):
//   1. router GEMM + top-2, routing scan, dispatch into 128-row expert segments (the same
//      kernels as the single-GPU layer). Segments are ordered by expert, so the rows for
//      rank r are one contiguous run.
//   2. q writes its 64 per-expert route counts into every rank's `meta` inbox and raises
//      its meta flag there to the layer's epoch.
//   3. once every rank's counts have arrived, a one-CTA kernel plans on the device: the
//      receive layout (source-major, each source's segments of q's experts in expert
//      order, padded to 128 rows as the source holds them), where q's run for each rank r
//      starts in r's buffer, where each source's results go back, and the m-tile table of
//      the grouped GEMMs over the received rows (local expert indices).
//   4. q stores its run for each rank r (rows and route weights) into r's buffer, then
//      raises its rows flag there; the grouped gate_up + SwiGLU and down x route-weight
//      GEMMs run once every source's rows are in; the results go back into each source's
//      `ret` buffer at the rows its permuted layout holds them, and raise a results flag.
//   5. combine + residual + next RMSNorm from `ret` (single-GPU kernel).
// Writers store, fence at system scope and release the flag; readers acquire it. Every rank
// runs the same sequence of MoE layers, so the epochs agree; a rank can run at most one
// phase ahead of another, which the protocol tolerates (each flag is raised only after the
// data its peer was still reading has been consumed). Every wait is bounded (2 s, then the
// device error word records kErrTimeoutPeer and the kernel returns).
// A GEMM row depends only on its own inputs, so results equal the single-GPU forward's.
#include <algorithm>
#include <cstring>
#include <vector>

#include "model.h"
#include "nccl_dl.h"
#include "ptx.cuh"

namespace ce4b {

namespace {

constexpr int kExperts = 64;
constexpr int kRows = 128;
constexpr int kMaxWorld = 8;
constexpr int kErrTimeoutPeer = 9;
constexpr unsigned long long kPeerWaitNs = 2000ull * 1000ull * 1000ull;
enum EpPhase : int { kPhaseMeta = 0, kPhaseRows = 1, kPhaseResults = 2 };

// Everything the exchange kernels need, by value.
struct EpDev {
  uint8_t* peer[kMaxWorld];  // every rank's EP buffer (own included)
  uint8_t* local;            // this rank's buffer
  int world, rank, e_loc, d;
  int cap_rows;
  size_t off_x, off_p, off_meta, off_flags, off_ret;
  unsigned* epoch;  // local: epoch of the current MoE layer
  int* done;        // local [2]: completion counters of the two push kernels
  int* send_off;    // local [world]: where this rank's run for rank r starts in r's buffer
  int* recv_off;    // local [world]: where rows from rank r start in this rank's buffer
  int* recv_rows;   // local [world]
  int* ret_off;     // local [world]: where rank r holds this rank's experts' rows (in r's ret)
  int4* tiles;      // local m-tile table over the received rows
  int* num_tiles;
  int* err;
};

__device__ __forceinline__ int pad_rows(int c) { return (c + kRows - 1) / kRows * kRows; }

__device__ __forceinline__ unsigned* flag_ptr(const EpDev& dv, int r, int phase, int src) {
  return reinterpret_cast<unsigned*>(dv.peer[r] + dv.off_flags) + phase * kMaxWorld + src;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Waits until this rank's flags of `phase` from every rank have reached the epoch.
__device__ __forceinline__ bool wait_flags(const EpDev& dv, int phase, unsigned epoch) {
  const unsigned long long start = global_timer_ns();
  for (int r = 0; r < dv.world; ++r) {
    const unsigned* f = flag_ptr(dv, dv.rank, phase, r);
    while (static_cast<int>(ld_acquire_sys(f) - epoch) < 0) {
      if (global_timer_ns() - start > kPeerWaitNs) return false;
      __nanosleep(128);
    }
  }
  return true;
}

// 2 + 3. Counts into every rank's inbox and the meta flags, then (thread 0) the device-side
// plan once every rank's counts are in. One CTA of 64 threads.
__global__ void ep_counts_plan_kernel(EpDev dv, const int* __restrict__ counts) {
  __shared__ unsigned epoch_s;
  const int e = threadIdx.x;
  if (e == 0) epoch_s = *dv.epoch + 1u;
  __syncthreads();
  const unsigned epoch = epoch_s;
  const int c = counts[e];
  for (int r = 0; r < dv.world; ++r) {
    reinterpret_cast<volatile int*>(dv.peer[r] + dv.off_meta)[dv.rank * kExperts + e] = c;
  }
  // The barrier orders every thread's count stores before thread 0's system-scope fence,
  // which orders them before the flags.
  __syncthreads();
  if (e != 0) return;
  *dv.epoch = epoch;
  fence_acq_rel_sys();
  for (int r = 0; r < dv.world; ++r) st_release_sys(flag_ptr(dv, r, kPhaseMeta, dv.rank), epoch);
  if (!wait_flags(dv, kPhaseMeta, epoch)) {
    record_error(dv.err, kErrTimeoutPeer);
    *dv.num_tiles = 0;
    for (int r = 0; r < dv.world; ++r) dv.send_off[r] = dv.recv_off[r] = dv.recv_rows[r] = dv.ret_off[r] = 0;
    return;
  }
  const volatile int* meta = reinterpret_cast<const volatile int*>(dv.local + dv.off_meta);  // [src][64]
  const int q = dv.rank, el = dv.e_loc;
  // Where this rank's run for rank r starts in r's buffer: after the runs of lower sources.
  for (int r = 0; r < dv.world; ++r) {
    int off = 0;
    for (int src = 0; src < q; ++src)
      for (int j = 0; j < el; ++j) off += pad_rows(meta[src * kExperts + r * el + j]);
    dv.send_off[r] = off;
  }
  int row = 0, nt = 0;
  bool fits = true;
  for (int src = 0; src < dv.world; ++src) {
    dv.recv_off[src] = row;
    // Source src holds its rows for this rank's experts from its own padded start of
    // expert q * el on; results go back there.
    int start = 0;
    for (int e = 0; e < q * el; ++e) start += pad_rows(meta[src * kExperts + e]);
    dv.ret_off[src] = start;
    for (int j = 0; j < el; ++j) {
      const int c = meta[src * kExperts + q * el + j];
      for (int i = 0; i * kRows < c; ++i) {
        if (row + (i + 1) * kRows > dv.cap_rows) {
          fits = false;
          break;
        }
        dv.tiles[nt++] = make_int4(j, row + i * kRows, min(kRows, c - i * kRows), 0);
      }
      row += pad_rows(c);
    }
    dv.recv_rows[src] = row - dv.recv_off[src];
  }
  if (!fits || row > dv.cap_rows) {
    record_error(dv.err, kErrBadShape);
    nt = 0;
  }
  *dv.num_tiles = nt;
}


// Copies `rows` rows of d BF16 (and optionally one float each) with 16-byte stores,
// grid-strided.
__device__ __forceinline__ void copy_rows(bf16* dst, const bf16* src, float* dst_p, const float* src_p, int rows,
                                          int d) {
  const int chunks = d / 8;
  const size_t n = static_cast<size_t>(rows) * chunks;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  }
  if (dst_p != nullptr) {
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < static_cast<size_t>(rows);
         i += stride) {
      dst_p[i] = src_p[i];
    }
  }
}

// The last CTA to finish raises the phase's flag on the given ranks. The barrier orders the
// CTA's stores before thread 0's GPU-scope fence and count; the last CTA's system-scope fence
// then orders every CTA's stores (they happen before it) before the flags, so one system
// fence a push is paid instead of one a CTA.
__device__ __forceinline__ void finish_push(const EpDev& dv, int counter, int phase, bool to_all) {
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    const int old = atomicAdd(dv.done + counter, 1);
    if (old == static_cast<int>(gridDim.x) - 1) {
      dv.done[counter] = 0;
      fence_acq_rel_sys();
      const unsigned epoch = *dv.epoch;
      for (int r = 0; r < dv.world; ++r) {
        if (to_all) st_release_sys(flag_ptr(dv, r, phase, dv.rank), epoch);
      }
    }
  }
}

// 4a. This rank's run for each rank into that rank's receive buffer.
__global__ void ep_push_rows_kernel(EpDev dv, const bf16* __restrict__ xperm, const float* __restrict__ pprob,
                                    const int* __restrict__ expert_start) {
  for (int r = 0; r < dv.world; ++r) {
    const int first = expert_start[r * dv.e_loc];
    const int rows = expert_start[(r + 1) * dv.e_loc] - first;
    const size_t at = static_cast<size_t>(dv.send_off[r]);
    if (at + rows > static_cast<size_t>(dv.cap_rows)) continue;  // the receiver's plan reports it
    bf16* dst = reinterpret_cast<bf16*>(dv.peer[r] + dv.off_x) + at * dv.d;
    float* dst_p = reinterpret_cast<float*>(dv.peer[r] + dv.off_p) + at;
    copy_rows(dst, xperm + static_cast<size_t>(first) * dv.d, dst_p, pprob + first, rows, dv.d);
  }
  finish_push(dv, 0, kPhaseRows, true);
}

// 4b/5. Waits for a phase's flags from every rank; the data is then read by TMA (async
// proxy) in the following kernels.
__global__ void ep_wait_kernel(EpDev dv, int phase) {
  if (threadIdx.x != 0) return;
  if (!wait_flags(dv, phase, *dv.epoch)) {
    record_error(dv.err, kErrTimeoutPeer);
    if (phase == kPhaseRows) *dv.num_tiles = 0;  // nothing runs on missing rows
  }
  fence_proxy_async_global();
}

// 4c. Results of each source's rows back into that source's `ret` buffer.
__global__ void ep_push_results_kernel(EpDev dv, const bf16* __restrict__ y) {
  const int d = dv.d;
  for (int src = 0; src < dv.world; ++src) {
    bf16* dst = reinterpret_cast<bf16*>(dv.peer[src] + dv.off_ret) + static_cast<size_t>(dv.ret_off[src]) * d;
    copy_rows(dst, y + static_cast<size_t>(dv.recv_off[src]) * d, nullptr, nullptr, dv.recv_rows[src], d);
  }
  finish_push(dv, 1, kPhaseResults, true);
}

EpDev ep_dev(const Model& m) {
  EpDev dv{};
  for (int r = 0; r < m.ep_world; ++r) dv.peer[r] = m.ep_peer[r];
  dv.local = m.ep_buf;
  dv.world = m.ep_world;
  dv.rank = m.ep_rank;
  dv.e_loc = kExperts / m.ep_world;
  dv.d = m.cfg.d_model;
  dv.cap_rows = static_cast<int>(m.ep_cap_rows);
  dv.off_x = m.ep_off.x;
  dv.off_p = m.ep_off.p;
  dv.off_meta = m.ep_off.meta;
  dv.off_flags = m.ep_off.flags;
  dv.off_ret = m.ep_off.ret;
  auto at = [&](size_t o) { return m.ep_buf + o; };
  dv.epoch = reinterpret_cast<unsigned*>(at(m.ep_off.epoch));
  dv.done = reinterpret_cast<int*>(at(m.ep_off.done));
  dv.send_off = reinterpret_cast<int*>(at(m.ep_off.send_off));
  dv.recv_off = reinterpret_cast<int*>(at(m.ep_off.recv_off));
  dv.recv_rows = reinterpret_cast<int*>(at(m.ep_off.recv_rows));
  dv.ret_off = reinterpret_cast<int*>(at(m.ep_off.ret_off));
  dv.tiles = reinterpret_cast<int4*>(at(m.ep_off.tiles));
  dv.num_tiles = reinterpret_cast<int*>(at(m.ep_off.num_tiles));
  dv.err = device_error_word();
  return dv;
}

}  // namespace

EpPlan ep_plan(int world, int rank, const int2* meta_send, const int2* meta_recv) {
  require(world >= 1 && kExperts % world == 0 && rank >= 0 && rank < world,
          "expert parallel: world must divide 64");
  const int e_loc = kExperts / world;
  EpPlan p;
  p.send_off.assign(world, 0);
  p.send_rows.assign(world, 0);
  p.recv_off.assign(world, 0);
  p.recv_rows.assign(world, 0);
  int off = 0;
  for (int r = 0; r < world; ++r) {
    p.send_off[r] = off;
    for (int e = 0; e < e_loc; ++e) p.send_rows[r] += meta_send[r * e_loc + e].x;
    off += p.send_rows[r];
  }
  int roff = 0;
  for (int r = 0; r < world; ++r) {
    p.recv_off[r] = roff;
    int seg = roff;
    for (int e = 0; e < e_loc; ++e) {
      const int2 m = meta_recv[r * e_loc + e];
      require(m.x >= 0 && m.y >= 0 && m.x % kRows == 0 && m.y <= m.x && m.x - m.y < kRows,
              "expert parallel: malformed segment metadata");
      for (int i = 0; i * kRows < m.y; ++i) {
        p.tiles.push_back({rank * e_loc + e, seg + i * kRows, std::min(kRows, m.y - i * kRows), 0});
      }
      seg += m.x;
      p.recv_rows[r] += m.x;
    }
    roff += p.recv_rows[r];
  }
  p.recv_total = roff;
  return p;
}

void Model::repack_experts(int rank, int world) {
  const int e_loc = kExperts / world;
  const std::map<std::string, Slot> old_slots = slots;
  uint8_t* old_arena = arena;
  slots.clear();
  plan_weights(e_loc);
  uint8_t* fresh = nullptr;
  check_cuda(cudaMalloc(&fresh, arena_bytes), "cudaMalloc expert-parallel weights");
  for (auto& kv : slots) {
    const Slot& o = old_slots.at(kv.first);
    Slot& n = kv.second;
    // Expert tensors keep this rank's e_loc consecutive experts; the rest is copied whole.
    const bool expert = n.shape.size() == 3 && n.shape[0] == e_loc && o.shape[0] == kExperts;
    const size_t src = o.offset + (expert ? n.bytes * static_cast<size_t>(rank) : 0);
    check_cuda(cudaMemcpy(fresh + n.offset, old_arena + src, n.bytes, cudaMemcpyDeviceToDevice),
               "repack weights");
    n.set = true;
  }
  arena = fresh;
  check_cuda(cudaFree(old_arena), "free full weights");
  experts_held = e_loc;
}

void Model::enable_expert_parallel(int rank, int world, const void* unique_id) {
  require(cfg.arch == CE4B_ARCH_MOE64A2, "expert parallelism needs a moe64a2 model");
  require(world >= 2 && world <= kMaxWorld && kExperts % world == 0,
          "expert parallel world size must divide 64 and be at most 8");
  require(rank >= 0 && rank < world && unique_id != nullptr, "bad expert parallel rank");
  require(ep_comm == nullptr, "expert parallelism is already enabled");
  require(finalized, "expert parallelism needs a finalized model");
  check_cuda(cudaSetDevice(device), "cudaSetDevice");
  const int d = cfg.d_model;
  const int e_loc = kExperts / world;
  // Worst case received rows: every source sends all 2 * max_batch routes to this rank's
  // experts, each of its e_loc segments padded by up to 127 rows.
  ep_cap_rows = static_cast<size_t>(world) * (2 * static_cast<size_t>(rows_cap) + e_loc * (kRows - 1));
  ep_cap_rows = (ep_cap_rows + kRows - 1) / kRows * kRows;
  const size_t cap = ep_cap_rows;
  size_t cur = 0;
  auto take = [&](size_t bytes) {
    const size_t o = (cur + 255) / 256 * 256;
    cur = o + bytes;
    return o;
  };
  ep_off.x = take(cap * d * 2);
  ep_off.p = take(cap * 4);
  ep_off.meta = take(static_cast<size_t>(kMaxWorld) * kExperts * 4);
  ep_off.flags = take(3 * kMaxWorld * 4);
  ep_off.ret = take(static_cast<size_t>(perm_rows) * d * 2);
  ep_off.h = take(cap * expert_hidden * 2);
  ep_off.y = take(cap * d * 2);
  ep_off.counts = take(kExperts * 4);
  ep_off.epoch = take(4);
  ep_off.done = take(2 * 4);
  ep_off.send_off = take(kMaxWorld * 4);
  ep_off.recv_off = take(kMaxWorld * 4);
  ep_off.recv_rows = take(kMaxWorld * 4);
  ep_off.ret_off = take(kMaxWorld * 4);
  ep_off.tiles = take((cap / kRows) * 16);
  ep_off.num_tiles = take(16);
  ep_buf_bytes = cur;
  check_cuda(cudaMalloc(&ep_buf, ep_buf_bytes), "cudaMalloc expert-parallel buffers");
  check_cuda(cudaMemset(ep_buf, 0, ep_buf_bytes), "clear expert-parallel buffers");
  // Every rank's buffer handle to every rank (NCCL send/recv of the 64-byte IPC handles);
  // the exchange also orders every rank's clearing of its flags before any peer write.
  cudaIpcMemHandle_t own{};
  check_cuda(cudaIpcGetMemHandle(&own, ep_buf), "cudaIpcGetMemHandle");
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  ncclComm_t comm = nullptr;
  const NcclApi& api = nccl();
  check_nccl(api.CommInitRank(&comm, world, id, rank), "ncclCommInitRank");
  ep_comm = comm;
  uint8_t* handles = nullptr;
  check_cuda(cudaMalloc(&handles, 2 * kMaxWorld * sizeof(cudaIpcMemHandle_t)), "cudaMalloc handles");
  check_cuda(cudaMemcpy(handles, &own, sizeof(own), cudaMemcpyHostToDevice), "copy handle");
  check_cuda(cudaDeviceSynchronize(), "clear expert-parallel buffers");
  check_nccl(api.GroupStart(), "ncclGroupStart");
  for (int r = 0; r < world; ++r) {
    check_nccl(api.Send(handles, sizeof(own), ncclUint8, r, comm, stream), "ncclSend handle");
    check_nccl(api.Recv(handles + (kMaxWorld + r) * sizeof(own), sizeof(own), ncclUint8, r, comm, stream),
               "ncclRecv handle");
  }
  check_nccl(api.GroupEnd(), "ncclGroupEnd");
  std::vector<cudaIpcMemHandle_t> all(world);
  check_cuda(cudaMemcpyAsync(all.data(), handles + kMaxWorld * sizeof(own), world * sizeof(own),
                             cudaMemcpyDeviceToHost, stream),
             "copy handles");
  check_cuda(cudaStreamSynchronize(stream), "handle exchange");
  cudaFree(handles);
  ep_peer.assign(world, nullptr);
  for (int r = 0; r < world; ++r) {
    if (r == rank) {
      ep_peer[r] = ep_buf;
      continue;
    }
    void* p = nullptr;
    check_cuda(cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    ep_peer[r] = static_cast<uint8_t*>(p);
  }
  ep_world = world;
  ep_rank = rank;
  // Only this rank's experts stay resident.
  repack_experts(rank, world);
  finalize();
  tm_ep_x = make_tmap_bf16(ep_buf + ep_off.x, cap, d, d, 128);
  tm_ep_h = make_tmap_bf16(ep_buf + ep_off.h, cap, expert_hidden, expert_hidden, 128);
  tm_ep_y = make_tmap_bf16(ep_buf + ep_off.y, cap, d, d, 128);
  graphs_clear();
}

void Model::disable_expert_parallel() {
  for (int r = 0; r < static_cast<int>(ep_peer.size()); ++r) {
    if (r != ep_rank && ep_peer[r] != nullptr) cudaIpcCloseMemHandle(ep_peer[r]);
  }
  ep_peer.clear();
  if (ep_comm != nullptr) {
    nccl().CommDestroy(static_cast<ncclComm_t>(ep_comm));
    ep_comm = nullptr;
  }
  if (ep_buf != nullptr) cudaFree(ep_buf);
  ep_buf = nullptr;
  ep_world = 1;
  ep_rank = 0;
}

void Model::moe_layer_ep(const Layer& L, int moe_index, const bf16* next_norm, int batch,
                         int32_t* tokens_per_expert, cudaStream_t s) {
  const int d = cfg.d_model;
  const int he = expert_hidden;
  auto at = [&](size_t off) { return workspace + off; };
  auto* route_expert = reinterpret_cast<int2*>(at(ws_off.route_expert));
  auto* route_prob = reinterpret_cast<float2*>(at(ws_off.route_prob));
  auto* route_pos = reinterpret_cast<int*>(at(ws_off.route_pos));
  auto* block_hist = reinterpret_cast<int*>(at(ws_off.block_hist));
  auto* block_off = reinterpret_cast<int*>(at(ws_off.block_off));
  auto* expert_start = reinterpret_cast<int*>(at(ws_off.expert_start));
  auto* m_tiles = reinterpret_cast<int4*>(at(ws_off.m_tiles));
  auto* num_m_tiles = reinterpret_cast<int*>(at(ws_off.num_m_tiles));
  auto* xperm = reinterpret_cast<bf16*>(at(ws_off.xperm));
  auto* pprob = reinterpret_cast<float*>(at(ws_off.pprob));
  auto* x = reinterpret_cast<bf16*>(at(ws_off.x));
  auto* n = reinterpret_cast<bf16*>(at(ws_off.n));
  auto* counts = reinterpret_cast<int*>(ep_buf + ep_off.counts);
  const EpDev dv = ep_dev(*this);

  moe_router_gemm(tm_n, L.tm_router, L.beta, route_expert, route_prob, block_hist, batch, d, s);
  trace("moe_router", s);
  moe_scan(block_hist, (batch + 127) / 128, expert_start, block_off, m_tiles, num_m_tiles, counts, s);
  trace("moe_scan", s);
  moe_dispatch(n, route_expert, route_prob, expert_start, block_off, xperm, pprob, route_pos,
               batch, d, s);
  trace("moe_dispatch", s);
  if (tokens_per_expert != nullptr) {
    check_cuda(cudaMemcpyAsync(tokens_per_expert + kExperts * moe_index, counts, kExperts * 4,
                               cudaMemcpyDeviceToDevice, s),
               "copy expert counts");
  }
  ep_counts_plan_kernel<<<1, kExperts, 0, s>>>(dv, counts);
  check_cuda(cudaGetLastError(), "ep_counts_plan launch");
  trace("ep_counts_plan", s);
  const int copy_grid = std::max(1, std::min(4 * sm_count(), (batch * 2 * (d / 8) + 255) / 256));
  ep_push_rows_kernel<<<copy_grid, 256, 0, s>>>(dv, xperm, pprob, expert_start);
  check_cuda(cudaGetLastError(), "ep_push_rows launch");
  trace("ep_push_rows", s);
  ep_wait_kernel<<<1, 32, 0, s>>>(dv, kPhaseRows);
  check_cuda(cudaGetLastError(), "ep_wait launch");
  trace("ep_wait_rows", s);

  auto* ep_p = reinterpret_cast<float*>(ep_buf + ep_off.p);
  gemm_grouped_swiglu(tm_ep_x, L.tm_gate_up, tm_ep_h, dv.tiles, dv.num_tiles, he, d, s);
  trace("moe_experts_gate_up_swiglu", s);
  gemm_grouped_scale(tm_ep_h, L.tm_down, tm_ep_y, dv.tiles, dv.num_tiles, ep_p, d, he, s);
  trace("moe_experts_down", s);

  ep_push_results_kernel<<<copy_grid, 256, 0, s>>>(dv, reinterpret_cast<const bf16*>(ep_buf + ep_off.y));
  check_cuda(cudaGetLastError(), "ep_push_results launch");
  trace("ep_push_results", s);
  ep_wait_kernel<<<1, 32, 0, s>>>(dv, kPhaseResults);
  check_cuda(cudaGetLastError(), "ep_wait launch");
  trace("ep_wait_results", s);
  moe_combine_norm(x, reinterpret_cast<const bf16*>(ep_buf + ep_off.ret), route_pos, next_norm, n, batch, d,
                   cfg.rms_norm_eps, s);
  trace("moe_combine_rmsnorm", s);
}

}  // namespace ce4b
