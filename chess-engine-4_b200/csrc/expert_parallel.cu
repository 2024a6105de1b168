// Expert parallelism for moe64a2: the 64 experts are split over `world` ranks (64 / world
// consecutive experts each); every rank routes its own tokens and the routed rows travel
// to the rank that owns their expert and back with NCCL send/recv over NVLink.
//
// One MoE layer on one rank (the reference's static dispatch path, moe.py:226-287, with an
// all-to-all of the routed rows between the ranks that own the experts):
//   1. router GEMM + top-2, routing scan, dispatch into 128-row expert segments (the same
//      kernels as the single-GPU layer). Segments are ordered by expert, so the rows for
//      rank r are one contiguous run.
//   2. per-expert {padded rows, valid rows} go to every rank (NCCL), then to the host
//      (one synchronisation per layer): each rank plans its receive layout and the m-tile
//      table of the grouped GEMMs over the received rows.
//   3. rows and route weights travel (NCCL); the grouped gate_up + SwiGLU and down x route
//      weight GEMMs run on the received rows with this rank's experts; results travel back
//      to the same rows of the sender's permuted buffer.
//   4. combine + residual + next RMSNorm (single-GPU kernel).
// A GEMM row depends only on its own inputs, so results equal the single-GPU forward's.
#include <algorithm>
#include <cstring>
#include <vector>

#include "model.h"
#include "nccl_dl.h"

namespace ce4b {

namespace {

constexpr int kExperts = 64;
constexpr int kRows = 128;

// meta[g] = {rows of expert g's segment (padded to 128), valid rows}.
__global__ void ep_meta_kernel(const int* __restrict__ counts, int2* __restrict__ meta) {
  const int g = threadIdx.x;
  if (g < kExperts) {
    const int c = counts[g];
    meta[g] = make_int2((c + kRows - 1) / kRows * kRows, c);
  }
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

void Model::enable_expert_parallel(int rank, int world, const void* unique_id) {
  require(cfg.arch == CE4B_ARCH_MOE64A2, "expert parallelism needs a moe64a2 model");
  require(world >= 2 && kExperts % world == 0, "expert parallel world size must divide 64");
  require(rank >= 0 && rank < world && unique_id != nullptr, "bad expert parallel rank");
  require(ep_comm == nullptr, "expert parallelism is already enabled");
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
  const size_t o_x = take(cap * d * 2), o_h = take(cap * expert_hidden * 2), o_y = take(cap * d * 2);
  const size_t o_p = take(cap * 4), o_c = take(kExperts * 4), o_m = take(2 * kExperts * 8);
  const size_t o_t = take((cap / kRows) * 16), o_n = take(16);
  check_cuda(cudaMalloc(&ep_buf, cur), "cudaMalloc expert-parallel buffers");
  ep_x = reinterpret_cast<bf16*>(ep_buf + o_x);
  ep_h = reinterpret_cast<bf16*>(ep_buf + o_h);
  ep_y = reinterpret_cast<bf16*>(ep_buf + o_y);
  ep_p = reinterpret_cast<float*>(ep_buf + o_p);
  ep_counts = reinterpret_cast<int*>(ep_buf + o_c);
  ep_meta = reinterpret_cast<int2*>(ep_buf + o_m);
  ep_tiles = reinterpret_cast<int4*>(ep_buf + o_t);
  ep_num_tiles = reinterpret_cast<int*>(ep_buf + o_n);
  check_cuda(cudaMallocHost(&ep_host, 2 * kExperts * sizeof(int2) + (cap / kRows + 1) * sizeof(int4)),
             "cudaMallocHost expert-parallel staging");
  tm_ep_x = make_tmap_bf16(ep_x, cap, d, d, 128);
  tm_ep_h = make_tmap_bf16(ep_h, cap, expert_hidden, expert_hidden, 128);
  tm_ep_y = make_tmap_bf16(ep_y, cap, d, d, 128);
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  ncclComm_t comm = nullptr;
  check_nccl(nccl().CommInitRank(&comm, world, id, rank), "ncclCommInitRank");
  ep_comm = comm;
  ep_world = world;
  ep_rank = rank;
  graphs_clear();
}

void Model::disable_expert_parallel() {
  if (ep_comm != nullptr) {
    nccl().CommDestroy(static_cast<ncclComm_t>(ep_comm));
    ep_comm = nullptr;
  }
  if (ep_buf != nullptr) cudaFree(ep_buf);
  if (ep_host != nullptr) cudaFreeHost(ep_host);
  ep_buf = nullptr;
  ep_host = nullptr;
  ep_world = 1;
  ep_rank = 0;
}

void Model::moe_layer_ep(const Layer& L, int moe_index, const bf16* next_norm, int batch,
                         int32_t* tokens_per_expert, cudaStream_t s) {
  const int d = cfg.d_model;
  const int he = expert_hidden;
  const int world = ep_world;
  const int e_loc = kExperts / world;
  const NcclApi& api = nccl();
  auto comm = static_cast<ncclComm_t>(ep_comm);
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
  auto* yperm = reinterpret_cast<bf16*>(at(ws_off.yperm));
  auto* x = reinterpret_cast<bf16*>(at(ws_off.x));
  auto* n = reinterpret_cast<bf16*>(at(ws_off.n));

  moe_router_gemm(tm_n, L.tm_router, L.beta, route_expert, route_prob, block_hist, batch, d, s);
  trace("moe_router", s);
  moe_scan(block_hist, (batch + 127) / 128, expert_start, block_off, m_tiles, num_m_tiles,
           ep_counts, s);
  trace("moe_scan", s);
  moe_dispatch(n, route_expert, route_prob, expert_start, block_off, xperm, pprob, route_pos,
               batch, d, s);
  trace("moe_dispatch", s);
  if (tokens_per_expert != nullptr) {
    check_cuda(cudaMemcpyAsync(tokens_per_expert + kExperts * moe_index, ep_counts, kExperts * 4,
                               cudaMemcpyDeviceToDevice, s),
               "copy expert counts");
  }

  // Segment metadata to every rank, then to the host.
  int2* meta_send = ep_meta;
  int2* meta_recv = ep_meta + kExperts;
  ep_meta_kernel<<<1, kExperts, 0, s>>>(ep_counts, meta_send);
  check_cuda(cudaGetLastError(), "ep_meta launch");
  check_nccl(api.GroupStart(), "ncclGroupStart");
  for (int r = 0; r < world; ++r) {
    check_nccl(api.Send(meta_send + r * e_loc, 2 * e_loc, ncclInt32, r, comm, s), "ncclSend meta");
    check_nccl(api.Recv(meta_recv + r * e_loc, 2 * e_loc, ncclInt32, r, comm, s), "ncclRecv meta");
  }
  check_nccl(api.GroupEnd(), "ncclGroupEnd");
  auto* host_meta = reinterpret_cast<int2*>(ep_host);
  check_cuda(cudaMemcpyAsync(host_meta, ep_meta, 2 * kExperts * sizeof(int2), cudaMemcpyDeviceToHost, s),
             "copy expert metadata");
  check_cuda(cudaStreamSynchronize(s), "expert metadata");
  const EpPlan plan = ep_plan(world, ep_rank, host_meta, host_meta + kExperts);
  require(static_cast<size_t>(plan.recv_total) <= ep_cap_rows, "expert parallel receive overflow");
  auto* host_tiles = reinterpret_cast<int4*>(host_meta + 2 * kExperts);
  const int nt = static_cast<int>(plan.tiles.size());
  std::copy(plan.tiles.begin(), plan.tiles.end(), host_tiles);
  host_tiles[nt] = make_int4(nt, 0, 0, 0);
  check_cuda(cudaMemcpyAsync(ep_tiles, host_tiles, nt * sizeof(int4), cudaMemcpyHostToDevice, s),
             "copy expert tiles");
  check_cuda(cudaMemcpyAsync(ep_num_tiles, &host_tiles[nt].x, sizeof(int), cudaMemcpyHostToDevice, s),
             "copy expert tile count");

  // Rows and route weights to the experts' ranks.
  check_nccl(api.GroupStart(), "ncclGroupStart");
  for (int r = 0; r < world; ++r) {
    const size_t so = plan.send_off[r], sr = plan.send_rows[r];
    const size_t ro = plan.recv_off[r], rr = plan.recv_rows[r];
    if (sr > 0) {
      check_nccl(api.Send(xperm + so * d, sr * d, ncclBfloat16, r, comm, s), "ncclSend rows");
      check_nccl(api.Send(pprob + so, sr, ncclFloat32, r, comm, s), "ncclSend weights");
    }
    if (rr > 0) {
      check_nccl(api.Recv(ep_x + ro * d, rr * d, ncclBfloat16, r, comm, s), "ncclRecv rows");
      check_nccl(api.Recv(ep_p + ro, rr, ncclFloat32, r, comm, s), "ncclRecv weights");
    }
  }
  check_nccl(api.GroupEnd(), "ncclGroupEnd");
  trace("moe_dispatch_all_to_all", s);

  gemm_grouped_swiglu(tm_ep_x, L.tm_gate_up, tm_ep_h, ep_tiles, ep_num_tiles, he, d, s);
  trace("moe_experts_gate_up_swiglu", s);
  gemm_grouped_scale(tm_ep_h, L.tm_down, tm_ep_y, ep_tiles, ep_num_tiles, ep_p, d, he, s);
  trace("moe_experts_down", s);

  // Results back into the sender's permuted layout.
  check_nccl(api.GroupStart(), "ncclGroupStart");
  for (int r = 0; r < world; ++r) {
    const size_t so = plan.send_off[r], sr = plan.send_rows[r];
    const size_t ro = plan.recv_off[r], rr = plan.recv_rows[r];
    if (rr > 0) check_nccl(api.Send(ep_y + ro * d, rr * d, ncclBfloat16, r, comm, s), "ncclSend results");
    if (sr > 0) check_nccl(api.Recv(yperm + so * d, sr * d, ncclBfloat16, r, comm, s), "ncclRecv results");
  }
  check_nccl(api.GroupEnd(), "ncclGroupEnd");
  trace("moe_combine_all_to_all", s);
  moe_combine_norm(x, yperm, route_pos, next_norm, n, batch, d, cfg.rms_norm_eps, s);
  trace("moe_combine_rmsnorm", s);
}

}  // namespace ce4b
