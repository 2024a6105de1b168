// Model handle behind the opaque ce4b_model of the C ABI.
#pragma once

#include <algorithm>
#include <array>
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "internal.h"
#include "latency_types.h"

namespace ce4b {

// Host plan of one expert-parallel exchange (csrc/expert_parallel.cu): rows of the local
// permuted buffer sent to each rank, rows received from each rank (in rank order, each
// source's expert segments in expert order) and the m-tile table over the received rows
// ({global expert, first row, valid rows, 0}).
struct EpPlan {
  std::vector<int> send_off, send_rows, recv_off, recv_rows;
  std::vector<int4> tiles;
  int recv_total = 0;
};
// meta_send[g] / meta_recv[r * (64 / world) + e] = {segment rows padded to 128, valid rows}.
EpPlan ep_plan(int world, int rank, const int2* meta_send, const int2* meta_recv);

struct Model {
  struct Slot {
    size_t offset = 0;
    size_t bytes = 0;
    std::vector<int64_t> shape;
    int dtype = CE4B_DTYPE_BF16;
    bool set = false;
  };
  struct Layer {
    bool moe = false;
    const bf16* norm = nullptr;
    CUtensorMap tm_gate_up{};  // dense gate_up, or stacked expert gate_up [64*2h_e, d]
    CUtensorMap tm_down{};     // dense down, or stacked expert down [64*d, h_e]
    CUtensorMap tm_router{};   // MoE router [64, d]
    const float* beta = nullptr;  // MoE router_qb_beta [64]
    const uint8_t* gu_scales = nullptr;    // MXFP8 weight scales
    const uint8_t* down_scales = nullptr;
  };
  struct WorkspaceOffsets {
    size_t a_in = 0, x = 0, n = 0, hidden = 0;
    size_t route_expert = 0, route_prob = 0, route_pos = 0, block_hist = 0, block_off = 0;
    size_t expert_start = 0, m_tiles = 0, num_m_tiles = 0, xperm = 0, pprob = 0, hperm = 0;
    size_t yperm = 0;
    size_t a_codes = 0, a_scales = 0, n_codes = 0, n_scales = 0, h_codes = 0, h_scales = 0;
    size_t fwd_ss = 0, fwd_part = 0, fwd_sync = 0;  // persistent dense forward
    size_t lat_part_in = 0, lat_part_dn = 0, lat_sync = 0;  // small-batch forward
  };

  ce4b_model_config cfg{};
  int device = -1;
  int max_batch = 0;
  int rows_cap = 0;
  int dense_hidden = 0;
  int expert_hidden = 0;
  int sel = 0;
  int in_dim = 0;
  int policy_size = 0;
  int policy_storage = 0;
  int perm_rows = 0;  // MoE permuted-row capacity

  uint8_t* arena = nullptr;
  size_t arena_bytes = 0;
  std::map<std::string, Slot> slots;
  uint8_t* workspace = nullptr;
  bool mx = false;                // precision MXFP8
  // Dense BF16 towers run as one persistent kernel (forward.cuh): its tensor maps and
  // norm-weight table live in fwd_dev.
  bool fused = false;
  uint8_t* fwd_dev = nullptr;      // FwdMaps
  bf16* fwd_weights = nullptr;     // norm-folded gate_up [depth][2h, d], then heads [Ps + 64, d]
  size_t fwd_sync_bytes = 0;
  unsigned long long* fwd_trace = nullptr;  // optional per-task timeline (device buffer)
  int fwd_trace_cap = 0;
  // Optional routing tap (tests): each MoE layer's expert pair per token,
  // [depth/2][batch][2] int32, written by forwards outside stream capture.
  int32_t* moe_tap = nullptr;
  int moe_tap_tokens = 0;
  // Optional MXFP8 tap (tests): the operands of one layer's quantisation points.
  ce4b_mxfp8_tap mx_tap{-1, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
  // Column width of the persistent forward's input and down tiles for this batch: 256 once
  // a layer's 256-wide down tiles fill two waves of SMs (throughput-bound), else 128
  // (the per-row-block dependency chain bounds the forward; more, narrower tiles help it).
  int fused_xw(int batch) const {
    const int nb = (batch + 127) / 128;
    return cfg.d_model % 256 == 0 && nb * (cfg.d_model / 256) >= 2 * sm_count() ? 256 : 128;
  }
  // Input tiles: 256 columns where d allows.
  int fused_xwi() const { return cfg.d_model % 256 == 0 ? 256 : 128; }
  // Small batches leave most SMs idle while each row block's chain runs: the input tiles
  // are then split into 8 K parts, the parts summed in fixed order by the last finisher.
  // Row blocks up to which this applies:
  int fused_small_nb() const {
    const int per_rb = (cfg.d_model / fused_xwi()) * 8;
    return std::max(0, std::min(rows_cap / 128, sm_count() / per_rb));
  }
  bool fused_small(int batch) const {
    const int nb = (batch + 127) / 128;
    return nb <= fused_small_nb() && fused_xw(batch) == 128;
  }
  int fused_kis(int batch) const { return fused_small(batch) ? 8 : 2; }
  // Down tiles are not split along K: with 96-deep stages a 128-column down tile runs
  // 6 MMAs per stage, and splitting it in 2 or 4 parts measured equal or slower at every
  // batch (B = 64 249 vs 249 µs, 256: 253 vs 257, 640: 259 vs 266, 1152: 262 vs 275 with
  // 4 parts; 2 parts slower still). The kernel keeps the split (dks parts) as a parameter.
  int fused_dks(int) const { return 1; }
  int fused_head_tasks() const { return (policy_storage + 64 + 255) / 256; }
  int fused_task_count(int batch) const {
    const int nb = (batch + 127) / 128, xt = cfg.d_model / fused_xw(batch), nc = dense_hidden / 128;
    return nb * (cfg.d_model / fused_xwi()) * fused_kis(batch) +
           cfg.depth * nb * (nc + xt * fused_dks(batch)) + nb * fused_head_tasks();
  }
  // Small-batch forward (latency.cu): dense BF16 models with d <= 512 run batches of at
  // most kLatMaxRows positions as one cooperative launch of short transposed tiles spread
  // over the SMs. Planned at create (lat = the shape allows it); lat_enabled can turn it
  // off (ce4b_model_set_latency_path), which sends small batches to the persistent forward.
  bool lat = false;
  bool lat_enabled = true;
  int lat_grid = 0, lat_max_tasks = 0, lat_kp_in = 0, lat_kp_dn = 0;
  uint8_t* lat_dev = nullptr;  // LatMaps, then the [grid][max_tasks] task table
  size_t lat_sync_bytes = 0;
  bool latency_path(int batch) const { return lat && lat_enabled && batch <= kLatMaxRows; }
  void plan_latency();
  void build_latency();
  void forward_latency(int layout, void* input, const void* scalars, int batch, float* policy,
                       float* wdl, float* moves_left, int wdl_probs, int write_back, cudaStream_t s);
  uint8_t* mx_arena = nullptr;    // quantised weights (codes + scales)
  size_t mx_arena_bytes = 0;
  const uint8_t* w_in_scales = nullptr;
  const uint8_t* heads_scales = nullptr;
  int heads_rows_mx = 0;          // head rows padded to a multiple of 128
  size_t workspace_bytes = 0;
  WorkspaceOffsets ws_off;

  CUtensorMap tm_a_in{}, tm_x{}, tm_n{}, tm_hidden{}, tm_w_in{}, tm_heads{};
  CUtensorMap tm_xperm{}, tm_hperm{}, tm_yperm{};
  CUtensorMap tm_a_u8{}, tm_n_u8{}, tm_h_u8{};  // MXFP8 activation codes
  std::vector<Layer> layers;
  bool finalized = false;
  cudaStream_t stream = nullptr;
  // Host-buffer evaluation keeps kIoSlots sets of device planes / outputs so that the
  // copies of one call overlap the forward of the next when calls come on different
  // streams. A slot is reused only after its last D2H copy (io[slot].free); forwards share
  // the workspace and are ordered by forward_done.
  static constexpr int kIoSlots = 2;
  struct IoSlot {
    size_t planes = 0, policy = 0, wdl = 0, moves_left = 0;  // workspace offsets
    size_t move_offsets = 0, move_indices = 0, move_probs = 0;  // legal-move policy
    cudaEvent_t free = nullptr;
  };
  static constexpr int kMaxMovesPerPosition = 256;  // chess has at most 218 legal moves
  IoSlot io[kIoSlots];
  unsigned io_next = 0;
  cudaEvent_t forward_done = nullptr;
  std::map<int, cudaGraphExec_t> graphs;  // key: batch * kIoSlots + slot
  // Small-batch evaluations whose host buffers are pinned and mapped (device-accessible)
  // run without copies: the expansion kernel reads the records from host memory and the
  // heads write policy, WDL and moves-left into the caller's buffers. One graph per
  // (batch, buffers), at most kDirectGraphs of them (the set is dropped when full).
  static constexpr size_t kDirectGraphs = 16;
  bool direct_io = true;  // ce4b_model_set_direct_io
  std::map<std::array<uintptr_t, 5>, cudaGraphExec_t> direct_graphs;
  // Captures forward() of an lc0 batch with the given device-visible pointers on the
  // internal stream (run once outside the capture first, for kernel attributes). Blocks.
  cudaGraphExec_t capture_evaluate(const ce4b_input_plane* planes, int batch, float* policy,
                                   float* wdl, float* moves_left);
  // The direct graph for these host buffers, or nullptr when they are not all pinned and
  // mapped over their whole extent or the batch does not take the small-batch forward.
  cudaGraphExec_t direct_graph(const ce4b_input_plane* host_planes, int batch, float* host_policy,
                               float* host_wdl, float* host_moves_left);
  // Optional per-kernel trace: an event is recorded after each kernel of forward().
  std::vector<cudaEvent_t> trace_events;
  std::vector<std::string> trace_labels;
  size_t trace_next = 0;

  Model() = default;
  Model(const Model&) = delete;
  Model& operator=(const Model&) = delete;
  ~Model();

  bool is_moe_layer(int l) const { return cfg.arch == CE4B_ARCH_MOE64A2 && l % 2 == 0; }
  void create(const ce4b_model_config& c, int device, int max_batch);
  void set_tensor(const std::string& name, const void* data, int dtype,
                  const std::vector<int64_t>& shape, bool src_device);
  void finalize();
  void forward(int layout, void* input, const void* scalars, int batch, float* policy, float* wdl,
               float* moves_left, int wdl_probs, int normalize_in_place,
               int32_t* tokens_per_expert, cudaStream_t s);
  // forward() ordered after every earlier forward of this model on any stream (outside
  // stream capture), so calls on different streams never share the workspace in flight.
  void forward_ordered(int layout, void* input, const void* scalars, int batch, float* policy,
                       float* wdl, float* moves_left, int wdl_probs, int normalize_in_place,
                       int32_t* tokens_per_expert, cudaStream_t s);
  void evaluate(const ce4b_input_plane* host_planes, int batch, float* host_policy,
                float* host_wdl, float* host_moves_left);
  void enqueue_evaluate(const ce4b_input_plane* host_planes, int batch, float* host_policy,
                        float* host_wdl, float* host_moves_left, cudaStream_t s);
  // As enqueue_evaluate, but returns only legal-move probabilities (softmax of the gathered
  // logits times temperature) instead of the full policy.
  void enqueue_evaluate_legal(const ce4b_input_plane* host_planes, int batch,
                              const int32_t* host_offsets, const int32_t* host_indices,
                              float temperature, float* host_probs, float* host_wdl,
                              float* host_moves_left, cudaStream_t s);
  // Graph of the host-buffer forward for (batch, slot), built on first use.
  cudaGraphExec_t evaluate_graph(int batch, int slot);
  void trace(const char* label, cudaStream_t s);
  void quantize_weights();
  void forward_mx(int layout, void* input, const void* scalars, int batch, float* policy,
                  float* wdl, float* moves_left, int wdl_probs, int write_back, cudaStream_t s);
  void forward_fused(int layout, void* input, const void* scalars, int batch, float* policy,
                     float* wdl, float* moves_left, int wdl_probs, int write_back, cudaStream_t s);
  // Expert parallelism (moe64a2): each of ep_world ranks holds and computes 64 / ep_world
  // consecutive experts (the weight arena is repacked to them). Routed rows, their weights
  // and the results travel through every rank's shared EP buffer over NVLink peer memory
  // (CUDA IPC), ordered by per-layer epoch flags; NCCL only carries the IPC handles once.
  int ep_world = 1;
  int ep_rank = 0;
  void* ep_comm = nullptr;        // ncclComm_t used at set-up
  size_t ep_cap_rows = 0;         // received-row capacity
  uint8_t* ep_buf = nullptr;      // this rank's buffer: shared part, then local part
  size_t ep_buf_bytes = 0;
  std::vector<uint8_t*> ep_peer;  // every rank's buffer (own included), IPC-mapped
  struct EpOffsets {
    size_t x = 0, p = 0, meta = 0, flags = 0, ret = 0;  // shared: peers write these
    size_t h = 0, y = 0, counts = 0, epoch = 0, done = 0, send_off = 0, recv_off = 0, recv_rows = 0,
           ret_off = 0, tiles = 0, num_tiles = 0;       // local
  } ep_off;
  CUtensorMap tm_ep_x{}, tm_ep_h{}, tm_ep_y{};
  // Experts held per MoE layer (64, or 64 / ep_world once the arena is repacked).
  int experts_held = 64;
  void enable_expert_parallel(int rank, int world, const void* unique_id);
  void disable_expert_parallel();
  void moe_layer_ep(const Layer& L, int moe_index, const bf16* next_norm, int batch,
                    int32_t* tokens_per_expert, cudaStream_t s);
  void graphs_clear() {
    for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
    graphs.clear();
    for (auto& kv : direct_graphs) cudaGraphExecDestroy(kv.second);
    direct_graphs.clear();
  }
  void moe_layer(const Layer& L, int moe_index, const bf16* next_norm, int batch,
                 int32_t* tokens_per_expert, cudaStream_t s);

 private:
  void add_slot(const std::string& name, std::vector<int64_t> shape, int dtype, size_t& cursor,
                bool pack = false);
  void plan_weights(int experts = 64);
  // Keeps this rank's experts only (expert parallelism): new arena, tensors copied.
  void repack_experts(int rank, int world);
  void plan_workspace();
  bf16* w(const std::string& name) const;
};

std::unique_ptr<Model> load_safetensors_model(const std::string& path, int device, int max_batch,
                                              int precision);

}  // namespace ce4b

struct ce4b_model {
  std::unique_ptr<ce4b::Model> impl;
};
