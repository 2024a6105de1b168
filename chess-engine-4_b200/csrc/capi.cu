// extern "C" entry points of libce4b200 (declared in include/ce4b200.h). Every entry point
// converts exceptions to a status code and records the message for ce4b_last_error().
#include <algorithm>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include <cstring>

#include "internal.h"
#include "model.h"
#include "nccl_dl.h"

namespace ce4b {

namespace {

thread_local std::string g_last_error;

// Device error word written by bounded in-kernel waits (one per device context).
__device__ int g_device_error_word;

std::mutex g_mu;
std::map<int, int*> g_error_words;
std::map<int, int> g_sm_counts;

int current_device() {
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  return dev;
}

template <class F>
int guarded(F&& f) {
  try {
    f();
    return CE4B_OK;
  } catch (const Error& e) {
    set_last_error(e.what());
    return e.status;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return CE4B_ERR_INVALID_ARGUMENT;
  } catch (...) {
    set_last_error("unknown error");
    return CE4B_ERR_INVALID_ARGUMENT;
  }
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

}  // namespace

void set_last_error(const std::string& msg) { g_last_error = msg; }

int* device_error_word() {
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_error_words.find(dev);
  if (it != g_error_words.end()) return it->second;
  void* p = nullptr;
  check_cuda(cudaGetSymbolAddress(&p, g_device_error_word), "cudaGetSymbolAddress(error word)");
  g_error_words[dev] = static_cast<int*>(p);
  return static_cast<int*>(p);
}

int sm_count() {
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_sm_counts.find(dev);
  if (it != g_sm_counts.end()) return it->second;
  int n = 0;
  check_cuda(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev), "SM count");
  g_sm_counts[dev] = n;
  return n;
}

}  // namespace ce4b

using namespace ce4b;

extern "C" {

const char* ce4b_last_error(void) { return g_last_error.c_str(); }

const char* ce4b_version(void) { return "ce4b200 0.1.0 (sm_100a)"; }

int ce4b_check_device_error(int device, int* code_out) {
  return guarded([&] {
    require(code_out != nullptr, "code_out is null");
    check_cuda(cudaSetDevice(device), "cudaSetDevice");
    int* word = device_error_word();
    check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    int code = 0;
    check_cuda(cudaMemcpy(&code, word, sizeof(int), cudaMemcpyDeviceToHost), "read error word");
    const int zero = 0;
    check_cuda(cudaMemcpy(word, &zero, sizeof(int), cudaMemcpyHostToDevice), "clear error word");
    *code_out = code;
  });
}

// ------------------------------------------------------------------ model handle
int ce4b_model_create(const ce4b_model_config* config, int device, int max_batch,
                      ce4b_model** out) {
  return guarded([&] {
    require(config != nullptr && out != nullptr, "null argument");
    *out = nullptr;
    auto h = new ce4b_model;
    try {
      h->impl = std::make_unique<Model>();
      h->impl->create(*config, device, max_batch);
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

int ce4b_model_set_tensor(ce4b_model* model, const char* name, const void* data, int dtype,
                          int ndim, const int64_t* shape, int src_is_device) {
  return guarded([&] {
    require(model != nullptr && model->impl && name != nullptr, "null argument");
    require(ndim >= 1 && ndim <= 4 && shape != nullptr, "bad tensor rank");
    std::vector<int64_t> s(shape, shape + ndim);
    model->impl->set_tensor(name, data, dtype, s, src_is_device != 0);
  });
}

int ce4b_model_finalize(ce4b_model* model) {
  return guarded([&] {
    require(model != nullptr && model->impl, "null model");
    model->impl->finalize();
  });
}

int ce4b_model_load_safetensors(const char* path, int device, int max_batch, int precision,
                                ce4b_model** out) {
  return guarded([&] {
    require(path != nullptr && out != nullptr, "null argument");
    *out = nullptr;
    auto h = new ce4b_model;
    try {
      h->impl = load_safetensors_model(path, device, max_batch, precision);
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

int ce4b_model_info_get(const ce4b_model* model, ce4b_model_info* info) {
  return guarded([&] {
    require(model != nullptr && model->impl && info != nullptr, "null argument");
    const Model& m = *model->impl;
    info->d_model = m.cfg.d_model;
    info->depth = m.cfg.depth;
    info->history_length = m.cfg.history_length;
    info->policy_size = m.policy_size;
    info->maximum_batch_size = m.max_batch;
    info->hidden_dim = m.dense_hidden;
    info->expert_hidden_dim = m.expert_hidden;
    info->arch = m.cfg.arch;
    info->weight_bytes = static_cast<int64_t>(m.arena_bytes);
    info->workspace_bytes = static_cast<int64_t>(m.workspace_bytes);
  });
}

int ce4b_model_forward(ce4b_model* model, int input_layout, void* input_dev,
                       const void* scalars_dev, int batch, float* policy_dev, float* wdl_dev,
                       float* moves_left_dev, int wdl_probs, int normalize_in_place,
                       int32_t* tokens_per_expert_dev, void* stream) {
  return guarded([&] {
    require(model != nullptr && model->impl, "null model");
    check_cuda(cudaSetDevice(model->impl->device), "cudaSetDevice");
    model->impl->forward_ordered(input_layout, input_dev, scalars_dev, batch, policy_dev,
                                 wdl_dev, moves_left_dev, wdl_probs, normalize_in_place,
                                 tokens_per_expert_dev, as_stream(stream));
  });
}

int ce4b_model_evaluate(ce4b_model* model, const ce4b_input_plane* host_planes, int batch,
                        float* host_policy, float* host_wdl, float* host_moves_left) {
  return guarded([&] {
    require(model != nullptr && model->impl, "null model");
    model->impl->evaluate(host_planes, batch, host_policy, host_wdl, host_moves_left);
  });
}

int ce4b_model_evaluate_async(ce4b_model* model, const ce4b_input_plane* host_planes, int batch,
                              float* host_policy, float* host_wdl, float* host_moves_left,
                              void* stream) {
  return guarded([&] {
    require(model != nullptr && model->impl, "null model");
    model->impl->enqueue_evaluate(host_planes, batch, host_policy, host_wdl, host_moves_left,
                                  as_stream(stream));
  });
}

int ce4b_model_set_trace(ce4b_model* model, void* const* events, int count) {
  return guarded([&] {
    require(model != nullptr && model->impl, "null model");
    require(count >= 0 && (count == 0 || events != nullptr), "bad trace event array");
    model->impl->trace_events.assign(reinterpret_cast<const cudaEvent_t*>(events),
                                     reinterpret_cast<const cudaEvent_t*>(events) + count);
  });
}

int ce4b_policy_softmax(const float* policy_dev, int batch, int policy_size,
                        const int32_t* move_offsets_dev, const int32_t* move_indices_dev,
                        float temperature, float* probs_dev, void* stream) {
  return guarded([&] {
    require(batch >= 0 && policy_size >= 1, "bad policy shape");
    ce4b::policy_softmax(policy_dev, batch, policy_size, move_offsets_dev, move_indices_dev,
                         temperature, probs_dev, as_stream(stream));
  });
}

int ce4b_model_evaluate_legal(ce4b_model* model, const ce4b_input_plane* host_planes, int batch,
                              const int32_t* host_move_offsets, const int32_t* host_move_indices,
                              float temperature, float* host_move_probs, float* host_wdl,
                              float* host_moves_left) {
  return guarded([&] {
    require(model != nullptr && model->impl, "null model");
    ce4b::Model& m = *model->impl;
    m.enqueue_evaluate_legal(host_planes, batch, host_move_offsets, host_move_indices, temperature,
                             host_move_probs, host_wdl, host_moves_left, m.stream);
    ce4b::check_cuda(cudaStreamSynchronize(m.stream), "synchronize evaluation");
  });
}

int ce4b_nccl_unique_id(void* out, int out_len) {
  return guarded([&] {
    require(out != nullptr && out_len >= static_cast<int>(sizeof(ncclUniqueId)),
            "unique id buffer must hold 128 bytes");
    ncclUniqueId id;
    ce4b::check_nccl(ce4b::nccl().GetUniqueId(&id), "ncclGetUniqueId");
    std::memcpy(out, &id, sizeof(id));
  });
}

int ce4b_model_enable_expert_parallel(ce4b_model* model, int rank, int world, const void* unique_id) {
  return guarded([&] {
    require(model != nullptr && model->impl, "null model");
    model->impl->enable_expert_parallel(rank, world, unique_id);
  });
}

int ce4b_expert_parallel_plan(int world, int rank, const int32_t* meta_send, const int32_t* meta_recv,
                              int32_t* send_rows, int32_t* recv_rows, int32_t* tiles, int tiles_cap,
                              int* num_tiles) {
  return guarded([&] {
    require(meta_send && meta_recv && send_rows && recv_rows && num_tiles, "null argument");
    const ce4b::EpPlan p = ce4b::ep_plan(world, rank, reinterpret_cast<const int2*>(meta_send),
                                         reinterpret_cast<const int2*>(meta_recv));
    for (int r = 0; r < world; ++r) {
      send_rows[r] = p.send_rows[r];
      recv_rows[r] = p.recv_rows[r];
    }
    *num_tiles = static_cast<int>(p.tiles.size());
    require(tiles == nullptr || tiles_cap >= *num_tiles, "tile buffer too small");
    if (tiles != nullptr) std::memcpy(tiles, p.tiles.data(), p.tiles.size() * sizeof(int4));
  });
}

int ce4b_model_set_task_trace(ce4b_model* model, void* device_buffer, int capacity_tasks) {
  return guarded([&] {
    require(model != nullptr && model->impl, "null model");
    require(capacity_tasks >= 0 && (capacity_tasks == 0 || device_buffer != nullptr),
            "bad task trace buffer");
    require((reinterpret_cast<uintptr_t>(device_buffer) & 7u) == 0, "task trace buffer not 8-byte aligned");
    model->impl->fwd_trace = capacity_tasks > 0 ? static_cast<unsigned long long*>(device_buffer) : nullptr;
    model->impl->fwd_trace_cap = capacity_tasks;
  });
}

int ce4b_model_set_routing_tap(ce4b_model* model, int32_t* experts_dev, int capacity_tokens) {
  return guarded([&] {
    require(model != nullptr && model->impl, "null model");
    ce4b::Model& m = *model->impl;
    if (experts_dev == nullptr || capacity_tokens <= 0) {
      m.moe_tap = nullptr;
      m.moe_tap_tokens = 0;
      return;
    }
    if (m.cfg.arch != CE4B_ARCH_MOE64A2) fail(CE4B_ERR_UNSUPPORTED, "the routing tap needs a moe64a2 model");
    m.moe_tap = experts_dev;
    m.moe_tap_tokens = capacity_tokens;
  });
}

int ce4b_model_set_mxfp8_tap(ce4b_model* model, const ce4b_mxfp8_tap* tap) {
  return guarded([&] {
    require(model != nullptr && model->impl, "null model");
    ce4b::Model& m = *model->impl;
    if (tap == nullptr || tap->layer < 0) {
      m.mx_tap = ce4b_mxfp8_tap{-1, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
      return;
    }
    if (!m.mx) fail(CE4B_ERR_UNSUPPORTED, "the MXFP8 tap needs an MXFP8 model");
    require(tap->layer <= m.cfg.depth, "tap layer must be in [0, depth]");
    m.mx_tap = *tap;
  });
}

int ce4b_model_task_count(const ce4b_model* model, int batch, int* tasks) {
  return guarded([&] {
    require(model != nullptr && model->impl && tasks != nullptr, "null argument");
    const ce4b::Model& m = *model->impl;
    require(batch >= 1 && batch <= m.max_batch, "batch size exceeds model capacity");
    if (m.fused && m.latency_path(batch)) {
      *tasks = m.lat_grid * m.lat_max_tasks;
    } else {
      *tasks = m.fused ? m.fused_task_count(batch) : 0;
    }
  });
}

int ce4b_model_set_latency_path(ce4b_model* model, int enable) {
  return guarded([&] {
    require(model != nullptr && model->impl, "null model");
    ce4b::Model& m = *model->impl;
    if (m.lat_enabled != (enable != 0)) {
      m.lat_enabled = enable != 0;
      m.graphs_clear();  // captured forwards of small batches used the other path
    }
  });
}

int ce4b_model_set_direct_io(ce4b_model* model, int enable) {
  return guarded([&] {
    require(model != nullptr && model->impl, "null model");
    model->impl->direct_io = enable != 0;
  });
}

int ce4b_model_uses_latency_path(const ce4b_model* model, int batch, int* uses) {
  return guarded([&] {
    require(model != nullptr && model->impl && uses != nullptr, "null argument");
    const ce4b::Model& m = *model->impl;
    require(batch >= 1 && batch <= m.max_batch, "batch size exceeds model capacity");
    *uses = m.fused && m.latency_path(batch) ? 1 : 0;
  });
}

int ce4b_model_trace_label(const ce4b_model* model, int index, char* buffer, int buffer_len) {
  return guarded([&] {
    require(model != nullptr && model->impl && buffer != nullptr && buffer_len > 0,
            "null argument");
    const auto& labels = model->impl->trace_labels;
    require(index >= 0 && static_cast<size_t>(index) < labels.size(), "trace index out of range");
    const std::string& l = labels[static_cast<size_t>(index)];
    const size_t n = std::min(l.size(), static_cast<size_t>(buffer_len - 1));
    l.copy(buffer, n);
    buffer[n] = '\0';
  });
}

void ce4b_model_destroy(ce4b_model* model) { delete model; }

// ------------------------------------------------------------------ kernel-op API
int ce4b_bf16_gemm(const void* a_dev, const void* b_dev, void* c_dev, int m, int n, int k,
                   void* stream) {
  return guarded([&] {
    require(m >= 1 && n >= 1 && k >= 1, "GEMM extents must be positive");
    require(n % 16 == 0, "GEMM N must be a multiple of 16");
    require(k % 8 == 0, "GEMM K must be a multiple of 8");
    require(c_dev != nullptr, "null output");
    const CUtensorMap ta = make_tmap_bf16(a_dev, m, k, k, 128);
    const CUtensorMap tb = make_tmap_bf16(b_dev, n, k, k, 128);
    const CUtensorMap tc = make_tmap_bf16(c_dev, m, n, n, 128);
    gemm_store_bf16(ta, tb, tc, m, n, k, as_stream(stream));
  });
}

int ce4b_rmsnorm_forward(const void* x_dev, const void* weight_dev, void* out_dev, int rows,
                         int width, float eps, void* stream) {
  return guarded([&] {
    require(x_dev && weight_dev && out_dev, "null pointer");
    require(rows >= 1 && width >= 1, "extents must be positive");
    rmsnorm_rows(static_cast<const bf16*>(x_dev), static_cast<const bf16*>(weight_dev),
                 static_cast<bf16*>(out_dev), rows, width, eps, as_stream(stream));
  });
}

int ce4b_swiglu_forward(const void* gate_up_dev, void* hidden_dev, int rows, int hidden_dim,
                        void* stream) {
  return guarded([&] {
    require(gate_up_dev && hidden_dev, "null pointer");
    require(rows >= 1 && hidden_dim >= 1, "extents must be positive");
    swiglu_rows(static_cast<const bf16*>(gate_up_dev), static_cast<bf16*>(hidden_dev), rows,
                hidden_dim, as_stream(stream));
  });
}

int ce4b_residual_add(void* out_dev, const void* residual_dev, int64_t elements, void* stream) {
  return guarded([&] {
    require(out_dev && residual_dev, "null pointer");
    require(elements >= 0, "negative element count");
    if (elements == 0) return;
    residual_add(static_cast<bf16*>(out_dev), static_cast<const bf16*>(residual_dev), elements,
                 as_stream(stream));
  });
}

int64_t ce4b_dense_block_workspace_size(int rows, int d_model, int hidden_dim) {
  if (rows < 1 || d_model < 1 || hidden_dim < 1) return -1;
  const int64_t r = (static_cast<int64_t>(rows) + 127) / 128 * 128;
  const int64_t a = (r * d_model * 2 + 255) / 256 * 256;
  const int64_t b = (r * hidden_dim * 2 + 255) / 256 * 256;
  return a + b;
}

int ce4b_dense_block_forward(const void* x_dev, const void* norm_weight_dev,
                             const void* gate_up_weight_dev, const void* down_weight_dev,
                             void* out_dev, void* workspace_dev, int rows, int d_model,
                             int hidden_dim, float eps, int precision, void* stream) {
  return guarded([&] {
    require(x_dev && norm_weight_dev && gate_up_weight_dev && down_weight_dev && out_dev &&
                workspace_dev,
            "null pointer");
    require(rows >= 1, "rows must be positive");
    require(d_model >= 64 && d_model % 64 == 0, "d_model must be a multiple of 64");
    require(hidden_dim >= 64 && hidden_dim % 64 == 0, "hidden_dim must be a multiple of 64");
    if (precision != CE4B_PRECISION_BF16) {
      fail(CE4B_ERR_UNSUPPORTED, "dense block: only BF16 precision is available");
    }
    require((reinterpret_cast<uintptr_t>(workspace_dev) & 255u) == 0,
            "workspace must be 256-byte aligned");
    cudaStream_t s = as_stream(stream);
    const int64_t r = (static_cast<int64_t>(rows) + 127) / 128 * 128;
    auto* normalized = static_cast<bf16*>(workspace_dev);
    auto* hidden = reinterpret_cast<bf16*>(static_cast<uint8_t*>(workspace_dev) +
                                           (r * d_model * 2 + 255) / 256 * 256);
    rmsnorm_rows(static_cast<const bf16*>(x_dev), static_cast<const bf16*>(norm_weight_dev),
                 normalized, rows, d_model, eps, s);
    const CUtensorMap t_norm = make_tmap_bf16(normalized, rows, d_model, d_model, 128);
    const CUtensorMap t_gu = make_tmap_bf16(gate_up_weight_dev, 2 * hidden_dim, d_model, d_model,
                                            static_cast<uint32_t>(swiglu_chunk(hidden_dim)));
    const CUtensorMap t_hidden = make_tmap_bf16(hidden, rows, hidden_dim, hidden_dim, 128);
    gemm_swiglu(t_norm, t_gu, t_hidden, rows, hidden_dim, d_model, s);
    check_cuda(cudaMemcpyAsync(out_dev, x_dev, static_cast<size_t>(rows) * d_model * 2,
                               cudaMemcpyDeviceToDevice, s),
               "copy residual");
    const CUtensorMap t_down = make_tmap_bf16(down_weight_dev, d_model, hidden_dim, hidden_dim,
                                              static_cast<uint32_t>(resnorm_b_box(d_model)));
    const CUtensorMap t_out = make_tmap_bf16(out_dev, rows, d_model, d_model, 128);
    gemm_resnorm(t_hidden, t_down, t_out, t_out, nullptr, nullptr, rows, d_model, hidden_dim, eps, s);
  });
}

// ------------------------------------------------------------------ MoE kernel ops
int ce4b_moe_route(const void* logits_dev, const float* beta_dev, int32_t* experts_dev,
                   float* probs_dev, int32_t* counts_dev, int tokens, void* stream) {
  return guarded([&] {
    require(logits_dev && beta_dev && experts_dev && probs_dev, "null pointer");
    require(tokens >= 1, "tokens must be positive");
    moe_route_logits(static_cast<const bf16*>(logits_dev), beta_dev,
                     reinterpret_cast<int2*>(experts_dev), reinterpret_cast<float2*>(probs_dev),
                     counts_dev, tokens, as_stream(stream));
  });
}

int ce4b_moe_dispatch_capacity(int tokens) {
  if (tokens < 1) return -1;
  // Two routes per token; every expert segment padded to a multiple of 128 rows.
  return (2 * ((tokens + 127) / 128 * 128) + 64 * 127 + 127) / 128 * 128;
}

int64_t ce4b_moe_route_dispatch_workspace_size(int tokens) {
  if (tokens < 1) return -1;
  const int64_t tiles = (static_cast<int64_t>(tokens) + 127) / 128;
  const int64_t cap_tiles = ce4b_moe_dispatch_capacity(tokens) / 128;
  auto a = [](int64_t v) { return (v + 255) / 256 * 256; };
  return 2 * a(tiles * 64 * 4) + a(cap_tiles * 16) + a(4);
}

int ce4b_moe_route_dispatch(const void* n_dev, const void* router_weight_dev, const float* beta_dev,
                            void* logits_dev, int32_t* experts_dev, float* probs_dev,
                            int32_t* positions_dev, int32_t* expert_offsets_dev,
                            int32_t* counts_dev, void* xperm_dev, float* pprob_dev,
                            void* workspace_dev, int tokens, int d_model, void* stream) {
  return guarded([&] {
    require(n_dev && router_weight_dev && beta_dev && experts_dev && probs_dev && positions_dev &&
                expert_offsets_dev && xperm_dev && pprob_dev && workspace_dev,
            "null pointer");
    require(tokens >= 1, "tokens must be positive");
    require(d_model >= 64 && d_model % 64 == 0, "d_model must be a multiple of 64");
    require((reinterpret_cast<uintptr_t>(workspace_dev) & 255u) == 0,
            "workspace must be 256-byte aligned");
    cudaStream_t s = as_stream(stream);
    auto a = [](int64_t v) { return (v + 255) / 256 * 256; };
    const int tiles = (tokens + 127) / 128;
    auto* base = static_cast<uint8_t*>(workspace_dev);
    auto* block_hist = reinterpret_cast<int*>(base);
    auto* block_off = reinterpret_cast<int*>(base + a(tiles * 64 * 4));
    auto* m_tiles = reinterpret_cast<int4*>(base + 2 * a(tiles * 64 * 4));
    const int64_t cap_tiles = ce4b_moe_dispatch_capacity(tokens) / 128;
    auto* num_m_tiles = reinterpret_cast<int*>(base + 2 * a(tiles * 64 * 4) + a(cap_tiles * 16));
    const CUtensorMap t_n = make_tmap_bf16(n_dev, tokens, d_model, d_model, 128);
    const CUtensorMap t_r = make_tmap_bf16(router_weight_dev, 64, d_model, d_model, 64);
    auto* route_expert = reinterpret_cast<int2*>(experts_dev);
    auto* route_prob = reinterpret_cast<float2*>(probs_dev);
    moe_router_gemm(t_n, t_r, beta_dev, route_expert, route_prob, block_hist, tokens, d_model, s,
                    static_cast<bf16*>(logits_dev));
    moe_scan(block_hist, tiles, expert_offsets_dev, block_off, m_tiles, num_m_tiles, counts_dev, s);
    moe_dispatch(static_cast<const bf16*>(n_dev), route_expert, route_prob, expert_offsets_dev,
                 block_off, static_cast<bf16*>(xperm_dev), pprob_dev, positions_dev, tokens,
                 d_model, s);
  });
}

int64_t ce4b_moe_workspace_size(int rows, int d_model, int hidden_dim) {
  if (rows < 1 || d_model < 1 || hidden_dim < 1) return -1;
  const int64_t tiles = (static_cast<int64_t>(rows) + 127) / 128 + 64;
  const int64_t r = (static_cast<int64_t>(rows) + 127) / 128 * 128;
  auto a = [](int64_t v) { return (v + 255) / 256 * 256; };
  return a(tiles * 16) + a(4) + a(r * 4) + a(r * hidden_dim * 2);
}

int ce4b_moe_forward(const void* x_dev, const void* gate_up_weight_dev,
                     const void* down_weight_dev, const void* route_probs_dev,
                     const int32_t* expert_offsets_dev, void* out_dev, void* workspace_dev,
                     int rows, int d_model, int hidden_dim, void* stream) {
  return guarded([&] {
    require(x_dev && gate_up_weight_dev && down_weight_dev && route_probs_dev &&
                expert_offsets_dev && out_dev && workspace_dev,
            "null pointer");
    require(rows >= 1, "rows must be positive");
    require(d_model >= 64 && d_model % 64 == 0, "d_model must be a multiple of 64");
    require(hidden_dim >= 64 && hidden_dim % 64 == 0, "hidden_dim must be a multiple of 64");
    require((reinterpret_cast<uintptr_t>(workspace_dev) & 255u) == 0,
            "workspace must be 256-byte aligned");
    cudaStream_t s = as_stream(stream);
    auto a = [](int64_t v) { return (v + 255) / 256 * 256; };
    const int64_t tiles = (static_cast<int64_t>(rows) + 127) / 128 + 64;
    const int64_t r = (static_cast<int64_t>(rows) + 127) / 128 * 128;
    auto* base = static_cast<uint8_t*>(workspace_dev);
    auto* m_tiles = reinterpret_cast<int4*>(base);
    auto* num_m_tiles = reinterpret_cast<int*>(base + a(tiles * 16));
    auto* scale = reinterpret_cast<float*>(base + a(tiles * 16) + a(4));
    auto* hidden = reinterpret_cast<bf16*>(base + a(tiles * 16) + a(4) + a(r * 4));
    moe_tiles_from_offsets(expert_offsets_dev, m_tiles, num_m_tiles, s);
    bf16_to_f32(static_cast<const bf16*>(route_probs_dev), scale, rows, s);
    const CUtensorMap t_x = make_tmap_bf16(x_dev, rows, d_model, d_model, 128);
    const CUtensorMap t_gu = make_tmap_bf16(gate_up_weight_dev, 64ull * 2 * hidden_dim, d_model,
                                            d_model, static_cast<uint32_t>(swiglu_chunk(hidden_dim)));
    const CUtensorMap t_h = make_tmap_bf16(hidden, rows, hidden_dim, hidden_dim, 128);
    gemm_grouped_swiglu(t_x, t_gu, t_h, m_tiles, num_m_tiles, hidden_dim, d_model, s);
    const CUtensorMap t_dn = make_tmap_bf16(down_weight_dev, 64ull * d_model, hidden_dim, hidden_dim,
                                            static_cast<uint32_t>(grouped_bn(d_model)));
    const CUtensorMap t_y = make_tmap_bf16(out_dev, rows, d_model, d_model, 128);
    gemm_grouped_scale(t_h, t_dn, t_y, m_tiles, num_m_tiles, scale, d_model, hidden_dim, s);
  });
}

// ------------------------------------------------------------------ MXFP8 kernel ops
int ce4b_quantize_mxfp8(const void* x_dev, void* codes_dev, void* scales_dev, int rows, int cols,
                        void* stream) {
  return guarded([&] {
    require(x_dev && codes_dev && scales_dev, "null pointer");
    require(rows >= 128 && cols >= 128, "MXFP8 tensors need at least 128 rows and columns");
    mx_quantize(static_cast<const bf16*>(x_dev), static_cast<uint8_t*>(codes_dev),
                static_cast<uint8_t*>(scales_dev), rows, cols, as_stream(stream));
  });
}

int ce4b_quantize_mxfp8_transpose(const void* x_dev, void* codes_dev, void* scales_dev, int rows,
                                  int cols, void* stream) {
  return guarded([&] {
    require(x_dev && codes_dev && scales_dev, "null pointer");
    require(rows >= 128 && cols >= 128, "MXFP8 tensors need at least 128 rows and columns");
    mx_quantize_transpose(static_cast<const bf16*>(x_dev), static_cast<uint8_t*>(codes_dev),
                          static_cast<uint8_t*>(scales_dev), rows, cols, as_stream(stream));
  });
}

int ce4b_mxfp8_gemm(const void* a_codes_dev, const void* a_scales_dev, const void* b_codes_dev,
                    const void* b_scales_dev, void* c_dev, int m, int n, int k, void* stream) {
  return guarded([&] {
    require(a_codes_dev && a_scales_dev && b_codes_dev && b_scales_dev && c_dev, "null pointer");
    require(m >= 128 && n >= 128 && k >= 128, "MXFP8 GEMM extents must be at least 128");
    require(m % 128 == 0 && n % 128 == 0 && k % 128 == 0,
            "MXFP8 GEMM extents must be multiples of 128");
    const CUtensorMap ta = make_tmap_u8(a_codes_dev, m, k, k, 128);
    const CUtensorMap tb = make_tmap_u8(b_codes_dev, n, k, k, 128);
    const CUtensorMap tc = make_tmap_bf16(c_dev, m, n, n, 128);
    gemm_mx_store_bf16(ta, tb, tc, static_cast<const uint8_t*>(a_scales_dev),
                       static_cast<const uint8_t*>(b_scales_dev), m, n, k, as_stream(stream));
  });
}

}  // extern "C"
