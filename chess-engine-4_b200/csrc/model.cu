// Model handle: weight arena in the Safetensors v1 layout, activation workspace sized for
// the maximum batch, TMA descriptors built once, and the per-layer forward schedule.
//
// Forward of a dense tower (B positions, width d, hidden h, L layers):
//   expand planes -> A_in [B, 64*sel] BF16
//   GEMM A_in . W_in^T, epilogue: x = bf16(acc + b_in), n = RMSNorm(x; block 0 weight)
//   per layer: GEMM n . W_gu^T, epilogue SwiGLU -> hidden [B, h]
//              GEMM hidden . W_d^T, epilogue: x = bf16(x + bf16(acc)), n = RMSNorm(x; next)
//   GEMM n . [W_policy; W_wdl; W_ml]^T, epilogue: bias, BF16 round, FP32 outputs, WDL softmax
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "internal.h"
#include "model.h"

#include "forward_types.h"

#include "safetensors.h"

namespace ce4b {

namespace {

size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

int64_t numel(const std::vector<int64_t>& s) {
  int64_t n = 1;
  for (auto v : s) n *= v;
  return n;
}

std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + "]";
}

}  // namespace

Model::~Model() {
  if (device >= 0) cudaSetDevice(device);
  disable_expert_parallel();
  graphs_clear();
  if (fwd_dev) cudaFree(fwd_dev);
  if (fwd_weights) cudaFree(fwd_weights);
  if (lat_dev) cudaFree(lat_dev);
  for (auto& slot : io)
    if (slot.free) cudaEventDestroy(slot.free);
  if (forward_done) cudaEventDestroy(forward_done);
  if (stream) cudaStreamDestroy(stream);
  if (arena) cudaFree(arena);
  if (mx_arena) cudaFree(mx_arena);
  if (workspace) cudaFree(workspace);
}

void Model::add_slot(const std::string& name, std::vector<int64_t> shape, int dtype,
                     size_t& cursor, bool pack) {
  if (!pack) cursor = align256(cursor);
  Slot s;
  s.offset = cursor;
  s.shape = std::move(shape);
  s.dtype = dtype;
  s.bytes = static_cast<size_t>(numel(s.shape)) * (dtype == CE4B_DTYPE_F32 ? 4 : 2);
  cursor += s.bytes;
  slots.emplace(name, s);
}

void Model::plan_weights(int experts) {
  const int d = cfg.d_model;
  size_t cur = 0;
  add_slot("input.weight", {d, in_dim}, CE4B_DTYPE_BF16, cur);
  add_slot("input.bias", {d}, CE4B_DTYPE_BF16, cur);
  add_slot("final_norm.weight", {d}, CE4B_DTYPE_BF16, cur);
  // The three head matrices (and their biases) are packed back to back so the heads run
  // as one GEMM over [policy_storage + 64, d].
  add_slot("policy.weight", {policy_storage, d}, CE4B_DTYPE_BF16, cur);
  add_slot("wdl.weight", {32, d}, CE4B_DTYPE_BF16, cur, true);
  add_slot("moves_left.weight", {32, d}, CE4B_DTYPE_BF16, cur, true);
  add_slot("policy.bias", {policy_storage}, CE4B_DTYPE_BF16, cur);
  add_slot("wdl.bias", {32}, CE4B_DTYPE_BF16, cur, true);
  add_slot("moves_left.bias", {32}, CE4B_DTYPE_BF16, cur, true);
  for (int l = 0; l < cfg.depth; ++l) {
    const std::string p = "blocks." + std::to_string(l);
    add_slot(p + ".norm.weight", {d}, CE4B_DTYPE_BF16, cur);
    if (is_moe_layer(l)) {
      add_slot(p + ".router.weight", {64, d}, CE4B_DTYPE_BF16, cur);
      add_slot(p + ".router_qb_beta", {64}, CE4B_DTYPE_F32, cur);
      add_slot(p + ".experts.gate_up.weight", {experts, 2 * expert_hidden, d}, CE4B_DTYPE_BF16, cur);
      add_slot(p + ".experts.down.weight", {experts, d, expert_hidden}, CE4B_DTYPE_BF16, cur);
    } else {
      add_slot(p + ".gate_up.weight", {2 * dense_hidden, d}, CE4B_DTYPE_BF16, cur);
      add_slot(p + ".down.weight", {d, dense_hidden}, CE4B_DTYPE_BF16, cur);
    }
  }
  arena_bytes = align256(cur);
}

void Model::plan_workspace() {
  const int d = cfg.d_model;
  size_t cur = 0;
  auto take = [&](size_t bytes) {
    const size_t off = align256(cur);
    cur = off + bytes;
    return off;
  };
  const size_t r = static_cast<size_t>(rows_cap);
  for (auto& slot : io) {
    slot.planes = take(r * kInputPlanes * sizeof(ce4b_input_plane));
    slot.policy = take(r * policy_size * 4);
    slot.wdl = take(r * 3 * 4);
    slot.moves_left = take(r * 4);
    slot.move_offsets = take((r + 1) * 4);
    slot.move_indices = take(r * kMaxMovesPerPosition * 4);
    slot.move_probs = take(r * kMaxMovesPerPosition * 4);
  }
  ws_off.a_in = take(r * in_dim * 2);
  ws_off.x = take(r * d * 2);
  ws_off.n = take(r * d * 2);
  ws_off.hidden = take(r * std::max(dense_hidden, expert_hidden) * 2);
  if (mx) {
    const size_t t = r / 128;
    ws_off.a_codes = take(r * in_dim);
    ws_off.a_scales = take(t * (in_dim / 128) * 512);
    ws_off.n_codes = take(r * d);
    ws_off.n_scales = take(t * (d / 128) * 512);
    ws_off.h_codes = take(r * dense_hidden);
    ws_off.h_scales = take(t * (dense_hidden / 128) * 512);
  }
  if (fused) {
    const size_t sj = static_cast<size_t>(d / 128);
    const size_t nb = r / 128;
    ws_off.fwd_ss = take(r * sj * kFwdG * 4);
    // K-part partial sums: 2 parts for every row block, or 8 for the small-batch schedule.
    const size_t chunk = 64 * 1024;
    ws_off.fwd_part = take(std::max(nb * sj * 2, static_cast<size_t>(fused_small_nb()) * sj * 8) * chunk);
    fwd_sync_bytes = (2 * nb + 2 * nb * sj + 1) * 4;
    ws_off.fwd_sync = take(fwd_sync_bytes);
  }
  if (lat) {
    // FP32 partial tiles [d / 128][K parts][64 positions][128] of the input and down GEMMs,
    // and the counters (x ready, hidden ready, one per 128-row block for each GEMM, CTAs
    // finished).
    const size_t mt = static_cast<size_t>(d / 128);
    ws_off.lat_part_in = take(mt * lat_kp_in * kLatMaxRows * 128 * 4);
    ws_off.lat_part_dn = take(mt * lat_kp_dn * kLatMaxRows * 128 * 4);
    lat_sync_bytes = (3 + 2 * mt) * 4;  // + the exit counter (the last CTA out zeroes all)
    ws_off.lat_sync = take(lat_sync_bytes);
  }
  if (cfg.arch == CE4B_ARCH_MOE64A2) {
    // Expert rows: 2 routes per token, each expert segment padded to 128 rows.
    perm_rows = static_cast<int>((2 * r + 64 * 127 + 127) / 128 * 128);
    const size_t p = static_cast<size_t>(perm_rows);
    const size_t tiles = r / 128;
    ws_off.route_expert = take(r * 8);
    ws_off.route_prob = take(r * 8);
    ws_off.route_pos = take(r * 8);
    ws_off.block_hist = take(tiles * 64 * 4);
    ws_off.block_off = take(tiles * 64 * 4);
    ws_off.expert_start = take(65 * 4);
    ws_off.m_tiles = take((p / 128) * 16);
    ws_off.num_m_tiles = take(4);
    ws_off.xperm = take(p * d * 2);
    ws_off.pprob = take(p * 4);
    ws_off.hperm = take(p * expert_hidden * 2);
    ws_off.yperm = take(p * d * 2);
  }
  workspace_bytes = align256(cur);
}

bf16* Model::w(const std::string& name) const {
  auto it = slots.find(name);
  if (it == slots.end()) fail(CE4B_ERR_INVALID_ARGUMENT, "unknown tensor " + name);
  return reinterpret_cast<bf16*>(arena + it->second.offset);
}

void Model::create(const ce4b_model_config& c, int dev, int maxb) {
  cfg = c;
  device = dev;
  require(c.arch == CE4B_ARCH_DENSE || c.arch == CE4B_ARCH_MOE64A2, "unknown architecture");
  require(c.d_model >= 64 && c.d_model % 64 == 0 && c.d_model <= 2048,
          "d_model must be a multiple of 64 in [64, 2048]");
  require(c.depth >= 1, "depth must be positive");
  require(c.history_length >= 1 && c.history_length <= 8, "history_length must be in [1, 8]");
  require(c.expansion_ratio > 0.0f, "expansion_ratio must be positive");
  require(c.policy_size >= 1 && c.policy_storage_size >= c.policy_size,
          "policy storage must hold the policy output");
  require(c.policy_storage_size % 32 == 0, "policy storage size must be a multiple of 32");
  require(maxb >= 1 && maxb <= (1 << 20), "max_batch must be in [1, 2^20]");
  require(c.precision == CE4B_PRECISION_BF16 || c.precision == CE4B_PRECISION_MXFP8,
          "unknown precision");
  mx = c.precision == CE4B_PRECISION_MXFP8;
  if (c.arch == CE4B_ARCH_MOE64A2) {
    require(c.depth % 2 == 0, "moe64a2 depth must be a positive even number");
    if (mx) fail(CE4B_ERR_UNSUPPORTED, "moe64a2 runs in BF16 (the reference's MoE kernels are BF16)");
  }
  const int hid = static_cast<int>(static_cast<double>(c.d_model) * c.expansion_ratio);
  dense_hidden = c.arch == CE4B_ARCH_DENSE ? hid : 4 * c.d_model;
  expert_hidden = c.arch == CE4B_ARCH_MOE64A2 ? hid : 0;
  require(dense_hidden % 64 == 0, "dense hidden dimension must be a multiple of 64");
  require(expert_hidden % 64 == 0, "expert hidden dimension must be a multiple of 64");
  sel = selected_planes(c.history_length);
  in_dim = sel * 64;
  if (mx) {
    require(c.d_model % 128 == 0 && (c.d_model <= 1024 || (c.d_model % 256 == 0 && c.d_model <= 2048)),
            "MXFP8 needs d_model a multiple of 128 up to 1024, or of 256 up to 2048");
    require(dense_hidden % 128 == 0, "MXFP8 needs a hidden width that is a multiple of 128");
    require(in_dim % 128 == 0, "MXFP8 needs an even history_length (input width multiple of 128)");
  }
  policy_size = c.policy_size;
  policy_storage = c.policy_storage_size;
  max_batch = maxb;
  rows_cap = (maxb + 127) / 128 * 128;
  fused = c.arch == CE4B_ARCH_DENSE && !mx && c.d_model % 128 == 0 &&
          c.d_model / 128 <= kFwdMaxSlices && dense_hidden % 128 == 0 && c.depth <= kFwdMaxDepth;
  (void)resnorm_bn(c.d_model);  // validates width against the cluster limit

  check_cuda(cudaSetDevice(device), "cudaSetDevice");
  plan_latency();
  plan_weights();
  plan_workspace();
  check_cuda(cudaMalloc(&arena, arena_bytes), "cudaMalloc weights");
  check_cuda(cudaMemset(arena, 0, arena_bytes), "cudaMemset weights");
  check_cuda(cudaMalloc(&workspace, workspace_bytes), "cudaMalloc workspace");
  check_cuda(cudaMemset(workspace, 0, workspace_bytes), "cudaMemset workspace");
  check_cuda(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "create stream");
  check_cuda(cudaEventCreateWithFlags(&forward_done, cudaEventDisableTiming), "create event");
  for (auto& slot : io)
    check_cuda(cudaEventCreateWithFlags(&slot.free, cudaEventDisableTiming), "create event");
}

void Model::set_tensor(const std::string& name, const void* data, int dtype,
                       const std::vector<int64_t>& shape, bool src_device) {
  auto it = slots.find(name);
  if (it == slots.end()) fail(CE4B_ERR_INVALID_ARGUMENT, "model has no tensor named " + name);
  Slot& s = it->second;
  if (shape != s.shape) {
    fail(CE4B_ERR_INVALID_ARGUMENT,
         "tensor " + name + " has shape " + shape_str(shape) + ", expected " + shape_str(s.shape));
  }
  if (dtype != s.dtype) fail(CE4B_ERR_INVALID_ARGUMENT, "tensor " + name + " has the wrong dtype");
  if (experts_held != 64) {
    fail(CE4B_ERR_UNSUPPORTED, "an expert-parallel model holds only its own experts; its weights are fixed");
  }
  require(data != nullptr, "tensor data is null");
  check_cuda(cudaSetDevice(device), "cudaSetDevice");
  check_cuda(cudaMemcpy(arena + s.offset, data, s.bytes,
                        src_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice),
             "copy tensor");
  s.set = true;
}

void Model::finalize() {
  for (const auto& kv : slots) {
    if (!kv.second.set) fail(CE4B_ERR_NOT_READY, "model is missing tensor " + kv.first);
  }
  check_cuda(cudaSetDevice(device), "cudaSetDevice");
  const int d = cfg.d_model;
  bf16* ws_a_in = reinterpret_cast<bf16*>(workspace + ws_off.a_in);
  bf16* ws_n = reinterpret_cast<bf16*>(workspace + ws_off.n);
  bf16* ws_hidden = reinterpret_cast<bf16*>(workspace + ws_off.hidden);
  tm_a_in = make_tmap_bf16(ws_a_in, rows_cap, in_dim, in_dim, 128);
  tm_n = make_tmap_bf16(ws_n, rows_cap, d, d, 128);
  tm_x = make_tmap_bf16(workspace + ws_off.x, rows_cap, d, d, 128);
  tm_hidden = make_tmap_bf16(ws_hidden, rows_cap, dense_hidden, dense_hidden, 128);
  const uint32_t bn = static_cast<uint32_t>(resnorm_b_box(d));
  tm_w_in = make_tmap_bf16(w("input.weight"), d, in_dim, in_dim, bn);
  tm_heads = make_tmap_bf16(w("policy.weight"), policy_storage + 64, d, d, 256);
  layers.clear();
  for (int l = 0; l < cfg.depth; ++l) {
    const std::string p = "blocks." + std::to_string(l);
    Layer L;
    L.moe = is_moe_layer(l);
    L.norm = w(p + ".norm.weight");
    if (!L.moe) {
      const uint32_t hc = static_cast<uint32_t>(swiglu_chunk(dense_hidden));
      L.tm_gate_up = make_tmap_bf16(w(p + ".gate_up.weight"), 2 * dense_hidden, d, d, hc);
      L.tm_down = make_tmap_bf16(w(p + ".down.weight"), d, dense_hidden, dense_hidden, bn);
    } else {
      const int he = expert_hidden;
      L.tm_router = make_tmap_bf16(w(p + ".router.weight"), 64, d, d, 64);
      L.beta = reinterpret_cast<const float*>(w(p + ".router_qb_beta"));
      const uint64_t held = static_cast<uint64_t>(experts_held);
      L.tm_gate_up = make_tmap_bf16(w(p + ".experts.gate_up.weight"), held * 2 * he, d, d,
                                    static_cast<uint32_t>(swiglu_chunk(he)));
      L.tm_down = make_tmap_bf16(w(p + ".experts.down.weight"), held * d, he, he,
                                 static_cast<uint32_t>(grouped_bn(d)));
    }
    layers.push_back(L);
  }
  if (cfg.arch == CE4B_ARCH_MOE64A2) {
    tm_xperm = make_tmap_bf16(workspace + ws_off.xperm, perm_rows, d, d, 128);
    tm_hperm = make_tmap_bf16(workspace + ws_off.hperm, perm_rows, expert_hidden, expert_hidden, 128);
    tm_yperm = make_tmap_bf16(workspace + ws_off.yperm, perm_rows, d, d, 128);
  }
  if (fused) {
    // Norm-folded weights: gate_up of layer l times blocks.l.norm.weight, heads times
    // final_norm.weight (column scaling, one BF16 rounding each).
    const size_t gu_elems = static_cast<size_t>(2) * dense_hidden * d;
    const size_t heads_rows = static_cast<size_t>(policy_storage) + 64;
    if (fwd_weights == nullptr) {
      check_cuda(cudaMalloc(&fwd_weights, (cfg.depth * gu_elems + heads_rows * d) * sizeof(bf16)),
                 "cudaMalloc folded weights");
    }
    FwdMaps maps{};
    maps.a_in = make_tmap_bf16(ws_a_in, rows_cap, in_dim, in_dim, 128);
    maps.x = make_tmap_bf16(workspace + ws_off.x, rows_cap, d, d, 128);
    maps.hidden = make_tmap_bf16(ws_hidden, rows_cap, dense_hidden, dense_hidden, 128);
    maps.hidden32 = make_tmap_bf16_sw64(ws_hidden, rows_cap, dense_hidden, dense_hidden, 128);
    maps.w_in = make_tmap_bf16(w("input.weight"), d, in_dim, in_dim, 128);
    for (int l = 0; l < cfg.depth; ++l) {
      const std::string p = "blocks." + std::to_string(l);
      bf16* gu = fwd_weights + l * gu_elems;
      fold_columns(w(p + ".gate_up.weight"), w(p + ".norm.weight"), gu, 2 * dense_hidden, d, stream);
      maps.gate_up[l] = make_tmap_bf16(gu, 2 * dense_hidden, d, d, 128);
      maps.down[l] = make_tmap_bf16(w(p + ".down.weight"), d, dense_hidden, dense_hidden, 128);
      maps.down32[l] = make_tmap_bf16_sw64(w(p + ".down.weight"), d, dense_hidden, dense_hidden, 128);
    }
    bf16* heads = fwd_weights + cfg.depth * gu_elems;
    fold_columns(w("policy.weight"), w("final_norm.weight"), heads, static_cast<int64_t>(heads_rows), d,
                 stream);
    maps.heads = make_tmap_bf16(heads, heads_rows, d, d, 128);
    check_cuda(cudaStreamSynchronize(stream), "fold norm weights");
    if (fwd_dev == nullptr) {
      check_cuda(cudaMalloc(&fwd_dev, sizeof(FwdMaps)), "cudaMalloc forward tensor maps");
    }
    check_cuda(cudaMemcpy(fwd_dev, &maps, sizeof(FwdMaps), cudaMemcpyHostToDevice),
               "copy forward tensor maps");
  }
  if (lat) build_latency();
  if (mx) quantize_weights();
  graphs_clear();
  finalized = true;
}

// MXFP8 weights: every linear's BF16 weight is quantised once (the reference re-quantises
// its weights on every call, src/chess_engine_4/kernels/dense.py:395-406; the codes are
// the same). The head matrix [policy_storage + 64, d] is padded with zero rows to a
// multiple of 128.
void Model::quantize_weights() {
  const int d = cfg.d_model;
  const int h = dense_hidden;
  heads_rows_mx = (policy_storage + 64 + 127) / 128 * 128;
  auto mx_size = [](size_t rows, size_t cols) {
    return align256(rows * cols) + align256((rows / 128) * (cols / 128) * 512);
  };
  size_t total = mx_size(d, in_dim) + mx_size(heads_rows_mx, d);
  for (int l = 0; l < cfg.depth; ++l) total += mx_size(2 * h, d) + mx_size(d, h);
  if (mx_arena == nullptr) {
    mx_arena_bytes = total;
    check_cuda(cudaMalloc(&mx_arena, mx_arena_bytes), "cudaMalloc MXFP8 weights");
  }
  bf16* padded = nullptr;
  check_cuda(cudaMalloc(&padded, static_cast<size_t>(heads_rows_mx) * d * 2), "cudaMalloc heads");
  size_t cur = 0;
  auto quant = [&](const bf16* src, int rows, int cols, const uint8_t** scales_out) {
    uint8_t* codes = mx_arena + cur;
    cur += align256(static_cast<size_t>(rows) * cols);
    uint8_t* scales = mx_arena + cur;
    cur += align256(static_cast<size_t>(rows / 128) * (cols / 128) * 512);
    mx_quantize(src, codes, scales, rows, cols, stream);
    *scales_out = scales;
    return codes;
  };
  const uint8_t* w_in_codes = quant(w("input.weight"), d, in_dim, &w_in_scales);
  tm_w_in = make_tmap_u8(w_in_codes, d, in_dim, in_dim, 128);
  check_cuda(cudaMemsetAsync(padded, 0, static_cast<size_t>(heads_rows_mx) * d * 2, stream), "zero");
  check_cuda(cudaMemcpyAsync(padded, w("policy.weight"),
                             static_cast<size_t>(policy_storage + 64) * d * 2,
                             cudaMemcpyDeviceToDevice, stream),
             "copy heads");
  const uint8_t* heads_codes = quant(padded, heads_rows_mx, d, &heads_scales);
  tm_heads = make_tmap_u8(heads_codes, heads_rows_mx, d, d, 256);
  for (int l = 0; l < cfg.depth; ++l) {
    const std::string p = "blocks." + std::to_string(l);
    Layer& L = layers[l];
    const uint8_t* gu = quant(w(p + ".gate_up.weight"), 2 * h, d, &L.gu_scales);
    const uint8_t* dn = quant(w(p + ".down.weight"), d, h, &L.down_scales);
    L.tm_gate_up = make_tmap_u8(gu, 2 * h, d, d, 128);
    L.tm_down = make_tmap_u8(dn, d, h, h, 128);
  }
  check_cuda(cudaStreamSynchronize(stream), "quantise weights");
  cudaFree(padded);
  tm_a_u8 = make_tmap_u8(workspace + ws_off.a_codes, rows_cap, in_dim, in_dim, 128);
  tm_n_u8 = make_tmap_u8(workspace + ws_off.n_codes, rows_cap, d, d, 128);
  tm_h_u8 = make_tmap_u8(workspace + ws_off.h_codes, rows_cap, h, h, 128);
}

// MXFP8 forward: the same schedule as the BF16 one on block-scaled GEMMs; each producing
// epilogue quantises its output (n, hidden) for the next GEMM, x stays BF16.
void Model::forward_mx(int layout, void* input, const void* scalars, int batch, float* policy,
                       float* wdl, float* moves_left, int wdl_probs, int write_back,
                       cudaStream_t s) {
  const int d = cfg.d_model;
  const int h = dense_hidden;
  const float eps = cfg.rms_norm_eps;
  auto* a_codes = workspace + ws_off.a_codes;
  auto* a_scales = workspace + ws_off.a_scales;
  auto* n_scales = workspace + ws_off.n_scales;
  auto* h_scales = workspace + ws_off.h_scales;
  // Test tap (outside stream capture only): the BF16 operands of one layer's quantisation
  // points and the codes and scales written for them.
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  check_cuda(cudaStreamIsCapturing(s, &capture), "query stream capture");
  const ce4b_mxfp8_tap* tap = mx_tap.layer >= 0 && capture == cudaStreamCaptureStatusNone ? &mx_tap : nullptr;
  const size_t rows_pad = static_cast<size_t>(batch + 127) / 128 * 128;
  auto copy_out = [&](void* dst, const void* src, size_t bytes) {
    if (dst != nullptr) check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s), "MXFP8 tap copy");
  };
  auto tap_n = [&](int layer) { return tap != nullptr && tap->layer == layer ? static_cast<bf16*>(tap->n_bf16_dev) : nullptr; };
  auto tap_n_codes = [&](int layer) {
    if (tap == nullptr || tap->layer != layer) return;
    copy_out(tap->n_codes_dev, workspace + ws_off.n_codes, rows_pad * d);
    copy_out(tap->n_scales_dev, n_scales, rows_pad / 128 * (d / 128) * 512);
  };
  expand_input_mx(layout, input, scalars, batch, cfg.history_length, a_codes, a_scales, write_back,
                  s);
  trace("expand_planes_mxfp8", s);
  if (tap != nullptr) {
    copy_out(tap->a_codes_dev, a_codes, rows_pad * in_dim);
    copy_out(tap->a_scales_dev, a_scales, rows_pad / 128 * (in_dim / 128) * 512);
  }
  const bf16* first_norm = cfg.depth > 0 ? layers[0].norm : w("final_norm.weight");
  gemm_mx_resnorm(tm_a_u8, tm_w_in, tm_x, tm_n_u8, a_scales, w_in_scales, n_scales,
                  w("input.bias"), first_norm, batch, d, in_dim, eps, s, tap_n(0));
  trace("input_gemm_bias_rmsnorm", s);
  tap_n_codes(0);
  for (int l = 0; l < cfg.depth; ++l) {
    const Layer& L = layers[l];
    const bf16* next_norm = l + 1 < cfg.depth ? layers[l + 1].norm : w("final_norm.weight");
    const bool tap_h = tap != nullptr && tap->layer == l;
    gemm_mx_swiglu(tm_n_u8, L.tm_gate_up, tm_h_u8, n_scales, L.gu_scales, h_scales, batch, h, d, s,
                   tap_h ? static_cast<bf16*>(tap->h_bf16_dev) : nullptr);
    trace("gate_up_swiglu", s);
    if (tap_h) {
      copy_out(tap->h_codes_dev, workspace + ws_off.h_codes, rows_pad * h);
      copy_out(tap->h_scales_dev, h_scales, rows_pad / 128 * (h / 128) * 512);
    }
    gemm_mx_resnorm(tm_h_u8, L.tm_down, tm_x, tm_n_u8, h_scales, L.down_scales, n_scales, nullptr,
                    next_norm, batch, d, h, eps, s, tap_n(l + 1));
    trace("down_residual_rmsnorm", s);
    tap_n_codes(l + 1);
  }
  gemm_mx_heads(tm_n_u8, tm_heads, n_scales, heads_scales, w("policy.bias"), policy, wdl,
                moves_left, batch, d, policy_size, policy_storage, wdl_probs, s);
  trace("heads", s);
}

// Dense BF16 forward as one persistent kernel (input GEMM, every layer, heads) after the
// plane expansion.
void Model::forward_fused(int layout, void* input, const void* scalars, int batch, float* policy,
                          float* wdl, float* moves_left, int wdl_probs, int write_back,
                          cudaStream_t s) {
  const int d = cfg.d_model;
  auto* sync = reinterpret_cast<int*>(workspace + ws_off.fwd_sync);
  // Counters restart from zero every forward (before the expansion, so that the
  // persistent kernel's predecessor in the stream is a kernel).
  check_cuda(cudaMemsetAsync(sync, 0, fwd_sync_bytes, s), "reset forward counters");
  expand_input(layout, input, scalars, batch, cfg.history_length,
               reinterpret_cast<bf16*>(workspace + ws_off.a_in), write_back, s);
  trace("expand_planes", s);
  const int nb_cap = rows_cap / 128;
  FwdParams p{};
  p.maps = reinterpret_cast<const FwdMaps*>(fwd_dev);
  p.bias = w("input.bias");
  p.x = reinterpret_cast<bf16*>(workspace + ws_off.x);
  p.hidden = reinterpret_cast<bf16*>(workspace + ws_off.hidden);
  p.ss = reinterpret_cast<float*>(workspace + ws_off.fwd_ss);
  p.sj = d / 128;
  p.part = reinterpret_cast<float*>(workspace + ws_off.fwd_part);
  p.hid_cnt = sync;
  p.slice_cnt = sync + nb_cap;
  p.part_cnt = sync + 2 * nb_cap;
  p.dpart_cnt = p.part_cnt + nb_cap * p.sj;
  p.task_counter = p.dpart_cnt + nb_cap * p.sj;
  p.err = device_error_word();
  p.rows_cap = rows_cap;
  p.nb = (batch + 127) / 128;
  p.d = d;
  p.h = dense_hidden;
  p.depth = cfg.depth;
  p.nc = dense_hidden / 128;
  p.xw = fused_xw(batch);
  p.xt = d / p.xw;
  p.xwi = fused_xwi();
  p.kis = fused_kis(batch);
  p.dks = fused_dks(batch);
  p.part_rb_chunks = (d / 128) * std::max(p.kis, p.dks);
  p.xti = d / p.xwi;
  p.kb_in = in_dim / kFwdKBlock;
  p.d96 = dense_hidden % kFwdDownStep == 0 && dense_hidden / kFwdDownStep >= p.dks ? 1 : 0;
  // A layer's down tiles of row block i are queued right after the gate_up tiles of row
  // block i + lag: with lag = 5/8 nb they are claimed close to when their inputs complete
  // (c1: 335 -> 330 us; lag = nb, all gate_up tiles first, and lag = nb / 4 are slower).
  p.lag = std::max(1, std::min(p.nb, (5 * p.nb + 7) / 8));
  p.head_bias = w("policy.bias");
  p.policy = policy;
  p.wdl = wdl;
  p.moves_left = moves_left;
  p.batch = batch;
  p.policy_size = policy_size;
  p.policy_storage = policy_storage;
  p.head_cols = policy_storage + 64;
  p.nht = fused_head_tasks();
  p.wdl_probs = wdl_probs;
  p.total_tasks = fused_task_count(batch);
  p.eps = cfg.rms_norm_eps;
  p.trace = fwd_trace;
  p.trace_cap = fwd_trace_cap;
  // One launch: input GEMM, every layer, and the heads of each row block as soon as its
  // last layer is published.
  dense_forward(p, s);
  trace("dense_tower", s);
}

// Shapes of the small-batch forward (latency.cu). Input GEMM: the most K parts of at most 4
// k-blocks that fit the SMs with d / 128 row blocks each. Down GEMMs: K parts of 2 k-blocks
// (1 when h / 64 is odd). gate_up tiles of even and odd layers, down tiles and head tiles
// each get their own CTAs, so a CTA's next weights load while it waits for its inputs.
void Model::plan_latency() {
  lat = false;
  const int d = cfg.d_model, h = dense_hidden;
  if (!fused || d > kLatMaxD || d % 128 != 0 || h % 64 != 0 || cfg.depth > kFwdMaxDepth) return;
  const int sms = sm_count();
  const int mt = d / 128, kb_in = in_dim / 64, hb = h / 64;
  int kp_in = 0;
  for (int kp = 1; kp <= kb_in; ++kp) {
    if (kb_in % kp == 0 && kb_in / kp <= kLatMaxKbSlot && mt * kp <= sms) kp_in = kp;
  }
  const int kc_dn = hb % 2 == 0 ? 2 : 1;
  const int kp_dn = hb / kc_dn;
  const int ht = (policy_storage + 64 + 127) / 128;
  const int gt = h / kLatGuUnits;
  // Two gate_up sets (even, odd layers); the heads go to the set the last layer leaves idle
  // when they fit there.
  const int layer_ctas = 2 * gt + mt * kp_dn + (ht <= gt ? 0 : ht);
  const int grid = std::max(layer_ctas, mt * kp_in);
  if (kp_in == 0 || grid > sms) return;
  lat = true;
  lat_kp_in = kp_in;
  lat_kp_dn = kp_dn;
  lat_grid = grid;
}

// Tensor maps and the per-CTA task lists of the small-batch forward (one device buffer).
void Model::build_latency() {
  const int d = cfg.d_model, h = dense_hidden, depth = cfg.depth;
  const int mt = d / 128, gt = h / kLatGuUnits, ht = (policy_storage + 64 + 127) / 128;
  LatMaps maps{};
  maps.a_in = make_tmap_bf16(workspace + ws_off.a_in, rows_cap, in_dim, in_dim, 64);
  maps.x = make_tmap_bf16(workspace + ws_off.x, rows_cap, d, d, 64);
  maps.hidden = make_tmap_bf16(workspace + ws_off.hidden, rows_cap, h, h, 64);
  maps.w_in = make_tmap_bf16(w("input.weight"), d, in_dim, in_dim, 128);
  for (int l = 0; l < depth; ++l) {
    const std::string p = "blocks." + std::to_string(l);
    // RMSNorm folded into the weight, as in the persistent forward (built just before).
    maps.gate_up[l] = make_tmap_bf16(fwd_weights + static_cast<size_t>(l) * 2 * h * d, 2 * h, d, d, kLatGuUnits);
    maps.down[l] = make_tmap_bf16(w(p + ".down.weight"), d, h, h, 128);
  }
  maps.heads = make_tmap_bf16(fwd_weights + static_cast<size_t>(depth) * 2 * h * d, policy_storage + 64, d, d, 128);
  // Task lists, each in dependency order (input, layers, heads), so that with every CTA
  // resident no wait can form a cycle.
  std::vector<std::vector<int4>> lists(lat_grid);
  const int n_in = mt * lat_kp_in;
  for (int m = 0; m < mt; ++m) {
    for (int k = 0; k < lat_kp_in; ++k) lists[lat_grid - n_in + m * lat_kp_in + k].push_back({kLatInput, 0, m, k});
  }
  const int down0 = 2 * gt;
  // Heads on the gate_up set that the last layer does not use (their weights load after its
  // last gate_up tile), else on CTAs of their own.
  const int heads0 = ht <= gt ? (depth % 2) * gt : down0 + mt * lat_kp_dn;
  for (int l = 0; l < depth; ++l) {
    for (int j = 0; j < gt; ++j) lists[(l % 2) * gt + j].push_back({kLatGateUp, l, j, 0});
    for (int m = 0; m < mt; ++m) {
      for (int k = 0; k < lat_kp_dn; ++k) lists[down0 + m * lat_kp_dn + k].push_back({kLatDown, l, m, k});
    }
  }
  for (int t = 0; t < ht; ++t) lists[heads0 + t].push_back({kLatHeads, depth, t, 0});
  lat_max_tasks = 1;
  for (const auto& v : lists) lat_max_tasks = std::max(lat_max_tasks, static_cast<int>(v.size()) + 1);
  std::vector<int4> table(static_cast<size_t>(lat_grid) * lat_max_tasks, int4{kLatEnd, 0, 0, 0});
  for (int c = 0; c < lat_grid; ++c) {
    for (size_t i = 0; i < lists[c].size(); ++i) table[static_cast<size_t>(c) * lat_max_tasks + i] = lists[c][i];
  }
  const size_t maps_bytes = align256(sizeof(LatMaps));
  if (lat_dev != nullptr) cudaFree(lat_dev);
  lat_dev = nullptr;
  check_cuda(cudaMalloc(&lat_dev, maps_bytes + table.size() * sizeof(int4)), "cudaMalloc small-batch plan");
  check_cuda(cudaMemcpy(lat_dev, &maps, sizeof(LatMaps), cudaMemcpyHostToDevice), "copy small-batch maps");
  check_cuda(cudaMemcpy(lat_dev + maps_bytes, table.data(), table.size() * sizeof(int4), cudaMemcpyHostToDevice),
             "copy small-batch tasks");
}

void Model::forward_latency(int layout, void* input, const void* scalars, int batch, float* policy,
                            float* wdl, float* moves_left, int wdl_probs, int write_back, cudaStream_t s) {
  const int d = cfg.d_model;
  // The counters are zero: from the workspace reset at create, then from the last CTA of
  // each launch.
  auto* sync = reinterpret_cast<int*>(workspace + ws_off.lat_sync);
  expand_input(layout, input, scalars, batch, cfg.history_length,
               reinterpret_cast<bf16*>(workspace + ws_off.a_in), write_back, s);
  trace("expand_planes", s);
  LatParams p{};
  p.maps = reinterpret_cast<const LatMaps*>(lat_dev);
  p.tasks = reinterpret_cast<const int4*>(lat_dev + align256(sizeof(LatMaps)));
  p.max_tasks = lat_max_tasks;
  p.in_bias = w("input.bias");
  p.head_bias = w("policy.bias");
  p.x = reinterpret_cast<bf16*>(workspace + ws_off.x);
  p.hidden = reinterpret_cast<bf16*>(workspace + ws_off.hidden);
  p.part_in = reinterpret_cast<float*>(workspace + ws_off.lat_part_in);
  p.part_dn = reinterpret_cast<float*>(workspace + ws_off.lat_part_dn);
  p.cnt = sync;
  p.err = device_error_word();
  p.policy = policy;
  p.wdl = wdl;
  p.moves_left = moves_left;
  p.batch = batch;
  p.n = (batch + 15) / 16 * 16;
  p.d = d;
  p.h = dense_hidden;
  p.depth = cfg.depth;
  p.mt = d / 128;
  p.kb_in = in_dim / 64;
  p.kp_in = lat_kp_in;
  p.kp_dn = lat_kp_dn;
  p.gt = dense_hidden / kLatGuUnits;
  p.ht = (policy_storage + 64 + 127) / 128;
  p.policy_size = policy_size;
  p.policy_storage = policy_storage;
  p.head_cols = policy_storage + 64;
  p.wdl_probs = wdl_probs;
  p.eps = cfg.rms_norm_eps;
  p.trace = fwd_trace;
  p.trace_cap = fwd_trace_cap;
  latency_forward(p, lat_grid, s);
  trace("dense_latency", s);
}

void Model::forward(int layout, void* input, const void* scalars, int batch, float* policy,
                    float* wdl, float* moves_left, int wdl_probs, int normalize_in_place,
                    int32_t* tokens_per_expert, cudaStream_t s) {
  if (!finalized) fail(CE4B_ERR_NOT_READY, "model is not finalized");
  require(batch >= 1 && batch <= max_batch,
          "batch size " + std::to_string(batch) + " exceeds model capacity " +
              std::to_string(max_batch));
  require(input != nullptr && policy != nullptr && wdl != nullptr && moves_left != nullptr,
          "null input or output pointer");
  const int d = cfg.d_model;
  const float eps = cfg.rms_norm_eps;
  bf16* a_in = reinterpret_cast<bf16*>(workspace + ws_off.a_in);
  const int write_back = normalize_in_place && cfg.history_length == 8;

  trace_next = 0;
  trace_labels.clear();
  if (fused) {
    if (latency_path(batch)) {
      forward_latency(layout, input, scalars, batch, policy, wdl, moves_left, wdl_probs, write_back, s);
    } else {
      forward_fused(layout, input, scalars, batch, policy, wdl, moves_left, wdl_probs, write_back, s);
    }
    return;
  }
  if (mx) {
    forward_mx(layout, input, scalars, batch, policy, wdl, moves_left, wdl_probs, write_back, s);
    return;
  }
  expand_input(layout, input, scalars, batch, cfg.history_length, a_in, write_back, s);
  trace("expand_planes", s);
  const bf16* first_norm = cfg.depth > 0 ? layers[0].norm : w("final_norm.weight");
  gemm_resnorm(tm_a_in, tm_w_in, tm_x, tm_n, w("input.bias"), first_norm, batch, d, in_dim, eps, s);
  trace("input_gemm_bias_rmsnorm", s);
  for (int l = 0; l < cfg.depth; ++l) {
    const Layer& L = layers[l];
    const bf16* next_norm = l + 1 < cfg.depth ? layers[l + 1].norm : w("final_norm.weight");
    if (L.moe) {
      if (ep_world > 1) {
        moe_layer_ep(L, l / 2, next_norm, batch, tokens_per_expert, s);
      } else {
        moe_layer(L, l / 2, next_norm, batch, tokens_per_expert, s);
      }
      continue;
    }
    gemm_swiglu(tm_n, L.tm_gate_up, tm_hidden, batch, dense_hidden, d, s);
    trace("gate_up_swiglu", s);
    gemm_resnorm(tm_hidden, L.tm_down, tm_x, tm_n, nullptr, next_norm, batch, d, dense_hidden, eps,
                 s);
    trace("down_residual_rmsnorm", s);
  }
  gemm_heads(tm_n, tm_heads, w("policy.bias"), policy, wdl, moves_left, batch, d, policy_size,
             policy_storage, wdl_probs, s);
  trace("heads", s);
}

// One moe64a2 expert layer (src/chess_engine_4/model/moe.py:160-180, static dispatch path
// :226-287): router GEMM with the top-2 epilogue, scan, dispatch, grouped gate_up+SwiGLU,
// grouped down scaled by the route weight, combine + residual + next layer's RMSNorm.
void Model::moe_layer(const Layer& L, int moe_index, const bf16* next_norm, int batch,
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
  auto* yperm = reinterpret_cast<bf16*>(at(ws_off.yperm));
  auto* x = reinterpret_cast<bf16*>(at(ws_off.x));
  auto* n = reinterpret_cast<bf16*>(at(ws_off.n));
  moe_router_gemm(tm_n, L.tm_router, L.beta, route_expert, route_prob, block_hist, batch, d, s);
  trace("moe_router", s);
  if (moe_tap != nullptr && batch <= moe_tap_tokens) {
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    check_cuda(cudaStreamIsCapturing(s, &capture), "query stream capture");
    if (capture == cudaStreamCaptureStatusNone) {
      check_cuda(cudaMemcpyAsync(moe_tap + static_cast<size_t>(moe_index) * batch * 2, route_expert,
                                 static_cast<size_t>(batch) * 8, cudaMemcpyDeviceToDevice, s),
                 "routing tap copy");
    }
  }
  moe_scan(block_hist, (batch + 127) / 128, expert_start, block_off, m_tiles, num_m_tiles,
           tokens_per_expert != nullptr ? tokens_per_expert + 64 * moe_index : nullptr, s);
  trace("moe_scan", s);
  moe_dispatch(n, route_expert, route_prob, expert_start, block_off, xperm, pprob, route_pos,
               batch, d, s);
  trace("moe_dispatch", s);
  gemm_grouped_swiglu(tm_xperm, L.tm_gate_up, tm_hperm, m_tiles, num_m_tiles, he, d, s);
  trace("moe_experts_gate_up_swiglu", s);
  gemm_grouped_scale(tm_hperm, L.tm_down, tm_yperm, m_tiles, num_m_tiles, pprob, d, he, s);
  trace("moe_experts_down", s);
  moe_combine_norm(x, yperm, route_pos, next_norm, n, batch, d, cfg.rms_norm_eps, s);
  trace("moe_combine_rmsnorm", s);
}

void Model::forward_ordered(int layout, void* input, const void* scalars, int batch,
                            float* policy, float* wdl, float* moves_left, int wdl_probs,
                            int normalize_in_place, int32_t* tokens_per_expert, cudaStream_t s) {
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  check_cuda(cudaStreamIsCapturing(s, &capture), "query stream capture");
  // Under the caller's stream capture the graph's own edges order the launches.
  const bool order = capture == cudaStreamCaptureStatusNone;
  if (order) check_cuda(cudaStreamWaitEvent(s, forward_done, 0), "wait previous forward");
  forward(layout, input, scalars, batch, policy, wdl, moves_left, wdl_probs, normalize_in_place,
          tokens_per_expert, s);
  if (order) check_cuda(cudaEventRecord(forward_done, s), "record forward");
}

void Model::trace(const char* label, cudaStream_t s) {
  if (trace_next >= trace_events.size()) return;
  check_cuda(cudaEventRecord(trace_events[trace_next++], s), "record trace event");
  trace_labels.emplace_back(label);
}

cudaGraphExec_t Model::capture_evaluate(const ce4b_input_plane* planes, int batch, float* pol,
                                        float* wdl, float* ml) {
  const std::vector<cudaEvent_t> saved = std::move(trace_events);
  trace_events.clear();
  cudaGraphExec_t exec = nullptr;
  try {
    check_cuda(cudaStreamWaitEvent(stream, forward_done, 0), "wait previous forward");
    forward(CE4B_INPUT_LC0, const_cast<ce4b_input_plane*>(planes), nullptr, batch, pol, wdl, ml, 1, 0,
            nullptr, stream);
    check_cuda(cudaStreamSynchronize(stream), "warm-up forward");
    check_cuda(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "begin capture");
    try {
      forward(CE4B_INPUT_LC0, const_cast<ce4b_input_plane*>(planes), nullptr, batch, pol, wdl, ml, 1, 0,
              nullptr, stream);
    } catch (...) {
      cudaGraph_t g = nullptr;
      cudaStreamEndCapture(stream, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    cudaGraph_t graph = nullptr;
    check_cuda(cudaStreamEndCapture(stream, &graph), "end capture");
    const cudaError_t st = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    check_cuda(st, "instantiate graph");
  } catch (...) {
    trace_events = saved;
    throw;
  }
  trace_events = saved;
  return exec;
}

cudaGraphExec_t Model::evaluate_graph(int batch, int slot) {
  IoSlot& io_slot = io[slot];
  auto* planes = reinterpret_cast<ce4b_input_plane*>(workspace + io_slot.planes);
  float* pol = reinterpret_cast<float*>(workspace + io_slot.policy);
  float* wdl = reinterpret_cast<float*>(workspace + io_slot.wdl);
  float* ml = reinterpret_cast<float*>(workspace + io_slot.moves_left);
  const int key = batch * kIoSlots + slot;
  auto it = graphs.find(key);
  if (it != graphs.end()) return it->second;
  // First use of this batch size and slot (the slot's earlier copies are done first).
  check_cuda(cudaStreamWaitEvent(stream, io_slot.free, 0), "wait I/O slot");
  return graphs.emplace(key, capture_evaluate(planes, batch, pol, wdl, ml)).first->second;
}

namespace {

using PointerAttributeFn = CUresult (*)(void*, CUpointer_attribute, CUdeviceptr);

PointerAttributeFn pointer_attribute_fn() {
  static PointerAttributeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuPointerGetAttribute", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PointerAttributeFn>(p);
    }
  });
  return fn;
}

// The device address of host buffer [ptr, ptr + bytes) when it is pinned and mapped for the
// current device over its whole extent, else nullptr: its first and last byte must both be
// mapped, lie in one CUDA allocation or registration (the same process-unique buffer id, so
// no unmapped hole can sit between them) and resolve to device addresses bytes - 1 apart.
void* mapped_view(const void* ptr, size_t bytes) {
  auto view = [](const void* p) -> char* {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
      (void)cudaGetLastError();
      return nullptr;
    }
    return a.type == cudaMemoryTypeHost ? static_cast<char*>(a.devicePointer) : nullptr;
  };
  auto buffer_id = [](const void* p, unsigned long long* id) {
    const PointerAttributeFn fn = pointer_attribute_fn();
    return fn != nullptr &&
           fn(id, CU_POINTER_ATTRIBUTE_BUFFER_ID, reinterpret_cast<CUdeviceptr>(p)) == CUDA_SUCCESS;
  };
  if (ptr == nullptr || bytes == 0) return nullptr;
  const void* end = static_cast<const char*>(ptr) + bytes - 1;
  char* first = view(ptr);
  char* last = view(end);
  if (first == nullptr || last == nullptr || last - first != static_cast<ptrdiff_t>(bytes - 1)) return nullptr;
  unsigned long long id_first = 0, id_last = 0;
  if (!buffer_id(ptr, &id_first) || !buffer_id(end, &id_last) || id_first != id_last) return nullptr;
  return first;
}

}  // namespace

cudaGraphExec_t Model::direct_graph(const ce4b_input_plane* host_planes, int batch, float* host_policy,
                                    float* host_wdl, float* host_moves_left) {
  if (!latency_path(batch)) return nullptr;
  const size_t b = static_cast<size_t>(batch);
  auto* planes = static_cast<ce4b_input_plane*>(mapped_view(host_planes, b * kInputPlanes * sizeof(ce4b_input_plane)));
  auto* pol = static_cast<float*>(mapped_view(host_policy, b * policy_size * 4));
  auto* wdl = static_cast<float*>(mapped_view(host_wdl, b * 3 * 4));
  auto* ml = static_cast<float*>(mapped_view(host_moves_left, b * 4));
  if (planes == nullptr || pol == nullptr || wdl == nullptr || ml == nullptr) return nullptr;
  const std::array<uintptr_t, 5> key{static_cast<uintptr_t>(batch), reinterpret_cast<uintptr_t>(planes),
                                     reinterpret_cast<uintptr_t>(pol), reinterpret_cast<uintptr_t>(wdl),
                                     reinterpret_cast<uintptr_t>(ml)};
  auto it = direct_graphs.find(key);
  if (it != direct_graphs.end()) return it->second;
  if (direct_graphs.size() >= kDirectGraphs) {
    for (auto& kv : direct_graphs) cudaGraphExecDestroy(kv.second);
    direct_graphs.clear();
  }
  return direct_graphs.emplace(key, capture_evaluate(planes, batch, pol, wdl, ml)).first->second;
}

void Model::enqueue_evaluate_legal(const ce4b_input_plane* host_planes, int batch,
                                   const int32_t* host_offsets, const int32_t* host_indices,
                                   float temperature, float* host_probs, float* host_wdl,
                                   float* host_moves_left, cudaStream_t s) {
  if (!finalized) fail(CE4B_ERR_NOT_READY, "model is not finalized");
  require(batch >= 1 && batch <= max_batch, "batch size exceeds model capacity");
  require(host_planes && host_offsets && host_probs && host_wdl && host_moves_left,
          "null host buffer");
  require(host_offsets[0] == 0, "move offsets must start at 0");
  for (int b = 0; b < batch; ++b) {
    require(host_offsets[b + 1] >= host_offsets[b] &&
                host_offsets[b + 1] - host_offsets[b] <= kMaxMovesPerPosition,
            "move offsets must be non-decreasing, at most 256 moves per position");
  }
  const int nnz = host_offsets[batch];
  require(nnz == 0 || host_indices != nullptr, "null move indices");
  check_cuda(cudaSetDevice(device), "cudaSetDevice");
  const int slot = static_cast<int>(io_next % kIoSlots);
  IoSlot& io_slot = io[slot];
  auto* planes = reinterpret_cast<ce4b_input_plane*>(workspace + io_slot.planes);
  float* pol = reinterpret_cast<float*>(workspace + io_slot.policy);
  float* wdl = reinterpret_cast<float*>(workspace + io_slot.wdl);
  float* ml = reinterpret_cast<float*>(workspace + io_slot.moves_left);
  auto* offsets = reinterpret_cast<int32_t*>(workspace + io_slot.move_offsets);
  auto* indices = reinterpret_cast<int32_t*>(workspace + io_slot.move_indices);
  auto* probs = reinterpret_cast<float*>(workspace + io_slot.move_probs);
  cudaGraphExec_t graph = evaluate_graph(batch, slot);
  ++io_next;
  check_cuda(cudaStreamWaitEvent(s, io_slot.free, 0), "wait I/O slot");
  check_cuda(cudaMemcpyAsync(planes, host_planes,
                             static_cast<size_t>(batch) * kInputPlanes * sizeof(ce4b_input_plane),
                             cudaMemcpyHostToDevice, s),
             "copy input planes");
  check_cuda(cudaMemcpyAsync(offsets, host_offsets, (batch + 1) * 4, cudaMemcpyHostToDevice, s),
             "copy move offsets");
  if (nnz > 0) {
    check_cuda(cudaMemcpyAsync(indices, host_indices, static_cast<size_t>(nnz) * 4,
                               cudaMemcpyHostToDevice, s),
               "copy move indices");
  }
  check_cuda(cudaStreamWaitEvent(s, forward_done, 0), "wait previous forward");
  if (graph != nullptr) {
    check_cuda(cudaGraphLaunch(graph, s), "launch graph");
  } else {
    forward(CE4B_INPUT_LC0, planes, nullptr, batch, pol, wdl, ml, 1, 0, nullptr, s);
  }
  policy_softmax(pol, batch, policy_size, offsets, indices, temperature, probs, s);
  check_cuda(cudaEventRecord(forward_done, s), "record forward");
  if (nnz > 0) {
    check_cuda(cudaMemcpyAsync(host_probs, probs, static_cast<size_t>(nnz) * 4,
                               cudaMemcpyDeviceToHost, s),
               "copy move probabilities");
  }
  check_cuda(cudaMemcpyAsync(host_wdl, wdl, static_cast<size_t>(batch) * 3 * 4,
                             cudaMemcpyDeviceToHost, s),
             "copy wdl");
  check_cuda(cudaMemcpyAsync(host_moves_left, ml, static_cast<size_t>(batch) * 4,
                             cudaMemcpyDeviceToHost, s),
             "copy moves left");
  check_cuda(cudaEventRecord(io_slot.free, s), "record I/O slot");
}

void Model::enqueue_evaluate(const ce4b_input_plane* host_planes, int batch, float* host_policy,
                             float* host_wdl, float* host_moves_left, cudaStream_t s) {
  if (!finalized) fail(CE4B_ERR_NOT_READY, "model is not finalized");
  require(batch >= 1 && batch <= max_batch, "batch size exceeds model capacity");
  require(host_planes && host_policy && host_wdl && host_moves_left, "null host buffer");
  check_cuda(cudaSetDevice(device), "cudaSetDevice");
  if (direct_io) {
    cudaGraphExec_t direct = direct_graph(host_planes, batch, host_policy, host_wdl, host_moves_left);
    if (direct != nullptr) {
      check_cuda(cudaStreamWaitEvent(s, forward_done, 0), "wait previous forward");
      check_cuda(cudaGraphLaunch(direct, s), "launch graph");
      check_cuda(cudaEventRecord(forward_done, s), "record forward");
      return;
    }
  }
  const int slot = static_cast<int>(io_next % kIoSlots);
  IoSlot& io_slot = io[slot];
  auto* planes = reinterpret_cast<ce4b_input_plane*>(workspace + io_slot.planes);
  float* pol = reinterpret_cast<float*>(workspace + io_slot.policy);
  float* wdl = reinterpret_cast<float*>(workspace + io_slot.wdl);
  float* ml = reinterpret_cast<float*>(workspace + io_slot.moves_left);
  cudaGraphExec_t graph = evaluate_graph(batch, slot);
  ++io_next;
  // This slot's previous D2H copies are done before its planes are overwritten; the H2D
  // copy may overlap the previous call's forward, which the graph then waits for.
  check_cuda(cudaStreamWaitEvent(s, io_slot.free, 0), "wait I/O slot");
  check_cuda(cudaMemcpyAsync(planes, host_planes,
                             static_cast<size_t>(batch) * kInputPlanes * sizeof(ce4b_input_plane),
                             cudaMemcpyHostToDevice, s),
             "copy input planes");
  check_cuda(cudaStreamWaitEvent(s, forward_done, 0), "wait previous forward");
  if (graph != nullptr) {
    check_cuda(cudaGraphLaunch(graph, s), "launch graph");
  } else {
    forward(CE4B_INPUT_LC0, planes, nullptr, batch, pol, wdl, ml, 1, 0, nullptr, s);
  }
  check_cuda(cudaEventRecord(forward_done, s), "record forward");
  check_cuda(cudaMemcpyAsync(host_policy, pol, static_cast<size_t>(batch) * policy_size * 4,
                             cudaMemcpyDeviceToHost, s),
             "copy policy");
  check_cuda(cudaMemcpyAsync(host_wdl, wdl, static_cast<size_t>(batch) * 3 * 4,
                             cudaMemcpyDeviceToHost, s),
             "copy wdl");
  check_cuda(cudaMemcpyAsync(host_moves_left, ml, static_cast<size_t>(batch) * 4,
                             cudaMemcpyDeviceToHost, s),
             "copy moves left");
  check_cuda(cudaEventRecord(io_slot.free, s), "record I/O slot");
}

void Model::evaluate(const ce4b_input_plane* host_planes, int batch, float* host_policy,
                     float* host_wdl, float* host_moves_left) {
  enqueue_evaluate(host_planes, batch, host_policy, host_wdl, host_moves_left, stream);
  check_cuda(cudaStreamSynchronize(stream), "synchronize evaluation");
}

// ------------------------------------------------------------------ Safetensors loading
namespace {

const std::string& meta(const SafetensorsFile& f, const std::string& key) {
  auto it = f.metadata.find(key);
  if (it == f.metadata.end()) fail(CE4B_ERR_IO, "model metadata is missing " + key);
  return it->second;
}

int meta_int(const SafetensorsFile& f, const std::string& key) {
  try {
    return std::stoi(meta(f, key));
  } catch (const Error&) {
    throw;
  } catch (...) {
    fail(CE4B_ERR_IO, "model metadata " + key + " is not an integer");
  }
}

float meta_float(const SafetensorsFile& f, const std::string& key) {
  try {
    return std::stof(meta(f, key));
  } catch (const Error&) {
    throw;
  } catch (...) {
    fail(CE4B_ERR_IO, "model metadata " + key + " is not a number");
  }
}

}  // namespace

std::unique_ptr<Model> load_safetensors_model(const std::string& path, int device, int max_batch,
                                              int precision) {
  const SafetensorsFile f = read_safetensors(path);
  // Contract checks of kernels/src/inference/runtime.cu:348-396.
  if (meta(f, "format") != "chess-engine-4" || meta(f, "format_version") != "1") {
    fail(CE4B_ERR_UNSUPPORTED, "unsupported model format");
  }
  const std::string arch = meta(f, "architecture");
  if (arch != "dense" && arch != "moe64a2") {
    fail(CE4B_ERR_UNSUPPORTED, "unsupported model architecture: " + arch);
  }
  if (meta(f, "activation") != "swiglu" || meta(f, "input_format") != "lc0-classical-112" ||
      meta(f, "input_normalization") != "history-select-rule50-div99-v1" ||
      meta_int(f, "input_planes") != kInputPlanes || meta_int(f, "board_size") != 8) {
    fail(CE4B_ERR_UNSUPPORTED, "unsupported model contract");
  }
  if (arch == "moe64a2" &&
      (meta_int(f, "num_experts") != 64 || meta_int(f, "num_active_experts") != 2 ||
       meta(f, "layer_pattern") != "alternating-moe-dense")) {
    fail(CE4B_ERR_UNSUPPORTED, "unsupported MoE model contract");
  }
  ce4b_model_config c{};
  c.arch = arch == "dense" ? CE4B_ARCH_DENSE : CE4B_ARCH_MOE64A2;
  c.d_model = meta_int(f, "d_model");
  c.depth = meta_int(f, "depth");
  c.history_length = meta_int(f, "history_length");
  c.expansion_ratio = meta_float(f, "expansion_ratio");
  c.rms_norm_eps = meta_float(f, "rms_norm_eps");
  c.policy_size = meta_int(f, "policy_size");
  c.policy_storage_size = meta_int(f, "policy_storage_size");
  c.precision = precision;
  auto m = std::make_unique<Model>();
  m->create(c, device, max_batch);
  for (const auto& kv : m->slots) {
    auto it = f.tensors.find(kv.first);
    if (it == f.tensors.end()) fail(CE4B_ERR_IO, "model is missing tensor " + kv.first);
    const SafetensorsTensor& t = it->second;
    const int dtype = t.dtype == "BF16" ? CE4B_DTYPE_BF16 : (t.dtype == "F32" ? CE4B_DTYPE_F32 : -1);
    if (dtype < 0) fail(CE4B_ERR_IO, "tensor " + kv.first + " has an unsupported dtype");
    if (t.bytes != kv.second.bytes) fail(CE4B_ERR_IO, "tensor " + kv.first + " has a wrong size");
    m->set_tensor(kv.first, t.data, dtype, t.shape, false);
  }
  m->finalize();
  return m;
}

}  // namespace ce4b
