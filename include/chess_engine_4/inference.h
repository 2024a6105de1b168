// chess_engine_4::inference over libce4b200: a header-only drop-in for the engine API the
// lc0 `ce4` backend links (kernels/include/chess_engine_4/inference.h:10-51 of the
// reference; third_party/lc0/src/neural/backends/ce4/backend.cc:77-78, 160-168). Same
// names, types and error behaviour (std::runtime_error); the work runs in libce4b200's
// C ABI (ce4b200.h): Load = ce4b_model_load_safetensors, Evaluate = ce4b_model_evaluate
// (blocking; policy logits [B, policy_size], WDL probabilities [B, 3], moves-left [B]).
// Needs C++20 (std::span) in the including translation unit; link with -lce4b200.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <span>
#include <stdexcept>
#include <string>

#include "ce4b200.h"

namespace chess_engine_4::inference {

struct InputPlane {
  std::uint64_t mask;
  float value;
};
static_assert(sizeof(InputPlane) == sizeof(ce4b_input_plane), "InputPlane is 16 bytes");
static_assert(offsetof(InputPlane, value) == offsetof(ce4b_input_plane, value), "InputPlane layout");

struct ModelInfo {
  int d_model;
  int depth;
  int history_length;
  int policy_size;
  int maximum_batch_size;
};

struct Outputs {
  std::span<float> policy;
  std::span<float> wdl;
  std::span<float> moves_left;
};

class Model {
 public:
  // Reads a Safetensors v1 model file onto GPU `gpu` for batches of up to
  // `maximum_batch_size` positions (BF16 forward).
  static std::unique_ptr<Model> Load(const std::string& path, int gpu, int maximum_batch_size) {
    ce4b_model* handle = nullptr;
    Check(ce4b_model_load_safetensors(path.c_str(), gpu, maximum_batch_size, CE4B_PRECISION_BF16,
                                      &handle));
    ce4b_model_info raw{};
    const int status = ce4b_model_info_get(handle, &raw);
    if (status != CE4B_OK) {
      const std::string message = ce4b_last_error();
      ce4b_model_destroy(handle);
      throw std::runtime_error("ce4b200: " + message);
    }
    ModelInfo info{raw.d_model, raw.depth, raw.history_length, raw.policy_size,
                   raw.maximum_batch_size};
    return std::unique_ptr<Model>(new Model(handle, info));
  }

  ~Model() {
    if (handle_ != nullptr) ce4b_model_destroy(handle_);
  }
  Model(Model&& other) noexcept : handle_(other.handle_), info_(other.info_) { other.handle_ = nullptr; }
  Model& operator=(Model&& other) noexcept {
    if (this != &other) {
      if (handle_ != nullptr) ce4b_model_destroy(handle_);
      handle_ = other.handle_;
      info_ = other.info_;
      other.handle_ = nullptr;
    }
    return *this;
  }
  Model(const Model&) = delete;
  Model& operator=(const Model&) = delete;

  const ModelInfo& info() const { return info_; }

  // planes: batch_size * 112 records; outputs sized batch_size * {policy_size, 3, 1}.
  // Not thread-safe (serialise calls on one model, as lc0 does with its mutex). Spans over
  // pinned, mapped host memory (cudaHostAlloc / cudaHostRegister) let small batches run
  // without copies (see ce4b_model_evaluate).
  void Evaluate(std::span<const InputPlane> planes, int batch_size, Outputs outputs) {
    if (batch_size < 1 || batch_size > info_.maximum_batch_size) {
      throw std::runtime_error("ce4b200: batch size out of range");
    }
    const auto b = static_cast<std::size_t>(batch_size);
    if (planes.size() < b * 112 || outputs.policy.size() < b * info_.policy_size ||
        outputs.wdl.size() < b * 3 || outputs.moves_left.size() < b) {
      throw std::runtime_error("ce4b200: input or output span too small for the batch");
    }
    Check(ce4b_model_evaluate(handle_, reinterpret_cast<const ce4b_input_plane*>(planes.data()),
                              batch_size, outputs.policy.data(), outputs.wdl.data(),
                              outputs.moves_left.data()));
  }

 private:
  Model(ce4b_model* handle, ModelInfo info) : handle_(handle), info_(info) {}
  static void Check(int status) {
    if (status != CE4B_OK) throw std::runtime_error(std::string("ce4b200: ") + ce4b_last_error());
  }

  ce4b_model* handle_ = nullptr;
  ModelInfo info_{};
};

}  // namespace chess_engine_4::inference
