// Safetensors reader used by ce4b_model_load_safetensors.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <unordered_map>
#include <vector>

namespace ce4b {

struct SafetensorsTensor {
  std::string dtype;  // "BF16", "F32", ...
  std::vector<int64_t> shape;
  const uint8_t* data = nullptr;
  uint64_t bytes = 0;
};

struct SafetensorsFile {
  std::map<std::string, std::string> metadata;
  std::unordered_map<std::string, SafetensorsTensor> tensors;
  std::vector<uint8_t> storage;
};

SafetensorsFile read_safetensors(const std::string& path);

}  // namespace ce4b
