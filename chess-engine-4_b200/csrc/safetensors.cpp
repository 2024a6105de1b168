// Minimal Safetensors reader: 8-byte little-endian header length, a JSON header mapping
// tensor names to {dtype, shape, data_offsets} plus an optional "__metadata__" map of
// strings, then the raw tensor bytes. Only the JSON subset that format uses is parsed.
#include "safetensors.h"

#include <cstring>
#include <fstream>

#include "internal.h"

namespace ce4b {

namespace {

struct JsonValue;
using JsonObject = std::vector<std::pair<std::string, JsonValue>>;

struct JsonValue {
  enum Kind { kNull, kBool, kNumber, kString, kArray, kObject } kind = kNull;
  double number = 0.0;
  bool boolean = false;
  std::string str;
  std::vector<JsonValue> array;
  JsonObject object;
};

class JsonParser {
 public:
  JsonParser(const char* begin, const char* end) : p_(begin), end_(end) {}

  JsonValue parse() {
    JsonValue v = value();
    skip_ws();
    if (p_ != end_) bad("trailing characters");
    return v;
  }

 private:
  [[noreturn]] void bad(const char* what) {
    fail(CE4B_ERR_IO, std::string("invalid Safetensors header JSON: ") + what);
  }
  void skip_ws() {
    while (p_ != end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  char peek() {
    skip_ws();
    if (p_ == end_) bad("unexpected end");
    return *p_;
  }
  void expect(char c) {
    if (peek() != c) bad("unexpected character");
    ++p_;
  }
  JsonValue value() {
    const char c = peek();
    JsonValue v;
    if (c == '{') {
      v.kind = JsonValue::kObject;
      ++p_;
      if (peek() == '}') {
        ++p_;
        return v;
      }
      while (true) {
        std::string key = string_body();
        expect(':');
        v.object.emplace_back(std::move(key), value());
        const char n = peek();
        ++p_;
        if (n == '}') break;
        if (n != ',') bad("expected , or }");
      }
    } else if (c == '[') {
      v.kind = JsonValue::kArray;
      ++p_;
      if (peek() == ']') {
        ++p_;
        return v;
      }
      while (true) {
        v.array.push_back(value());
        const char n = peek();
        ++p_;
        if (n == ']') break;
        if (n != ',') bad("expected , or ]");
      }
    } else if (c == '"') {
      v.kind = JsonValue::kString;
      v.str = string_body();
    } else if (c == 't' || c == 'f' || c == 'n') {
      const char* word = c == 't' ? "true" : (c == 'f' ? "false" : "null");
      const size_t len = std::strlen(word);
      if (static_cast<size_t>(end_ - p_) < len || std::strncmp(p_, word, len) != 0) bad("literal");
      p_ += len;
      v.kind = c == 'n' ? JsonValue::kNull : JsonValue::kBool;
      v.boolean = c == 't';
    } else {
      v.kind = JsonValue::kNumber;
      const char* start = p_;
      while (p_ != end_ && (std::strchr("+-0123456789.eE", *p_) != nullptr)) ++p_;
      if (start == p_) bad("number");
      v.number = std::stod(std::string(start, p_));
    }
    return v;
  }
  std::string string_body() {
    expect('"');
    std::string out;
    while (true) {
      if (p_ == end_) bad("unterminated string");
      const char c = *p_++;
      if (c == '"') break;
      if (c != '\\') {
        out.push_back(c);
        continue;
      }
      if (p_ == end_) bad("bad escape");
      const char e = *p_++;
      switch (e) {
        case '"': out.push_back('"'); break;
        case '\\': out.push_back('\\'); break;
        case '/': out.push_back('/'); break;
        case 'b': out.push_back('\b'); break;
        case 'f': out.push_back('\f'); break;
        case 'n': out.push_back('\n'); break;
        case 'r': out.push_back('\r'); break;
        case 't': out.push_back('\t'); break;
        case 'u': {
          if (end_ - p_ < 4) bad("bad \\u escape");
          const unsigned code = static_cast<unsigned>(std::stoul(std::string(p_, p_ + 4), nullptr, 16));
          p_ += 4;
          if (code < 0x80) {
            out.push_back(static_cast<char>(code));
          } else if (code < 0x800) {
            out.push_back(static_cast<char>(0xC0 | (code >> 6)));
            out.push_back(static_cast<char>(0x80 | (code & 0x3F)));
          } else {
            out.push_back(static_cast<char>(0xE0 | (code >> 12)));
            out.push_back(static_cast<char>(0x80 | ((code >> 6) & 0x3F)));
            out.push_back(static_cast<char>(0x80 | (code & 0x3F)));
          }
          break;
        }
        default: bad("bad escape");
      }
    }
    return out;
  }

  const char* p_;
  const char* end_;
};

const JsonValue* find(const JsonObject& obj, const std::string& key) {
  for (const auto& kv : obj) {
    if (kv.first == key) return &kv.second;
  }
  return nullptr;
}

}  // namespace

SafetensorsFile read_safetensors(const std::string& path) {
  std::ifstream in(path, std::ios::binary | std::ios::ate);
  if (!in) fail(CE4B_ERR_IO, "cannot open model: " + path);
  const auto size = static_cast<uint64_t>(in.tellg());
  in.seekg(0);
  SafetensorsFile file;
  file.storage.resize(size);
  in.read(reinterpret_cast<char*>(file.storage.data()), static_cast<std::streamsize>(size));
  if (!in || size < 8) fail(CE4B_ERR_IO, "invalid Safetensors file: " + path);
  uint64_t header_len = 0;
  std::memcpy(&header_len, file.storage.data(), 8);
  if (header_len > size - 8) fail(CE4B_ERR_IO, "invalid Safetensors header size");
  const char* hbegin = reinterpret_cast<const char*>(file.storage.data() + 8);
  const JsonValue root = JsonParser(hbegin, hbegin + header_len).parse();
  if (root.kind != JsonValue::kObject) fail(CE4B_ERR_IO, "Safetensors header is not an object");
  const uint64_t data_start = 8 + header_len;
  for (const auto& [name, v] : root.object) {
    if (name == "__metadata__") {
      if (v.kind != JsonValue::kObject) fail(CE4B_ERR_IO, "__metadata__ is not an object");
      for (const auto& [k, mv] : v.object) {
        if (mv.kind != JsonValue::kString) fail(CE4B_ERR_IO, "metadata value is not a string");
        file.metadata[k] = mv.str;
      }
      continue;
    }
    if (v.kind != JsonValue::kObject) fail(CE4B_ERR_IO, "tensor entry is not an object");
    const JsonValue* dtype = find(v.object, "dtype");
    const JsonValue* shape = find(v.object, "shape");
    const JsonValue* offsets = find(v.object, "data_offsets");
    if (dtype == nullptr || shape == nullptr || offsets == nullptr ||
        dtype->kind != JsonValue::kString || shape->kind != JsonValue::kArray ||
        offsets->kind != JsonValue::kArray || offsets->array.size() != 2) {
      fail(CE4B_ERR_IO, "tensor " + name + " has a malformed entry");
    }
    SafetensorsTensor t;
    t.dtype = dtype->str;
    for (const auto& d : shape->array) t.shape.push_back(static_cast<int64_t>(d.number));
    const auto b = static_cast<uint64_t>(offsets->array[0].number);
    const auto e = static_cast<uint64_t>(offsets->array[1].number);
    if (b > e || data_start + e > size) fail(CE4B_ERR_IO, "tensor " + name + " has invalid offsets");
    t.data = file.storage.data() + data_start + b;
    t.bytes = e - b;
    file.tensors.emplace(name, std::move(t));
  }
  return file;
}

}  // namespace ce4b
