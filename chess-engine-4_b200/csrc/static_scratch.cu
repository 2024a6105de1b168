// Dense-block forward for callers that must not allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc at the point where they run a block:
// an engine thread inside a memory-pool-managed process whose allocator is frozen after
// start-up, code running under a capture or a real-time budget that forbids allocation,
// or plugins that are handed only input and output buffers. ce4b_dense_block_forward
// needs scratch (the normalised rows and the SwiGLU hidden rows), which its caller
// allocates. This variant keeps that scratch in a file-scope __device__ array of fixed
// size instead, so the call allocates nothing.
//
// The array is part of the library's device image: every GPU on which the library is
// loaded holds kStaticScratchBytes for the life of the process. With CUDA's lazy module
// loading (the default of recent toolkits) the image is loaded, and the 8 MiB reserved,
// on the first call on each device: a host whose allocator freezes after start-up should
// make one call per device during start-up. All calls on a device
// share it and it keeps the previous call's contents; the block writes every scratch
// element it reads before reading it, so nothing needs clearing. Calls whose GPU work
// overlaps (different streams, or different host threads on one device) race on the
// array and must be serialised by the caller.
#include <atomic>
#include <mutex>

#include "internal.h"

namespace ce4b {

namespace {

// 8 MiB: enough for rows * (d_model + hidden_dim) * 2 bytes (each part rounded up to
// 128 rows and 256 bytes), e.g. 2048 rows at d_model 512 / hidden 1536.
constexpr int64_t kStaticScratchBytes = int64_t{8} << 20;

__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::atomic<void*> g_scratch_address[kMaxDevices];
std::mutex g_scratch_mu;

// Device address of g_static_scratch on the current device. The name of a __device__
// array in host code is a host-side stand-in, so the address is looked up once per
// device (with that device current) and cached. The first call on a device does this
// lookup, which also loads the library's device image there (reserving the array); it
// should come during the host's start-up, before any stream capture.
void* scratch_address() {
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  require(dev >= 0 && dev < kMaxDevices, "device ordinal out of range");
  void* p = g_scratch_address[dev].load(std::memory_order_acquire);
  if (p != nullptr) return p;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  p = g_scratch_address[dev].load(std::memory_order_relaxed);
  if (p == nullptr) {
    check_cuda(cudaGetSymbolAddress(&p, g_static_scratch), "cudaGetSymbolAddress(static scratch)");
    g_scratch_address[dev].store(p, std::memory_order_release);
  }
  return p;
}

int64_t round256(int64_t v) { return (v + 255) / 256 * 256; }

}  // namespace

}  // namespace ce4b

using namespace ce4b;

extern "C" int ce4b_dense_block_forward_static(const void* x_dev, const void* norm_weight_dev,
                                               const void* gate_up_weight_dev,
                                               const void* down_weight_dev, void* out_dev,
                                               int rows, int d_model, int hidden_dim, float eps,
                                               int precision, void* stream) {
  try {
    require(x_dev && norm_weight_dev && gate_up_weight_dev && down_weight_dev && out_dev,
            "null pointer");
    require(rows >= 1, "rows must be positive");
    require(d_model >= 64 && d_model % 64 == 0, "d_model must be a multiple of 64");
    require(hidden_dim >= 64 && hidden_dim % 64 == 0, "hidden_dim must be a multiple of 64");
    if (precision != CE4B_PRECISION_BF16) {
      fail(CE4B_ERR_UNSUPPORTED, "dense block: only BF16 precision is available");
    }
    const int64_t r = (static_cast<int64_t>(rows) + 127) / 128 * 128;
    const int64_t norm_bytes = round256(r * d_model * 2);
    const int64_t need = norm_bytes + round256(r * hidden_dim * 2);
    if (need > kStaticScratchBytes) {
      fail(CE4B_ERR_INVALID_ARGUMENT,
           "dense block needs " + std::to_string(need) + " scratch bytes; the static scratch "
           "holds " + std::to_string(kStaticScratchBytes) + " (use ce4b_dense_block_forward)");
    }
    auto* base = static_cast<uint8_t*>(scratch_address());
    auto* normalized = reinterpret_cast<bf16*>(base);
    auto* hidden = reinterpret_cast<bf16*>(base + norm_bytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
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
