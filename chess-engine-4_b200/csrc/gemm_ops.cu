// Host launchers for the tcgen05 GEMM instantiations used by the forward path, plus the
// TMA tensor-map helper.
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>
#include <set>
#include <utility>

#include "forward.cuh"
#include "gemm.cuh"
#include "internal.h"

namespace ce4b {

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  if (fn == nullptr) fail(CE4B_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  return fn;
}

// Opt each kernel instantiation into the dynamic shared memory it needs, once per device.
template <class K>
void ensure_smem(K kernel, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> done;
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  const auto key = std::make_pair(dev, reinterpret_cast<const void*>(kernel));
  std::lock_guard<std::mutex> lock(mu);
  if (done.count(key)) return;
  check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
             "cudaFuncSetAttribute(max dynamic smem)");
  done.insert(key);
}

// Clusters of `cluster` CTAs of `kernel` that fit on the device at once (cached).
template <class K>
int max_active_clusters(K kernel, int threads, int smem, int cluster) {
  static std::mutex mu;
  static std::map<std::tuple<int, const void*, int>, int> cache;
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  const auto key = std::make_tuple(dev, reinterpret_cast<const void*>(kernel), cluster);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(cluster), 1, 1);
  cfg.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  check_cuda(cudaOccupancyMaxActiveClusters(&n, kernel, &cfg), "cudaOccupancyMaxActiveClusters");
  require(n >= 1, "no cluster of " + std::to_string(cluster) + " CTAs fits on this device");
  cache.emplace(key, n);
  return n;
}

template <class K, class... Args>
void launch(K kernel, dim3 grid, int threads, int smem, int cluster_x, cudaStream_t s,
            Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = s;
  // Every GEMM kernel waits for its predecessor (grid_dependency_wait) before touching
  // global memory, so it may be launched programmatically: its CTAs take SMs as the
  // previous kernel's CTAs leave and run their prologue under that kernel's tail.
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  unsigned n_attr = 1;
  if (cluster_x > 0) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(cluster_x);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    n_attr = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n_attr;
  check_cuda(cudaLaunchKernelEx(&cfg, kernel, args...), "gemm launch");
}

int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Epilogue column groups per TMEM lane quarter (4 * kG epilogue warps per CTA).
constexpr int kG = 4;

// Placeholder for unused tensor-map arguments.
const CUtensorMap& null_map() {
  static const CUtensorMap m{};
  return m;
}

}  // namespace

namespace {
CUtensorMap encode_bf16(const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                        uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  require(ptr != nullptr, "tensor map: null pointer");
  require((reinterpret_cast<uintptr_t>(ptr) & 15u) == 0, "tensor map: base not 16-byte aligned");
  require((ld_elems * 2) % 16 == 0, "tensor map: row stride not a multiple of 16 bytes");
  require(rows >= 1 && cols >= 1 && box_rows >= 1 && box_rows <= 256, "tensor map: bad extent");
  CUtensorMap map;
  const cuuint64_t gdim[2] = {cols, rows};
  const cuuint64_t gstride[1] = {ld_elems * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr),
                                 gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(CE4B_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
  return map;
}
}  // namespace

CUtensorMap make_tmap_bf16_sw64(const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                                uint32_t box_rows) {
  return encode_bf16(ptr, rows, cols, ld_elems, 32, box_rows, CU_TENSOR_MAP_SWIZZLE_64B);
}

CUtensorMap make_tmap_bf16(const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                           uint32_t box_rows) {
  require(ptr != nullptr, "tensor map: null pointer");
  require((reinterpret_cast<uintptr_t>(ptr) & 15u) == 0, "tensor map: base not 16-byte aligned");
  require((ld_elems * 2) % 16 == 0, "tensor map: row stride not a multiple of 16 bytes");
  require(rows >= 1 && cols >= 1 && box_rows >= 1 && box_rows <= 256, "tensor map: bad extent");
  CUtensorMap map;
  const cuuint64_t gdim[2] = {cols, rows};
  const cuuint64_t gstride[1] = {ld_elems * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), box_rows};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr),
                                 gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                 CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(CE4B_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
  return map;
}

CUtensorMap make_tmap_u8(const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld_bytes,
                         uint32_t box_rows) {
  require(ptr != nullptr, "tensor map: null pointer");
  require((reinterpret_cast<uintptr_t>(ptr) & 15u) == 0, "tensor map: base not 16-byte aligned");
  require(ld_bytes % 16 == 0, "tensor map: row stride not a multiple of 16 bytes");
  require(rows >= 1 && cols >= 1 && box_rows >= 1 && box_rows <= 256, "tensor map: bad extent");
  CUtensorMap map;
  const cuuint64_t gdim[2] = {cols, rows};
  const cuuint64_t gstride[1] = {ld_bytes};
  const cuuint32_t box[2] = {128, box_rows};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr),
                                 gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                 CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(CE4B_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
  return map;
}

// ------------------------------------------------------------------ MXFP8 GEMMs
void gemm_mx_store_bf16(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tC,
                        const uint8_t* sfa, const uint8_t* sfb, int m, int n, int k,
                        cudaStream_t s) {
  require(m % 128 == 0 && n % 128 == 0 && k % 128 == 0,
          "MXFP8 GEMM extents must be multiples of 128");
  constexpr int BN = 128, NS = 5, NA = 2;
  using Epi = EpiStoreBF16<BN>;
  auto kernel = gemm_mx_kernel<BN, NS, NA, 1, kG, false, DenseSched, Epi>;
  constexpr int smem = GemmMxSmem<BN, NS, NA, Epi>::kBytes;
  ensure_smem(kernel, smem);
  DenseSched sched{m, n / BN, (m / kBM) * (n / BN), BN, 0};
  typename Epi::Params ep{n};
  const MxScales sf{sfa, sfb, k / 128};
  const int grid = std::min(sched.num_tiles, sm_count());
  launch(kernel, dim3(grid), gemm_threads(kG), smem, 0, s, tA, tB, tC, null_map(), sched, ep, sf,
         k / 128, device_error_word());
}

void gemm_mx_swiglu(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tH,
                    const uint8_t* sfa, const uint8_t* sfb, uint8_t* h_scales, int m,
                    int hidden_dim, int k, cudaStream_t s, bf16* tap) {
  require(hidden_dim % 128 == 0 && k % 128 == 0, "MXFP8 SwiGLU needs multiples of 128");
  using Epi = EpiSwiGLU<128, true>;
  const int chunks = hidden_dim / 128;
  DenseSched sched{m, chunks, ceil_div(m, kBM) * chunks, 128, hidden_dim};
  typename Epi::Params ep{h_scales, chunks, tap};
  const MxScales sf{sfa, sfb, k / 128};
  constexpr int kStatKb = 4;
  if (k / 128 <= kStatKb && chunks <= sm_count() && sched.num_tiles >= sm_count()) {
    // Short K: each CTA keeps one chunk's gate/up codes resident and streams A only. The
    // grid is a multiple of the chunk count so that a CTA's chunk is fixed.
    constexpr int NS = 4;
    auto kernel = gemm_mx_bstat_kernel<kStatKb, NS, kG, Epi>;
    constexpr int smem = GemmMxBStatSmem<kStatKb, NS, Epi>::kBytes;
    ensure_smem(kernel, smem);
    const int grid = (sm_count() / chunks) * chunks;
    launch(kernel, dim3(grid), gemm_threads(kG), smem, 0, s, tA, tB, tH, sched, ep, sf, k / 128,
           device_error_word());
    return;
  }
  constexpr int BN = 256, NS = 4, NA = 1;
  auto kernel = gemm_mx_kernel<BN, NS, NA, 2, kG, false, DenseSched, Epi>;
  constexpr int smem = GemmMxSmem<BN, NS, NA, Epi>::kBytes;
  ensure_smem(kernel, smem);
  const int grid = std::min(sched.num_tiles, sm_count());
  launch(kernel, dim3(grid), gemm_threads(kG), smem, 0, s, tA, tB, tH, null_map(), sched, ep, sf,
         k / 128, device_error_word());
}

void gemm_mx_resnorm(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tX,
                     const CUtensorMap& tN, const uint8_t* sfa, const uint8_t* sfb,
                     uint8_t* n_scales, const bf16* bias, const bf16* norm_w, int m, int d, int k,
                     float eps, cudaStream_t s, bf16* tap) {
  require(d % 128 == 0 && k % 128 == 0 && (d / 128 <= kMaxClusterN || (d % 256 == 0 && d / 256 <= kMaxClusterN)),
          "MXFP8 residual GEMM needs d a multiple of 128 up to 1024 (of 256 up to 2048) and K a multiple of 128");
  if (d > 1024) {
    // d / 256 CTAs per row (up to 8): the x tile moves into the stage ring after the main
    // loop, which leaves room for four operand stages beside the cluster's receive buffer.
    constexpr int BN = 256, NS = 4, NA = 1;
    using Epi = EpiResNorm<BN, true, kMaxClusterN, true>;
    auto kernel = gemm_mx_kernel<BN, NS, NA, 2, kG, true, DenseSched, Epi>;
    constexpr int smem = GemmMxSmem<BN, NS, NA, Epi>::kBytes;
    static_assert(GemmMxSmem<BN, NS, NA, Epi>::kRingBytes >= Epi::kXBytes + kBM * BN,
                  "the ring must hold the x tile and the n codes");
    ensure_smem(kernel, smem);
    const int cn = d / BN;
    DenseSched sched{m, cn, ceil_div(m, kBM) * cn, BN, 128};
    typename Epi::Params ep{bias, norm_w, d, bias != nullptr ? Epi::kBias : Epi::kResidual,
                            cn,   eps,    n_scales, tap};
    const MxScales sf{sfa, sfb, k / 128};
    launch(kernel, dim3(sched.num_tiles), gemm_threads(kG), smem, cn, s, tA, tB, tX, tN, sched, ep,
           sf, k / 128, device_error_word());
    return;
  }
  if (d % 256 == 0 && d / 256 <= 4) {
    // 128 x 256 tiles (B as two 128-row boxes): a 256-column MMA keeps the tensor core busy
    // per ring stage where a 128-column one runs at half rate, and half as many CTAs.
    constexpr int BN = 256, NS = 3, NA = 1;
    using Epi = EpiResNorm<BN, true, 4>;
    auto kernel = gemm_mx_kernel<BN, NS, NA, 2, kG, true, DenseSched, Epi>;
    constexpr int smem = GemmMxSmem<BN, NS, NA, Epi>::kBytes;
    ensure_smem(kernel, smem);
    const int cn = d / BN;
    DenseSched sched{m, cn, ceil_div(m, kBM) * cn, BN, 128};
    typename Epi::Params ep{bias, norm_w, d, bias != nullptr ? Epi::kBias : Epi::kResidual,
                            cn,   eps,    n_scales, tap};
    const MxScales sf{sfa, sfb, k / 128};
    launch(kernel, dim3(sched.num_tiles), gemm_threads(kG), smem, cn, s, tA, tB, tX, tN, sched, ep,
           sf, k / 128, device_error_word());
    return;
  }
  constexpr int BN = 128, NS = 5, NA = 1;
  using Epi = EpiResNorm<BN, true>;
  auto kernel = gemm_mx_kernel<BN, NS, NA, 1, kG, true, DenseSched, Epi>;
  constexpr int smem = GemmMxSmem<BN, NS, NA, Epi>::kBytes;
  ensure_smem(kernel, smem);
  const int cn = d / BN;
  DenseSched sched{m, cn, ceil_div(m, kBM) * cn, BN, 0};
  typename Epi::Params ep{bias, norm_w, d, bias != nullptr ? Epi::kBias : Epi::kResidual,
                          cn,   eps,    n_scales, tap};
  const MxScales sf{sfa, sfb, k / 128};
  launch(kernel, dim3(sched.num_tiles), gemm_threads(kG), smem, cn, s, tA, tB, tX, tN, sched, ep,
         sf, k / 128, device_error_word());
}

void gemm_mx_heads(const CUtensorMap& tA, const CUtensorMap& tB, const uint8_t* sfa,
                   const uint8_t* sfb, const bf16* bias, float* policy, float* wdl,
                   float* moves_left, int m, int d, int policy_size, int policy_storage,
                   int wdl_probs, cudaStream_t s) {
  constexpr int BN = 256, NS = 3, NA = 1;
  using Epi = EpiHeads;
  auto kernel = gemm_mx_kernel<BN, NS, NA, 1, kG, false, DenseSched, Epi>;
  constexpr int smem = GemmMxSmem<BN, NS, NA, Epi>::kBytes;
  ensure_smem(kernel, smem);
  const int n_total = policy_storage + 64;
  DenseSched sched{m, ceil_div(n_total, BN), ceil_div(m, kBM) * ceil_div(n_total, BN), BN, 0};
  typename Epi::Params ep{bias, policy, wdl, moves_left, policy_size, policy_storage, n_total,
                          wdl_probs};
  const MxScales sf{sfa, sfb, d / 128};
  const int grid = std::min(sched.num_tiles, sm_count());
  launch(kernel, dim3(grid), gemm_threads(kG), smem, 0, s, tA, tB, null_map(), null_map(), sched,
         ep, sf, d / 128, device_error_word());
}

// ------------------------------------------------------------------ plain store
void gemm_store_bf16(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tC, int m,
                     int n, int k, cudaStream_t s) {
  constexpr int BN = 128, NS = 6, NA = 2;
  using Epi = EpiStoreBF16<BN>;
  auto kernel = gemm_tc_kernel<BN, NS, NA, 1, kG, false, DenseSched, Epi>;
  constexpr int smem = GemmSmem<BN, NS, NA, Epi>::kBytes;
  ensure_smem(kernel, smem);
  DenseSched sched{m, ceil_div(n, BN), ceil_div(m, kBM) * ceil_div(n, BN), BN, 0};
  typename Epi::Params ep{n};
  const int grid = std::min(sched.num_tiles, sm_count());
  launch(kernel, dim3(grid), gemm_threads(kG), smem, 0, s, tA, tB, tC, null_map(), sched, ep,
         ceil_div(k, kBK), device_error_word());
}

// ------------------------------------------------------------------ SwiGLU
int swiglu_chunk(int hidden) { return hidden % 128 == 0 ? 128 : 64; }

void gemm_swiglu(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tH, int m,
                 int hidden_dim, int k, cudaStream_t s) {
  const int hc = swiglu_chunk(hidden_dim);
  require(hidden_dim % hc == 0, "SwiGLU hidden dim must be a multiple of 64");
  DenseSched sched{m, hidden_dim / hc, ceil_div(m, kBM) * (hidden_dim / hc), hc, hidden_dim};
  const int grid = std::min(sched.num_tiles, sm_count());
  if (hc == 128) {
    // Single-CTA tiles: measured as fast as CTA pairs here (the per-tile MMA rate is the
    // same; the kernel's span is set by its prologue, first loads and last epilogue).
    constexpr int BN = 256, NS = 4, NA = 2;
    using Epi = EpiSwiGLU<128>;
    auto kernel = gemm_tc_kernel<BN, NS, NA, 2, kG, false, DenseSched, Epi>;
    constexpr int smem = GemmSmem<BN, NS, NA, Epi>::kBytes;
    ensure_smem(kernel, smem);
    typename Epi::Params ep{0};
    launch(kernel, dim3(grid), gemm_threads(kG), smem, 0, s, tA, tB, tH, null_map(), sched, ep,
           ceil_div(k, kBK), device_error_word());
  } else {
    constexpr int BN = 128, NS = 6, NA = 2;
    using Epi = EpiSwiGLU<64>;
    auto kernel = gemm_tc_kernel<BN, NS, NA, 2, kG, false, DenseSched, Epi>;
    constexpr int smem = GemmSmem<BN, NS, NA, Epi>::kBytes;
    ensure_smem(kernel, smem);
    typename Epi::Params ep{0};
    launch(kernel, dim3(grid), gemm_threads(kG), smem, 0, s, tA, tB, tH, null_map(), sched, ep,
           ceil_div(k, kBK), device_error_word());
  }
}

// ------------------------------------------------------------------ residual + RMSNorm
int resnorm_bn(int d) {
  if (d % 128 == 0 && d / 128 <= kMaxClusterN) return 128;
  if (d % 256 == 0 && d / 256 <= kMaxClusterN) return 256;
  if (d % 64 == 0 && d / 64 <= kMaxClusterN) return 64;
  fail(CE4B_ERR_UNSUPPORTED, "d_model " + std::to_string(d) +
                                 " is not supported (multiple of 64, at most 2048)");
}

// CTA pairs with 256-column slices for the wide models (768, 1024: clusters of 6 and 8).
// Narrower models keep single-CTA 128-column slices: the MMA rate per SM is set by the
// slice width N (about 50 % of peak at N = 128, 68-71 % at N = 256, single CTA or pair
// alike), and at d <= 512 a cluster of 2 * d / 128 CTAs would not all fit at once (15
// clusters of 8 are resident at this shared-memory size) while 4-CTA clusters do.
int resnorm_pair_bn(int d) {
  if (d % 256 == 0 && d >= 768 && d / 256 <= 4) return 256;
  return 0;
}

int resnorm_b_box(int d) {
  const int pair_bn = resnorm_pair_bn(d);
  return pair_bn != 0 ? pair_bn / 2 : resnorm_bn(d);
}

// CTA pairs: a cluster of 2 * cn CTAs covers 256 rows across the full width d; pair j
// (ranks 2j, 2j+1) owns column slice j, each CTA 128 rows of it. One tile per CTA.
template <int BN, int NS>
static void gemm_resnorm_pair(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tX,
                              const CUtensorMap& tN, const bf16* bias, const bf16* norm_w, int m,
                              int d, int k, float eps, cudaStream_t s) {
  using Epi = EpiResNorm<BN>;
  auto kernel = gemm_pair_kernel<BN, NS, 1, kG, 4, Epi>;
  constexpr int smem = GemmPairSmem<BN, NS, 1, Epi>::kBytes;
  ensure_smem(kernel, smem);
  const int cn = d / BN;
  DensePairSched ps{m, cn, ceil_div(m, 2 * kBM) * cn, BN, BN / 2, 0};
  typename Epi::Params ep{bias, norm_w, d, bias != nullptr ? Epi::kBias : Epi::kResidual, cn, eps};
  launch(kernel, dim3(2 * ps.num_tiles), gemm_threads(kG), smem, 2 * cn, s, tA, tB, tX, tN, ps,
         ep, ceil_div(k, kBK), device_error_word());
}

template <int BN, int NS>
static void gemm_resnorm_bn(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tX,
                            const CUtensorMap& tN, const bf16* bias, const bf16* norm_w, int m,
                            int d, int k, float eps, cudaStream_t s) {
  using Epi = EpiResNorm<BN>;
  auto kernel = gemm_tc_kernel<BN, NS, 1, 1, kG, true, DenseSched, Epi>;
  constexpr int smem = GemmSmem<BN, NS, 1, Epi>::kBytes;
  ensure_smem(kernel, smem);
  const int cn = d / BN;
  DenseSched sched{m, cn, ceil_div(m, kBM) * cn, BN, 0};
  typename Epi::Params ep{bias, norm_w, d, bias != nullptr ? Epi::kBias : Epi::kResidual, cn, eps};
  // One tile per CTA: the cluster's CTAs cover one 128-row block across the full width.
  launch(kernel, dim3(sched.num_tiles), gemm_threads(kG), smem, cn, s, tA, tB, tX, tN, sched, ep,
         ceil_div(k, kBK), device_error_word());
}

void gemm_resnorm(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tX,
                  const CUtensorMap& tN, const bf16* bias, const bf16* norm_w, int m, int d, int k,
                  float eps, cudaStream_t s) {
  if (resnorm_pair_bn(d) == 256) {
    gemm_resnorm_pair<256, 4>(tA, tB, tX, tN, bias, norm_w, m, d, k, eps, s);
    return;
  }
  switch (resnorm_bn(d)) {
    case 64: gemm_resnorm_bn<64, 7>(tA, tB, tX, tN, bias, norm_w, m, d, k, eps, s); break;
    case 128: gemm_resnorm_bn<128, 5>(tA, tB, tX, tN, bias, norm_w, m, d, k, eps, s); break;
    default: gemm_resnorm_bn<256, 3>(tA, tB, tX, tN, bias, norm_w, m, d, k, eps, s); break;
  }
}

// ------------------------------------------------------------------ persistent dense forward
void dense_forward(const FwdParams& p, cudaStream_t s) {
  require(p.total_tasks >= 1 && p.depth >= 1 && p.depth <= kFwdMaxDepth && p.kb_in >= 1 &&
              p.d % 128 == 0 && p.d / 128 <= kFwdMaxSlices && p.h % 128 == 0 &&
              (p.xw == 128 || p.xw == 256) && p.d % p.xw == 0 && p.xt == p.d / p.xw &&
              (p.xwi == 128 || p.xwi == 256) && p.d % p.xwi == 0 && p.xti == p.d / p.xwi &&
              p.kis >= 2 && p.kis <= 8 && p.kb_in >= p.kis && p.dks >= 1 && p.dks <= 4 &&
              (p.dks == 1 || (p.xw == 128 && (p.h / kFwdKBlock) % p.dks == 0)) &&
              p.part_rb_chunks == (p.d / 128) * std::max(p.kis, p.dks) && p.batch >= 1 &&
              p.batch <= p.nb * 128 && p.policy != nullptr && p.wdl != nullptr &&
              p.moves_left != nullptr && p.head_bias != nullptr && p.policy_size <= p.policy_storage &&
              p.policy_storage % 32 == 0 && p.head_cols == p.policy_storage + 64 &&
              p.nht == (p.head_cols + 255) / 256 && p.lag >= 1 && p.lag <= p.nb,
          "persistent forward: unsupported shape");
  auto kernel = dense_forward_kernel;
  ensure_smem(kernel, FwdSmem::kBytes);
  const int grid = std::min(sm_count(), p.total_tasks);
  launch(kernel, dim3(grid), kFwdThreads, FwdSmem::kBytes, 0, s, p);
}

// ------------------------------------------------------------------ heads
void gemm_heads(const CUtensorMap& tA, const CUtensorMap& tB, const bf16* bias, float* policy,
                float* wdl, float* moves_left, int m, int d, int policy_size, int policy_storage,
                int wdl_probs, cudaStream_t s) {
  constexpr int BN = 256, NS = 3, NA = 2;
  using Epi = EpiHeads;
  auto kernel = gemm_tc_kernel<BN, NS, NA, 1, kG, false, DenseSched, Epi>;
  constexpr int smem = GemmSmem<BN, NS, NA, Epi>::kBytes;
  ensure_smem(kernel, smem);
  const int n_total = policy_storage + 64;
  DenseSched sched{m, ceil_div(n_total, BN), ceil_div(m, kBM) * ceil_div(n_total, BN), BN, 0};
  typename Epi::Params ep{bias, policy, wdl, moves_left, policy_size, policy_storage, n_total,
                          wdl_probs};
  const int grid = std::min(sched.num_tiles, sm_count());
  launch(kernel, dim3(grid), gemm_threads(kG), smem, 0, s, tA, tB, null_map(), null_map(), sched,
         ep, ceil_div(d, kBK), device_error_word());
}

// ------------------------------------------------------------------ MoE GEMMs
void moe_router_gemm(const CUtensorMap& tA, const CUtensorMap& tB, const float* beta,
                     int2* route_expert, float2* route_prob, int* block_hist, int tokens, int d,
                     cudaStream_t s, bf16* logits_out) {
  constexpr int BN = 64, NS = 8, NA = 1;
  using Epi = EpiRouter;
  auto kernel = gemm_tc_kernel<BN, NS, NA, 1, kG, false, DenseSched, Epi>;
  constexpr int smem = GemmSmem<BN, NS, NA, Epi>::kBytes;
  ensure_smem(kernel, smem);
  DenseSched sched{tokens, 1, ceil_div(tokens, kBM), BN, 0};
  typename Epi::Params ep{beta, route_expert, route_prob, block_hist, logits_out};
  // One tile (128 tokens) per CTA: block_hist row = tile index.
  launch(kernel, dim3(sched.num_tiles), gemm_threads(kG), smem, 0, s, tA, tB, null_map(),
         null_map(), sched, ep, ceil_div(d, kBK), device_error_word());
}

void gemm_grouped_swiglu(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tH,
                         const int4* m_tiles, const int* num_m_tiles, int hidden, int k,
                         cudaStream_t s) {
  const int hc = swiglu_chunk(hidden);
  require(hidden % hc == 0, "expert hidden dim must be a multiple of 64");
  GroupedSched sched{m_tiles, num_m_tiles, hidden / hc, hc, 2 * hidden, hidden};
  const int grid = sm_count();
  if (hc == 128) {
    constexpr int BN = 256, NS = 4, NA = 2;
    using Epi = EpiSwiGLU<128>;
    auto kernel = gemm_tc_kernel<BN, NS, NA, 2, kG, false, GroupedSched, Epi>;
    constexpr int smem = GemmSmem<BN, NS, NA, Epi>::kBytes;
    ensure_smem(kernel, smem);
    typename Epi::Params ep{0};
    launch(kernel, dim3(grid), gemm_threads(kG), smem, 0, s, tA, tB, tH, null_map(), sched, ep,
           ceil_div(k, kBK), device_error_word());
  } else {
    constexpr int BN = 128, NS = 6, NA = 2;
    using Epi = EpiSwiGLU<64>;
    auto kernel = gemm_tc_kernel<BN, NS, NA, 2, kG, false, GroupedSched, Epi>;
    constexpr int smem = GemmSmem<BN, NS, NA, Epi>::kBytes;
    ensure_smem(kernel, smem);
    typename Epi::Params ep{0};
    launch(kernel, dim3(grid), gemm_threads(kG), smem, 0, s, tA, tB, tH, null_map(), sched, ep,
           ceil_div(k, kBK), device_error_word());
  }
}

int grouped_bn(int n) {
  if (n % 256 == 0) return 256;
  if (n % 128 == 0) return 128;
  require(n % 64 == 0, "expert output width must be a multiple of 64");
  return 64;
}

template <int BN, int NS>
static void gemm_grouped_scale_bn(const CUtensorMap& tA, const CUtensorMap& tB,
                                  const CUtensorMap& tY, const int4* m_tiles,
                                  const int* num_m_tiles, const float* row_scale, int n, int k,
                                  cudaStream_t s) {
  using Epi = EpiScaleStore<BN>;
  auto kernel = gemm_tc_kernel<BN, NS, 2, 1, kG, false, GroupedSched, Epi>;
  constexpr int smem = GemmSmem<BN, NS, 2, Epi>::kBytes;
  ensure_smem(kernel, smem);
  GroupedSched sched{m_tiles, num_m_tiles, n / BN, BN, n, 0};
  typename Epi::Params ep{row_scale};
  launch(kernel, dim3(sm_count()), gemm_threads(kG), smem, 0, s, tA, tB, tY, null_map(), sched, ep,
         ceil_div(k, kBK), device_error_word());
}

void gemm_grouped_scale(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tY,
                        const int4* m_tiles, const int* num_m_tiles, const float* row_scale, int n,
                        int k, cudaStream_t s) {
  switch (grouped_bn(n)) {
    case 256: gemm_grouped_scale_bn<256, 4>(tA, tB, tY, m_tiles, num_m_tiles, row_scale, n, k, s); break;
    case 128: gemm_grouped_scale_bn<128, 5>(tA, tB, tY, m_tiles, num_m_tiles, row_scale, n, k, s); break;
    default: gemm_grouped_scale_bn<64, 7>(tA, tB, tY, m_tiles, num_m_tiles, row_scale, n, k, s); break;
  }
}

}  // namespace ce4b
