// Internal host-side declarations shared by the translation units of libce4b200.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

#include "../../include/ce4b200.h"

#ifdef __CUDACC__
#define CE4B_HD __host__ __device__
#else
#define CE4B_HD
#endif

namespace ce4b {

using bf16 = __nv_bfloat16;

// Error carrying a C-ABI status code; converted to a return value at the ABI edge.
struct Error : std::runtime_error {
  int status;
  Error(int s, const std::string& msg) : std::runtime_error(msg), status(s) {}
};

[[noreturn]] inline void fail(int status, const std::string& msg) { throw Error(status, msg); }

inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(CE4B_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

inline void require(bool cond, const std::string& msg) {
  if (!cond) fail(CE4B_ERR_INVALID_ARGUMENT, msg);
}

// Per-thread message of the last failed ABI call.
void set_last_error(const std::string& msg);

// Device error word shared by all kernels of the current device (bounded-wait timeouts).
int* device_error_word();

int sm_count();

// ---------------------------------------------------------------- tensor maps
// 2-D BF16 tensor map, 128-byte swizzle, box = 64 (K) x box_rows. Throws on bad alignment.
CUtensorMap make_tmap_bf16(const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                           uint32_t box_rows);
// Same with a 64-byte swizzle and box = 32 (K) x box_rows.
CUtensorMap make_tmap_bf16_sw64(const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                                uint32_t box_rows);

// ---------------------------------------------------------------- GEMM launchers
// Every map is a BF16 map from make_tmap_bf16 (box 64 columns x box_rows rows); output
// maps (tC, tH, tX, tN) use 128-row boxes and the exact row count of the output.
// C[M,N] = A[M,K] . B[N,K]^T, BF16 out, N % 16 == 0 (B box 128 rows).
void gemm_store_bf16(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tC, int m,
                     int n, int k, cudaStream_t s);
// hidden[M,h] = SwiGLU over W_gu [2h, K] (gate rows first); tB box rows must equal hc.
int swiglu_chunk(int hidden);  // 128 if hidden % 128 == 0, else 64
void gemm_swiglu(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tH, int m,
                 int hidden_dim, int k, cudaStream_t s);
// Residual/bias epilogue with optional fused RMSNorm; tB box rows must equal resnorm_b_box(d).
// tX is the residual stream x [M, d] (read for the residual mode, written), tN the
// normalised output [M, d] (used when norm_w is set).
int resnorm_bn(int d);
// Persistent dense forward (input GEMM, all layers, RMSNorm passes) in one launch.
struct FwdParams;
void dense_forward(const FwdParams& p, cudaStream_t s);
// Small-batch dense forward (latency.cu) in one cooperative launch of `grid` CTAs.
struct LatParams;
void latency_forward(const LatParams& p, int grid, cudaStream_t s);
// Rows of the tB box that gemm_resnorm expects for width d (BN, or BN/2 on CTA pairs).
int resnorm_b_box(int d);
void gemm_resnorm(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tX,
                  const CUtensorMap& tN, const bf16* bias, const bf16* norm_w, int m, int d, int k,
                  float eps, cudaStream_t s);
// Heads over the concatenated [policy | wdl | moves-left] matrix; tB box rows 256.
void gemm_heads(const CUtensorMap& tA, const CUtensorMap& tB, const bf16* bias, float* policy,
                float* wdl, float* moves_left, int m, int d, int policy_size, int policy_storage,
                int wdl_probs, cudaStream_t s);
// Per position b: probs[i] = softmax over i in [offsets[b], offsets[b+1]) of
// policy[b, indices[i]] * temperature (legal-move policy of the lc0 backend).
void policy_softmax(const float* policy, int batch, int policy_size, const int32_t* offsets,
                    const int32_t* indices, float temperature, float* probs, cudaStream_t s);
// out[r, c] = bf16(W[r, c] * w[c]) for a row-major [rows, cols] BF16 matrix.
void fold_columns(const bf16* W, const bf16* w, bf16* out, int64_t rows, int cols, cudaStream_t s);

// ---------------------------------------------------------------- MoE
// Router GEMM (A = normalised rows [T, d], B = router weight [64, d] with 64-row boxes)
// with the top-2 routing epilogue; block_hist receives [ceil(T/128)][64] counts and, when
// logits_out is set, the BF16 logits [T, 64] the selection used.
void moe_router_gemm(const CUtensorMap& tA, const CUtensorMap& tB, const float* beta,
                     int2* route_expert, float2* route_prob, int* block_hist, int tokens, int d,
                     cudaStream_t s, bf16* logits_out = nullptr);
// expert_start receives 65 entries: segment starts (each padded to 128 rows), then the
// total number of permuted rows.
void moe_scan(const int* block_hist, int ntiles, int* expert_start, int* block_off,
              int4* m_tiles, int* num_m_tiles, int* counts_out, cudaStream_t s);
void moe_dispatch(const bf16* n, const int2* route_expert, const float2* route_prob,
                  const int* expert_start, const int* block_off, bf16* xperm, float* pprob,
                  int* route_pos, int tokens, int d, cudaStream_t s);
// Grouped expert GEMMs over the device-side m-tile table. B rows per expert: 2*hidden for
// gate_up (box rows = swiglu_chunk(hidden)), n for down (box rows = grouped_bn(n)).
void gemm_grouped_swiglu(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tH,
                         const int4* m_tiles, const int* num_m_tiles, int hidden, int k,
                         cudaStream_t s);
int grouped_bn(int n);
void gemm_grouped_scale(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tY,
                        const int4* m_tiles, const int* num_m_tiles, const float* row_scale, int n,
                        int k, cudaStream_t s);
void moe_combine_norm(bf16* x, const bf16* yperm, const int* route_pos, const bf16* norm_w,
                      bf16* nout, int tokens, int d, float eps, cudaStream_t s);
void moe_tiles_from_offsets(const int* offsets, int4* m_tiles, int* num_m_tiles, cudaStream_t s);
void moe_route_logits(const bf16* logits, const float* beta, int2* experts, float2* probs,
                      int* counts, int tokens, cudaStream_t s);
void bf16_to_f32(const bf16* in, float* out, int n, cudaStream_t s);

// ---------------------------------------------------------------- MXFP8
// BF16 [rows, cols] -> E4M3 codes [rows, cols] + E8M0 scales [rows/128][cols/128][512].
void mx_quantize(const bf16* x, uint8_t* codes, uint8_t* scales, int rows, int cols,
                 cudaStream_t s);
// The same for the transpose: codes [cols, rows] + scales [cols/128][rows/128][512].
void mx_quantize_transpose(const bf16* x, uint8_t* codes, uint8_t* scales, int rows, int cols,
                           cudaStream_t s);
// 2-D byte (E4M3 code) tensor map, 128-byte swizzle, box = 128 codes x box_rows.
CUtensorMap make_tmap_u8(const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld_bytes,
                         uint32_t box_rows);
// C[M,N] BF16 = block-scaled E4M3 A[M,K] . B[N,K]^T (M, N, K multiples of 128; maps with
// 128-row boxes; C map BF16 with 128-row boxes).
void gemm_mx_store_bf16(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tC,
                        const uint8_t* sfa, const uint8_t* sfb, int m, int n, int k,
                        cudaStream_t s);
// MXFP8 forms of the forward's GEMMs (code maps from make_tmap_u8 with 128-row boxes; the
// x map of the residual GEMM stays BF16). sfa/sfb are the A/B scale tiles.
// `tap` (tests): when set, the BF16 values the epilogue quantised are also written there
// ([m, hidden_dim] / [m, d] row-major).
void gemm_mx_swiglu(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tH,
                    const uint8_t* sfa, const uint8_t* sfb, uint8_t* h_scales, int m,
                    int hidden_dim, int k, cudaStream_t s, bf16* tap = nullptr);
void gemm_mx_resnorm(const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tX,
                     const CUtensorMap& tN, const uint8_t* sfa, const uint8_t* sfb,
                     uint8_t* n_scales, const bf16* bias, const bf16* norm_w, int m, int d, int k,
                     float eps, cudaStream_t s, bf16* tap = nullptr);
void gemm_mx_heads(const CUtensorMap& tA, const CUtensorMap& tB, const uint8_t* sfa,
                   const uint8_t* sfb, const bf16* bias, float* policy, float* wdl,
                   float* moves_left, int m, int d, int policy_size, int policy_storage,
                   int wdl_probs, cudaStream_t s);
// Input planes -> MXFP8 codes [B, 64*sel] + scales (sel*64 a multiple of 128).
void expand_input_mx(int layout, const void* input, const void* scalars, int batch, int history,
                     uint8_t* codes, uint8_t* scales, int write_back_rule50, cudaStream_t s);

// ---------------------------------------------------------------- elementwise
// Expand an input batch into the BF16 GEMM operand [B, selected_planes * 64].
void expand_input(int layout, const void* input, const void* scalars, int batch, int history,
                  bf16* out, int write_back_rule50, cudaStream_t s);
void rmsnorm_rows(const bf16* x, const bf16* w, bf16* out, int rows, int width, float eps,
                  cudaStream_t s);
void swiglu_rows(const bf16* gate_up, bf16* hidden, int rows, int hidden_dim, cudaStream_t s);
void residual_add(bf16* out, const bf16* residual, int64_t elements, cudaStream_t s);

constexpr int kInputPlanes = 112;
constexpr int kHistoryPlanes = 104;
constexpr int kPlanesPerHistory = 13;
CE4B_HD inline int selected_planes(int history) {
  return history * kPlanesPerHistory + (kInputPlanes - kHistoryPlanes);
}

}  // namespace ce4b
