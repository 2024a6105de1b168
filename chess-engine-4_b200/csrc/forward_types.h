// Types shared by the persistent dense forward kernel (forward.cuh) and its host side.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

namespace ce4b {

constexpr int kFwdKBlock = 64;  // BF16 k-block (one 128-byte swizzle span)
constexpr int kFwdMaxDepth = 32;
constexpr int kFwdMaxSlices = 8;  // d / 128 <= 8 (d <= 1024)
constexpr int kFwdNStage = 4;
constexpr int kFwdTaskRing = 4;
constexpr int kFwdG = 4;
// warp 0 TMA producer, warp 1 MMA issuer, 16 epilogue warps, then one store warp
constexpr int kFwdEpiThreads = 128 * kFwdG;
constexpr int kFwdStoreWarp = 2 + 4 * kFwdG;
constexpr int kFwdThreads = 64 + kFwdEpiThreads + 32;
constexpr int kErrTimeoutDependency = 7;

enum FwdTaskType : int { kTaskEnd = -1, kTaskInput = 0, kTaskGateUp = 1, kTaskDown = 2, kTaskHeads = 3 };

// Tensor maps in global memory (64-byte aligned), written once by the host.
struct FwdMaps {
  CUtensorMap a_in;    // expanded planes [rows, in_dim], box 64 x 128
  CUtensorMap x;       // residual stream [rows, d], box 64 x 128 (A of the gate_up tiles)
  CUtensorMap hidden;  // [rows, h], box 64 x 128
  CUtensorMap w_in;    // input.weight [d, in_dim], box 64 x 128
  CUtensorMap gate_up[kFwdMaxDepth];  // bf16(gate_up.weight * norm.weight) [2h, d], box 64 x 128
  CUtensorMap down[kFwdMaxDepth];     // [d, h], box 64 x 128
  // 64-byte-swizzled maps (box 32 x 128) of hidden and down.weight: the second box of a
  // 96-deep down-tile stage.
  CUtensorMap hidden32;
  CUtensorMap down32[kFwdMaxDepth];
  // bf16(final_norm.weight * [policy.weight | wdl.weight | moves_left.weight]) rows
  // [head_cols, d], box 64 x 128.
  CUtensorMap heads;
};

// 128-column down tiles move K in steps of 96 when h allows: a 48 KB ring stage holds A
// and B as a 64-wide (128-byte swizzle) and a 32-wide (64-byte swizzle) box each, so each
// wait for a stage feeds 6 MMAs instead of 4. (A stage costs the MMA thread a roughly fixed
// ~520 cycles when its MMAs take less, so 128-column MMAs run at half rate with 4 per stage.)
constexpr int kFwdDownStep = 96;
constexpr uint32_t kFwdD96A1 = 16384;  // stage offsets: A 64-wide @0, A 32-wide, B 64-wide, B 32-wide
constexpr uint32_t kFwdD96B0 = 24576;
constexpr uint32_t kFwdD96B1 = 40960;

struct FwdParams {
  const FwdMaps* maps;
  const __nv_bfloat16* bias;  // input.bias [d]
  __nv_bfloat16* x;           // [rows_cap, d]
  __nv_bfloat16* hidden;      // [rows_cap, h]
  float* ss;                  // [rows_cap, sj * kFwdG] partial sums of squares of x
  float* part;                // FP32 partial sums of the K parts of input (and down) tiles
  int* hid_cnt;               // [nb] finished gate_up tiles
  int* slice_cnt;             // [nb] finished 128-column x slices
  int* part_cnt;              // [nb * xti] K parts of each input tile that finished
  int* dpart_cnt;             // [nb * xt] K parts of each down tile that finished (dks a layer)
  int* task_counter;          // [1]
  int* err;
  // Heads (the tasks after the last layer): [policy | wdl | moves-left] logits of each row
  // block, 256 head columns a task.
  const __nv_bfloat16* head_bias;  // [head_cols] (policy, wdl, moves-left biases back to back)
  float* policy;                   // [batch, policy_size]
  float* wdl;                      // [batch, 3] probabilities (wdl_probs) or logits
  float* moves_left;               // [batch]
  int batch;
  int policy_size;                 // 1858
  int policy_storage;              // 1888: first wdl column; moves-left at policy_storage + 32
  int head_cols;                   // policy_storage + 64
  int nht;                         // head tasks per row block (head_cols / 256, rounded up)
  int wdl_probs;
  int rows_cap;
  int nb;      // row blocks of 128
  int d, h, depth;
  int sj;      // d / 128 column slices (the granularity of slice_cnt and ss)
  int nc;      // h / 128 hidden chunks
  int xw;      // column width of the down tiles (128 or 256, per forward)
  int xt;      // d / xw down tiles per row block
  int xwi;     // column width of the input tiles (256 where d allows, else 128)
  int xti;     // d / xwi input tiles per row block
  int kis;     // K parts of an input tile: 2, or 8 for batches that leave most SMs idle
  int dks;     // K parts of a down tile: 1, or 4 for batches that leave most SMs idle
  int part_rb_chunks;  // 64 KB partial-sum chunks per row block: (d / 128) * max(kis, dks)
  int kb_in;   // k-blocks of the input GEMM (in_dim / 64)
  int d96;     // 1: 128-column down tiles use 96-deep stages (h % 96 == 0)
  int lag;     // 1..nb: a layer's down tiles of row block i follow its gate_up tiles of i + lag
  int total_tasks;
  float eps;
  // Optional per-task timeline (nullptr: off): kFwdTraceWords u64 per task id < trace_cap,
  // %globaltimer ns of {0 fetched, 1 dependencies met, 2 last load issued, 3 first MMA
  // issued, 4 accumulator committed, 5 epilogue started, 6 epilogue done, 7 epilogue
  // results staged, 8 results published, 9 store warp took the staged tile, 11 its stores
  // completed}, and the CTA index in word 10.
  unsigned long long* trace;
  int trace_cap;
};

constexpr int kFwdTraceWords = 12;

}  // namespace ce4b
