// Types shared by the small-batch dense forward kernel (latency.cu) and its host side.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include "forward_types.h"

namespace ce4b {

// Positions a small-batch forward takes: the batch is the N side of every MMA (N = batch
// rounded up to 16, at most 64), weights the 128-row M side.
constexpr int kLatMaxRows = 64;
constexpr int kLatMaxD = 512;
constexpr int kLatWSlotBytes = 64 * 1024;  // one of two weight slots in shared memory
constexpr int kLatMaxKbSlot = kLatWSlotBytes / (128 * 64 * 2);  // 4 k-blocks of a 128-row tile
constexpr int kLatThreads = 256;
constexpr int kLatTraceWords = 12;
constexpr int kLatGuUnits = 32;  // hidden units of a gate_up tile (32 gate + 32 up weight rows)

enum LatTaskType : int { kLatEnd = -1, kLatInput = 0, kLatGateUp = 1, kLatDown = 2, kLatHeads = 3 };

// Tensor maps in global memory (64-byte aligned), written once by the host. Activations
// are the MMA's B operand (box 64 columns x 64 rows), weights its A operand.
struct LatMaps {
  CUtensorMap a_in;    // expanded planes [rows, in_dim]
  CUtensorMap x;       // residual stream [rows, d]
  CUtensorMap hidden;  // [rows, h]
  CUtensorMap w_in;    // input.weight [d, in_dim], box 64 x 128
  CUtensorMap gate_up[kFwdMaxDepth];  // bf16(gate_up.weight * norm.weight) [2h, d], box 64 x 32
  CUtensorMap down[kFwdMaxDepth];     // down.weight [d, h], box 64 x 128
  // bf16(final_norm.weight * [policy | wdl | moves-left].weight) [head_cols, d], box 64 x 128
  CUtensorMap heads;
};

struct LatParams {
  const LatMaps* maps;
  const int4* tasks;  // [grid][max_tasks] {type, layer, tile, part}; type -1 ends a list
  int max_tasks;
  const __nv_bfloat16* in_bias;              // input.bias [d]
  const __nv_bfloat16* head_bias;            // [head_cols]
  __nv_bfloat16* x;       // [rows_cap, d]
  __nv_bfloat16* hidden;  // [rows_cap, h]
  float* part_in;         // [d / 128][kp_in][n][128] FP32 partial sums of the input GEMM
  float* part_dn;         // [d / 128][kp_dn][n][128] of each layer's down GEMM
  int* cnt;               // [0] x slices ready, [1] hidden tiles ready, [2 + m] input and
                          // [2 + mt + m] down partial tiles of 128-row block m, [2 + 2 mt]
                          // CTAs finished (zero at launch; the last CTA zeroes them all)
  int* err;
  float* policy;
  float* wdl;
  float* moves_left;
  int batch;
  int n;        // MMA N: batch rounded up to 16
  int d, h, depth;
  int mt;       // d / 128
  int kb_in;    // in_dim / 64
  int kp_in;    // K parts of the input GEMM (kb_in / kp_in k-blocks each)
  int kp_dn;    // K parts of each down GEMM
  int gt;       // gate_up tiles a layer: h / kLatGuUnits
  int ht;       // head tiles: ceil(head_cols / 128)
  int policy_size, policy_storage, head_cols, wdl_probs;
  float eps;
  unsigned long long* trace;  // optional: kLatTraceWords per (CTA, task) index
  int trace_cap;
};

}  // namespace ce4b
