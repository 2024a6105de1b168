/*
 * ce4b200 — C ABI of the B200 (sm_100a) forward path for the chess-engine-4
 * position-evaluation networks (dense and moe64a2 SwiGLU towers).
 *
 * Conventions
 *  - Every entry point returns an int status (CE4B_OK == 0). No exception crosses the
 *    ABI. ce4b_last_error() returns the message of the calling thread's last failure.
 *  - Pointers named *_dev are device pointers on the handle's (or current) device;
 *    pointers named host_* are host pointers. BF16 tensors are raw uint16 storage.
 *  - `stream` is a cudaStream_t passed as void*; NULL means the legacy default stream.
 *    Work is enqueued asynchronously unless the function says it blocks.
 *  - Matrices are row-major. "A . B^T" GEMMs take B as [N, K] (the nn.Linear weight
 *    layout), K contiguous.
 *  - One model handle belongs to one GPU. Calls on one handle must be serialised by
 *    the caller; handles on different GPUs may be used concurrently.
 */
#ifndef CE4B200_H
#define CE4B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CE4B_OK 0
#define CE4B_ERR_INVALID_ARGUMENT 1
#define CE4B_ERR_CUDA 2
#define CE4B_ERR_UNSUPPORTED 3
#define CE4B_ERR_IO 4
#define CE4B_ERR_DEVICE_TIMEOUT 5
#define CE4B_ERR_NOT_READY 6

#define CE4B_ARCH_DENSE 0
#define CE4B_ARCH_MOE64A2 1

#define CE4B_PRECISION_BF16 0
#define CE4B_PRECISION_MXFP8 1

/* Input layouts accepted by ce4b_model_forward. */
#define CE4B_INPUT_F32_PLANES 0  /* float  [B, 112, 8, 8]  (PyTorch model input)            */
#define CE4B_INPUT_BF16_PLANES 1 /* bf16   [B, 112, 8, 8]                                    */
#define CE4B_INPUT_LC0 2         /* ce4b_input_plane [B, 112] (lc0 engine input)             */
#define CE4B_INPUT_PACKED_F32 3  /* uint8 [B, 104, 8] bit-packed MSB-first + float [B, 8]    */
#define CE4B_INPUT_PACKED_BF16 4 /* uint8 [B, 104, 8] bit-packed MSB-first + bf16  [B, 8]    */

#define CE4B_DTYPE_BF16 0
#define CE4B_DTYPE_F32 1

/* One lc0 input plane: square s (0..63) holds `value` if bit s of `mask` is set, else 0.
 * Replaces chess_engine_4::inference::InputPlane
 * (kernels/include/chess_engine_4/inference.h:10-13); same 16-byte size and layout. */
typedef struct ce4b_input_plane {
  uint64_t mask;
  float value;
  uint32_t reserved;
} ce4b_input_plane;

/* Model hyper-parameters; the fields of the Safetensors v1 metadata
 * (src/chess_engine_4/release/export.py:199-219) and of DenseChessNetConfig /
 * Moe64A2ChessNetConfig (src/chess_engine_4/model/dense.py:59-82, moe.py:74-102). */
typedef struct ce4b_model_config {
  int32_t arch;                /* CE4B_ARCH_*                                              */
  int32_t d_model;             /* multiple of 64, <= 2048                                  */
  int32_t depth;               /* layers; even for moe64a2                                 */
  int32_t history_length;      /* 1..8                                                     */
  float expansion_ratio;       /* dense hidden = int(d * ratio); moe: expert hidden        */
  float rms_norm_eps;          /* 1e-6 in every reference config                           */
  int32_t policy_size;         /* 1858                                                     */
  int32_t policy_storage_size; /* 1888 (rows of policy.weight)                             */
  int32_t precision;           /* CE4B_PRECISION_*                                         */
} ce4b_model_config;

typedef struct ce4b_model_info {
  int32_t d_model;
  int32_t depth;
  int32_t history_length;
  int32_t policy_size;
  int32_t maximum_batch_size;
  int32_t hidden_dim;       /* dense FFN hidden of dense layers                          */
  int32_t expert_hidden_dim; /* 0 for dense models                                       */
  int32_t arch;
  int64_t weight_bytes;
  int64_t workspace_bytes;
} ce4b_model_info;

typedef struct ce4b_model ce4b_model;

/* Message of the calling thread's last failed call ("" if none). */
const char* ce4b_last_error(void);

/* Library version string. */
const char* ce4b_version(void);

/* Reads and clears the device error word written by bounded in-kernel waits that ran
 * out (0 = no error). Blocks on `device` until prior work is done. */
int ce4b_check_device_error(int device, int* code_out);

/* ------------------------------------------------------------------ model handle
 * Replaces chess_engine_4::inference::Model (kernels/include/chess_engine_4/inference.h:29-51,
 * kernels/src/inference/runtime.cu:340-787) and the custom-kernel forward reached from
 * DenseChessNet / Moe64A2ChessNet.forward (src/chess_engine_4/model/dense.py:188-199,
 * moe.py:389-410). */

/* Creates an empty model on `device` for batches up to `max_batch` positions. Weights
 * are uploaded with ce4b_model_set_tensor and sealed with ce4b_model_finalize. */
int ce4b_model_create(const ce4b_model_config* config, int device, int max_batch,
                      ce4b_model** out);

/* Copies one tensor into the model's weight arena. `name` and shape follow the
 * Safetensors v1 contract (kernels/src/inference/runtime.cu:398-452), e.g.
 * "input.weight" [d, 7168], "blocks.3.gate_up.weight" [2h, d]. `src_is_device` selects
 * device-to-device or host-to-device copy. Blocks until the copy is done. */
int ce4b_model_set_tensor(ce4b_model* model, const char* name, const void* data, int dtype,
                          int ndim, const int64_t* shape, int src_is_device);

/* Checks that every tensor is present and prepares derived data. Must be called after
 * the last ce4b_model_set_tensor and before a forward. */
int ce4b_model_finalize(ce4b_model* model);

/* Loads a Safetensors v1 file (release/export.py format) and finalizes the model. */
int ce4b_model_load_safetensors(const char* path, int device, int max_batch, int precision,
                                ce4b_model** out);

int ce4b_model_info_get(const ce4b_model* model, ce4b_model_info* info);

/* Device-side forward on `stream`. `input_dev` is in layout `input_layout`;
 * `scalars_dev` is the [B, 8] aux-plane scalars for the packed layouts (else NULL).
 * Outputs: policy [B, policy_size] f32, wdl [B, 3] f32 (logits, or probabilities when
 * wdl_probs != 0), moves_left [B] f32. For moe64a2, tokens_per_expert_dev receives
 * [depth/2, 64] int32 counts (may be NULL). For CE4B_INPUT_F32_PLANES with
 * `normalize_in_place` != 0 the rule-50 plane of the input is divided by 99 in place,
 * as normalize_lc0_planes does (src/chess_engine_4/model/dense.py:34-42).
 * Outside stream capture the forward is ordered after the model's previous forward on
 * any stream (it shares the model's workspace); under capture the caller's graph orders it. */
int ce4b_model_forward(ce4b_model* model, int input_layout, void* input_dev,
                       const void* scalars_dev, int batch, float* policy_dev, float* wdl_dev,
                       float* moves_left_dev, int wdl_probs, int normalize_in_place,
                       int32_t* tokens_per_expert_dev, void* stream);

/* Host-buffer evaluation, blocking: H2D of the planes, forward (CUDA graph per batch
 * size), D2H of policy [B, policy_size], WDL probabilities [B, 3], moves-left [B].
 * Mirrors Model::Evaluate (kernels/src/inference/runtime.cu:532-564).
 * Batches that take the small-batch forward skip the copies when all four host buffers are
 * pinned and mapped for the model's device over their whole extent, each inside one
 * cudaHostAlloc allocation or cudaHostRegister registration (e.g. torch pin_memory): the
 * expansion kernel reads the records from host memory and the heads write the outputs
 * into the caller's buffers (one CUDA graph per batch size and buffer set, built on first
 * use, which blocks).
 * Results are identical either way. Other buffers take the copy path. */
int ce4b_model_evaluate(ce4b_model* model, const ce4b_input_plane* host_planes, int batch,
                        float* host_policy, float* host_wdl, float* host_moves_left);

/* Turns the copy-free evaluation of pinned host buffers above on (default) or off
 * (enable = 0: every evaluation copies through device buffers). */
int ce4b_model_set_direct_io(ce4b_model* model, int enable);

/* Asynchronous form of ce4b_model_evaluate on `stream`: enqueues the H2D copy, the
 * graph and the D2H copies (or, for pinned buffers of a small batch, the copy-free graph)
 * and returns. Host buffers must stay valid and untouched (and should be pinned) until the
 * stream reaches that point. The first call for a batch size (and, copy-free, for a
 * buffer set) builds its graph and blocks.
 * The model owns two device I/O slots used in turn. Consecutive calls on different
 * streams overlap: a call's H2D copy and the previous call's D2H copies run while a
 * forward computes. Forwards of one model never overlap one another (each waits for the
 * previous one on any stream), and a slot's planes are overwritten only after its last
 * D2H copies have finished. Calls on one handle must still be serialised on the host. */
int ce4b_model_evaluate_async(ce4b_model* model, const ce4b_input_plane* host_planes, int batch,
                              float* host_policy, float* host_wdl, float* host_moves_left,
                              void* stream);

/* Legal-move policy (the lc0 backend's post-processing, third_party/lc0/src/neural/
 * backends/ce4/backend.cc:182-195, on the device): for position b the probabilities of
 * its legal moves, move_indices[move_offsets[b] .. move_offsets[b+1]) (NN policy indices,
 * board transform applied by the caller), are softmax((logit - max) * temperature) of the
 * gathered logits. expf is used (the backend's FastExp approximates it).
 * ce4b_policy_softmax works on device buffers (policy [batch, policy_size] f32, offsets
 * [batch + 1], indices and probs [offsets[batch]]) on `stream`.
 * ce4b_model_evaluate_legal is ce4b_model_evaluate returning move probabilities instead
 * of the 1858 logits (blocking; host buffers; at most 256 moves per position), so only
 * ~4 bytes per legal move cross PCIe instead of 7.4 KB per position. */
int ce4b_policy_softmax(const float* policy_dev, int batch, int policy_size,
                        const int32_t* move_offsets_dev, const int32_t* move_indices_dev,
                        float temperature, float* probs_dev, void* stream);
int ce4b_model_evaluate_legal(ce4b_model* model, const ce4b_input_plane* host_planes, int batch,
                              const int32_t* host_move_offsets, const int32_t* host_move_indices,
                              float temperature, float* host_move_probs, float* host_wdl,
                              float* host_moves_left);

/* Per-kernel tracing of ce4b_model_forward: when `count` > 0, forward records
 * events[i] (cudaEvent_t) on its stream after its i-th kernel; count 0 disables.
 * ce4b_model_trace_label names kernel i of the last traced forward. */
int ce4b_model_set_trace(ce4b_model* model, void* const* events, int count);
/* ------------------------------------------------------------------ expert parallelism
 * moe64a2 across `world` GPUs of one node (one process and one model handle per GPU, world
 * in {2, 4, 8}): each rank holds and computes only 64 / world consecutive experts (its
 * weight arena is repacked to them when this is enabled, so weights are fixed from then on).
 * Every MoE layer sends each routed row to the rank of its expert and the result back
 * (expert parallelism over the reference's static dispatch path,
 * src/chess_engine_4/model/moe.py:226-287) through the ranks' shared buffers over NVLink
 * peer memory (CUDA IPC), with the receive layout and the grouped GEMMs' tile table built
 * on the device: no host synchronisation, so forwards may be captured in CUDA graphs. Each
 * rank passes its own batch of positions to ce4b_model_forward / ce4b_model_evaluate, and
 * every rank must run the same sequence of forwards; results equal the single-GPU forward
 * of those positions. A peer that stops answering turns into a device error
 * (ce4b_check_device_error) after 2 s instead of a hang. ce4b_nccl_unique_id fills the
 * 128-byte NCCL unique id used once to exchange the buffer handles (rank 0 makes it, every
 * rank passes the same bytes); ce4b_model_enable_expert_parallel is collective over the
 * ranks and needs a finalized model. */
int ce4b_nccl_unique_id(void* out, int out_len);
int ce4b_model_enable_expert_parallel(ce4b_model* model, int rank, int world, const void* unique_id);

/* Host restatement of the exchange plan that the forward builds on the device (no GPU;
 * the forward's tile table uses local expert indices): meta_send[64][2] holds
 * this rank's {segment rows padded to 128, valid rows} per expert, meta_recv[world][64 /
 * world][2] the same from every rank for this rank's experts. Outputs rows sent to / received
 * from each rank and the m-tile table over the received rows (int32 x4 per tile: global
 * expert, first row, valid rows, 0); tiles may be NULL to only count them. */
int ce4b_expert_parallel_plan(int world, int rank, const int32_t* meta_send, const int32_t* meta_recv,
                              int32_t* send_rows, int32_t* recv_rows, int32_t* tiles, int tiles_cap,
                              int* num_tiles);

/* Per-task timeline of the persistent dense forward (dense BF16 models). With
 * capacity_tasks > 0, each forward writes 12 uint64 per task id < capacity_tasks into the
 * device buffer: %globaltimer ns when the task was fetched, its inputs were ready, its
 * last load was issued, its first MMA was issued, its accumulator was committed, its
 * epilogue started and finished, its results were staged in shared memory and published,
 * the store warp took the staged tile; then the CTA index; then the tile's global stores
 * completed. 0 disables. Task ids are numbered input-GEMM tiles first (row block, slice,
 * k split); then per layer the gate_up tiles of row block i (hidden chunk) each followed by
 * the down tiles of row block i - lag (slice, k split), lag = ceil(5/8 of the row blocks),
 * the remaining down tiles last; then the head tiles (row block, 256 head columns).
 * ce4b_model_task_count gives the number of tasks of a forward at `batch` (0 when the
 * model does not use the persistent forward). */
int ce4b_model_set_task_trace(ce4b_model* model, void* device_buffer, int capacity_tasks);
int ce4b_model_task_count(const ce4b_model* model, int batch, int* tasks);

/* Small-batch forward of dense BF16 models with d_model <= 512: batches of at most 64
 * positions run as one cooperative launch in which every GEMM is computed transposed
 * (weights on the MMA's 128-row side, positions on its N side) and split over most SMs,
 * with the same folded-RMSNorm arithmetic as the persistent forward (the norm weight in
 * the next linear's weight, the row's rsqrt(mean(x^2)+eps) on the FP32 accumulator;
 * the reference rounds n = bf16(x * r * w) first, kernels/src/inference/runtime.cu:182-336).
 * It is the latency path of the lc0 backend's
 * per-search-batch evaluation (third_party/lc0/src/neural/backends/ce4/backend.cc:163-168,
 * Model::Evaluate in kernels/src/inference/runtime.cu:532-564). Enabled by default;
 * enable = 0 sends small batches to the persistent forward instead (for comparisons).
 * With the task trace on, task index = CTA * max_tasks + position in the CTA's list
 * (ce4b_model_task_count gives grid * max_tasks), words 0..7 = task start, inputs ready,
 * activations landed, MMAs issued, MMAs done, results stored and published, all K parts
 * in, this CTA's share of the sum published; word 10 = CTA, word 11 = type << 48 |
 * layer << 32 | tile << 16 | part. ce4b_model_uses_latency_path reports the choice for a
 * batch size. */
int ce4b_model_set_latency_path(ce4b_model* model, int enable);
int ce4b_model_uses_latency_path(const ce4b_model* model, int batch, int* uses);

int ce4b_model_trace_label(const ce4b_model* model, int index, char* buffer, int buffer_len);

/* Routing tap (testing hook) of a moe64a2 model: with experts_dev set, each later
 * single-GPU ce4b_model_forward outside stream capture whose batch B <= capacity_tokens
 * writes every MoE layer's expert pair per token, [depth/2][B][2] int32 (best first), as
 * MoeBlock.forward selects them (src/chess_engine_4/model/moe.py:160-177). NULL turns the
 * tap off. No counterpart in the reference's API. */
int ce4b_model_set_routing_tap(ce4b_model* model, int32_t* experts_dev, int capacity_tokens);

/* MXFP8 tap (testing hook) of an MXFP8 model: the operands of the quantisation points of
 * one layer, as the reference's custom MXFP8 path quantises them (the BF16 activations fed
 * to quantize_mxfp8 before each mxfp8_gemm, src/chess_engine_4/kernels/dense.py:395,
 * 403-406). With tap->layer = l in [0, depth], each later ce4b_model_forward outside
 * stream capture writes, for its batch B (rows_pad = B rounded up to 128):
 *  - a_codes [rows_pad, 64 * planes] and a_scales [rows_pad/128][planes/2][512]: the input
 *    planes' codes and scales (planes = selected input planes; NULL: not recorded);
 *  - n_bf16 [B, d]: the normalised rows (BF16) that the epilogue producing layer l's input
 *    quantised (l = 0: the input GEMM's; l = depth: the heads' input), with n_codes
 *    [rows_pad, d] and n_scales [rows_pad/128][d/128][512] written for them;
 *  - for l < depth, h_bf16 [B, h], h_codes [rows_pad, h], h_scales [rows_pad/128][h/128][512]:
 *    layer l's SwiGLU hidden rows and their codes and scales.
 * Scales use the ce4b_quantize_mxfp8 layout. Any pointer may be NULL. tap = NULL or
 * tap->layer < 0 turns the tap off. No counterpart in the reference's API. */
typedef struct ce4b_mxfp8_tap {
  int32_t layer;
  void* a_codes_dev;
  void* a_scales_dev;
  void* n_bf16_dev;
  void* n_codes_dev;
  void* n_scales_dev;
  void* h_bf16_dev;
  void* h_codes_dev;
  void* h_scales_dev;
} ce4b_mxfp8_tap;
int ce4b_model_set_mxfp8_tap(ce4b_model* model, const ce4b_mxfp8_tap* tap);

void ce4b_model_destroy(ce4b_model* model);

/* Self-test of the bounded in-kernel waits (no counterpart in the reference): launches
 * one single-thread kernel on `stream` that waits, with the given limit (at most 100 ms),
 * for something that never happens: kind 0, a global counter nobody publishes (the
 * persistent forward's cross-CTA dependency wait); kind 1, an mbarrier nobody arrives on
 * (a pipeline-stage wait). The kernel gives up after the limit, records the timeout code
 * (kind 0: 7, dependency; kind 1: 1, producer) in the device error word that
 * ce4b_check_device_error reads and clears, and returns. Blocks until the kernel is done;
 * waited_ns receives the wait the kernel measured. Nothing faults, traps or hangs. */
int ce4b_selftest_bounded_wait(int kind, long long limit_ns, long long* waited_ns, void* stream);

/* ------------------------------------------------------------------ kernel-op API
 * Replaces the pybind operators of the reference extension (kernels/src/sm100/dense.cu:760-774)
 * reached through src/chess_engine_4/kernels/dense.py. */

/* C[M,N] = A[M,K] . B[N,K]^T in BF16 (FP32 accumulate). N % 16 == 0, K % 8 == 0.
 * Replaces dense_bf16_gemm (src/chess_engine_4/kernels/dense.py:116-129). */
int ce4b_bf16_gemm(const void* a_dev, const void* b_dev, void* c_dev, int m, int n, int k,
                   void* stream);

/* out = bf16(x * rsqrt(mean(x^2) + eps) * w) per row.
 * Replaces dense_rmsnorm_forward (kernels/src/sm100/dense.cu:313-348). */
int ce4b_rmsnorm_forward(const void* x_dev, const void* weight_dev, void* out_dev, int rows,
                         int width, float eps, void* stream);

/* hidden[r, j] = bf16(silu(gate_up[r, j]) * gate_up[r, H + j]).
 * Replaces dense_swiglu_forward (kernels/src/sm100/dense.cu:350-377). */
int ce4b_swiglu_forward(const void* gate_up_dev, void* hidden_dev, int rows, int hidden_dim,
                        void* stream);

/* out = bf16(out + residual), elementwise.
 * Replaces dense_residual_add (kernels/src/sm100/dense.cu:379-390). */
int ce4b_residual_add(void* out_dev, const void* residual_dev, int64_t elements, void* stream);

/* Scratch bytes ce4b_dense_block_forward needs for `rows` rows. */
int64_t ce4b_dense_block_workspace_size(int rows, int d_model, int hidden_dim);

/* out = x + down(SwiGLU(gate_up(RMSNorm(x)))) for one dense block, BF16.
 * gate_up_weight [2H, d] (gate rows first), down_weight [d, H]. `workspace_dev` holds
 * ce4b_dense_block_workspace_size() bytes (256-byte aligned). precision must be
 * CE4B_PRECISION_BF16. Replaces dense_block_forward
 * (src/chess_engine_4/kernels/dense.py:141-160, 357-392). */
int ce4b_dense_block_forward(const void* x_dev, const void* norm_weight_dev,
                             const void* gate_up_weight_dev, const void* down_weight_dev,
                             void* out_dev, void* workspace_dev, int rows, int d_model,
                             int hidden_dim, float eps, int precision, void* stream);

/* Top-2 routing of BF16 router logits [tokens, 64] with the quantile-balancing offsets
 * beta [64] (FP32): experts [tokens, 2] int32 (best first; the lower index wins ties),
 * probs [tokens, 2] FP32 holding the BF16-rounded softmax weights over all 64 logits,
 * counts [64] int32 incremented per route (may be NULL; zero it first). Replaces the
 * selection in MoeBlock.forward (src/chess_engine_4/model/moe.py:160-177) and the
 * runtime's RouteKernel (kernels/src/inference/moe_bf16_impl.cuh:18-68). */
int ce4b_moe_route(const void* logits_dev, const float* beta_dev, int32_t* experts_dev,
                   float* probs_dev, int32_t* counts_dev, int tokens, void* stream);

/* Routing and dispatch of one moe64a2 layer, with the kernels the model's forward runs
 * (router GEMM with the top-2 epilogue and per-tile expert histograms, histogram scan,
 * dispatch). Replaces the eval-path selection and static dispatch of MoeBlock.forward
 * (src/chess_engine_4/model/moe.py:160-177, 232-267) with its route order _route_slots
 * (moe.py:36-47), and the runtime's RouteKernel / PrefixOffsetsKernel / DispatchKernel
 * (kernels/src/inference/moe_bf16_impl.cuh:18-106).
 * Inputs: n [tokens, d_model] BF16 normalised rows, router_weight [64, d_model] BF16,
 * beta [64] FP32 (router_qb_beta). Outputs: logits [tokens, 64] BF16 as the selection
 * used them (may be NULL), experts [tokens, 2] int32 (best first; the lower index wins
 * ties of logit - beta), probs [tokens, 2] FP32 (BF16-rounded softmax over all 64 logits),
 * positions [tokens, 2] int32 (row of each route in the permuted layout), expert_offsets
 * [65] int32 (segment starts, each a multiple of 128, then the total permuted rows),
 * counts [64] int32 (routes per expert; may be NULL), xperm [capacity, d_model] BF16
 * (row positions[t][k] = n[t]; padding rows are not written) and pprob [capacity] FP32.
 * Within an expert, routes are ordered by 2 * token + k. capacity =
 * ce4b_moe_dispatch_capacity(tokens); workspace holds
 * ce4b_moe_route_dispatch_workspace_size(tokens) bytes (256-byte aligned). The outputs feed
 * ce4b_moe_forward (xperm, pprob as BF16, expert_offsets) directly. */
int ce4b_moe_dispatch_capacity(int tokens);
int64_t ce4b_moe_route_dispatch_workspace_size(int tokens);
int ce4b_moe_route_dispatch(const void* n_dev, const void* router_weight_dev, const float* beta_dev,
                            void* logits_dev, int32_t* experts_dev, float* probs_dev,
                            int32_t* positions_dev, int32_t* expert_offsets_dev,
                            int32_t* counts_dev, void* xperm_dev, float* pprob_dev,
                            void* workspace_dev, int tokens, int d_model, void* stream);

/* Scratch bytes ce4b_moe_forward needs. */
int64_t ce4b_moe_workspace_size(int rows, int d_model, int hidden_dim);

/* Expert MLP over rows already sorted by expert: rows [offsets[e], offsets[e+1]) of x
 * [rows, d] go through expert e: out = ((silu(x.Wg^T) * (x.Wu^T)) . Wd^T) * route_probs
 * per row (BF16, FP32 accumulate). gate_up [64, 2H, d] (gate rows first), down [64, d, H],
 * route_probs [rows] BF16, expert_offsets [65] int32 on the device, each a multiple of 128
 * (the reference's static path pads segments to 128 rows); a misaligned offset sets the
 * device error word and that expert is skipped. Rows past offsets[64] are not written.
 * Replaces moe_forward (src/chess_engine_4/kernels/moe.py:24-46). */
int ce4b_moe_forward(const void* x_dev, const void* gate_up_weight_dev,
                     const void* down_weight_dev, const void* route_probs_dev,
                     const int32_t* expert_offsets_dev, void* out_dev, void* workspace_dev,
                     int rows, int d_model, int hidden_dim, void* stream);

/* MXFP8 quantisation of a BF16 [rows, cols] matrix (rows, cols multiples of 128):
 * E4M3 codes [rows, cols] and E8M0 scales [rows/128, cols/128, 32, 16] (one per row and
 * 32 columns; byte (r%32)*16 + (r/32)*4 + kb of each 128x128 tile). Bit-exact to the
 * reference's quantiser recipe: scale = E8M0 round-up of max(amax * 0.002232142857, 1e-12),
 * codes = E4M3 round-to-nearest-even satfinite of x / scale. Replaces quantize_mxfp8
 * (src/chess_engine_4/kernels/dense.py:46-60). */
int ce4b_quantize_mxfp8(const void* x_dev, void* codes_dev, void* scales_dev, int rows, int cols,
                        void* stream);

/* The quantisation of the transpose of a BF16 [rows, cols] matrix without materialising it:
 * codes [cols, rows] and scales [cols/128, rows/128, 32, 16], equal to ce4b_quantize_mxfp8 of
 * the transposed matrix. Replaces quantize_mxfp8_transpose
 * (src/chess_engine_4/kernels/dense.py:63-84). */
int ce4b_quantize_mxfp8_transpose(const void* x_dev, void* codes_dev, void* scales_dev, int rows,
                                  int cols, void* stream);

/* C[M,N] BF16 = sum over 32-element K blocks of (A codes * 2^(sa-127)) (B codes *
 * 2^(sb-127)), FP32 accumulate: A, B E4M3 codes [M,K], [N,K] with scales in the
 * ce4b_quantize_mxfp8 layout; M, N, K multiples of 128. Block-scaled tcgen05 MMA
 * (kind::mxf8f6f4). Replaces mxfp8_gemm (src/chess_engine_4/kernels/dense.py:87-113). */
int ce4b_mxfp8_gemm(const void* a_codes_dev, const void* a_scales_dev, const void* b_codes_dev,
                    const void* b_scales_dev, void* c_dev, int m, int n, int k, void* stream);

/* ce4b_dense_block_forward for callers that cannot allocate device memory (an engine
 * thread whose process freezes its allocator after start-up, a plugin that is handed only
 * its input and output buffers, code under a no-allocation budget). Same arguments and
 * result, without the workspace: the scratch lives in a fixed 8 MiB __device__ array of
 * the library (held on every GPU that loads it), so rows * (d_model + hidden_dim) * 2
 * bytes, each part rounded up to 128 rows and 256 bytes, must fit in 8 MiB; larger calls
 * fail with CE4B_ERR_INVALID_ARGUMENT. The first call on a device looks up the array's
 * device address, which (under CUDA's default lazy module loading) loads the library's
 * device image there and reserves the 8 MiB: make that first call during start-up, before
 * any stream capture and before the allocator is frozen. All calls on a device share
 * the array: calls whose GPU work overlaps race and must be serialised by the caller.
 * Allocates nothing. This entry point has no counterpart in the reference. */
int ce4b_dense_block_forward_static(const void* x_dev, const void* norm_weight_dev,
                                    const void* gate_up_weight_dev, const void* down_weight_dev,
                                    void* out_dev, int rows, int d_model, int hidden_dim,
                                    float eps, int precision, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CE4B200_H */
