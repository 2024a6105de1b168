// Legal-move policy on the device: the lc0 ce4 backend's post-processing
// (third_party/lc0/src/neural/backends/ce4/backend.cc:182-195): for each position, gather
// the logits of its legal moves (NN indices computed by the caller), subtract their
// maximum, exponentiate with the policy temperature and normalise. Only the legal-move
// probabilities then need to cross PCIe instead of the 1858 logits per position.
// The exponential is expf (the backend's FastExp is a low-order approximation; the two
// differ by FastExp's own error).
#include "internal.h"
#include "ptx.cuh"

namespace ce4b {

namespace {

// One warp per position.
__global__ void policy_softmax_kernel(const float* __restrict__ policy, int batch, int policy_size,
                                      const int32_t* __restrict__ offsets,
                                      const int32_t* __restrict__ indices, float temperature,
                                      float* __restrict__ probs, int* __restrict__ err) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= batch) return;
  const int begin = offsets[warp];
  const int end = offsets[warp + 1];
  if (end <= begin) return;
  const float* row = policy + static_cast<size_t>(warp) * policy_size;
  float mx = -INFINITY;
  for (int i = begin + lane; i < end; i += 32) {
    const int idx = indices[i];
    if (idx < 0 || idx >= policy_size) {
      record_error(err, kErrBadShape);
      continue;
    }
    mx = fmaxf(mx, row[idx]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float total = 0.0f;
  for (int i = begin + lane; i < end; i += 32) {
    const int idx = indices[i];
    const float e = (idx >= 0 && idx < policy_size) ? expf((row[idx] - mx) * temperature) : 0.0f;
    probs[i] = e;
    total += e;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
  const float scale = total > 0.0f ? 1.0f / total : 1.0f;
  for (int i = begin + lane; i < end; i += 32) probs[i] *= scale;
}

}  // namespace

void policy_softmax(const float* policy, int batch, int policy_size, const int32_t* offsets,
                    const int32_t* indices, float temperature, float* probs, cudaStream_t s) {
  require(batch >= 0 && policy_size > 0, "bad policy shape");
  if (batch == 0) return;
  require(policy && offsets && indices && probs, "null policy pointer");
  const int threads = 256;
  const int blocks = (batch * 32 + threads - 1) / threads;
  policy_softmax_kernel<<<blocks, threads, 0, s>>>(policy, batch, policy_size, offsets, indices,
                                                   temperature, probs, device_error_word());
  check_cuda(cudaGetLastError(), "policy_softmax launch");
}

}  // namespace ce4b
