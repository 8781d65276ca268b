// heads.cu — linear decision heads on the [CLS] hidden state of each request.
//
// A serving call needs only the [CLS] (position 0) hidden state of each
// request, so the engine applies final_norm to those rows alone (the
// reference normalises every row, src/model.cpp:292) and this kernel runs the
// linear heads (softmax or sigmoid) on them in fp32.  One block per request,
// one warp per output logit.
#include "common.cuh"
#include "kernels.h"

namespace sjb {
namespace {

__global__ void __launch_bounds__(128) dec_heads_kernel(const float* __restrict__ Hc, int D,
                                                        const float* __restrict__ W,
                                                        const float* __restrict__ bias,
                                                        HeadSpec spec, float* __restrict__ probs) {
  __shared__ float logits[64];
  const int b = blockIdx.x;
  const float* y = Hc + (int64_t)b * D;
  // one warp per output logit
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int o = wid; o < spec.n_total; o += 4) {
    float acc = 0.f;
    for (int j = lane; j < D; j += 32) acc = fmaf(y[j], W[(int64_t)o * D + j], acc);
    acc = warp_sum(acc);
    if (lane == 0) logits[o] = acc + bias[o];
  }
  __syncthreads();
  if (threadIdx.x < spec.n_heads) {
    const int h = threadIdx.x, off = spec.off[h], n = spec.n_out[h];
    float* out = probs + (int64_t)b * spec.n_total + off;
    if (spec.kind[h] == 1) {
      for (int k = 0; k < n; ++k) out[k] = 1.0f / (1.0f + expf(-logits[off + k]));
    } else {
      float mx = logits[off];
      for (int k = 1; k < n; ++k) mx = fmaxf(mx, logits[off + k]);
      float sum = 0.f;
      for (int k = 0; k < n; ++k) sum += expf(logits[off + k] - mx);
      for (int k = 0; k < n; ++k) out[k] = expf(logits[off + k] - mx) / sum;
    }
  }
}

}  // namespace

cudaError_t dec_heads(const float* Hc, int B, int D, const float* W, const float* bias,
                      HeadSpec spec, float* probs, cudaStream_t st) {
  if (B <= 0) return cudaSuccess;
  if (spec.n_total > 64 || spec.n_heads > 8) return cudaErrorInvalidValue;
  dec_heads_kernel<<<B, 128, 0, st>>>(Hc, D, W, bias, spec, probs);
  return cudaGetLastError();
}

}  // namespace sjb
