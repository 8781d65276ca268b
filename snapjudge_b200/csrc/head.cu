// head.cu — the decision-model tail of DecisionModel::forward (src/model.cpp:402-535)
// on device: type embedding, marker gather and the act head.  The head's
// TransformerEncoderLayers and the scorer's LN / Linear layers reuse the
// encoder's LN, GEMM and attention kernels (engine.cu).
#include <cmath>

#include "common.cuh"
#include "kernels.h"

namespace sjb {
namespace {

// h[r] += type_emb[qtype[b]] for every row r of segment b (model.cpp:402-408)
__global__ void type_emb_kernel(float* __restrict__ h, const int32_t* __restrict__ cu, int B,
                                const int64_t* __restrict__ qtype, const float* __restrict__ te,
                                int D, int T) {
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= T) return;
  const int b = seq_of_row(cu, B, r);
  const float* t = te + qtype[b] * (int64_t)D;
  float* row = h + (int64_t)r * D;
  for (int j = threadIdx.x & 31; j < D; j += 32) row[j] += t[j];
}

// m[b*K + k] = h[cu[b] + clamp(marker_pos[b*K + k], 0, n_b - 1)]   (model.cpp:463-474)
__global__ void gather_markers_kernel(const float* __restrict__ h, const int32_t* __restrict__ cu,
                                      const int64_t* __restrict__ pos, int K, int D, int BK,
                                      float* __restrict__ m) {
  const int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (i >= BK) return;
  const int b = i / K;
  const int n = cu[b + 1] - cu[b];
  int64_t p = pos[i];
  p = p < 0 ? 0 : (p >= n ? n - 1 : p);
  const float* src = h + ((int64_t)cu[b] + p) * D;
  float* dst = m + (int64_t)i * D;
  for (int j = threadIdx.x & 31; j < D; j += 32) dst[j] = src[j];
}

// pooled[b, d] = sum over rows i < n_b of h[cu[b] + i, d], then / max(1, n_b):
// Agent::embed's mean over non-padding positions (agent.cpp:347-354), summed
// in row order in fp32 as there.  Block (b, column slab): one thread per column.
__global__ void mean_pool_kernel(const float* __restrict__ h, const int32_t* __restrict__ cu,
                                 int D, float* __restrict__ pooled) {
  const int b = blockIdx.x;
  const int d = blockIdx.y * blockDim.x + threadIdx.x;
  if (d >= D) return;
  const int s0 = cu[b], n = cu[b + 1] - s0;
  const float* src = h + (int64_t)s0 * D + d;
  float acc = 0.f;
  for (int i = 0; i < n; ++i) acc += src[(int64_t)i * D];
  pooled[(int64_t)b * D + d] = acc / (float)max(1, n);
}

// One block per segment: the masked scorer logits, their softmax statistics
// (fp64 sums of fp32 exponentials, model.cpp:490-508), the act features
// [CLS row, top1, top1 - top2, normalised entropy, k / 255] and the act MLP
// (Linear(D+4, 256) + GELU, Linear(256, n_act)) with its softmax (:510-533).
// top1_only: SjModel's act, [top1, 1 - top1] (sj_model.cpp:355-366).
constexpr int kActThreads = 256;
__global__ void __launch_bounds__(kActThreads)
    act_head_kernel(const float* __restrict__ h, const int32_t* __restrict__ cu,
                    const float* __restrict__ score, const uint8_t* __restrict__ mask, int K,
                    const float* __restrict__ w1, const float* __restrict__ b1,
                    const float* __restrict__ w2, const float* __restrict__ b2, int n_act, int D,
                    float* __restrict__ logits, float* __restrict__ act, int top1_only) {
  extern __shared__ unsigned char sm_raw[];
  double* p = reinterpret_cast<double*>(sm_raw);       // [K]
  float* feats = reinterpret_cast<float*>(p + K);      // [D + 4]
  float* a1 = feats + D + 4;                           // [256]
  float* a2 = a1 + 256;                                // [n_act]
  const int b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int kWarps = kActThreads / 32;

  for (int k = tid; k < K; k += kActThreads) {
    const float lg = mask[b * K + k] ? score[b * K + k] : -1e4f;
    logits[b * K + k] = lg;
    p[k] = lg;  // staged; turned into probabilities below
  }
  const float* cls = h + (int64_t)cu[b] * D;
  for (int j = tid; j < D; j += kActThreads) feats[j] = cls[j];
  __syncthreads();
  if (tid == 0) {
    float mx = static_cast<float>(p[0]);
    for (int k = 1; k < K; ++k) mx = fmaxf(mx, static_cast<float>(p[k]));
    double z = 0;
    for (int k = 0; k < K; ++k) {
      p[k] = expf(static_cast<float>(p[k]) - mx);
      z += p[k];
    }
    double top1 = 0, top2 = 0, ent = 0, ks = 0;
    for (int k = 0; k < K; ++k) {
      const double v = p[k] / z;
      if (v > top1) {
        top2 = top1;
        top1 = v;
      } else if (v > top2) {
        top2 = v;
      }
      ent -= v * log(v > 1e-9 ? v : 1e-9);
      ks += mask[b * K + k];
    }
    if (top1_only) {  // SjModel (src/sj_model.cpp:355-366): act = [top1, 1 - top1]
      act[(int64_t)b * 2] = static_cast<float>(top1);
      act[(int64_t)b * 2 + 1] = static_cast<float>(1.0 - top1);
    }
    const double kf = ks > 2.0 ? ks : 2.0;
    ent /= log(kf);
    feats[D] = static_cast<float>(top1);
    feats[D + 1] = static_cast<float>(top1 - top2);
    feats[D + 2] = static_cast<float>(ent);
    feats[D + 3] = static_cast<float>(kf / 255.0);
  }
  __syncthreads();
  if (top1_only) return;
  // a1 = gelu(W1 feats + b1): one warp per output, lanes across the D+4 inputs
  for (int j = warp; j < 256; j += kWarps) {
    const float* wr = w1 + (int64_t)j * (D + 4);
    float s = 0.f;
    for (int i = lane; i < D + 4; i += 32) s += wr[i] * feats[i];
    s = warp_sum(s);
    if (lane == 0) a1[j] = gelu_erf(s + b1[j]);
  }
  __syncthreads();
  for (int j = warp; j < n_act; j += kWarps) {
    const float* wr = w2 + (int64_t)j * 256;
    float s = 0.f;
    for (int i = lane; i < 256; i += 32) s += wr[i] * a1[i];
    s = warp_sum(s);
    if (lane == 0) a2[j] = s + b2[j];
  }
  __syncthreads();
  if (tid == 0) {
    float amx = a2[0];
    for (int j = 1; j < n_act; ++j) amx = fmaxf(amx, a2[j]);
    double as = 0;
    for (int j = 0; j < n_act; ++j) {
      a2[j] = expf(a2[j] - amx);
      as += a2[j];
    }
    for (int j = 0; j < n_act; ++j) act[(int64_t)b * n_act + j] = static_cast<float>(a2[j] / as);
  }
}

}  // namespace

cudaError_t type_emb_add(float* h, const int32_t* cu, int B, const int64_t* qtype,
                         const float* te, int D, int T, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  type_emb_kernel<<<(T + 7) / 8, 256, 0, st>>>(h, cu, B, qtype, te, D, T);
  return cudaGetLastError();
}

cudaError_t gather_markers(const float* h, const int32_t* cu, const int64_t* pos, int B, int K,
                           int D, float* m, cudaStream_t st) {
  const int BK = B * K;
  if (BK <= 0) return cudaSuccess;
  gather_markers_kernel<<<(BK + 7) / 8, 256, 0, st>>>(h, cu, pos, K, D, BK, m);
  return cudaGetLastError();
}

cudaError_t mean_pool(const float* h, const int32_t* cu, int B, int D, float* pooled,
                      cudaStream_t st) {
  if (B <= 0 || D <= 0) return cudaSuccess;
  const dim3 grid(B, (D + 127) / 128);
  mean_pool_kernel<<<grid, 128, 0, st>>>(h, cu, D, pooled);
  return cudaGetLastError();
}

size_t act_head_smem(int K, int D, int n_act) {
  return (size_t)K * sizeof(double) + (size_t)(D + 4 + 256 + n_act) * sizeof(float);
}

cudaError_t act_head(const float* h, const int32_t* cu, int B, const float* score,
                     const uint8_t* mask, int K, const float* w1, const float* b1,
                     const float* w2, const float* b2, int n_act, int D, float* logits,
                     float* act, bool top1_only, cudaStream_t st) {
  if (B <= 0) return cudaSuccess;
  const size_t smem = act_head_smem(K, D, n_act);
  if (smem > 48 * 1024) {
    cudaError_t rc = cudaFuncSetAttribute(act_head_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (rc != cudaSuccess) return rc;
  }
  act_head_kernel<<<B, kActThreads, smem, st>>>(h, cu, score, mask, K, w1, b1, w2, b2, n_act, D,
                                                logits, act, top1_only ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace sjb
