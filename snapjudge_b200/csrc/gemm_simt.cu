// gemm_simt.cu — CUDA-core GEMM for the fp32 mode and for shapes the tcgen05
// GEMM does not take (tiny hidden sizes).
//
// C = A W^T with W in the checkpoint's [N, K] layout, the contraction of the
// reference gemm_nt / gemm_geglu (src/tensor.cpp:108-151).  64x64 output tile
// per 256-thread block, 4x4 outputs per thread, fp32 accumulation over K in
// order.  Epilogues: bias + activation store, fp32 residual add (Wo / Wo2 of an
// encoder layer), and the GEGLU gate gelu(A Wg^T) * (A Wu^T) with W = [Wg; Wu].
#include "common.cuh"
#include "kernels.h"

namespace sjb {
namespace {

constexpr int BM = 64, BN = 64, BK = 16;

template <typename TA, typename TC, bool GEGLU>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const TA* __restrict__ A,
                                                        const TA* __restrict__ W,
                                                        const float* __restrict__ bias,
                                                        TC* __restrict__ C,
                                                        float* __restrict__ resid, int M, int N,
                                                        int K, int act) {
  __shared__ float As[BK][BM + 4];
  __shared__ float Ws[BK][BN + 4];
  __shared__ float Us[GEGLU ? BK : 1][BN + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  float acc[4][4] = {};
  float accu[4][4] = {};  // up-projection accumulators (GEGLU only)
  for (int k0 = 0; k0 < K; k0 += BK) {
    for (int e = threadIdx.x; e < BM * BK; e += 256) {
      int r = e / BK, k = e % BK;
      int gr = m0 + r, gk = k0 + k;
      As[k][r] = (gr < M && gk < K) ? io<TA>::to_f(A[(int64_t)gr * K + gk]) : 0.f;
      int gn = n0 + r;
      Ws[k][r] = (gn < N && gk < K) ? io<TA>::to_f(W[(int64_t)gn * K + gk]) : 0.f;
      if (GEGLU) Us[k][r] = (gn < N && gk < K) ? io<TA>::to_f(W[(int64_t)(gn + N) * K + gk]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float a[4], w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[k][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) w[j] = Ws[k][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], w[j], acc[i][j]);
      if (GEGLU) {
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = Us[k][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) accu[i][j] = fmaf(a[i], w[j], accu[i][j]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int r = m0 + ty * 4 + i;
    if (r >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int c = n0 + tx * 4 + j;
      if (c >= N) continue;
      float v = acc[i][j];
      if (GEGLU) {
        v = gelu_erf(v) * accu[i][j];
        C[(int64_t)r * N + c] = io<TC>::cvt(v);
        continue;
      }
      if (bias) v += bias[c];
      if (resid) {
        resid[(int64_t)r * N + c] += v;
        continue;
      }
      if (act == ACT_GELU) v = gelu_erf(v);
      else if (act == ACT_RELU) v = fmaxf(v, 0.f);
      C[(int64_t)r * N + c] = io<TC>::cvt(v);
    }
  }
}

}  // namespace

template <typename TA, typename TC>
cudaError_t gemm_simt(const TA* A, const TA* W, const float* bias, TC* C, float* resid, int M,
                      int N, int K, int act, bool geglu, cudaStream_t st) {
  if (M <= 0 || N <= 0) return cudaSuccess;
  dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
  if (geglu)
    gemm_simt_kernel<TA, TC, true><<<grid, 256, 0, st>>>(A, W, nullptr, C, nullptr, M, N, K, 0);
  else
    gemm_simt_kernel<TA, TC, false><<<grid, 256, 0, st>>>(A, W, bias, C, resid, M, N, K, act);
  return cudaGetLastError();
}

template cudaError_t gemm_simt<float, float>(const float*, const float*, const float*, float*,
                                             float*, int, int, int, int, bool, cudaStream_t);
template cudaError_t gemm_simt<bf16, bf16>(const bf16*, const bf16*, const float*, bf16*, float*,
                                           int, int, int, int, bool, cudaStream_t);

}  // namespace sjb
