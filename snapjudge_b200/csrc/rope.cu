// rope.cu — rotate-half RoPE on packed qkv and per-row positions.
//
// Follows the reference rope_inplace (src/tensor.cpp:257-279): pairs
// (d, d + Dh/2) of every q and k head, x0' = x0 c - x1 s, x1' = x1 c + x0 s in
// fp32, with the reference's fp32 tables (src/model.cpp:173-190).  The
// reference takes position = r % L on a padded batch; the packed varlen form
// takes position = r - cu_seqlens[b], which is the same number for every row.
#include "common.cuh"
#include "kernels.h"

namespace sjb {
namespace {

template <typename T>
__global__ void rope_kernel(T* __restrict__ qkv, const float* __restrict__ cos_t,
                            const float* __restrict__ sin_t, const int32_t* __restrict__ pos,
                            const int32_t* __restrict__ cu, int B, int M, int H, int Dh) {
  const int half = Dh / 2;
  const int pairs = 2 * H * half;  // q and k heads
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)M * pairs) return;
  int r = (int)(idx / pairs);
  int c = (int)(idx % pairs);
  int hh = c / half, d = c % half;
  int p = pos ? pos[r] : r - cu[seq_of_row(cu, B, r)];
  float cs = cos_t[(int64_t)p * half + d], sn = sin_t[(int64_t)p * half + d];
  T* row = qkv + (int64_t)r * 3 * H * Dh + hh * Dh;
  float x0 = io<T>::to_f(row[d]), x1 = io<T>::to_f(row[d + half]);
  row[d] = io<T>::cvt(x0 * cs - x1 * sn);
  row[d + half] = io<T>::cvt(x1 * cs + x0 * sn);
}

__global__ void positions_kernel(const int32_t* __restrict__ cu, int B, int32_t* __restrict__ pos,
                                 int32_t* __restrict__ seq) {
  const int b = blockIdx.x;
  if (b >= B) return;
  const int s = cu[b], e = cu[b + 1];
  for (int r = s + threadIdx.x; r < e; r += blockDim.x) {
    pos[r] = r - s;
    if (seq) seq[r] = b;
  }
}

}  // namespace

template <typename T>
cudaError_t rope(T* qkv, const float* cos_t, const float* sin_t, const int32_t* pos, int M, int H,
                 int Dh, cudaStream_t st) {
  int64_t n = (int64_t)M * H * Dh;  // 2*H*(Dh/2) pairs per row
  if (n <= 0) return cudaSuccess;
  rope_kernel<T><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(qkv, cos_t, sin_t, pos, nullptr, 0,
                                                               M, H, Dh);
  return cudaGetLastError();
}

cudaError_t rope_cu(bf16* qkv, const float* cos_t, const float* sin_t, const int32_t* cu, int B,
                    int M, int H, int Dh, cudaStream_t st) {
  int64_t n = (int64_t)M * H * Dh;
  if (n <= 0 || B <= 0) return cudaSuccess;
  rope_kernel<bf16><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(qkv, cos_t, sin_t, nullptr, cu,
                                                                  B, M, H, Dh);
  return cudaGetLastError();
}

cudaError_t positions(const int32_t* cu, int B, int T, int32_t* pos, int32_t* seq,
                      cudaStream_t st) {
  if (B <= 0 || T <= 0) return cudaSuccess;
  positions_kernel<<<B, 128, 0, st>>>(cu, B, pos, seq);
  return cudaGetLastError();
}

template cudaError_t rope<float>(float*, const float*, const float*, const int32_t*, int, int, int,
                                 cudaStream_t);
template cudaError_t rope<bf16>(bf16*, const float*, const float*, const int32_t*, int, int, int,
                                cudaStream_t);

}  // namespace sjb
