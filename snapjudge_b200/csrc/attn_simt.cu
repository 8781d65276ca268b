// attn_simt.cu — packed varlen attention on CUDA cores.
//
// Used in fp32 mode and for head dims the tcgen05 kernel does not take
// (Dh = 8, 16, 32).  Semantics follow the reference attention
// (src/tensor.cpp:156-228): query i of segment b attends keys
// j in [max(0, i - w), min(kv_len, i + w + 1)) (w = 0: [0, kv_len)), scores
// scaled by 1/sqrt(Dh), max-subtracted softmax, probability-weighted V sum.
// The softmax is evaluated online over key tiles of 32 (one rescale per tile);
// fp32 throughout.
//
// One block = 64 query rows of one (segment, head); one thread per query row
// keeps q and the output accumulator in registers; K/V tiles are staged in
// shared memory as fp32.
#include "common.cuh"
#include "kernels.h"

namespace sjb {
namespace {

constexpr int QT = 64;   // query rows per block
constexpr int KT = 32;   // keys per shared-memory tile

template <typename T, int DH>
__global__ void __launch_bounds__(QT) attn_simt_kernel(const T* __restrict__ qkv,
                                                       const int32_t* __restrict__ cu,
                                                       const int32_t* __restrict__ kv_lens,
                                                       T* __restrict__ O, int H, int window,
                                                       const int2* __restrict__ tiles) {
  __shared__ float Ks[KT][DH + 1];
  __shared__ float Vs[KT][DH + 1];
  const int2 tl = tiles ? tiles[blockIdx.x] : make_int2(blockIdx.z, blockIdx.x * QT);
  const int b = tl.x, q0 = tl.y, h = blockIdx.y;
  const int s0 = cu[b];
  const int n = cu[b + 1] - s0;
  if (q0 >= n) return;  // idle tile of the grid form (block-uniform exit)
  int nk = kv_lens ? kv_lens[b] : n;
  if (nk > n) nk = n;
  const int D3 = 3 * H * DH;
  const int i = q0 + threadIdx.x;
  const bool valid = i < n;
  const float scale = rsqrtf((float)DH) * 1.4426950408889634f;  // log2(e) / sqrt(Dh)

  float q[DH], o[DH];
#pragma unroll
  for (int d = 0; d < DH; ++d) {
    q[d] = valid ? io<T>::to_f(qkv[(int64_t)(s0 + i) * D3 + h * DH + d]) : 0.f;
    o[d] = 0.f;
  }
  int lo = 0, hi = nk;        // this thread's key range
  int blo = 0, bhi = nk;      // the block's key range (union over its rows)
  if (window > 0) {
    lo = max(0, i - window);
    hi = min(nk, i + window + 1);
    blo = max(0, q0 - window);
    bhi = min(nk, q0 + QT - 1 + window + 1);
  }
  float m = -INFINITY, l = 0.f;
  for (int k0 = blo; k0 < bhi; k0 += KT) {
    __syncthreads();
    for (int e = threadIdx.x; e < KT * DH; e += QT) {
      int kk = e / DH, d = e % DH;
      int j = k0 + kk;
      bool ok = j < bhi;
      Ks[kk][d] = ok ? io<T>::to_f(qkv[(int64_t)(s0 + j) * D3 + H * DH + h * DH + d]) : 0.f;
      Vs[kk][d] = ok ? io<T>::to_f(qkv[(int64_t)(s0 + j) * D3 + 2 * H * DH + h * DH + d]) : 0.f;
    }
    __syncthreads();
    if (!valid) continue;
    float s[KT];
    float tmax = -INFINITY;
#pragma unroll
    for (int kk = 0; kk < KT; ++kk) {
      int j = k0 + kk;
      float acc = 0.f;
#pragma unroll
      for (int d = 0; d < DH; ++d) acc = fmaf(q[d], Ks[kk][d], acc);
      s[kk] = (j >= lo && j < hi) ? acc * scale : -INFINITY;
      tmax = fmaxf(tmax, s[kk]);
    }
    if (tmax == -INFINITY) continue;  // no key of this tile is visible to row i
    float mn = fmaxf(m, tmax);
    float corr = exp2f(m - mn);  // m = -inf on the first visible tile -> 0
    l *= corr;
#pragma unroll
    for (int d = 0; d < DH; ++d) o[d] *= corr;
#pragma unroll
    for (int kk = 0; kk < KT; ++kk) {
      float p = exp2f(s[kk] - mn);
      l += p;
#pragma unroll
      for (int d = 0; d < DH; ++d) o[d] = fmaf(p, Vs[kk][d], o[d]);
    }
    m = mn;
  }
  if (!valid) return;
  float inv = l > 0.f ? 1.0f / l : 0.f;
  T* orow = O + (int64_t)(s0 + i) * H * DH + h * DH;
#pragma unroll
  for (int d = 0; d < DH; ++d) orow[d] = io<T>::cvt(o[d] * inv);
}

}  // namespace

template <typename T>
cudaError_t attn_simt(const T* qkv, const int32_t* cu, const int32_t* kv_lens, T* O, int H, int Dh,
                      int window, const int2* tiles, int n_tiles, int B, int max_seqlen,
                      cudaStream_t st) {
  dim3 grid(n_tiles, H, 1);
  if (!tiles) grid = dim3((max_seqlen + QT - 1) / QT, H, B);
  if (grid.x == 0 || grid.z == 0) return cudaSuccess;
  switch (Dh) {
    case 8: attn_simt_kernel<T, 8><<<grid, QT, 0, st>>>(qkv, cu, kv_lens, O, H, window, tiles); break;
    case 16: attn_simt_kernel<T, 16><<<grid, QT, 0, st>>>(qkv, cu, kv_lens, O, H, window, tiles); break;
    case 32: attn_simt_kernel<T, 32><<<grid, QT, 0, st>>>(qkv, cu, kv_lens, O, H, window, tiles); break;
    case 64: attn_simt_kernel<T, 64><<<grid, QT, 0, st>>>(qkv, cu, kv_lens, O, H, window, tiles); break;
    case 128: attn_simt_kernel<T, 128><<<grid, QT, 0, st>>>(qkv, cu, kv_lens, O, H, window, tiles); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

template cudaError_t attn_simt<float>(const float*, const int32_t*, const int32_t*, float*, int,
                                      int, int, const int2*, int, int, int, cudaStream_t);
template cudaError_t attn_simt<bf16>(const bf16*, const int32_t*, const int32_t*, bf16*, int, int,
                                     int, const int2*, int, int, int, cudaStream_t);

}  // namespace sjb
