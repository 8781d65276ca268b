// common.cuh — shared device helpers for the snapjudge B200 kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sjb {

using bf16 = __nv_bfloat16;

// Element-type traits for kernels that run in fp32 mode (fp32 activations) or
// bf16 mode (bf16 activations, fp32 accumulation).
template <typename T> struct io;
template <> struct io<float> {
  static __device__ __forceinline__ float ld(const float* p) { return *p; }
  static __device__ __forceinline__ float cvt(float v) { return v; }
  static __device__ __forceinline__ float to_f(float v) { return v; }
};
template <> struct io<bf16> {
  static __device__ __forceinline__ float ld(const bf16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ bf16 cvt(float v) { return __float2bfloat16(v); }
  static __device__ __forceinline__ float to_f(bf16 v) { return __bfloat162float(v); }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// exact erf GELU, as the reference's gelu_erf (src/tensor.cpp:96-98)
__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654757f));
}

// Index of the sequence that owns packed row r: largest b with cu[b] <= r.
__device__ __forceinline__ int seq_of_row(const int32_t* cu, int B, int r) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= r) lo = mid; else hi = mid - 1;
  }
  return lo;
}

}  // namespace sjb
