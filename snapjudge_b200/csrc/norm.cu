// norm.cu — embedding gather + LayerNorm, and residual add + LayerNorm.
//
// Follows the reference layer_norm (src/tensor.cpp:54-79): population
// variance, eps inside the square root, weight then optional bias; the
// residual stream X stays fp32 (src/model.cpp:333-397).  Statistics are
// two-pass fp32 over the row held in registers (the reference accumulates in
// fp64; the difference is far below every tolerance used here).
//
// One warp per row, 16-byte loads: each lane owns D/128 float4 chunks
// (D <= 1024 in registers).  Rows of other widths use a block-per-row kernel.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace sjb {
namespace {

constexpr int kMaxChunks = 8;  // float4 chunks per lane -> D <= 1024

template <typename TY>
__device__ __forceinline__ void store4(TY* p, float4 v);
template <>
__device__ __forceinline__ void store4<float>(float* p, float4 v) {
  *reinterpret_cast<float4*>(p) = v;
}
template <>
__device__ __forceinline__ void store4<bf16>(bf16* p, float4 v) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
  __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

template <typename TR>
__device__ __forceinline__ float4 load4(const TR* p);
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
template <>
__device__ __forceinline__ float4 load4<bf16>(const bf16* p) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&u.x);
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&u.y);
  float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

// Normalise the lane-held chunks v[0..nc) of a D-wide row; returns inv std.
// Chunk c of a lane is float4 index lane + 32 c; chunks past the row end are
// zero and excluded from the variance.
__device__ __forceinline__ void row_stats(const float4 (&v)[kMaxChunks], int lane, int nc4, int D,
                                          float eps, float& mean, float& inv) {
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) s += (v[c].x + v[c].y) + (v[c].z + v[c].w);
  mean = warp_sum(s) / (float)D;
  float q = 0.f;
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c) {
    if (lane + 32 * c >= nc4) break;
    float a = v[c].x - mean, b = v[c].y - mean, cc = v[c].z - mean, d = v[c].w - mean;
    q += (a * a + b * b) + (cc * cc + d * d);
  }
  float var = warp_sum(q) / (float)D;
  inv = 1.0f / sqrtf(var + eps);
}

template <typename TY>
__global__ void __launch_bounds__(256) embed_ln_warp(const int64_t* __restrict__ ids, int T,
                                                     const float* __restrict__ emb, int V, int D,
                                                     const float* __restrict__ w, float eps,
                                                     float* __restrict__ X, TY* __restrict__ Y,
                                                     int* __restrict__ bad,
                                                     const float* __restrict__ pos_emb,
                                                     const int32_t* __restrict__ pos, int max_pos,
                                                     const float* __restrict__ b) {
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= T) return;
  const int nc4 = D >> 2;  // float4 chunks in the row
  int64_t id = ids[r];
  bool ok = id >= 0 && id < V;
  if (!ok && lane == 0) *bad = 1;
  float4 v[kMaxChunks];
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = lane + 32 * k;
    v[k] = (ok && c < nc4) ? load4<float>(emb + id * (int64_t)D + 4 * c)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (pos_emb) {  // learned absolute positions, clamped to the table
    int p = pos[r];
    p = p < max_pos ? p : max_pos - 1;
#pragma unroll
    for (int k = 0; k < kMaxChunks; ++k) {
      const int c = lane + 32 * k;
      if (ok && c < nc4) {
        const float4 e = load4<float>(pos_emb + (int64_t)p * D + 4 * c);
        v[k].x += e.x;
        v[k].y += e.y;
        v[k].z += e.z;
        v[k].w += e.w;
      }
    }
  }
  float mean, inv;
  row_stats(v, lane, nc4, D, eps, mean, inv);
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = lane + 32 * k;
    if (c >= nc4) break;
    float4 g = load4<float>(w + 4 * c);
    float4 o = make_float4((v[k].x - mean) * inv * g.x, (v[k].y - mean) * inv * g.y,
                           (v[k].z - mean) * inv * g.z, (v[k].w - mean) * inv * g.w);
    if (b) {
      const float4 bb = load4<float>(b + 4 * c);
      o.x += bb.x;
      o.y += bb.y;
      o.z += bb.z;
      o.w += bb.w;
    }
    store4<float>(X + (int64_t)r * D + 4 * c, o);
    if (Y) store4<TY>(Y + (int64_t)r * D + 4 * c, o);
  }
}

template <typename TR, typename TY>
__global__ void __launch_bounds__(256) add_ln_warp(float* __restrict__ X, const TR* __restrict__ R,
                                                   const float* __restrict__ w,
                                                   const float* __restrict__ b,
                                                   TY* __restrict__ Y, int M, int D, float eps,
                                                   const int32_t* __restrict__ rows) {
  const int lane = threadIdx.x & 31;
  const int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (i >= M) return;
  const int src = rows ? rows[i] : i;
  const int nc4 = D >> 2;
  float4 v[kMaxChunks];
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = lane + 32 * k;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < nc4) {
      x = load4<float>(X + (int64_t)src * D + 4 * c);
      if (R && !rows) {
        float4 rr = load4<TR>(R + (int64_t)src * D + 4 * c);
        x.x += rr.x; x.y += rr.y; x.z += rr.z; x.w += rr.w;
        store4<float>(X + (int64_t)src * D + 4 * c, x);
      }
    }
    v[k] = x;
  }
  float mean, inv;
  row_stats(v, lane, nc4, D, eps, mean, inv);
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = lane + 32 * k;
    if (c >= nc4) break;
    float4 g = load4<float>(w + 4 * c);
    float4 o = make_float4((v[k].x - mean) * inv * g.x, (v[k].y - mean) * inv * g.y,
                           (v[k].z - mean) * inv * g.z, (v[k].w - mean) * inv * g.w);
    if (b) {
      float4 bb = load4<float>(b + 4 * c);
      o.x += bb.x; o.y += bb.y; o.z += bb.z; o.w += bb.w;
    }
    store4<TY>(Y + (int64_t)i * D + 4 * c, o);
  }
}

// ---- e4m3 (the FP8 variant's GEMM operands) ----
// Two floats to an e4m3 pair, rounded to nearest even, saturating at +-448;
// the low byte holds a (cvt puts its first source in the high byte).
__device__ __forceinline__ uint32_t e4m3x2(float a, float b) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(b), "f"(a));
  return r;
}
// four consecutive values times s -> four e4m3 codes in memory order
__device__ __forceinline__ uint32_t e4m3x4(float4 v, float s) {
  const float a = v.x * s, b = v.y * s, c = v.z * s, d = v.w * s;
  return e4m3x2(a, b) | (e4m3x2(c, d) << 16);
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// the row scale amax / 448 and its inverse 448 / amax, both correctly rounded
__device__ __forceinline__ void e4m3_scales(float amax, float& scale, float& inv) {
  if (amax > 0.f) {
    scale = __fdiv_rn(amax, 448.f);
    inv = __fdiv_rn(448.f, amax);
  } else {
    scale = 1.f;
    inv = 0.f;
  }
}

// one warp per row, two passes over the row (amax, then the codes); cols % 4 == 0
template <typename T>
__global__ void __launch_bounds__(256) quant_rows_kernel(const T* __restrict__ x, int64_t rows,
                                                         int cols, uint8_t* __restrict__ q,
                                                         float* __restrict__ scale) {
  const int lane = threadIdx.x & 31;
  const int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (i >= rows) return;
  const T* row = x + i * cols;
  float amax = 0.f;
  for (int c = 4 * lane; c < cols; c += 128) {
    const float4 v = load4<T>(row + c);
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  amax = warp_max(amax);
  float sc, inv;
  e4m3_scales(amax, sc, inv);
  uint32_t* qrow = reinterpret_cast<uint32_t*>(q + i * cols);
  for (int c = 4 * lane; c < cols; c += 128) qrow[c >> 2] = e4m3x4(load4<T>(row + c), inv);
  if (lane == 0) scale[i] = sc;
}

// LN(X) * w (+ b) of a row held in registers (as add_ln_warp), then quantised
__global__ void __launch_bounds__(256) ln_e4m3_warp(const float* __restrict__ X,
                                                    const float* __restrict__ w,
                                                    const float* __restrict__ b,
                                                    uint8_t* __restrict__ q,
                                                    float* __restrict__ scale, int64_t M, int D,
                                                    float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (i >= M) return;
  const int nc4 = D >> 2;
  float4 v[kMaxChunks];
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = lane + 32 * k;
    v[k] = c < nc4 ? load4<float>(X + i * D + 4 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float mean, invs;
  row_stats(v, lane, nc4, D, eps, mean, invs);
  float amax = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = lane + 32 * k;
    if (c >= nc4) break;
    const float4 g = load4<float>(w + 4 * c);
    float4 o = make_float4((v[k].x - mean) * invs * g.x, (v[k].y - mean) * invs * g.y,
                           (v[k].z - mean) * invs * g.z, (v[k].w - mean) * invs * g.w);
    if (b) {
      const float4 bb = load4<float>(b + 4 * c);
      o.x += bb.x; o.y += bb.y; o.z += bb.z; o.w += bb.w;
    }
    v[k] = o;
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(o.x), fabsf(o.y)), fmaxf(fabsf(o.z), fabsf(o.w))));
  }
  amax = warp_max(amax);
  float sc, inv;
  e4m3_scales(amax, sc, inv);
  uint32_t* qrow = reinterpret_cast<uint32_t*>(q + i * D);
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = lane + 32 * k;
    if (c >= nc4) break;
    qrow[c] = e4m3x4(v[k], inv);
  }
  if (lane == 0) scale[i] = sc;
}

// ---- e4m3 with one static scale per tensor (SJ_PREC_FP8_TENSOR) ----
// The scale s is read from device memory (calibrated by the engine); every row
// is quantised as x / s (RN, saturating) and its entry of the row-scale array
// the GEMM epilogue reads is set to s.
__device__ __forceinline__ float static_inv(float s) { return s > 0.f ? __fdiv_rn(1.f, s) : 0.f; }

// LN(X) * w (+ b) as ln_e4m3_warp, quantised with the tensor's scale
template <typename TX>
__global__ void __launch_bounds__(256) ln_e4m3_static_warp(const TX* __restrict__ X,
                                                           const float* __restrict__ w,
                                                           const float* __restrict__ b,
                                                           uint8_t* __restrict__ q,
                                                           float* __restrict__ sa,
                                                           const float* __restrict__ s_t,
                                                           int64_t M, int D, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (i >= M) return;
  const int nc4 = D >> 2;
  float4 v[kMaxChunks];
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = lane + 32 * k;
    v[k] = c < nc4 ? load4<TX>(X + i * D + 4 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float mean, invs;
  row_stats(v, lane, nc4, D, eps, mean, invs);
  const float st = *s_t, inv = static_inv(st);
  uint32_t* qrow = reinterpret_cast<uint32_t*>(q + i * D);
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = lane + 32 * k;
    if (c >= nc4) break;
    const float4 g = load4<float>(w + 4 * c);
    float4 o = make_float4((v[k].x - mean) * invs * g.x, (v[k].y - mean) * invs * g.y,
                           (v[k].z - mean) * invs * g.z, (v[k].w - mean) * invs * g.w);
    if (b) {
      const float4 bb = load4<float>(b + 4 * c);
      o.x += bb.x; o.y += bb.y; o.z += bb.z; o.w += bb.w;
    }
    qrow[c] = e4m3x4(o, inv);
  }
  if (lane == 0) sa[i] = st;
}

// ln_e4m3_static_warp for a bf16 X with D = 256 NC (the per-tensor FP8
// variant's LayerNorm, whose output is rounded to e4m3): each lane holds NC
// chunks of 8 values (16-byte loads), chunk k at columns 8 (lane + 32 k).
// Fewer instructions per row than the generic kernel: the mean and variance
// are multiplied by the constant 1/D and the inverse deviation is rsqrtf
// (each within a few ulp of the division and 1/sqrtf the bf16 mode uses).
template <int NC>
__global__ void __launch_bounds__(128) ln_e4m3_static_bf16x8(const bf16* __restrict__ X,
                                                             const float* __restrict__ w,
                                                             const float* __restrict__ b,
                                                             uint8_t* __restrict__ q,
                                                             float* __restrict__ sa,
                                                             const float* __restrict__ s_t,
                                                             int64_t M, float eps) {
  constexpr int D = 256 * NC;
  constexpr float kInvD = 1.0f / (float)D;
  const int lane = threadIdx.x & 31;
  const int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (i >= M) return;
  float v[NC][8];
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    const uint4 t = *reinterpret_cast<const uint4*>(X + i * D + 8 * (lane + 32 * k));
    const uint32_t tw[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&tw[e]));
      v[k][2 * e] = f.x;
      v[k][2 * e + 1] = f.y;
    }
  }
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < NC; ++k)
#pragma unroll
    for (int e = 0; e < 8; ++e) s += v[k][e];
  const float mean = warp_sum(s) * kInvD;
  float d2 = 0.f;
#pragma unroll
  for (int k = 0; k < NC; ++k)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      v[k][e] -= mean;
      d2 = fmaf(v[k][e], v[k][e], d2);
    }
  const float invs = rsqrtf(warp_sum(d2) * kInvD + eps);
  const float st = *s_t, inv = static_inv(st);
#pragma unroll
  for (int k = 0; k < NC; ++k) {
    const int c = 8 * (lane + 32 * k);
    uint32_t code[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float4 g = load4<float>(w + c + 4 * h);
      float4 o = make_float4(v[k][4 * h] * invs * g.x, v[k][4 * h + 1] * invs * g.y,
                             v[k][4 * h + 2] * invs * g.z, v[k][4 * h + 3] * invs * g.w);
      if (b) {
        const float4 bb = load4<float>(b + c + 4 * h);
        o.x += bb.x; o.y += bb.y; o.z += bb.z; o.w += bb.w;
      }
      code[h] = e4m3x4(o, inv);
    }
    *reinterpret_cast<uint2*>(q + i * D + c) = make_uint2(code[0], code[1]);
  }
  if (lane == 0) sa[i] = st;
}

// rows of x quantised with the tensor's scale (the identity norm of layer 0)
template <typename TX>
__global__ void __launch_bounds__(256) quant_rows_static_kernel(const TX* __restrict__ x,
                                                                int64_t rows, int cols,
                                                                uint8_t* __restrict__ q,
                                                                float* __restrict__ sa,
                                                                const float* __restrict__ s_t) {
  const int lane = threadIdx.x & 31;
  const int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (i >= rows) return;
  const float st = *s_t, inv = static_inv(st);
  uint32_t* qrow = reinterpret_cast<uint32_t*>(q + i * cols);
  for (int c = 4 * lane; c < cols; c += 128) qrow[c >> 2] = e4m3x4(load4<TX>(x + i * cols + c), inv);
  if (lane == 0) sa[i] = st;
}

// amax |x| over n values into *amax (float bits compared as unsigned, values >= 0)
template <typename T>
__global__ void __launch_bounds__(256) amax_kernel(const T* __restrict__ x, int64_t n,
                                                   unsigned* __restrict__ amax) {
  float m = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(static_cast<float>(x[i])));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0 && m > 0.f) atomicMax(amax, __float_as_uint(m));
}

// s[i] = amax[i] * margin / 448 (1 where nothing was seen)
__global__ void scales_from_amax_kernel(const unsigned* __restrict__ amax, float* __restrict__ s,
                                        int n, float margin) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float a = __uint_as_float(amax[i]);
  s[i] = a > 0.f ? __fdiv_rn(a * margin, 448.f) : 1.f;
}

// x quantised with one scale (weights, per tensor): q = e4m3(x * inv), and
// the row-scale array filled with s
__global__ void quant_tensor_kernel(const float* __restrict__ x, int64_t n4, float inv, float s,
                                    uint8_t* __restrict__ q, float* __restrict__ sw, int rows) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n4) reinterpret_cast<uint32_t*>(q)[i] = e4m3x4(reinterpret_cast<const float4*>(x)[i], inv);
  if (i < rows) sw[i] = s;
}

// ---- generic widths: one block per row, row staged in shared memory ----
__device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = 0.f;
  for (int k = 0; k < nw; ++k) t += red[k];
  return t;
}

template <typename TR, typename TY>
__global__ void add_ln_block(float* __restrict__ X, const TR* __restrict__ R,
                             const float* __restrict__ w, const float* __restrict__ b,
                             TY* __restrict__ Y, int M, int D, float eps,
                             const int32_t* __restrict__ rows, const int64_t* __restrict__ ids,
                             const float* __restrict__ emb, int V, int* __restrict__ bad) {
  extern __shared__ float srow[];
  __shared__ float red[32];
  const int i = blockIdx.x;
  if (i >= M) return;
  const int src = rows ? rows[i] : i;
  int64_t id = 0;
  bool ok = true;
  if (ids) {
    id = ids[i];
    ok = id >= 0 && id < V;
    if (!ok && threadIdx.x == 0) *bad = 1;
  }
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    float x;
    if (ids) {
      x = ok ? emb[id * (int64_t)D + j] : 0.f;
    } else {
      x = X[(int64_t)src * D + j];
      if (R && !rows) {
        x += io<TR>::to_f(R[(int64_t)src * D + j]);
        X[(int64_t)src * D + j] = x;
      }
    }
    srow[j] = x;
  }
  __syncthreads();
  float s = 0.f;
  for (int j = threadIdx.x; j < D; j += blockDim.x) s += srow[j];
  float mean = block_sum(s, red) / (float)D;
  float q = 0.f;
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    float d = srow[j] - mean;
    q += d * d;
  }
  float inv = 1.0f / sqrtf(block_sum(q, red) / (float)D + eps);
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    float o = (srow[j] - mean) * inv * w[j];
    if (b) o += b[j];
    if (ids) {
      X[(int64_t)i * D + j] = o;
      if (Y) Y[(int64_t)i * D + j] = io<TY>::cvt(o);
    } else {
      Y[(int64_t)i * D + j] = io<TY>::cvt(o);
    }
  }
}

__global__ void cast_bf16_kernel(const float* __restrict__ X, bf16* __restrict__ Y, int64_t n) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) Y[i] = __float2bfloat16(X[i]);
}

// rows[i] of X (bf16 [*, D]) -> the same rows of Y (fp32), one warp per row
__global__ void __launch_bounds__(256) widen_rows_kernel(const bf16* __restrict__ X,
                                                         float* __restrict__ Y,
                                                         const int32_t* __restrict__ rows, int n,
                                                         int D) {
  const int lane = threadIdx.x & 31;
  const int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (i >= n) return;
  const int64_t r = rows[i];
  for (int c = 4 * lane; c < D; c += 128) store4<float>(Y + r * D + c, load4<bf16>(X + r * D + c));
}

// bf16 -> fp32, four values per thread (n % 4 == 0)
__global__ void widen_f32_kernel(const bf16* __restrict__ X, float* __restrict__ Y, int64_t n4) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n4) store4<float>(Y + 4 * i, load4<bf16>(X + 4 * i));
}

bool warp_path(int D) { return D % 4 == 0 && D <= 4 * 32 * kMaxChunks; }

}  // namespace

template <typename TY>
cudaError_t embed_ln(const int64_t* ids, int T, const float* emb, int V, int D, const float* w,
                     float eps, float* X, TY* Y, int* bad, cudaStream_t st, const float* pos_emb,
                     const int32_t* pos, int max_pos, const float* b) {
  if (T <= 0) return cudaSuccess;
  if (warp_path(D)) {
    embed_ln_warp<TY><<<(T + 7) / 8, 256, 0, st>>>(ids, T, emb, V, D, w, eps, X, Y, bad, pos_emb,
                                                    pos, max_pos, b);
  } else if (pos_emb || b) {
    return cudaErrorInvalidValue;  // positions / bias: the warp-per-row form (D <= 1024) only
  } else {
    add_ln_block<float, TY><<<T, 128, D * sizeof(float), st>>>(X, nullptr, w, nullptr, Y, T, D,
                                                               eps, nullptr, ids, emb, V, bad);
  }
  return cudaGetLastError();
}

template <typename TR, typename TY>
cudaError_t add_ln(float* X, const TR* R, const float* w, const float* b, TY* Y, int M, int D,
                   float eps, const int32_t* rows, cudaStream_t st) {
  if (M <= 0) return cudaSuccess;
  if (warp_path(D)) {
    add_ln_warp<TR, TY><<<(M + 7) / 8, 256, 0, st>>>(X, R, w, b, Y, M, D, eps, rows);
  } else {
    add_ln_block<TR, TY><<<M, 128, D * sizeof(float), st>>>(X, R, w, b, Y, M, D, eps, rows,
                                                            nullptr, nullptr, 0, nullptr);
  }
  return cudaGetLastError();
}

cudaError_t cast_bf16(const float* X, bf16* Y, int64_t n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  cast_bf16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(X, Y, n);
  return cudaGetLastError();
}

template <typename T>
cudaError_t quant_rows_e4m3(const T* x, int64_t rows, int cols, uint8_t* q, float* scale,
                            cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (cols <= 0 || cols % 4 != 0) return cudaErrorInvalidValue;
  quant_rows_kernel<T><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(x, rows, cols, q, scale);
  return cudaGetLastError();
}
template cudaError_t quant_rows_e4m3<float>(const float*, int64_t, int, uint8_t*, float*,
                                            cudaStream_t);
template cudaError_t quant_rows_e4m3<bf16>(const bf16*, int64_t, int, uint8_t*, float*,
                                           cudaStream_t);

cudaError_t ln_e4m3(const float* X, const float* w, const float* b, uint8_t* q, float* scale,
                    int64_t rows, int D, float eps, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (D % 128 != 0 || D > 4 * 32 * kMaxChunks) return cudaErrorInvalidValue;
  ln_e4m3_warp<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(X, w, b, q, scale, rows, D, eps);
  return cudaGetLastError();
}

template <typename TX>
cudaError_t ln_e4m3_static(const TX* X, const float* w, const float* b, uint8_t* q, float* sa,
                           const float* s_t, int64_t rows, int D, float eps, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (D % 128 != 0 || D > 4 * 32 * kMaxChunks) return cudaErrorInvalidValue;
  if constexpr (std::is_same<TX, bf16>::value) {
    // 16-byte loads, registers for exactly the row's chunks; blocks of 4 rows
    const unsigned g4 = (unsigned)((rows + 3) / 4);
    switch (D) {
      case 512: ln_e4m3_static_bf16x8<2><<<g4, 128, 0, st>>>(X, w, b, q, sa, s_t, rows, eps);
        return cudaGetLastError();
      case 768: ln_e4m3_static_bf16x8<3><<<g4, 128, 0, st>>>(X, w, b, q, sa, s_t, rows, eps);
        return cudaGetLastError();
      case 1024: ln_e4m3_static_bf16x8<4><<<g4, 128, 0, st>>>(X, w, b, q, sa, s_t, rows, eps);
        return cudaGetLastError();
      default: break;
    }
  }
  ln_e4m3_static_warp<TX><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(X, w, b, q, sa, s_t, rows,
                                                                      D, eps);
  return cudaGetLastError();
}
template cudaError_t ln_e4m3_static<float>(const float*, const float*, const float*, uint8_t*,
                                           float*, const float*, int64_t, int, float, cudaStream_t);
template cudaError_t ln_e4m3_static<bf16>(const bf16*, const float*, const float*, uint8_t*,
                                          float*, const float*, int64_t, int, float, cudaStream_t);

template <typename TX>
cudaError_t quant_rows_static(const TX* x, int64_t rows, int cols, uint8_t* q, float* sa,
                              const float* s_t, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (cols <= 0 || cols % 4 != 0) return cudaErrorInvalidValue;
  quant_rows_static_kernel<TX><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(x, rows, cols, q, sa,
                                                                           s_t);
  return cudaGetLastError();
}
template cudaError_t quant_rows_static<float>(const float*, int64_t, int, uint8_t*, float*,
                                              const float*, cudaStream_t);
template cudaError_t quant_rows_static<bf16>(const bf16*, int64_t, int, uint8_t*, float*,
                                             const float*, cudaStream_t);

cudaError_t widen_rows_f32(const bf16* X, float* Y, const int32_t* rows, int n, int D,
                           cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  if (D % 4 != 0) return cudaErrorInvalidValue;
  widen_rows_kernel<<<(unsigned)((n + 7) / 8), 256, 0, st>>>(X, Y, rows, n, D);
  return cudaGetLastError();
}

cudaError_t widen_f32(const bf16* X, float* Y, int64_t n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  if (n % 4 != 0) return cudaErrorInvalidValue;
  const int64_t n4 = n / 4;
  widen_f32_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(X, Y, n4);
  return cudaGetLastError();
}

template <typename T>
cudaError_t amax_abs(const T* x, int64_t n, unsigned* amax, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 8);
  amax_kernel<T><<<(unsigned)blocks, 256, 0, st>>>(x, n, amax);
  return cudaGetLastError();
}
template cudaError_t amax_abs<float>(const float*, int64_t, unsigned*, cudaStream_t);
template cudaError_t amax_abs<bf16>(const bf16*, int64_t, unsigned*, cudaStream_t);

cudaError_t scales_from_amax(const unsigned* amax, float* s, int n, float margin,
                             cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  scales_from_amax_kernel<<<(n + 255) / 256, 256, 0, st>>>(amax, s, n, margin);
  return cudaGetLastError();
}

cudaError_t quant_tensor_e4m3(const float* x, int64_t n, int rows, float amax, uint8_t* q,
                              float* sw, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  if (n % 4 != 0) return cudaErrorInvalidValue;
  const float s = amax > 0.f ? amax / 448.f : 1.f, inv = amax > 0.f ? 448.f / amax : 0.f;
  const int64_t n4 = n / 4, work = std::max<int64_t>(n4, rows);
  quant_tensor_kernel<<<(unsigned)((work + 255) / 256), 256, 0, st>>>(x, n4, inv, s, q, sw, rows);
  return cudaGetLastError();
}

template cudaError_t embed_ln<float>(const int64_t*, int, const float*, int, int, const float*,
                                     float, float*, float*, int*, cudaStream_t,
                                     const float*, const int32_t*, int, const float*);
template cudaError_t embed_ln<bf16>(const int64_t*, int, const float*, int, int, const float*,
                                     float, float*, bf16*, int*, cudaStream_t,
                                     const float*, const int32_t*, int, const float*);
template cudaError_t add_ln<float, float>(float*, const float*, const float*, const float*,
                                          float*, int, int, float, const int32_t*, cudaStream_t);
template cudaError_t add_ln<bf16, bf16>(float*, const bf16*, const float*, const float*, bf16*,
                                        int, int, float, const int32_t*, cudaStream_t);
template cudaError_t add_ln<float, bf16>(float*, const float*, const float*, const float*, bf16*,
                                         int, int, float, const int32_t*, cudaStream_t);
template cudaError_t add_ln<bf16, float>(float*, const bf16*, const float*, const float*, float*,
                                         int, int, float, const int32_t*, cudaStream_t);

}  // namespace sjb
