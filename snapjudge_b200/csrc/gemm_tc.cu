// gemm_tc.cu — persistent warp-specialised tcgen05 GEMM for the encoder projections.
//
// C = A W^T with A [M, K] bf16 activations and W [N, K] bf16 weights in the
// checkpoint layout (both K-major), fp32 accumulation in TMEM — the
// contraction of the reference gemm_nt / gemm_geglu (src/tensor.cpp:108-151).
//
// CTA (320 threads, one per SM, persistent over output tiles of 128 x BN):
//   warp 0      TMA producer: A 128x64 and W BNx64 boxes, 128-byte swizzle,
//               STAGES-deep ring of shared-memory stages (full/empty mbarriers)
//   warp 1      TMEM owner + MMA issuer: 4 x tcgen05.mma (K = 16) per stage
//               into one of two TMEM accumulators (2 x BN fp32 columns)
//   warps 2-9   epilogue: tcgen05.ld of the accumulator (warp w reads TMEM
//               lanes 32*(w%4)..+31 = tile rows; warps 2-5 take the first half
//               of the tile's columns, warps 6-9 the second), then one of
//                 STORE  C = bf16(acc + bias, act)           (act: GELU-erf / ReLU)
//                 RESID  X += acc (+bias)                    (fp32 residual stream)
//                 GEGLU  G = bf16(gelu(acc_g) * acc_u)        (W tile = 128 gate rows
//                                                             + 128 up rows of [Wg; Wu];
//                                                             erf per A&S 7.1.26, packed fp32)
//                 ROPE   QKV = bf16(rotate-half(acc)) on q/k heads of 64, v as is
// F8 instances take e4m3 A and W (tcgen05 kind::f8f6f4, 128-element k-blocks:
// the same 128-byte swizzled rows) with a scale per A row and per W row; the
// epilogue multiplies the fp32 accumulator by both before its own work.
// The epilogue of tile i overlaps the MMAs of tile i+1 (double-buffered TMEM);
// each epilogue warp hands its accumulator back with a plain remote arrive.
// Every mbarrier wait is bounded and sleeps in hardware between tests
// (mbar_wait<true>: waiters that re-issue try_wait slow the MMA issue); a
// wait that runs out records an error code and the CTA winds down (no trap).
#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"
#include "tc_host.h"

namespace sjb {

__device__ int g_gemm_tc_err;  // error sink when the caller passes no flag

namespace {
using namespace tc;

constexpr int BM = 128, BK = 64;
constexpr int kEpiWarps = 8;  // epilogue warps of every instance but TC_GEGLU8's
// GEGLU with e4m3 output codes (SJ_PREC_FP8_TENSOR's Wi projection): an
// instance of its own with 16 epilogue warps, 32 output columns each, and no
// staging buffers.  Its epilogue is short of registers, not of work, so twice
// the warps hide twice the TMEM-load and arithmetic latency.
constexpr int TC_GEGLU8 = 5;
template <int EPI>
__host__ __device__ constexpr bool is_geglu() { return EPI == TC_GEGLU || EPI == TC_GEGLU8; }
template <int EPI>
__host__ __device__ constexpr int epi_warps() { return EPI == TC_GEGLU8 ? 16 : kEpiWarps; }
template <int EPI>
__host__ __device__ constexpr int threads_for() { return 64 + 32 * epi_warps<EPI>(); }

struct EpiArgs {
  const float* bias;
  int act;
  bf16* C;
  int ldc;               // output row pitch in elements
  float* resid;          // fp32 [M, ldr]
  int ldr;
  const float* cos_t;    // [max_pos, 32]
  const float* sin_t;
  const int32_t* pos;    // [M]
  int rope_cols;         // columns [0, rope_cols) are rotated q/k heads
  const float* sa;       // F8: [M] scale of each A row
  const float* sw;       // F8: [w_rows] scale of each W row
  // GEGLU with e4m3 output (SJ_PREC_FP8_TENSOR): codes of v / *c8_scale into
  // C8 [M, ldc] (bytes) instead of bf16 C, c8_rowscale[row] = *c8_scale
  uint8_t* C8;
  const float* c8_scale;
  float* c8_rowscale;
  int uniform;           // F8: sa and sw hold one value each (per-tensor scales)
  int* err;
};

// Epilogues move data through a per-warp pair of 4 KB swizzled shared-memory
// buffers (8 KB x 8 warps): bf16 outputs are staged as 32 x 64 chunks and
// written with TMA stores; the fp32 residual X is read as 32 x 32 chunks with
// TMA loads (two in flight), updated, and written back with TMA.  GEGLU on
// 128-column tiles (32 outputs per warp) and 64-column tiles store directly.
template <int BN, int EPI>
__host__ __device__ constexpr bool staged() {
  return EPI != TC_GEGLU8 && (BN == 256 || (BN == 128 && EPI != TC_GEGLU));
}
constexpr int kStageBytesPerWarp = 2 * 32 * 128;
template <int BN, int EPI>
__host__ __device__ constexpr int out_bytes() { return staged<BN, EPI>() ? kEpiWarps * kStageBytesPerWarp : 0; }
template <int BN, int EPI, bool PAIR>
__host__ __device__ constexpr int stages_for() {
  return PAIR ? (staged<BN, EPI>() ? 5 : 6)
              : (BN >= 256 ? (staged<BN, EPI>() ? 3 : 4) : (staged<BN, EPI>() ? 5 : 6));
}

__device__ __forceinline__ void record_err(int* err, int code) {
  atomicCAS(err ? err : &g_gemm_tc_err, 0, code);
}

// ---- GEGLU gate on column pairs, packed fp32 (fma/mul .f32x2) ----
// erf by Abramowitz & Stegun, Handbook of Mathematical Functions, eq. 7.1.26:
//   erfc(z) = (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-z^2),
//   t = 1 / (1 + p z), z >= 0, |error| <= 1.5e-7,
// with z = |x| / sqrt(2), so 1 - Phi(|x|) = erfc(z) / 2 and
//   gelu(x) = x Phi(x) = relu(x) - |x| (1 - Phi(|x|)).
// The reciprocal and exponential are the approximate hardware ones (relative
// error ~2^-22); the gate is then rounded to bf16, so the result matches the
// erf GELU to within one bf16 rounding step.
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 pk2(float a, float b) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 unpk2(f32x2 v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f32x2 splat2(float a) { return pk2(a, a); }
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The GEGLU gate with the tanh form of GELU,
//   gelu(x) ~ x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))) / 2,
// one MUFU operation per value instead of two.  It differs from the erf form
// by at most 4.7e-4 (at |x| ~ 2.7), far below the e4m3 rounding of the values
// it is used for: only the GEGLU with e4m3 output (TC_GEGLU8).
__device__ __forceinline__ float2 geglu_pair_tanh(float ga, float gb, float ua, float ub) {
  constexpr float k0 = 0.7978845608028654f;          // sqrt(2 / pi)
  constexpr float k1 = 0.044715f * 0.7978845608028654f;
  const f32x2 g = pk2(ga, gb);
  const float2 in = unpk2(mul2(g, fma2(mul2(g, g), splat2(k1), splat2(k0))));
  const f32x2 t = pk2(tanh_approx(in.x), tanh_approx(in.y));
  const f32x2 hg = mul2(g, splat2(0.5f));
  return unpk2(mul2(fma2(hg, t, hg), pk2(ua, ub)));
}

// (gelu(ga), gelu(gb)), packed
__device__ __forceinline__ f32x2 gelu2(float ga, float gb) {
  constexpr float kP = 0.3275911f * 0.70710678118654752f;  // p / sqrt(2)
  // -a_i / 2: the polynomial comes out as -erfc(z) / 2 before the exponential
  constexpr float kA1 = -0.5f * 0.254829592f, kA2 = 0.5f * 0.284496736f,
                  kA3 = -0.5f * 1.421413741f, kA4 = 0.5f * 1.453152027f,
                  kA5 = -0.5f * 1.061405429f;
  constexpr float kE = -0.5f * 1.4426950408889634f;  // -z^2 log2(e) = x^2 * kE
  const f32x2 ax = pk2(fabsf(ga), fabsf(gb));
  const float2 d = unpk2(fma2(ax, splat2(kP), splat2(1.f)));
  const f32x2 t = pk2(rcp_approx(d.x), rcp_approx(d.y));
  f32x2 p = fma2(t, splat2(kA5), splat2(kA4));
  p = fma2(t, p, splat2(kA3));
  p = fma2(t, p, splat2(kA2));
  p = fma2(t, p, splat2(kA1));
  p = mul2(p, t);
  const f32x2 g = pk2(ga, gb);
  const float2 e = unpk2(mul2(mul2(g, g), splat2(kE)));
  const f32x2 h = mul2(p, pk2(ex2_approx(e.x), ex2_approx(e.y)));  // -(1 - Phi(|x|))
  return fma2(ax, h, pk2(fmaxf(ga, 0.f), fmaxf(gb, 0.f)));
}

// (gelu(ga) * ua, gelu(gb) * ub)
__device__ __forceinline__ float2 geglu_pair(float ga, float gb, float ua, float ub) {
  return unpk2(mul2(gelu2(ga, gb), pk2(ua, ub)));
}

// The STORE epilogue's 32 accumulator values: + bias[0..32) (when given), then
// the activation, chosen once per call so that the unrolled loop holds one
// activation's code; GELU is the GEGLU gate's erf approximation above.
template <int ACT>
__device__ __forceinline__ void bias_act32(const uint32_t (&r)[32], const float* bias, float* v) {
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    float a0 = __uint_as_float(r[j]), a1 = __uint_as_float(r[j + 1]);
    if (bias) {
      const float2 bb = *reinterpret_cast<const float2*>(bias + j);
      a0 += bb.x;
      a1 += bb.y;
    }
    if (ACT == ACT_GELU) {
      const float2 g = unpk2(gelu2(a0, a1));
      a0 = g.x;
      a1 = g.y;
    } else if (ACT == ACT_RELU) {
      a0 = fmaxf(a0, 0.f);
      a1 = fmaxf(a1, 0.f);
    }
    v[j] = a0;
    v[j + 1] = a1;
  }
}
__device__ __forceinline__ void bias_act32(const uint32_t (&r)[32], const float* bias, int act,
                                           float* v) {
  if (act == ACT_GELU) bias_act32<ACT_GELU>(r, bias, v);
  else if (act == ACT_RELU) bias_act32<ACT_RELU>(r, bias, v);
  else bias_act32<ACT_NONE>(r, bias, v);
}

// 32 values to e4m3 codes (x * inv, RN, saturating at +-448) in memory order,
// written as two 16-byte stores
__device__ __forceinline__ void store_e4m3x32(uint8_t* dst, const float* v, float inv) {
  uint32_t w[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint16_t lo, hi;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(v[4 * j + 1] * inv), "f"(v[4 * j] * inv));
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(v[4 * j + 3] * inv), "f"(v[4 * j + 2] * inv));
    w[j] = (uint32_t)lo | ((uint32_t)hi << 16);
  }
  uint4* d = reinterpret_cast<uint4*>(dst);
  d[0] = make_uint4(w[0], w[1], w[2], w[3]);
  d[1] = make_uint4(w[4], w[5], w[6], w[7]);
}
// four values to four e4m3 codes (RN, saturating) in memory order
__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d) {
  uint16_t lo, hi;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(b), "f"(a));
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(d), "f"(c));
  return (uint32_t)lo | ((uint32_t)hi << 16);
}
__device__ __forceinline__ void store_bf16x32(bf16* dst, const float* v) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[q * 8 + 2 * e], v[q * 8 + 2 * e + 1]);
      w[e] = *reinterpret_cast<uint32_t*>(&h);
    }
    d[q] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// r[j] *= sa * sw[j] for 32 accumulator columns (sw 16-byte aligned): the
// e4m3 operands' row and channel scales
__device__ __forceinline__ void unscale32(uint32_t (&r)[32], float sa, const float* sw, float su) {
  if (su != 0.f) {  // per-tensor scales: one product for every element
#pragma unroll
    for (int k = 0; k < 32; ++k) r[k] = __float_as_uint(__uint_as_float(r[k]) * su);
    return;
  }
  const float4* s4 = reinterpret_cast<const float4*>(sw);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float4 w = __ldg(s4 + k);
    r[4 * k] = __float_as_uint(__uint_as_float(r[4 * k]) * (sa * w.x));
    r[4 * k + 1] = __float_as_uint(__uint_as_float(r[4 * k + 1]) * (sa * w.y));
    r[4 * k + 2] = __float_as_uint(__uint_as_float(r[4 * k + 2]) * (sa * w.z));
    r[4 * k + 3] = __float_as_uint(__uint_as_float(r[4 * k + 3]) * (sa * w.w));
  }
}

// unscale16 with the channel scales already in registers
__device__ __forceinline__ void unscale16w(uint32_t (&r)[16], float sa, const float4 (&w)[4],
                                           float su) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float m0 = su != 0.f ? su : sa * w[k].x, m1 = su != 0.f ? su : sa * w[k].y;
    const float m2 = su != 0.f ? su : sa * w[k].z, m3 = su != 0.f ? su : sa * w[k].w;
    r[4 * k] = __float_as_uint(__uint_as_float(r[4 * k]) * m0);
    r[4 * k + 1] = __float_as_uint(__uint_as_float(r[4 * k + 1]) * m1);
    r[4 * k + 2] = __float_as_uint(__uint_as_float(r[4 * k + 2]) * m2);
    r[4 * k + 3] = __float_as_uint(__uint_as_float(r[4 * k + 3]) * m3);
  }
}

// 8 floats -> 8 bf16 (16 bytes)
__device__ __forceinline__ uint4 pack_bf16x8(const float* v) {
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
    w[e] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <int BN, int EPI, bool PAIR, bool F8>
__global__ void __launch_bounds__(threads_for<EPI>(), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
                   const __grid_constant__ CUtensorMap mapC, int M, int n_tiles, int K, int up_row0,
                   EpiArgs ep) {
  // PAIR: a cluster of 2 CTAs computes 256 x BN tiles with the pair MMA; each CTA
  // holds 128 rows of A and BN/2 rows of B per stage and 128 rows of the result.
  constexpr int STAGES = stages_for<BN, EPI, PAIR>();
  constexpr bool STAGED = staged<BN, EPI>();
  // the residual epilogue releases the accumulator as soon as it is in registers
  constexpr bool EARLY = (EPI == TC_RESID || EPI == TC_RESID16) && STAGED;
  constexpr int BROWS = PAIR ? BN / 2 : BN;  // B rows this CTA loads per stage
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int B_BYTES = BROWS * BK * 2;
  constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  constexpr int TILE_M = PAIR ? 2 * BM : BM;
  constexpr uint32_t IDESC = F8 ? idesc_e4m3(TILE_M, BN) : idesc_bf16(TILE_M, BN, false, false);
  constexpr int BKE = F8 ? 2 * BK : BK;  // elements per k-block (128 bytes per row either way)

  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full_bar[STAGES], empty_bar[STAGES], tfull_bar[2], tempty_bar[2], drain_bar;
  constexpr int EPI_WARPS = epi_warps<EPI>();
  __shared__ uint64_t xload_bar[EPI_WARPS][2];  // residual chunk loads (RESID epilogue)
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;

  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_rank() : 0;
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;  // cluster (or CTA) index
  const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int m_tiles = (M + TILE_M - 1) / TILE_M;
  const int num_tiles = m_tiles * n_tiles;
  const int k_blocks = K / BKE;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], EPI_WARPS * (PAIR ? 2 : 1));
    }
    mbar_init(&drain_bar, 1);
    for (int w = 0; w < EPI_WARPS; ++w) {
      mbar_init(&xload_bar[w][0], 1);
      mbar_init(&xload_bar[w][1], 1);
    }
    abort_sh = 0;
    fence_barrier_init();
    tma_prefetch(&mapA);
    tma_prefetch(&mapB);
    if (STAGED) tma_prefetch(&mapC);
  }
  if (warp == 1) {
    if (PAIR) tmem_alloc_pair(&tmem_base_sh, TMEM_COLS);
    else tmem_alloc(&tmem_base_sh, TMEM_COLS);
  }
  fence_before_sync();
  if (PAIR) cluster_sync();  // the peer's barriers exist before anyone signals them
  else __syncthreads();
  fence_after_sync();
  const uint32_t tmem_base = tmem_base_sh;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer (both CTAs of a pair) ----------------
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    for (int t = unit; t < num_tiles && !abort_sh; t += units) {
      const int m0 = (t / n_tiles) * TILE_M + (int)rank * BM, nb = t % n_tiles;
      for (int kb = 0; kb < k_blocks; ++kb) {
        if (!mbar_wait<true>(&empty_bar[stage], phase ^ 1)) {
          record_err(ep.err, 1);
          abort_sh = 1;
          break;
        }
        uint8_t* sa = smem + stage * STAGE_BYTES;
        uint8_t* sb = sa + A_BYTES;
        if (PAIR) {
          // both CTAs' bytes are counted on rank 0's barrier
          const uint32_t bar0 = mapa_shared(smem_u32(&full_bar[stage]), 0);
          if (rank == 0) mbar_expect_tx(&full_bar[stage], 2 * STAGE_BYTES);
          tma_load_2d_pair(sa, &mapA, bar0, kb * BKE, m0);
          const int brow = is_geglu<EPI>() ? (rank == 0 ? nb * BROWS : up_row0 + nb * BROWS)
                                           : nb * BN + (int)rank * BROWS;
          tma_load_2d_pair(sb, &mapB, bar0, kb * BKE, brow);
        } else {
          mbar_expect_tx(&full_bar[stage], STAGE_BYTES);
          tma_load_2d(sa, &mapA, &full_bar[stage], kb * BKE, m0);
          if (is_geglu<EPI>()) {
            tma_load_2d(sb, &mapB, &full_bar[stage], kb * BKE, nb * (BN / 2));
            tma_load_2d(sb + B_BYTES / 2, &mapB, &full_bar[stage], kb * BKE,
                        up_row0 + nb * (BN / 2));
          } else {
            tma_load_2d(sb, &mapB, &full_bar[stage], kb * BKE, nb * BN);
          }
        }
        ++issued;
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
    // drain: every issued copy has landed before the CTA can exit (in a pair,
    // rank 0's barriers count both CTAs' copies; the cluster barrier at the end
    // keeps rank 1 resident until then)
    if (!PAIR || rank == 0) {
      for (int i = 0; i < STAGES && i < issued; ++i) {
        if (--stage < 0) { stage = STAGES - 1; phase ^= 1; }
        if (!mbar_wait<true>(&full_bar[stage], phase)) record_err(ep.err, 2);
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ---------------- MMA issuer (rank 0 of a pair) ----------------
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    for (int t = unit; t < num_tiles && !abort_sh; t += units, ++local) {
      const int b = local & 1;
      const uint32_t aphase = (local >> 1) & 1;
      if (!mbar_wait<true>(&tempty_bar[b], aphase ^ 1)) {
        record_err(ep.err, 3);
        abort_sh = 1;
        break;
      }
      fence_after_sync();
      const uint32_t d = tmem_base + b * BN;
      for (int kb = 0; kb < k_blocks; ++kb) {
        if (!mbar_wait<true>(&full_bar[stage], phase)) {
          record_err(ep.err, 4);
          abort_sh = 1;
          break;
        }
        fence_after_sync();
        const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
        const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // 32 bytes of K per instruction: 16 bf16 or 32 e4m3
          const uint64_t ad = desc_kmajor_sw128(a_addr + kk * 32);
          const uint64_t bd = desc_kmajor_sw128(b_addr + kk * 32);
          if (F8) {
            if (PAIR) mma_e4m3_pair(d, ad, bd, IDESC, (kb | kk) != 0);
            else mma_e4m3(d, ad, bd, IDESC, (kb | kk) != 0);
          } else {
            if (PAIR) mma_bf16_pair(d, ad, bd, IDESC, (kb | kk) != 0);
            else mma_bf16(d, ad, bd, IDESC, (kb | kk) != 0);
          }
        }
        if (PAIR) mma_commit_pair(&empty_bar[stage], 0x3);
        else mma_commit(&empty_bar[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (PAIR) mma_commit_pair(&tfull_bar[b], 0x3);
      else mma_commit(&tfull_bar[b]);
    }
    if (PAIR) mma_commit_pair(&drain_bar, 0x1);
    else mma_commit(&drain_bar);
    if (!mbar_wait<true>(&drain_bar, 0)) record_err(ep.err, 5);
  } else if (warp >= 2) {
    // ---------------- epilogue ----------------
    const int q = warp & 3;             // TMEM lane quarter this warp may access
    const int hf = (warp - 2) >> 2;     // which half of the tile's columns
    // staged store of a 32-row x 64-column bf16 chunk (row = lane): write it
    // 128-byte-swizzled into this warp's staging buffer, then one TMA store
    uint8_t* stg = smem + STAGES * STAGE_BYTES + (warp - 2) * kStageBytesPerWarp;
    int sbuf = 0;
    uint32_t xphase = 0u;  // bit b: parity of this warp's residual-load barrier b
    uint64_t* xb = xload_bar[warp - 2];
    // per-tensor scales (ep.uniform): the product of the row and channel
    // scales is one value, read once; the e4m3 GEGLU output's static scale too
    const float su = F8 && ep.uniform ? ep.sa[0] * ep.sw[0] : 0.f;
    const float s8 = ep.C8 ? *ep.c8_scale : 0.f, inv8 = s8 > 0.f ? 1.f / s8 : 0.f;
    // hand accumulator buffer b back to the MMA warp (rank 0's barrier in a pair)
    auto release = [&](int b) {
      fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        if (PAIR) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty_bar[b]), 0));
        else mbar_arrive(&tempty_bar[b]);
      }
    };
    auto store_chunk = [&](const float* v, int col, int row0) {
      if (lane == 0) bulk_wait_read<1>();  // this buffer's previous store has read it
      __syncwarp();
      uint8_t* rowp = stg + sbuf * (32 * 128) + lane * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          __nv_bfloat162 h = __floats2bfloat162_rn(v[c * 8 + 2 * e], v[c * 8 + 2 * e + 1]);
          w[e] = *reinterpret_cast<uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(rowp + ((c ^ (lane & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&mapC, stg + sbuf * (32 * 128), col, row0);
        bulk_commit();
      }
      sbuf ^= 1;
    };
    int local = 0;
    for (int t = unit; t < num_tiles; t += units, ++local) {
      const int b = local & 1;
      const uint32_t aphase = (local >> 1) & 1;
      const int m0 = (t / n_tiles) * TILE_M + (int)rank * BM, nb = t % n_tiles;
      if (EARLY && lane == 0) {
        // request this tile's first two X chunks while its MMAs still run
        bulk_wait_read<0>();  // the previous tile's stores have read both buffers
        // chunks of 32 rows x 128 bytes: 32 fp32 or (TC_RESID16) 64 bf16 columns
        constexpr int XW = EPI == TC_RESID16 ? 64 : 32;
#pragma unroll
        for (int k = 0; k < 2 && k < BN / 2 / XW; ++k) {
          mbar_expect_tx(&xb[k], 32 * 128);
          tma_load_2d(stg + k * 4096, &mapC, &xb[k], nb * BN + hf * BN / 2 + XW * k, m0 + q * 32);
        }
      }
      // RoPE: this row's cos/sin (32 each, 16-byte loads), fetched before the
      // accumulator is ready so that their latency hides behind the wait
      float cs[32], sn[32];
      if constexpr (EPI == TC_ROPE) {
        constexpr int HEADS = BN / 64;
        const int r = m0 + q * 32 + lane;
        const int h0 = hf * ((HEADS + 1) / 2), h1 = min(HEADS, (hf + 1) * ((HEADS + 1) / 2));
        if (r < M && nb * BN + h0 * 64 < ep.rope_cols && h0 < h1) {
          const int p = ep.pos[r];
          const float4* c4 = reinterpret_cast<const float4*>(ep.cos_t + (int64_t)p * 32);
          const float4* s4 = reinterpret_cast<const float4*>(ep.sin_t + (int64_t)p * 32);
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float4 a = __ldg(c4 + k), z = __ldg(s4 + k);
            cs[4 * k] = a.x; cs[4 * k + 1] = a.y; cs[4 * k + 2] = a.z; cs[4 * k + 3] = a.w;
            sn[4 * k] = z.x; sn[4 * k + 1] = z.y; sn[4 * k + 2] = z.z; sn[4 * k + 3] = z.w;
          }
        } else {
#pragma unroll
          for (int k = 0; k < 32; ++k) { cs[k] = 1.f; sn[k] = 0.f; }
        }
      }
      // the row scale (written before this kernel started) is read before
      // the accumulator wait too
      const int row = m0 + q * 32 + lane;
      const bool live = row < M;
      const float sa = F8 && live && su == 0.f ? ep.sa[row] : 0.f;
      int ok = 1;
      if (lane == 0) ok = mbar_wait<true>(&tfull_bar[b], aphase) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok || abort_sh) {
        if (lane == 0 && !ok) { record_err(ep.err, 6); abort_sh = 1; }
        break;
      }
      fence_after_sync();
      const uint32_t tacc = tmem_base + ((uint32_t)(q * 32) << 16) + b * BN;
      uint32_t r0[32], r1[32];
      if constexpr (EPI == TC_GEGLU8) {
        // this warp: rows q*32 .. q*32+31 of the CTA's 128, output columns
        // hf*32 .. hf*32+31 of the tile's HALF (gate at c, up at HALF + c);
        // codes packed as they are made, 32 bytes per row
        constexpr int HALF = BN / 2;
        static_assert(HALF == 4 * 32, "TC_GEGLU8 runs on 256-column tiles");
        const int c = hf * 32, col = nb * HALF + c;
        tmem_ld32(tacc + c, r0);
        tmem_ld32(tacc + HALF + c, r1);
        tmem_ld_wait();
        release(b);  // the accumulator is in registers
        if constexpr (F8) {
          unscale32(r0, sa, ep.sw + col, su);
          unscale32(r1, sa, ep.sw + up_row0 + col, su);
        }
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float2 o0 = geglu_pair_tanh(__uint_as_float(r0[j]), __uint_as_float(r0[j + 1]),
                                            __uint_as_float(r1[j]), __uint_as_float(r1[j + 1]));
          const float2 o1 = geglu_pair_tanh(__uint_as_float(r0[j + 2]), __uint_as_float(r0[j + 3]),
                                            __uint_as_float(r1[j + 2]), __uint_as_float(r1[j + 3]));
          w[j / 4] = e4m3x4(o0.x * inv8, o0.y * inv8, o1.x * inv8, o1.y * inv8);
        }
        if (live) {
          uint4* d = reinterpret_cast<uint4*>(ep.C8 + (int64_t)row * ep.ldc + col);
          d[0] = make_uint4(w[0], w[1], w[2], w[3]);
          d[1] = make_uint4(w[4], w[5], w[6], w[7]);
          if (nb == 0 && hf == 0) ep.c8_rowscale[row] = s8;
        }
      } else if (EPI == TC_GEGLU && STAGED) {
        constexpr int HALF = BN / 2;    // output columns of the tile
        const int col_base = nb * HALF;
#pragma unroll 1
        for (int c = hf * HALF / 2; c < (hf + 1) * HALF / 2; c += 64) {
          float v[64];
#pragma unroll
          for (int k2 = 0; k2 < 2; ++k2) {
            tmem_ld32(tacc + c + 32 * k2, r0);
            tmem_ld32(tacc + HALF + c + 32 * k2, r1);
            tmem_ld_wait();
            if constexpr (F8) {
              unscale32(r0, sa, ep.sw + col_base + c + 32 * k2, su);
              unscale32(r1, sa, ep.sw + up_row0 + col_base + c + 32 * k2, su);
            }
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const float2 o = geglu_pair(__uint_as_float(r0[j]), __uint_as_float(r0[j + 1]),
                                          __uint_as_float(r1[j]), __uint_as_float(r1[j + 1]));
              v[32 * k2 + j] = o.x;
              v[32 * k2 + j + 1] = o.y;
            }
          }
          if (ep.C8) {  // e4m3 codes at the tensor's static scale, direct stores
            if (live) {
              uint8_t* dst = ep.C8 + (int64_t)row * ep.ldc + col_base + c;
              store_e4m3x32(dst, v, inv8);
              store_e4m3x32(dst + 32, v + 32, inv8);
              if (nb == 0 && c == 0) ep.c8_rowscale[row] = s8;
            }
          } else {
            store_chunk(v, col_base + c, m0 + q * 32);
          }
        }
      } else if (EPI == TC_GEGLU) {
        constexpr int HALF = BN / 2;    // output columns of the tile
        const int col_base = nb * HALF;
#pragma unroll 1
        for (int c = hf * HALF / 2; c < (hf + 1) * HALF / 2; c += 32) {
          tmem_ld32(tacc + c, r0);
          tmem_ld32(tacc + HALF + c, r1);
          tmem_ld_wait();
          if constexpr (F8) {
            unscale32(r0, sa, ep.sw + col_base + c, su);
            unscale32(r1, sa, ep.sw + up_row0 + col_base + c, su);
          }
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float2 o = geglu_pair(__uint_as_float(r0[j]), __uint_as_float(r0[j + 1]),
                                        __uint_as_float(r1[j]), __uint_as_float(r1[j + 1]));
            v[j] = o.x;
            v[j + 1] = o.y;
          }
          if (live && ep.C8) {
            store_e4m3x32(ep.C8 + (int64_t)row * ep.ldc + col_base + c, v, inv8);
            if (nb == 0 && c == 0) ep.c8_rowscale[row] = s8;
          } else if (live) {
            store_bf16x32(ep.C + (int64_t)row * ep.ldc + col_base + c, v);
          }
        }
      } else if (EPI == TC_ROPE) {
        constexpr int HEADS = BN / 64;
        const int col_base = nb * BN;
        const int h0 = hf * ((HEADS + 1) / 2), h1 = min(HEADS, (hf + 1) * ((HEADS + 1) / 2));
#pragma unroll 1
        for (int hh = h0; hh < h1; ++hh) {
          const int c = hh * 64;
          if constexpr (F8) {
            // the head in two passes of 16 + 16 columns, so that the row's
            // cos/sin stay in registers beside them; staged like store_chunk
            const bool rot = col_base + c < ep.rope_cols;
            uint8_t* rowp = stg + sbuf * (32 * 128) + lane * 128;
            if (STAGED) {
              if (lane == 0) bulk_wait_read<1>();
              __syncwarp();
            }
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              uint32_t a[16], z[16];
              // the channel scales are requested before the TMEM loads, so
              // that the two latencies overlap
              float4 wa[4], wz[4];
              if (su == 0.f) {
                const float4* pa = reinterpret_cast<const float4*>(ep.sw + col_base + c + 16 * h2);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  wa[k] = __ldg(pa + k);
                  wz[k] = __ldg(pa + 8 + k);
                }
              }
              tmem_ld16(tacc + c + 16 * h2, a);
              tmem_ld16(tacc + c + 32 + 16 * h2, z);
              tmem_ld_wait();
              unscale16w(a, sa, wa, su);
              unscale16w(z, sa, wz, su);
              float va[16], vz[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float x0 = __uint_as_float(a[j]), x1 = __uint_as_float(z[j]);
                va[j] = rot ? x0 * cs[16 * h2 + j] - x1 * sn[16 * h2 + j] : x0;
                vz[j] = rot ? x1 * cs[16 * h2 + j] + x0 * sn[16 * h2 + j] : x1;
              }
              if (STAGED) {
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                  *reinterpret_cast<uint4*>(rowp + (((2 * h2 + u) ^ (lane & 7)) << 4)) =
                      pack_bf16x8(va + 8 * u);
                  *reinterpret_cast<uint4*>(rowp + (((4 + 2 * h2 + u) ^ (lane & 7)) << 4)) =
                      pack_bf16x8(vz + 8 * u);
                }
              } else if (live) {
                uint4* d0 = reinterpret_cast<uint4*>(ep.C + (int64_t)row * ep.ldc + col_base + c + 16 * h2);
                uint4* d1 = reinterpret_cast<uint4*>(ep.C + (int64_t)row * ep.ldc + col_base + c + 32 + 16 * h2);
                d0[0] = pack_bf16x8(va);
                d0[1] = pack_bf16x8(va + 8);
                d1[0] = pack_bf16x8(vz);
                d1[1] = pack_bf16x8(vz + 8);
              }
            }
            if (STAGED) {
              fence_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&mapC, stg + sbuf * (32 * 128), col_base + c, m0 + q * 32);
                bulk_commit();
              }
              sbuf ^= 1;
            }
            continue;
          }
          tmem_ld32(tacc + c, r0);
          tmem_ld32(tacc + c + 32, r1);
          tmem_ld_wait();
          float v[64];
          const bool rot = col_base + c < ep.rope_cols;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float x0 = __uint_as_float(r0[j]), x1 = __uint_as_float(r1[j]);
            v[j] = rot ? x0 * cs[j] - x1 * sn[j] : x0;
            v[32 + j] = rot ? x1 * cs[j] + x0 * sn[j] : x1;
          }
          if (STAGED) {
            store_chunk(v, col_base + c, m0 + q * 32);
          } else if (live) {
            store_bf16x32(ep.C + (int64_t)row * ep.ldc + col_base + c, v);
            store_bf16x32(ep.C + (int64_t)row * ep.ldc + col_base + c + 32, v + 32);
          }
        }
      } else if (EPI == TC_RESID && STAGED) {
        // X += acc through TMA: the warp's half of the accumulator is read into
        // registers and released at once; X arrives as 32 x 32 fp32 chunks in
        // two buffers (the first two requested before the accumulator was
        // ready), is updated and written back; rows past M are neither read
        // nor written
        constexpr int NCH = BN / 64;  // 32-column chunks in this warp's half
        const int c0 = hf * BN / 2;
        const int xcol = nb * BN + c0, xrow = m0 + q * 32;
        uint32_t acc[NCH][32];
#pragma unroll
        for (int k = 0; k < NCH; ++k) tmem_ld32(tacc + c0 + 32 * k, acc[k]);
        tmem_ld_wait();
        release(b);
#pragma unroll
        for (int k = 0; k < NCH; ++k) {
          int okx = 1;
          if (lane == 0) okx = mbar_wait<true>(&xb[k & 1], (xphase >> (k & 1)) & 1u) ? 1 : 0;
          okx = __shfl_sync(0xffffffffu, okx, 0);
          xphase ^= 1u << (k & 1);
          if (!okx) {
            if (lane == 0) { record_err(ep.err, 7); abort_sh = 1; }
            break;
          }
          if constexpr (F8) unscale32(acc[k], sa, ep.sw + xcol + 32 * k, su);  // e4m3 operands
          uint8_t* rowp = stg + (k & 1) * 4096 + lane * 128;
          const float4* bias4 =
              ep.bias ? reinterpret_cast<const float4*>(ep.bias + xcol + 32 * k) : nullptr;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            float4* cell = reinterpret_cast<float4*>(rowp + ((c ^ (lane & 7)) << 4));
            float4 o = *cell;
            float4 a = make_float4(__uint_as_float(acc[k][4 * c]), __uint_as_float(acc[k][4 * c + 1]),
                                   __uint_as_float(acc[k][4 * c + 2]),
                                   __uint_as_float(acc[k][4 * c + 3]));
            if (bias4) {
              const float4 bv = bias4[c];
              a.x += bv.x;
              a.y += bv.y;
              a.z += bv.z;
              a.w += bv.w;
            }
            o.x += a.x;
            o.y += a.y;
            o.z += a.z;
            o.w += a.w;
            *cell = o;
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&mapC, stg + (k & 1) * 4096, xcol + 32 * k, xrow);
            bulk_commit();
            if (k + 2 < NCH) {  // chunk k + 2 into this buffer once the store has read it
              bulk_wait_read<0>();
              mbar_expect_tx(&xb[k & 1], 32 * 128);
              tma_load_2d(stg + (k & 1) * 4096, &mapC, &xb[k & 1], xcol + 32 * (k + 2), xrow);
            }
          }
        }
      } else if constexpr (EPI == TC_RESID16) {
        // bf16 X += acc (+ bias) through TMA, as the fp32 path above with
        // chunks of 32 rows x 64 bf16 columns (the same 4 KB swizzled
        // buffers); each chunk takes two 32-column accumulator pieces
        constexpr int NCH = BN / 64;   // 32-column accumulator pieces in this warp's half
        constexpr int NX = BN / 128;   // 64-column X chunks in this warp's half (<= 2)
        static_assert(NX >= 1 && NX <= 2, "TC_RESID16 runs on 128- or 256-column tiles");
        const int c0 = hf * BN / 2;
        const int xcol = nb * BN + c0, xrow = m0 + q * 32;
        uint32_t acc[NCH][32];
#pragma unroll
        for (int k = 0; k < NCH; ++k) tmem_ld32(tacc + c0 + 32 * k, acc[k]);
        tmem_ld_wait();
        release(b);
#pragma unroll
        for (int k = 0; k < NX; ++k) {
          int okx = 1;
          if (lane == 0) okx = mbar_wait<true>(&xb[k], (xphase >> k) & 1u) ? 1 : 0;
          okx = __shfl_sync(0xffffffffu, okx, 0);
          xphase ^= 1u << k;
          if (!okx) {
            if (lane == 0) { record_err(ep.err, 7); abort_sh = 1; }
            break;
          }
          uint8_t* rowp = stg + k * 4096 + lane * 128;
          const float* bias = ep.bias ? ep.bias + xcol + 64 * k : nullptr;
#pragma unroll
          for (int c = 0; c < 8; ++c) {  // 16-byte cell c: columns 8c .. 8c+7 of the chunk
            uint4* cell = reinterpret_cast<uint4*>(rowp + ((c ^ (lane & 7)) << 4));
            uint4 o = *cell;
            uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
            const uint32_t* a = acc[2 * k + (c >> 2)] + 8 * (c & 3);
            float bv[8], mul[8];
            if constexpr (F8) {  // e4m3 operands: row x channel scales, per cell
              if (su != 0.f) {
#pragma unroll
                for (int e = 0; e < 8; ++e) mul[e] = su;
              } else {
                const float4 w0 = __ldg(reinterpret_cast<const float4*>(ep.sw + xcol + 64 * k + 8 * c));
                const float4 w1 = __ldg(reinterpret_cast<const float4*>(ep.sw + xcol + 64 * k + 8 * c + 4));
                mul[0] = sa * w0.x; mul[1] = sa * w0.y; mul[2] = sa * w0.z; mul[3] = sa * w0.w;
                mul[4] = sa * w1.x; mul[5] = sa * w1.y; mul[6] = sa * w1.z; mul[7] = sa * w1.w;
              }
            }
            if (bias) {
              const float4 b0 = *reinterpret_cast<const float4*>(bias + 8 * c);
              const float4 b1 = *reinterpret_cast<const float4*>(bias + 8 * c + 4);
              bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w;
              bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e) bv[e] = 0.f;
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              __nv_bfloat162 x = *reinterpret_cast<__nv_bfloat162*>(&ow[e]);
              const float2 xf = __bfloat1622float2(x);
              float a0 = __uint_as_float(a[2 * e]), a1 = __uint_as_float(a[2 * e + 1]);
              if constexpr (F8) {
                a0 *= mul[2 * e];
                a1 *= mul[2 * e + 1];
              }
              const float s0 = xf.x + (a0 + bv[2 * e]);
              const float s1 = xf.y + (a1 + bv[2 * e + 1]);
              __nv_bfloat162 r = __floats2bfloat162_rn(s0, s1);
              ow[e] = *reinterpret_cast<uint32_t*>(&r);
            }
            *cell = o;
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&mapC, stg + k * 4096, xcol + 64 * k, xrow);
            bulk_commit();
          }
        }
      } else if (EPI == TC_RESID) {
        // narrow tiles: X += acc with direct loads and stores, the next
        // chunk's residual loads in flight while the current one is added
        constexpr int NCH = BN / 64;  // 32-column chunks in this warp's half
        const int c0 = hf * BN / 2;
        float* xrow = ep.resid + (int64_t)row * ep.ldr + nb * BN + c0;
        float4 xv[2][8];
        if (live) {
#pragma unroll
          for (int j = 0; j < 8; ++j) xv[0][j] = reinterpret_cast<const float4*>(xrow)[j];
        }
#pragma unroll
        for (int k = 0; k < NCH; ++k) {
          if (k + 1 < NCH && live) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              xv[(k + 1) & 1][j] = reinterpret_cast<const float4*>(xrow + 32 * (k + 1))[j];
          }
          tmem_ld32(tacc + c0 + 32 * k, r0);
          tmem_ld_wait();
          if constexpr (F8) unscale32(r0, sa, ep.sw + nb * BN + c0 + 32 * k, su);
          if (live) {
            const float* bk = ep.bias ? ep.bias + nb * BN + c0 + 32 * k : nullptr;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float4 a = make_float4(__uint_as_float(r0[4 * j]), __uint_as_float(r0[4 * j + 1]),
                                     __uint_as_float(r0[4 * j + 2]), __uint_as_float(r0[4 * j + 3]));
              if (bk) {
                const float4 bv = reinterpret_cast<const float4*>(bk)[j];
                a.x += bv.x;
                a.y += bv.y;
                a.z += bv.z;
                a.w += bv.w;
              }
              float4 o = xv[k & 1][j];
              o.x += a.x;
              o.y += a.y;
              o.z += a.z;
              o.w += a.w;
              reinterpret_cast<float4*>(xrow + 32 * k)[j] = o;
            }
          }
        }
      } else if (STAGED) {
        const int col_base = nb * BN;
#pragma unroll 1
        for (int c = hf * BN / 2; c < (hf + 1) * BN / 2; c += 64) {
          float v[64];
#pragma unroll
          for (int k2 = 0; k2 < 2; ++k2) {
            tmem_ld32(tacc + c + 32 * k2, r0);
            tmem_ld_wait();
            if constexpr (F8) unscale32(r0, sa, ep.sw + col_base + c + 32 * k2, su);
            bias_act32(r0, ep.bias ? ep.bias + col_base + c + 32 * k2 : nullptr, ep.act,
                       v + 32 * k2);
          }
          store_chunk(v, col_base + c, m0 + q * 32);
        }
      } else {
        const int col_base = nb * BN;
#pragma unroll 1
        for (int c = hf * BN / 2; c < (hf + 1) * BN / 2; c += 32) {
          tmem_ld32(tacc + c, r0);
          tmem_ld_wait();
          if (!live) continue;
          if constexpr (F8) unscale32(r0, sa, ep.sw + col_base + c, su);
          float v[32];
          bias_act32(r0, ep.bias ? ep.bias + col_base + c : nullptr, ep.act, v);
          store_bf16x32(ep.C + (int64_t)row * ep.ldc + col_base + c, v);
        }
      }
      if constexpr (!EARLY && EPI != TC_GEGLU8) release(b);
    }
    if (STAGED && lane == 0) bulk_wait_all();  // staged stores done before the CTA exits
  }

  fence_before_sync();
  if (PAIR) cluster_sync();  // neither CTA leaves while the pair still uses the other
  else __syncthreads();
  if (warp == 1) {
    __syncwarp();
    fence_after_sync();
    if (PAIR) tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <int BN, int EPI, bool PAIR, bool F8>
cudaError_t launch(const void* A, const void* W, int M, int N_out, int K, int w_rows, EpiArgs ep,
                   cudaStream_t st) {
  constexpr int STAGES = stages_for<BN, EPI, PAIR>();
  constexpr int BROWS = PAIR ? BN / 2 : BN;
  constexpr int SMEM = STAGES * (BM * BK * 2 + BROWS * BK * 2) + out_bytes<BN, EPI>() + 1024;
  static std::atomic<uint64_t> attr_done{0};  // per device ordinal
  if (cudaError_t rc = ensure_smem_attr(gemm_tc_kernel<BN, EPI, PAIR, F8>, SMEM, attr_done))
    return rc;
  CUtensorMap ma, mb, mc;
  const int b_box = PAIR ? BROWS : (is_geglu<EPI>() ? BN / 2 : BN);
  if (F8) {
    if (!make_map_u8(&ma, A, K, M, (uint64_t)K, 2 * BK, BM) ||
        !make_map_u8(&mb, W, K, w_rows, (uint64_t)K, 2 * BK, b_box))
      return cudaErrorInvalidValue;
  } else if (!make_map_bf16(&ma, A, K, M, (uint64_t)K * 2, BK, BM) ||
             !make_map_bf16(&mb, W, K, w_rows, (uint64_t)K * 2, BK, b_box)) {
    return cudaErrorInvalidValue;
  }
  if (staged<BN, EPI>() && EPI == TC_RESID) {
    if (!make_map_f32(&mc, ep.resid, N_out, M, (uint64_t)N_out * 4, 32, 32))
      return cudaErrorInvalidValue;
  } else if (staged<BN, EPI>()) {
    if (!make_map_bf16(&mc, ep.C, N_out, M, (uint64_t)N_out * 2, 64, 32)) return cudaErrorInvalidValue;
  } else {
    mc = ma;  // unused
  }
  const int out_tile = is_geglu<EPI>() ? BN / 2 : BN;
  const int n_tiles = N_out / out_tile;
  const int tile_m = PAIR ? 2 * BM : BM;
  const int tiles = ((M + tile_m - 1) / tile_m) * n_tiles;
  const int up_row0 = is_geglu<EPI>() ? N_out : 0;
  if (!PAIR) {
    const int grid = std::min(tiles, sm_count());
    gemm_tc_kernel<BN, EPI, false, F8><<<grid, threads_for<EPI>(), SMEM, st>>>(ma, mb, mc, M, n_tiles, K,
                                                                      up_row0, ep);
    return cudaGetLastError();
  }
  const int pairs = std::min(tiles, sm_count() / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(threads_for<EPI>(), 1, 1);
  cfg.dynamicSmemBytes = SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, EPI, true, F8>, ma, mb, mc, M, n_tiles, K,
                            up_row0, ep);
}

// Pair tiles (256 x 256) for large GEMMs; single-CTA tiles otherwise.
constexpr int kPairMinRows = 2048;

template <int EPI, bool F8 = false>
cudaError_t dispatch_bn(const void* A, const void* W, int M, int N, int K, int w_rows, EpiArgs ep,
                        cudaStream_t st) {
  if constexpr (EPI == TC_GEGLU8) {  // 256-column tiles only
    if (N % 128 != 0) return cudaErrorInvalidValue;
    if (M >= kPairMinRows) return launch<256, EPI, true, F8>(A, W, M, N, K, w_rows, ep, st);
    return launch<256, EPI, false, F8>(A, W, M, N, K, w_rows, ep, st);
  } else if constexpr (EPI == TC_RESID16) {  // staged tiles only: 256 or 128 columns
    if (N % 256 == 0) {
      if (M >= kPairMinRows) return launch<256, EPI, true, F8>(A, W, M, N, K, w_rows, ep, st);
      return launch<256, EPI, false, F8>(A, W, M, N, K, w_rows, ep, st);
    }
    if (N % 128 == 0) return launch<128, EPI, false, F8>(A, W, M, N, K, w_rows, ep, st);
    return cudaErrorInvalidValue;
  } else {
    if (EPI == TC_GEGLU) {
      if (N % 128 == 0) {
        if (M >= kPairMinRows) return launch<256, EPI, true, F8>(A, W, M, N, K, w_rows, ep, st);
        return launch<256, EPI, false, F8>(A, W, M, N, K, w_rows, ep, st);
      }
      return launch<128, EPI, false, F8>(A, W, M, N, K, w_rows, ep, st);
    }
    if (N % 256 == 0) {
      if (M >= kPairMinRows) return launch<256, EPI, true, F8>(A, W, M, N, K, w_rows, ep, st);
      return launch<256, EPI, false, F8>(A, W, M, N, K, w_rows, ep, st);
    }
    if (N % 128 == 0) return launch<128, EPI, false, F8>(A, W, M, N, K, w_rows, ep, st);
    return launch<64, EPI, false, F8>(A, W, M, N, K, w_rows, ep, st);
  }
}

}  // namespace

bool gemm_tc_supported(int M, int N, int K, bool geglu) {
  if (M <= 0 || K < BK || K % BK != 0) return false;
  return geglu ? (N % 64 == 0) : (N % 64 == 0);
}

cudaError_t gemm_tc(const bf16* A, const bf16* W, const float* bias, bf16* C, float* resid, int M,
                    int N, int K, int epi, int act, TcRope rope, int* err, cudaStream_t st) {
  if (!gemm_tc_supported(M, N, K, epi == TC_GEGLU)) return cudaErrorInvalidValue;
  EpiArgs ep{};
  ep.bias = bias;
  ep.act = act;
  ep.C = C;
  ep.ldc = N;
  ep.resid = resid;
  ep.ldr = N;
  ep.cos_t = rope.cos_t;
  ep.sin_t = rope.sin_t;
  ep.pos = rope.pos;
  ep.rope_cols = 2 * rope.H * 64;
  ep.err = err;
  switch (epi) {
    case TC_STORE: return dispatch_bn<TC_STORE>(A, W, M, N, K, N, ep, st);
    case TC_RESID: return dispatch_bn<TC_RESID>(A, W, M, N, K, N, ep, st);
    case TC_GEGLU: return dispatch_bn<TC_GEGLU>(A, W, M, N, K, 2 * N, ep, st);
    case TC_ROPE: return dispatch_bn<TC_ROPE>(A, W, M, N, K, N, ep, st);
    case TC_RESID16:
      if (!C) return cudaErrorInvalidValue;
      return dispatch_bn<TC_RESID16>(A, W, M, N, K, N, ep, st);
  }
  return cudaErrorInvalidValue;
}

cudaError_t gemm_tc_take_status(int* code) {
  int v = 0;
  cudaError_t rc = cudaMemcpyFromSymbol(&v, g_gemm_tc_err, sizeof(int));
  if (rc == cudaSuccess && v != 0) {
    const int zero = 0;
    rc = cudaMemcpyToSymbol(g_gemm_tc_err, &zero, sizeof(int));
  }
  *code = v;
  return rc;
}

bool gemm_tc_f8_supported(int M, int N, int K, int epi) {
  if (M <= 0 || K < 2 * BK || K % (2 * BK) != 0 || N % 64 != 0) return false;
  return epi == TC_STORE || epi == TC_GEGLU || epi == TC_ROPE || epi == TC_RESID ||
         epi == TC_RESID16;
}

cudaError_t gemm_tc_f8(const uint8_t* A, const uint8_t* W, const float* sa, const float* sw,
                       const float* bias, bf16* C, int M, int N, int K, int epi, int act,
                       TcRope rope, int* err, cudaStream_t st, float* resid, TcQ8 q8) {
  if (!gemm_tc_f8_supported(M, N, K, epi) || !sa || !sw) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(sw) & 15) return cudaErrorInvalidValue;
  EpiArgs ep{};
  ep.bias = bias;
  ep.act = act;
  ep.C = C;
  ep.ldc = N;
  ep.cos_t = rope.cos_t;
  ep.sin_t = rope.sin_t;
  ep.pos = rope.pos;
  ep.rope_cols = 2 * rope.H * 64;
  ep.sa = sa;
  ep.sw = sw;
  ep.resid = resid;
  ep.ldr = N;
  ep.C8 = q8.C;
  ep.c8_scale = q8.scale;
  ep.c8_rowscale = q8.rowscale;
  ep.uniform = q8.uniform ? 1 : 0;
  ep.err = err;
  if ((epi == TC_RESID && !resid) || (epi == TC_RESID16 && !C)) return cudaErrorInvalidValue;
  if (q8.C && (epi != TC_GEGLU || !q8.scale || !q8.rowscale)) return cudaErrorInvalidValue;
  switch (epi) {
    case TC_STORE: return dispatch_bn<TC_STORE, true>(A, W, M, N, K, N, ep, st);
    case TC_RESID: return dispatch_bn<TC_RESID, true>(A, W, M, N, K, N, ep, st);
    case TC_RESID16: return dispatch_bn<TC_RESID16, true>(A, W, M, N, K, N, ep, st);
    case TC_GEGLU:
      if (q8.C) return dispatch_bn<TC_GEGLU8, true>(A, W, M, N, K, 2 * N, ep, st);
      return dispatch_bn<TC_GEGLU, true>(A, W, M, N, K, 2 * N, ep, st);
    case TC_ROPE: return dispatch_bn<TC_ROPE, true>(A, W, M, N, K, N, ep, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace sjb
