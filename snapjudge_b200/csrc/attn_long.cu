// attn_long.cu — tcgen05 flash attention for long segments (Dh = 64, no window).
//
// Semantics of the reference attention (src/tensor.cpp:156-228) with w = 0:
// query i of segment b attends keys j < kv_len (kv_lens null: the segment's
// length), scale 1/sqrt(64), max-subtracted softmax; bf16 q/k/v/o, fp32 scores
// and accumulation, P rounded to bf16 for the P.V MMA, the row normaliser
// summed in fp32.  Windowed layers and short segments stay on attn_tc.cu,
// whose four small CTAs per SM suit items of one or two key tiles.
//
// Built for segments of hundreds to thousands of tokens, where an item has
// many key tiles.  One persistent CTA per SM; a work item is 256 queries (two
// 128-row Q tiles, Q0 and Q1) of one (segment, head); items are walked with a
// stride of the grid.  Warp roles (512 threads):
//   warps 0-3   issue the MMAs, one kind each (warp-uniform bookkeeping, one
//               elected lane issues): S0 = Q0 K^T, S1 = Q1 K^T, O0 += P0 V,
//               O1 += P1 V;
//   warp 4      one thread issues every TMA load;
//   warp 5      one thread decodes the CTA's work items (segment bounds from
//               cu_seqlens) into a ring in shared memory, up to 8 ahead;
//   warps 8-11  softmax of Q0 (thread = query row = TMEM lane), output of Q0;
//   warps 12-15 the same for Q1.
// Shared memory: Q double-buffered (2 items x 2 tiles x 16 KB) and a 4-stage
// ring of 128-key K and V tiles (16 KB each), all 128-byte swizzled.
// TMEM (512 columns): S0, S1 (fp32 scores, 128 each), P0, P1 (bf16 pairs,
// 64 each) and O0, O1 (fp32, 64 each).  Because P has its own columns, S_t of
// the next key tile is issued as soon as softmax t has loaded S_t into
// registers, so the tensor pipe runs the next tile's QK^T and the previous
// tile's P.V while the softmax warps work.
// Hand-offs are mbarriers: s_full (S done, tcgen05.commit), s_free (softmax
// read S), p_full (P written to TMEM, O rescaled), o_done (P.V done), k/v_full
// (TMA), kv_empty and q_empty (the MMAs that read a stage / a Q buffer are
// done), it_full/it_empty (the item ring).
// Rescaling follows attn_tc.cu: each row moves its reference max only when a
// tile's max exceeds it by 2^8, then multiplies its O row (in TMEM, after the
// previous P.V is done) and running sum before publishing the new P.
// Every wait is bounded by wall time and also ends when another role has given
// up (a CTA-wide abort word in shared memory); after the loops, the loader
// waits for the copies it issued and the MMA warps for their MMAs, then TMEM
// is freed and the CTA returns.  Nothing traps.
#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"
#include "tc_host.h"

namespace sjb {

__device__ int g_attn_long_err;

namespace {
using namespace tc;

constexpr int QT = 128;  // rows per Q tile
constexpr int KT = 128;  // keys per K/V tile
constexpr int DH = 64;
constexpr int STAGES = 4;
constexpr int kThreads = 512;
// Warpgroup 0: four MMA-issuing warps, one per SM sub-partition (warp w on
// sub-partition w).  Each shares its issue port with two softmax warps that
// keep it busy; a single issuing warp for all 24 MMAs of a key tile got them
// accepted at ~150 cycles each (32-64 cycles alone).
// Warpgroup 1: the TMA loader (warp 4) and the item decoder (warp 5).
// Warpgroups 2 and 3: softmax of Q0 and Q1.  Registers move from the first
// two warpgroups to the softmax ones (setmaxnreg): 2 x 128 x 56 +
// 2 x 128 x 200 = 65536, the block's 512 threads x 128 at launch.
constexpr int kLoadWarp = 4, kDecodeWarp = 5, kSoftmaxWarp0 = 8;
constexpr int kCtrlRegs = 56, kSoftmaxRegs = 200;
constexpr int RING = 8;  // decoded work items in flight (shared memory)
// consumers of each decoded item: the loader, the 4 MMA warps, 8 softmax warps
constexpr int kItemReaders = 13;
// Of every 8 column pairs of a row, this many are exponentiated by ex2_poly on
// the FMA/ALU pipes and the rest on the MUFU.
constexpr int kPolyPairsOf8 = 1;
constexpr int TILE = QT * DH * 2;                 // 16 KB: one Q, K or V tile
constexpr int SMEM_BYTES = 4 * TILE + STAGES * 2 * TILE + 1024;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_S0 = 0, COL_P0 = 256, COL_O0 = 384;  // tile t: + t * 128 / 64 / 64
constexpr float kRescaleLog2 = 8.f;
constexpr uint32_t IDESC_S = idesc_bf16(QT, KT, false, false);
constexpr uint32_t IDESC_O = idesc_bf16(QT, DH, false, true);

__device__ __forceinline__ void record_err(int* err, int code) {
  atomicCAS(err ? err : &g_attn_long_err, 0, code);
}

__device__ __forceinline__ float ex2(float x) {  // 2^x on the MUFU (flush-to-zero)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
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
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// two bf16 (low = a) from fp32, round to nearest even
__device__ __forceinline__ uint32_t bf16x2(float a, float b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}
// 2^x for a pair on the FMA and ALU pipes (the MUFU computes 16 exponentials
// per clock per SM, fewer than a tile needs to keep pace with the tensor
// pipe, so part of every row goes here).  Cody-Waite split x = n + f with
// n = rint(x) (adding 1.5 * 2^23 rounds to an integer in the low mantissa
// bits) and f in [-0.5, 0.5]; 2^f from a cubic fitted by least squares on
// Chebyshev nodes of [-0.5, 0.5] (relative error <= 7.5e-5, far below the
// bf16 rounding of P); 2^n added into the exponent field.  Arguments below
// -125 are clamped (2^-125 vanishes next to the row maximum's 2^0).
constexpr float kRoundMagic = 12582912.f;
__device__ __forceinline__ f32x2 ex2_poly(f32x2 x) {
  float2 v = unpk2(x);
  v.x = fmaxf(v.x, -125.f);
  v.y = fmaxf(v.y, -125.f);
  const f32x2 xv = pk2(v.x, v.y);
  const f32x2 t = add2(xv, pk2(kRoundMagic, kRoundMagic));
  const f32x2 n = add2(t, pk2(-kRoundMagic, -kRoundMagic));
  const f32x2 f = fma2(n, pk2(-1.f, -1.f), xv);
  f32x2 q = fma2(pk2(0.0551716238f, 0.0551716238f), f, pk2(0.242611125f, 0.242611125f));
  q = fma2(q, f, pk2(0.693260968f, 0.693260968f));
  q = fma2(q, f, pk2(0.999928057f, 0.999928057f));
  const float2 qf = unpk2(q), tf = unpk2(t);
  return pk2(__uint_as_float(__float_as_uint(qf.x) + (__float_as_uint(tf.x) << 23)),
             __uint_as_float(__float_as_uint(qf.y) + (__float_as_uint(tf.y) << 23)));
}
// P for columns [C0, C1) of a row: p = 2^(s * scale - m), fp32 row sums in
// acc0/acc1, bf16 pairs packed over s[c / 2].  kPolyPairsOf8 of every 8
// column pairs go to ex2_poly, the rest to the MUFU (fp32 ex2).
template <int C0, int C1>
__device__ __forceinline__ void exp_cols(uint32_t (&s)[128], f32x2 scale2, f32x2 negm2,
                                         f32x2& acc0, f32x2& acc1) {
#pragma unroll
  for (int c = C0; c < C1; c += 2) {
    const f32x2 x = fma2(pk2(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), scale2, negm2);
    float2 p;
    if (((c >> 1) & 7) >= 8 - kPolyPairsOf8) {
      p = unpk2(ex2_poly(x));
    } else {
      const float2 xf = unpk2(x);
      p = make_float2(ex2(xf.x), ex2(xf.y));
    }
    if ((c >> 1) & 1) acc1 = add2(acc1, pk2(p.x, p.y));
    else acc0 = add2(acc0, pk2(p.x, p.y));
    s[c >> 1] = bf16x2(p.x, p.y);
  }
}
__device__ __forceinline__ void st_global_v8(void* p, const uint32_t (&v)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

// A work item: queries [q0, q0 + 256) of segment b (rows s0 + .), head h.
// nt: Q tiles with rows in the segment (1 or 2); n_kv: key tiles
// (0: no visible key, -1: idle slot of the grid form).
struct LItem {
  int s0, n, nk, q0, h, nt, n_kv;
};

// Item w.  List form (pairs != null): pairs[w / H] = (b, q0), head w % H.
// Grid form: w = (b * npp + (npp - 1 - p)) * H + h, q0 = 256 p (npp items per
// segment at most): a segment's items are adjacent, so the CTAs working on it
// at the same time share its K/V tiles through L2 (with the items of one
// segment and head spread over time, each re-read K/V from DRAM: 948 MB for
// 201 MB of Q/K/V on C4's shape); segments shorter than long_min belong to
// attn_tc and are idle here.
__device__ __forceinline__ LItem decode(int w, const int2* pairs, int H, int B, int npp,
                                        const int32_t* cu, const int32_t* kv_lens, int long_min) {
  LItem it;
  it.h = w % H;
  const int rest = w / H;
  int b;
  if (pairs) {
    const int2 p = pairs[rest];
    b = p.x;
    it.q0 = p.y;
  } else {
    b = rest / npp;
    it.q0 = (npp - 1 - rest % npp) * 2 * QT;
  }
  it.s0 = cu[b];
  it.n = cu[b + 1] - it.s0;
  if (it.q0 >= it.n || (!pairs && it.n < long_min)) {
    it.nk = it.nt = 0;
    it.n_kv = -1;
    return it;
  }
  it.nk = kv_lens ? min(kv_lens[b], it.n) : it.n;
  it.nt = it.q0 + QT < it.n ? 2 : 1;
  it.n_kv = it.nk > 0 ? (it.nk + KT - 1) / KT : 0;
  return it;
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_long_kernel(const __grid_constant__ CUtensorMap map, const int32_t* __restrict__ cu,
                     const int32_t* __restrict__ kv_lens, bf16* __restrict__ O, int H, int B,
                     const int2* __restrict__ pairs, int n_items, int npp, int long_min,
                     int* err) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t q_full[2], q_empty[2], k_full[STAGES], v_full[STAGES], kv_empty[STAGES];
  __shared__ uint64_t s_full[2], s_free[2], p_full[2], o_done[2], drain;
  __shared__ uint64_t it_full[RING], it_empty[RING];
  __shared__ LItem ring[RING];
  __shared__ uint32_t tmem_sh;
  __shared__ int abort_sh;
  // loader's issue counts, read at teardown: K/V tiles, Q loads per buffer
  __shared__ uint32_t kv_issued_sh, q_issued_sh[2];

  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem;                // buffer qb, tile t at (2 qb + t) * TILE
  uint8_t* sKV = smem + 4 * TILE;    // stage s: K at 2 s TILE, V at (2 s + 1) TILE
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = (int)gridDim.x;
  const int cnt = n_items > (int)blockIdx.x ? (n_items - 1 - (int)blockIdx.x) / G + 1 : 0;
  volatile int* abort_v = &abort_sh;

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 2);  // both S warps, after an item's last S
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);   // one arrive per warp of the softmax group
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 4);  // both S warps (K read) and both P.V warps (V read)
    }
    mbar_init(&drain, 4);  // the four MMA warps
    for (int i = 0; i < RING; ++i) {
      mbar_init(&it_full[i], 1);
      mbar_init(&it_empty[i], kItemReaders);
    }
    abort_sh = 0;
    kv_issued_sh = q_issued_sh[0] = q_issued_sh[1] = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&tmem_sh, TMEM_COLS);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = tmem_sh;

  // bounded wait that also gives up once another role has aborted
  auto wait = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (true) {
      for (int i = 0; i < 32; ++i)
        if (mbar_try(bar, parity)) return true;
      if (*abort_v) return false;
      if (globaltimer() - t0 > kWaitNs) {
        record_err(err, code);
        *abort_v = 1;
        return false;
      }
    }
  };
  // the same for the loader and decode threads, which mostly wait: the thread
  // sleeps in hardware until the phase completes (its polling would take
  // issue slots from the softmax warps on its SM sub-partition)
  auto wait_sleep = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
    if (mbar_try_sleep(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (true) {
      for (int i = 0; i < 4; ++i)
        if (mbar_try_sleep(bar, parity)) return true;
      if (*abort_v) return false;
      if (globaltimer() - t0 > kWaitNs) {
        record_err(err, code);
        *abort_v = 1;
        return false;
      }
    }
  };
  // lane 0 waits, the warp follows its result
  auto warp_wait = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
    int okw = 1;
    if (lane == 0) okw = wait(bar, parity, code) ? 1 : 0;
    return __shfl_sync(0xffffffffu, okw, 0) != 0;
  };
  // item k from the ring (one thread per call site; false if a wait gave up)
  auto take = [&](int k, LItem& it) -> bool {
    if (!wait(&it_full[k % RING], (k / RING) & 1, 36)) return false;
    it = ring[k % RING];
    return true;
  };
  auto give = [&](int k) { mbar_arrive(&it_empty[k % RING]); };
  // item k for a whole warp: lane 0 waits, every lane copies, lane 0 releases
  auto warp_take = [&](int k, LItem& it) -> bool {
    int okw = 1;
    if (lane == 0) okw = wait(&it_full[k % RING], (k / RING) & 1, 36) ? 1 : 0;
    if (__shfl_sync(0xffffffffu, okw, 0) == 0) return false;
    __syncwarp();
    it = ring[k % RING];
    __syncwarp();
    if (lane == 0) give(k);
    return true;
  };

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kCtrlRegs));
    // ---------------------------------------------------------------- MMA issue
    // Every lane runs the bookkeeping (warp-uniform control flow keeps the
    // descriptors and TMEM addresses in uniform registers, which tcgen05.mma
    // reads; issued from a single-lane branch, each MMA first waited on
    // per-lane to uniform register moves); one elected lane issues the MMAs
    // and the commits that track them.  Warps 0/1 issue S_t (t = warp & 1)
    // and release K; warps 2/3 issue P_t V and release V.  For an item without
    // Q tile t the warp still walks its key tiles in step and releases each
    // stage with a plain arrive.
    const int t = warp & 1;
    const bool is_s = warp < 2;
    uint32_t g = 0;            // K/V tiles walked
    uint32_t n = 0;            // MMA groups issued (S_t or P_t V)
    uint32_t nq[2] = {0, 0};   // items started per Q buffer
    int active = 0;
    bool ok = true;
    for (int k = 0; k < cnt && ok; ++k) {
      LItem it;
      if (!(ok = warp_take(k, it))) break;
      if (it.n_kv <= 0) continue;
      const int qb = active & 1;
      ++active;
      const bool mine = t < it.nt;
      if (is_s) {
        if (!(ok = warp_wait(&q_full[qb], nq[qb] & 1, 22))) break;
        ++nq[qb];
      }
      const uint32_t q_addr = smem_u32(sQ + (2 * qb + t) * TILE);
      for (int j = 0; j < it.n_kv && ok; ++j, ++g) {
        const int st = g % STAGES;
        const bool last = j == it.n_kv - 1;
        if (is_s) {
          if (!(ok = warp_wait(&k_full[st], (g / STAGES) & 1, 23))) break;
          if (mine) {
            if (n > 0 && !(ok = warp_wait(&s_free[t], (n - 1) & 1, 24))) break;
            fence_after_sync();
            const uint32_t k_addr = smem_u32(sKV + 2 * st * TILE);
            if (elect_one()) {
#pragma unroll
              for (int kk = 0; kk < DH / 16; ++kk)
                mma_bf16(tmem + COL_S0 + 128 * t, desc_kmajor_sw128(q_addr + kk * 32),
                         desc_kmajor_sw128(k_addr + kk * 32), IDESC_S, kk != 0);
              mma_commit(&s_full[t]);
              mma_commit(&kv_empty[st]);
              if (last) mma_commit(&q_empty[qb]);
            }
            __syncwarp();
            ++n;
          } else {
            if (elect_one()) {
              mbar_arrive(&kv_empty[st]);
              if (last) mbar_arrive(&q_empty[qb]);
            }
            __syncwarp();
          }
        } else {
          if (!(ok = warp_wait(&v_full[st], (g / STAGES) & 1, 20))) break;
          if (mine) {
            if (!(ok = warp_wait(&p_full[t], n & 1, 21))) break;
            fence_after_sync();
            const uint32_t v_addr = smem_u32(sKV + (2 * st + 1) * TILE);
            const int lim = min(KT, it.nk - j * KT);
            if (elect_one()) {
              if (lim > 64) {
#pragma unroll
                for (int kk = 0; kk < KT / 16; ++kk)
                  mma_bf16_ts(tmem + COL_O0 + 64 * t, tmem + COL_P0 + 64 * t + kk * 8,
                              desc_mnmajor_sw128(v_addr + kk * 16 * 128), IDESC_O,
                              (j > 0 || kk > 0) ? 1u : 0u);
              } else {  // at most 64 visible keys: P holds them in its first 32 columns
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                  mma_bf16_ts(tmem + COL_O0 + 64 * t, tmem + COL_P0 + 64 * t + kk * 8,
                              desc_mnmajor_sw128(v_addr + kk * 16 * 128), IDESC_O,
                              (j > 0 || kk > 0) ? 1u : 0u);
              }
              mma_commit(&o_done[t]);
              mma_commit(&kv_empty[st]);
            }
            __syncwarp();
            ++n;
          } else {
            if (elect_one()) mbar_arrive(&kv_empty[st]);
            __syncwarp();
          }
        }
      }
    }
  } else if (warp < kSoftmaxWarp0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kCtrlRegs));
    if (warp == kDecodeWarp) {
      // ---------------------------------------------------------------- decode
      if (lane == 0) {
        for (int k = 0; k < cnt; ++k) {
          if (k >= RING && !wait_sleep(&it_empty[k % RING], ((k / RING) - 1) & 1, 37)) break;
          ring[k % RING] = decode((int)blockIdx.x + k * G, pairs, H, B, npp, cu, kv_lens, long_min);
          mbar_arrive(&it_full[k % RING]);  // release: the item is visible to its readers
        }
      }
      __syncwarp();
    } else if (warp == kLoadWarp) {
      // ---------------------------------------------------------------- loader
      if (lane == 0) {
        tma_prefetch(&map);
        uint32_t gl = 0;  // K/V tiles issued
        uint32_t nq[2] = {0, 0};
        int active = 0;  // items with keys, in order (Q buffer = active & 1)
        bool ok = true;
        for (int k = 0; k < cnt && ok; ++k) {
          LItem it;
          if (!(ok = take(k, it))) break;
          give(k);
          if (it.n_kv <= 0) continue;
          const int qb = active & 1;
          ++active;
          if (nq[qb] > 0 && !(ok = wait_sleep(&q_empty[qb], (nq[qb] - 1) & 1, 30))) break;
          mbar_expect_tx(&q_full[qb], it.nt * TILE);
          for (int t = 0; t < it.nt; ++t)
            tma_load_2d(sQ + (2 * qb + t) * TILE, &map, &q_full[qb], it.h * DH,
                        it.s0 + it.q0 + t * QT);
          q_issued_sh[qb] = ++nq[qb];
          for (int j = 0; j < it.n_kv; ++j, ++gl) {
            const int s = gl % STAGES;
            if (gl >= STAGES && !(ok = wait_sleep(&kv_empty[s], ((gl / STAGES) - 1) & 1, 31)))
              break;
            const int row = it.s0 + j * KT;
            mbar_expect_tx(&k_full[s], TILE);
            tma_load_2d(sKV + 2 * s * TILE, &map, &k_full[s], (H + it.h) * DH, row);
            mbar_expect_tx(&v_full[s], TILE);
            tma_load_2d(sKV + (2 * s + 1) * TILE, &map, &v_full[s], (2 * H + it.h) * DH, row);
            kv_issued_sh = gl + 1;
          }
        }
      }
      __syncwarp();
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    // ---------------------------------------------------------------- softmax
    const int t = (warp - kSoftmaxWarp0) >> 2;  // Q tile of this warpgroup
    const int r = tid & 127;                      // row within the tile = TMEM lane
    const int sub = warp & 3;                     // SM sub-partition = TMEM lane quarter
    const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
    const uint32_t tS = tmem + COL_S0 + 128 * t + lane_off;
    const uint32_t tP = tmem + COL_P0 + 64 * t + lane_off;
    const uint32_t tO = tmem + COL_O0 + 64 * t + lane_off;
    const float scale = 0.125f * 1.4426950408889634f;  // log2(e) / sqrt(64)
    const bool o32 = (reinterpret_cast<uintptr_t>(O) & 31) == 0;
    uint32_t cs = 0, co = 0;  // s_full and o_done phases consumed
    bool ok = true;
    for (int k = 0; k < cnt && ok; ++k) {
      LItem it;
      if (!(ok = warp_take(k, it))) break;
      if (it.n_kv < 0 || t >= it.nt) continue;
      const int i_q = it.q0 + t * QT + r;
      const bool live = i_q < it.n;
      bf16* orow = O + (int64_t)(it.s0 + i_q) * H * DH + it.h * DH;
      if (it.n_kv == 0) {  // no visible key: the reference's empty sum gives 0
        if (live)
          for (int q = 0; q < 8; ++q) reinterpret_cast<uint4*>(orow)[q] = make_uint4(0, 0, 0, 0);
        continue;
      }
      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j < it.n_kv; ++j) {
        if (!(ok = warp_wait(&s_full[t], cs & 1, 25))) break;
        ++cs;
        fence_after_sync();
        const int lim = min(KT, it.nk - j * KT);  // visible keys of this tile (all rows)
        const bool full = lim > 64;
        uint32_t s[128];
        tmem_ld32(tS, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
        tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
        if (full) {
          tmem_ld32(tS + 64, *reinterpret_cast<uint32_t(*)[32]>(&s[64]));
          tmem_ld32(tS + 96, *reinterpret_cast<uint32_t(*)[32]>(&s[96]));
        }
        tmem_ld_wait();
        fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[t]);  // S_t may be overwritten now
        const int ncol = full ? 128 : 64;
        if (lim < ncol) {
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c < ncol && c >= lim) s[c] = __float_as_uint(-INFINITY);
        }
        float a0 = -INFINITY, a1 = -INFINITY, a2 = -INFINITY, a3 = -INFINITY;
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
          a0 = max3(a0, __uint_as_float(s[c]), __uint_as_float(s[c + 1]));
          a1 = max3(a1, __uint_as_float(s[c + 2]), __uint_as_float(s[c + 3]));
          a2 = max3(a2, __uint_as_float(s[c + 4]), __uint_as_float(s[c + 5]));
          a3 = max3(a3, __uint_as_float(s[c + 6]), __uint_as_float(s[c + 7]));
        }
        if (full) {
#pragma unroll
          for (int c = 64; c < 128; c += 8) {
            a0 = max3(a0, __uint_as_float(s[c]), __uint_as_float(s[c + 1]));
            a1 = max3(a1, __uint_as_float(s[c + 2]), __uint_as_float(s[c + 3]));
            a2 = max3(a2, __uint_as_float(s[c + 4]), __uint_as_float(s[c + 5]));
            a3 = max3(a3, __uint_as_float(s[c + 6]), __uint_as_float(s[c + 7]));
          }
        }
        const float m_tile = max3(a0, a1, fmaxf(a2, a3)) * scale;
        const bool first = m_ref == -INFINITY;
        const bool grow = !first && m_tile > m_ref + kRescaleLog2;
        const float m_new = (first || grow) ? m_tile : m_ref;
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const float resc = grow ? ex2(m_ref - m_new) : 1.f;
        if (grow) l *= resc;
        m_ref = m_new;
        // P = 2^(s * scale - m_use) as bf16 pairs, packed over s[0 .. ncol/2)
        const f32x2 scale2 = pk2(scale, scale), negm2 = pk2(-m_use, -m_use);
        f32x2 acc0 = pk2(0.f, 0.f), acc1 = pk2(0.f, 0.f);
        exp_cols<0, 64>(s, scale2, negm2, acc0, acc1);
        if (full) exp_cols<64, 128>(s, scale2, negm2, acc0, acc1);
        const float2 u0 = unpk2(acc0), u1 = unpk2(acc1);
        l += (u0.x + u0.y) + (u1.x + u1.y);
        // P_t(j - 1) must be consumed (and O_t final for the rescale) before
        // P_t(j) is written; P goes out first so that its registers are free
        // for the (rare) rescale of the O row
        if (j > 0) {
          if (!(ok = warp_wait(&o_done[t], co & 1, 26))) break;
          ++co;
          fence_after_sync();
        }
        tmem_st32(tP, *reinterpret_cast<const uint32_t(*)[32]>(&s[0]));
        if (full) tmem_st32(tP + 32, *reinterpret_cast<const uint32_t(*)[32]>(&s[32]));
        if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t ov[32];
            tmem_ld32(tO + 32 * half, ov);
            tmem_ld_wait();
#pragma unroll
            for (int d = 0; d < 32; ++d) ov[d] = __float_as_uint(__uint_as_float(ov[d]) * resc);
            tmem_st32(tO + 32 * half, ov);
          }
        }
        tmem_st_wait();
        fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
      }
      if (!ok) break;
      // the item's output: its last P.V, then O / l
      if (!(ok = warp_wait(&o_done[t], co & 1, 27))) break;
      ++co;
      fence_after_sync();
      uint32_t oa[32], ob[32];
      tmem_ld32(tO, oa);
      tmem_ld32(tO + 32, ob);
      tmem_ld_wait();
      fence_before_sync();
      if (live) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t wv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int d = q * 16 + 2 * e;
            const float x0 = __uint_as_float(d < 32 ? oa[d] : ob[d - 32]) * inv;
            const float x1 = __uint_as_float(d + 1 < 32 ? oa[d + 1] : ob[d - 31]) * inv;
            wv[e] = bf16x2(x0, x1);
          }
          if (o32) {
            st_global_v8(orow + 16 * q, wv);
          } else {
            reinterpret_cast<uint4*>(orow)[2 * q] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            reinterpret_cast<uint4*>(orow)[2 * q + 1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
          }
        }
      }
    }
  }

  // ---- teardown: every copy landed and every MMA done before TMEM and shared
  // memory are released
  __syncthreads();
  if (tid == kLoadWarp * 32) {
    const uint32_t gl = kv_issued_sh;
    for (int s = 0; s < STAGES; ++s) {
      if (gl <= (uint32_t)s) continue;
      const uint32_t last = gl - 1 - ((gl - 1 - s) % STAGES);  // last tile issued into stage s
      if (!mbar_wait(&k_full[s], (last / STAGES) & 1)) record_err(err, 32);
      if (!mbar_wait(&v_full[s], (last / STAGES) & 1)) record_err(err, 33);
    }
    for (int qb = 0; qb < 2; ++qb)
      if (q_issued_sh[qb] > 0 && !mbar_wait(&q_full[qb], (q_issued_sh[qb] - 1) & 1))
        record_err(err, 34);
  }
  if (warp < 4) {  // every MMA warp's MMAs are done
    if (elect_one()) {
      mma_commit(&drain);
      if (!mbar_wait(&drain, 0)) record_err(err, 35);
    }
    __syncwarp();
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

cudaError_t attn_long_take_status(int* code) {
  int v = 0;
  cudaError_t rc = cudaMemcpyFromSymbol(&v, g_attn_long_err, sizeof(int));
  if (rc == cudaSuccess && v != 0) {
    const int zero = 0;
    rc = cudaMemcpyToSymbol(g_attn_long_err, &zero, sizeof(int));
  }
  *code = v;
  return rc;
}

cudaError_t attn_long(const bf16* qkv, const int32_t* cu, const int32_t* kv_lens, bf16* O, int T,
                      int H, const int2* pairs, int n_pairs, int B, int max_seqlen, int* err,
                      cudaStream_t st) {
  static std::atomic<uint64_t> attr_done{0};  // per device ordinal
  if (cudaError_t rc = ensure_smem_attr(attn_long_kernel, SMEM_BYTES, attr_done)) return rc;
  if (T <= 0) return cudaSuccess;
  CUtensorMap map;
  const uint64_t cols = 3ull * H * DH;
  if (!make_map_bf16(&map, qkv, cols, T, cols * 2, DH, QT)) return cudaErrorInvalidValue;
  const int npp = (max_seqlen + 2 * QT - 1) / (2 * QT);
  const long long items = pairs ? (long long)n_pairs * H : (long long)B * npp * H;
  if (items <= 0) return cudaSuccess;
  if (items > 0x7fffffff) return cudaErrorInvalidValue;
  const int grid = (int)std::min<long long>(items, (long long)sm_count());
  attn_long_kernel<<<grid, kThreads, SMEM_BYTES, st>>>(map, cu, kv_lens, O, H, B, pairs,
                                                        (int)items, npp, kAttnLongMin, err);
  return cudaGetLastError();
}

}  // namespace sjb
