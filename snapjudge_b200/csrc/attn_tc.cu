// attn_tc.cu — tcgen05 flash attention for packed variable-length sequences (Dh = 64).
//
// Semantics of the reference attention (src/tensor.cpp:156-228): query i of
// segment b attends keys j in [max(0, i - w), min(kv_len, i + w + 1))
// (w = 0: all j < kv_len), scale 1/sqrt(64), max-subtracted softmax.  bf16
// q/k/v/o, fp32 scores and accumulation; P is rounded to bf16 for the P.V MMA
// (the row normaliser sums the fp32 probabilities).
//
// Built for many short items: 4 small CTAs per SM, each a complete pipeline of
// its own, so an SM always has several independent (S -> softmax -> P.V)
// chains in flight.  A work item is 128 queries of one segment x one head; a
// CTA walks a strided list of items, longest segments first.
//   128 threads: thread = query row = TMEM lane (softmax, output).  Thread 0
//   also issues the TMA loads and the MMAs:
//     Q of the item (one 16 KB buffer, loaded for the next item as soon as the
//     current item's last S is computed), K/V tiles of 64 keys through a
//     2-stage ring that runs on across items;
//     S = Q K^T (M=128, N=64, K=64) into TMEM, then O += P V with P read from
//     TMEM (the A operand) and V from shared memory (MN-major); the next S
//     (of this item, or of the next one once its Q is in) is issued as soon
//     as the P.V completes, before the loads that P.V frees.
//   TMEM (128 columns): S (fp32, 64) — P (bf16 pairs) overwrites its first 32
//   columns once S is in registers — and O (fp32, 64).
// Without a window every row of a tile sees the same keys [kbase, kbase +
// lim): a tile with lim <= 32 (short segments, last tiles) exponentiates 32
// columns and its P.V runs over 32 keys.
// Rescaling: each row keeps a reference max m_ref for its exponentials and
// moves it only when a tile's max exceeds it by more than 2^8 (exponent 8 in
// log2 units); then the row's O (in TMEM) and running sum are multiplied by
// 2^(m_ref_old - m_ref_new) before the next P.V accumulates.  The result is the
// same softmax (every term uses the same reference), with P <= 2^8.
// Keys past kv_len and outside the window are masked with -inf (interior tiles
// skip the mask); key tiles wholly outside the window are skipped.
// Work items are decoded into shared memory 64 at a time by all threads.  Every
// mbarrier wait is bounded; a failed wait is carried to the next block-wide
// barrier (__syncthreads_or), where all threads leave together (no trap).
#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"
#include "tc_host.h"

namespace sjb {

__device__ int g_attn_tc_err;

namespace {
using namespace tc;

constexpr int QT = 128;        // queries per work item
constexpr int KT = 64;         // keys per tile
constexpr int DH = 64;
constexpr int KV_STAGES = 2;
constexpr int kThreads = 128;
constexpr int kCtasPerSm = 4;
constexpr int CHUNK = 64;      // work items decoded at a time
constexpr int Q_BYTES = QT * DH * 2;       // 16 KB
constexpr int KV_BYTES = KT * DH * 2;      // 8 KB each for K and V
constexpr int SMEM_BYTES = Q_BYTES + KV_STAGES * 2 * KV_BYTES + 1024;
constexpr uint32_t TMEM_COLS = 128;
constexpr uint32_t COL_S = 0, COL_O = KT;  // P (bf16 pairs) in columns [0, 32) over S
constexpr float kRescaleLog2 = 8.f;  // move the reference max when exceeded by 2^8
constexpr uint32_t IDESC_S = idesc_bf16(QT, KT, false, false);
constexpr uint32_t IDESC_O = idesc_bf16(QT, DH, false, true);

__device__ __forceinline__ void record_err(int* err, int code) {
  atomicCAS(err ? err : &g_attn_tc_err, 0, code);
}

__device__ __forceinline__ float ex2(float x) {  // 2^x on the MUFU (ex2.approx, flush-to-zero)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- packed fp32 pairs (fma/add .f32x2) ----
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

// 2^x on both halves with one MUFU op: pack to f16 pairs, ex2.approx.f16x2, unpack.
__device__ __forceinline__ f32x2 ex2_pair(f32x2 x) {
  const float2 v = unpk2(x);
  uint32_t h;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(v.y), "f"(v.x));  // low half = v.x
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(h) : "r"(h));
  float a, b;
  asm("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
      "cvt.f32.f16 %0, lo;\n\tcvt.f32.f16 %1, hi;\n\t}"
      : "=f"(a), "=f"(b)
      : "r"(h));
  return pk2(a, b);
}

// Row halves of 32 S columns (thread = row).  Columns at or past `lim`
// (relative to the half) become -inf; with a window, those outside
// [lo, hi) (relative) do.
__device__ __forceinline__ void mask_hi(uint32_t (&r)[32], int lim) {
#pragma unroll
  for (int c = 0; c < 32; ++c)
    if (c >= lim) r[c] = __float_as_uint(-INFINITY);
}
__device__ __forceinline__ void mask_lohi(uint32_t (&r)[32], int lo, int hi) {
#pragma unroll
  for (int c = 0; c < 32; ++c)
    if (c < lo || c >= hi) r[c] = __float_as_uint(-INFINITY);
}
__device__ __forceinline__ float max32(const uint32_t (&r)[32]) {
  float a = -INFINITY, b = -INFINITY, c = -INFINITY, d = -INFINITY;
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    a = max3(a, __uint_as_float(r[i]), __uint_as_float(r[i + 1]));
    b = max3(b, __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
    c = max3(c, __uint_as_float(r[i + 4]), __uint_as_float(r[i + 5]));
    d = max3(d, __uint_as_float(r[i + 6]), __uint_as_float(r[i + 7]));
  }
  return max3(a, b, fmaxf(c, d));
}
// P = 2^(s * scale - m) for 32 columns -> 16 bf16 pairs; fp32 row sums in acc0/acc1
__device__ __forceinline__ void exp32(const uint32_t (&r)[32], f32x2 scale2, f32x2 negm2,
                                      uint32_t* pk, f32x2& acc0, f32x2& acc1) {
#pragma unroll
  for (int c = 0; c < 32; c += 2) {
    const f32x2 x = fma2(pk2(__uint_as_float(r[c]), __uint_as_float(r[c + 1])), scale2, negm2);
    const f32x2 p = ex2_pair(x);
    if ((c >> 1) & 1) acc1 = add2(acc1, p);
    else acc0 = add2(acc0, p);
    const float2 pf = unpk2(p);
    __nv_bfloat162 pb = __floats2bfloat162_rn(pf.x, pf.y);
    pk[c >> 1] = *reinterpret_cast<uint32_t*>(&pb);
  }
}

// 32 bytes to global memory in one store (address 32-byte aligned)
__device__ __forceinline__ void st_global_v8(void* p, const uint32_t (&v)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

struct __align__(16) Item {
  int q0, h, s0, n, nk, t_lo, n_kv, pad;  // n_kv: -1 idle grid slot, 0 no visible key
};

// Work item w: list form (tiles != null): tile w / H, head w % H; grid form:
// w = ((nqt - 1 - qtile) * B + b) * H + h, the highest query tiles first: only
// long segments have them, so without a schedule the longest work still goes
// first (C2's mixed lengths: 91 -> ~75 us).  Idle grid-form items get n_kv = -1.
__device__ __forceinline__ Item decode(int w, const int2* tiles, int H, int nqt, int B,
                                       const int32_t* cu, const int32_t* kv_lens, int window,
                                       int long_min) {
  Item it;
  it.h = w % H;
  const int rest = w / H;
  int b;
  if (tiles) {
    const int2 t = tiles[rest];
    b = t.x;
    it.q0 = t.y;
  } else {
    b = rest % B;
    it.q0 = (nqt - 1 - rest / B) * QT;
  }
  it.s0 = cu[b];
  it.n = cu[b + 1] - it.s0;
  it.pad = 0;
  if (it.q0 >= it.n || (!tiles && it.n >= long_min)) {
    it.nk = it.t_lo = 0;
    it.n_kv = -1;
    return it;
  }
  const int nk = kv_lens ? kv_lens[b] : it.n;
  it.nk = min(nk, it.n);
  int k_lo = 0, k_hi = it.nk;
  if (window > 0) {
    k_lo = max(0, it.q0 - window);
    k_hi = min(it.nk, it.q0 + QT - 1 + window + 1);
  }
  it.t_lo = k_lo / KT;
  it.n_kv = k_hi > k_lo ? (k_hi - 1) / KT - it.t_lo + 1 : 0;
  return it;
}

// A query-tile list carried in the launch's own parameter block (NS > 1):
// callers that allocate nothing still get a longest-first order, and every
// launch has its own copy.  NS = 1: no list in the parameters.
template <int NS>
struct TileList {
  int2 t[NS];
};

template <int NS>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    attn_tc_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapKV,
                   const int32_t* __restrict__ cu, const int32_t* __restrict__ kv_lens,
                   bf16* __restrict__ O, int H, int window, const int2* __restrict__ tiles_arg,
                   int n_items, int nqt, int B, int* err, int inject, int long_min,
                   const __grid_constant__ TileList<NS> plist) {
  const int2* tiles = NS > 1 ? plist.t : tiles_arg;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t q_full, kv_full[KV_STAGES], s_full, pv_done, drain;
  __shared__ Item items[2][CHUNK];  // this CTA's work items, chunk c in items[c & 1]
  __shared__ uint32_t tmem_sh;

  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem;
  uint8_t* sKV = smem + Q_BYTES;  // stage s: K at s * 2 * KV, V at + KV
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool leader = tid == 0;
  const bool o32 = (reinterpret_cast<uintptr_t>(O) & 31) == 0;

  // this CTA's items: w = blockIdx.x + k * gridDim.x, k < cnt
  const int cnt =
      n_items > (int)blockIdx.x ? (n_items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  auto decode_chunk = [&](int c) {
    const int k = c * CHUNK + tid;
    if (tid < CHUNK && k < cnt)
      items[c & 1][tid] = decode((int)blockIdx.x + k * (int)gridDim.x, tiles, H, nqt, B, cu,
                                 kv_lens, window, long_min);
  };

  if (leader) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < KV_STAGES; ++s) mbar_init(&kv_full[s], 1);
    mbar_init(&s_full, 1);
    mbar_init(&pv_done, 1);
    mbar_init(&drain, 1);
    fence_barrier_init();
    tma_prefetch(&mapQ);
    tma_prefetch(&mapKV);
  }
  if (warp == 0) tmem_alloc(&tmem_sh, TMEM_COLS);
  decode_chunk(0);
  decode_chunk(1);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = tmem_sh;

  // ---- loads (thread 96, the loader): K/V tiles in item order through the
  // ring, Q per item; MMAs (thread 0).  Both keep their bookkeeping in shared
  // memory (no registers in the other threads); thread 0 reads the loader's
  // counters (volatile, monotonic) only to decide whether a load is out.
  __shared__ struct {
    int lk, lj;            // loader: next K/V tile to load: item lk, tile lj
    uint32_t kv_issued;    // loader: K/V tiles loaded (tile t goes to stage t % KV_STAGES)
    uint32_t q_issued;     // loader: Q loads
    int q_item;            // loader: item whose Q is in the buffer or on its way
    uint32_t kv_done;      // thread 0: K/V tiles whose arrival it has seen
    uint32_t q_done;       // thread 0: Q loads whose arrival it has seen
    uint32_t s_issued;     // thread 0: S computed or on its way for tiles < s_issued
  } ls;
  const bool loader = tid == 96;  // lane 0 of warp 3
  if (leader) {
    ls.lk = ls.lj = 0;
    ls.kv_issued = ls.kv_done = ls.q_issued = ls.q_done = ls.s_issued = 0;
    ls.q_item = -1;
  }
  __syncthreads();
  int &lk = ls.lk, &lj = ls.lj, &q_item = ls.q_item;
  uint32_t &kv_issued = ls.kv_issued, &kv_done = ls.kv_done, &q_issued = ls.q_issued,
           &q_done = ls.q_done, &s_issued = ls.s_issued;
  auto kv_out = [&]() { return *reinterpret_cast<volatile uint32_t*>(&ls.kv_issued); };
  auto q_out_item = [&]() { return *reinterpret_cast<volatile int*>(&ls.q_item); };
  auto item_at = [&](int k) -> const Item& { return items[(k / CHUNK) & 1][k % CHUNK]; };
  // K/V loads while a stage is free (`released` tiles have finished their P.V)
  // and the item is decoded (chunks up to `chunk_hi`)
  auto issue_kv = [&](uint32_t released, int chunk_hi) {
    const int k_end = min(cnt, (chunk_hi + 1) * CHUNK);
    while (kv_issued < released + KV_STAGES && lk < k_end) {
      const Item& it = item_at(lk);
      if (it.n_kv <= 0) {
        ++lk;
        lj = 0;
        continue;
      }
      const int stage = kv_issued % KV_STAGES;
      const int row = it.s0 + (it.t_lo + lj) * KT;
      uint8_t* dst = sKV + stage * 2 * KV_BYTES;
      mbar_expect_tx(&kv_full[stage], 2 * KV_BYTES);
      tma_load_2d(dst, &mapKV, &kv_full[stage], (H + it.h) * DH, row);
      tma_load_2d(dst + KV_BYTES, &mapKV, &kv_full[stage], (2 * H + it.h) * DH, row);
      ++kv_issued;
      if (++lj == it.n_kv) {
        ++lk;
        lj = 0;
      }
    }
  };
  auto issue_q = [&](int k) {
    const Item& it = item_at(k);
    mbar_expect_tx(&q_full, Q_BYTES);
    tma_load_2d(sQ, &mapQ, &q_full, it.h * DH, it.s0 + it.q0);
    ++q_issued;
    q_item = k;
  };
  // S of K/V tile t (the first of its item: wait for Q too); false if a wait ran out
  auto issue_s = [&](bool first, uint32_t t) -> bool {
    if (first) {
      if (!mbar_wait(&q_full, q_done & 1)) return false;
      ++q_done;
    }
    if (!mbar_wait(&kv_full[t % KV_STAGES], (t / KV_STAGES) & 1)) return false;
    ++kv_done;
    fence_after_sync();
    const uint32_t q_addr = smem_u32(sQ);
    const uint32_t k_addr = smem_u32(sKV + (t % KV_STAGES) * 2 * KV_BYTES);
#pragma unroll
    for (int kk = 0; kk < DH / 16; ++kk)
      mma_bf16(tmem + COL_S, desc_kmajor_sw128(q_addr + kk * 32),
               desc_kmajor_sw128(k_addr + kk * 32), IDESC_S, kk != 0);
    mma_commit(&s_full);
    s_issued = t + 1;
    return true;
  };
  // Q for the first active item after k within the decoded chunks (loader)
  auto prefetch_q = [&](int k, int chunk_hi) {
    const int k_end = min(cnt, (chunk_hi + 1) * CHUNK);
    for (int k2 = k + 1; k2 < k_end; ++k2)
      if (item_at(k2).n_kv > 0) {
        issue_q(k2);
        break;
      }
  };

  // ---- per-thread state ----
  const float scale = 0.125f * 1.4426950408889634f;  // log2(e) / sqrt(64)
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  const uint32_t tS = tmem + COL_S + lane_off, tO = tmem + COL_O + lane_off;
  uint32_t g = 0;  // K/V tiles consumed (global over items)
  int fail = 0;    // a wait ran out (uniform within each warp)
  // bounded wait by lane 0, result broadcast to the warp (all 32 lanes call it)
  auto warp_wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    int okw = 1;
    if (lane == 0) okw = mbar_wait(bar, parity) ? 1 : 0;
    return __shfl_sync(0xffffffffu, okw, 0) != 0;
  };
  // after a section run by lane 0 of warp w alone (thread 0: w = 0, the
  // loader: w = 3): the warp reconverges and adopts lane 0's failure
  auto join = [&](int w) {
    if (warp == w) {
      __syncwarp();
      fail |= __shfl_sync(0xffffffffu, fail, 0);
    }
  };

  for (int k = 0; k < cnt; ++k) {
    if (k > 0 && k % CHUNK == 0) {
      // entering chunk c: decode chunk c + 1 into the buffer chunk c - 1 used
      if (__syncthreads_or(fail)) break;
      decode_chunk(k / CHUNK + 1);
      if (__syncthreads_or(fail)) break;
    }
    const int chunk_hi = k / CHUNK + 1;
    const Item it = item_at(k);
    if (it.n_kv < 0) continue;  // idle grid slot
    const int i_q = it.q0 + tid;
    const bool live = i_q < it.n;
    bf16* orow = O + (int64_t)(it.s0 + i_q) * H * DH + it.h * DH;
    if (it.n_kv == 0) {  // no visible key at all: the reference's empty sum gives 0
      if (live)
        for (int q = 0; q < 8; ++q) reinterpret_cast<uint4*>(orow)[q] = make_uint4(0, 0, 0, 0);
      continue;
    }
    // (inject: the failure-detection test's launch issues no load, so the
    // first wait below runs out with nothing in flight)
    if (loader && !fail && !inject) {
      if (q_item != k) issue_q(k);
      if (lk < k) {  // items lk..k-1 had no tiles (their buffer may be reused)
        lk = k;
        lj = 0;
      }
      issue_kv(g, chunk_hi);  // at least this item's first tiles
    }
    join(3);
    int lo = 0, hi = it.nk;
    if (window > 0) {
      lo = max(0, i_q - window);
      hi = min(it.nk, i_q + window + 1);
    }
    float m_ref = -INFINITY, l = 0.f;
    bool broke = false;
    for (int j = 0; j < it.n_kv; ++j, ++g) {
      // this tile's visible keys: without a window, [kbase, kbase + lim) for
      // every row (uniform); a tile with lim <= 32 uses its first 32 columns
      const int kbase = (it.t_lo + j) * KT;
      const int lim = window == 0 ? min(KT, it.nk - kbase) : KT;
      const bool two = lim > 32;
      // S = Q K_j^T (thread 0), unless issued right after the previous P.V
      if (leader && !fail && s_issued <= g) {
        if (!issue_s(j == 0, g)) {
          record_err(err, 10);
          fail = 1;
        }
      }
      join(0);
      // softmax: S_j -> P_j (every thread, its row)
      if (!fail && !warp_wait(&s_full, g & 1)) {
        if (lane == 0) record_err(err, 11);
        fail = 1;
      }
      // Q is free once this item's last S is done: the loader fetches the next item's
      if (loader && !fail && j == it.n_kv - 1) prefetch_q(k, chunk_hi);
      join(3);
      if (!fail) {
        fence_after_sync();
        uint32_t ra[32], rb[32];
        tmem_ld32(tS, ra);
        if (two) tmem_ld32(tS + 32, rb);
        tmem_ld_wait();
        if (window == 0) {
          if (lim < 32) mask_hi(ra, lim);
          if (two && lim < KT) mask_hi(rb, lim - 32);
        } else {
          mask_lohi(ra, lo - kbase, hi - kbase);
          mask_lohi(rb, lo - kbase - 32, hi - kbase - 32);
        }
        float mt = max32(ra);
        if (two) mt = fmaxf(mt, max32(rb));
        const float m_tile = mt * scale;
        // move the reference max on the first visible tile, or when exceeded by 2^8
        const bool first = m_ref == -INFINITY;
        const bool grow = !first && m_tile > m_ref + kRescaleLog2;
        const float m_new = (first || grow) ? m_tile : m_ref;
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const float resc = grow ? ex2(m_ref - m_new) : 1.f;
        if (grow) l *= resc;
        m_ref = m_new;
        // P_j = 2^(s * scale - m_use), two exponentials per MUFU op (ex2 on
        // f16 pairs: arguments <= 8, results <= 256; P is rounded to bf16
        // afterwards, below f16's precision); fp32 row sum
        const f32x2 scale2 = pk2(scale, scale), negm2 = pk2(-m_use, -m_use);
        f32x2 acc0 = pk2(0.f, 0.f), acc1 = pk2(0.f, 0.f);
        // P over the first 16 (32) columns of S, which is in registers
        uint32_t pk[16];
        exp32(ra, scale2, negm2, pk, acc0, acc1);
        tmem_st16(tS, pk);
        if (two) {
          exp32(rb, scale2, negm2, pk, acc0, acc1);
          tmem_st16(tS + 16, pk);
        }
        const float2 s0 = unpk2(acc0), s1 = unpk2(acc1);
        l += (s0.x + s0.y) + (s1.x + s1.y);
        if (__any_sync(0xffffffffu, grow) && j >= 1) {
          // O holds P_0..P_{j-1} V against the old reference (the P.V of tile
          // j - 1 is done: S_j was issued after it): rescale this warp's rows
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
      }
      fence_before_sync();
      if (__syncthreads_or(fail)) {
        broke = true;
        break;
      }
      // O += P_j V_j (thread 0; 32 keys when the tile's second half is
      // empty), then the next S at once; the loader issues the loads the
      // P.V frees
      if (leader) {
        fence_after_sync();
        const uint32_t v_addr = smem_u32(sKV + (g % KV_STAGES) * 2 * KV_BYTES + KV_BYTES);
        const int ksteps = two ? KT / 16 : 2;
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk)
          if (kk < ksteps)
            mma_bf16_ts(tmem + COL_O, tmem + COL_S + kk * 8,
                        desc_mnmajor_sw128(v_addr + kk * 16 * 128), IDESC_O,
                        (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&pv_done);
        if (!mbar_wait(&pv_done, g & 1)) {
          record_err(err, 12);
          fail = 1;
        } else {
          // tile g + 1 belongs to this item or to the item whose Q is loading;
          // issue its S now if the loader has its K/V load out (and, for a
          // new item, its Q is in)
          const bool same = j + 1 < it.n_kv;
          bool go = kv_out() > g + 1 && (same || q_out_item() > k);
          if (go && !same) go = mbar_test(&q_full, q_done & 1);
          if (go && !issue_s(!same, g + 1)) {
            record_err(err, 10);
            fail = 1;
          }
        }
      }
      join(0);
      if (loader) {
        if (!mbar_wait(&pv_done, g & 1)) {
          record_err(err, 12);
          fail = 1;
        } else {
          issue_kv(g + 1, chunk_hi);
        }
      }
      join(3);
    }
    if (broke) break;
    // the item's output: wait for its last P.V (thread 0 already has: the
    // phase is complete for it), then O / l
    if (!fail && !warp_wait(&pv_done, (g - 1) & 1)) {
      if (lane == 0) record_err(err, 13);
      fail = 1;
    }
    if (fail) continue;  // carried to the next block-wide barrier
    fence_after_sync();
    uint32_t oa[32], ob[32];
    tmem_ld32(tO, oa);
    tmem_ld32(tO + 32, ob);
    tmem_ld_wait();
    fence_before_sync();
    if (live) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      // the row's 64 outputs in four 32-byte stores when O is 32-byte aligned
      // (rows are then too: their pitch is H * 128 bytes), else eight of 16
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t wv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int d = q * 16 + 2 * e;
          const float a = __uint_as_float(d < 32 ? oa[d] : ob[d - 32]) * inv;
          const float b2 = __uint_as_float(d + 1 < 32 ? oa[d + 1] : ob[d - 31]) * inv;
          __nv_bfloat162 hb = __floats2bfloat162_rn(a, b2);
          wv[e] = *reinterpret_cast<uint32_t*>(&hb);
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

  // drain: every issued copy has landed and every MMA is done before TMEM and
  // shared memory are released (at most one Q and KV_STAGES K/V loads are open;
  // the barrier makes the loader's counters visible to thread 0)
  __syncthreads();
  if (leader) {
    if (q_issued > q_done && !mbar_wait(&q_full, q_done & 1)) record_err(err, 14);
    for (uint32_t t = kv_done; t < kv_issued; ++t)
      if (!mbar_wait(&kv_full[t % KV_STAGES], (t / KV_STAGES) & 1)) record_err(err, 15);
    mma_commit(&drain);
    if (!mbar_wait(&drain, 0)) record_err(err, 16);
  }
  fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    fence_after_sync();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

bool attn_tc_supported(int Dh) { return Dh == DH; }

namespace {
std::atomic<int> g_inject_timeout{0};
}

void attn_tc_inject_wait_timeout(bool enable) { g_inject_timeout.store(enable ? 1 : 0); }

cudaError_t attn_tc_take_status(int* code) {
  int v = 0;
  cudaError_t rc = cudaMemcpyFromSymbol(&v, g_attn_tc_err, sizeof(int));
  if (rc == cudaSuccess && v != 0) {
    const int zero = 0;
    rc = cudaMemcpyToSymbol(g_attn_tc_err, &zero, sizeof(int));
  }
  *code = v;
  return rc;
}

cudaError_t attn_tc(const bf16* qkv, const int32_t* cu, const int32_t* kv_lens, bf16* O, int T,
                    int H, int window, const int2* tiles, int n_tiles, int B, int max_seqlen,
                    int* err, cudaStream_t st, int long_min) {
  static std::atomic<uint64_t> attr_done{0};  // per device ordinal
  if (cudaError_t rc = ensure_smem_attr(attn_tc_kernel<1>, SMEM_BYTES, attr_done)) return rc;
  if (T <= 0) return cudaSuccess;
  CUtensorMap mq, mkv;
  const uint64_t cols = 3ull * H * DH;
  if (!make_map_bf16(&mq, qkv, cols, T, cols * 2, DH, QT) ||
      !make_map_bf16(&mkv, qkv, cols, T, cols * 2, DH, KT))
    return cudaErrorInvalidValue;
  const int nqt = tiles ? 0 : (max_seqlen + QT - 1) / QT;
  const long long items = tiles ? (long long)n_tiles * H : (long long)B * nqt * H;
  if (items <= 0) return cudaSuccess;
  if (items > 0x7fffffff) return cudaErrorInvalidValue;
  const int grid = (int)std::min<long long>(items, (long long)kCtasPerSm * sm_count());
  attn_tc_kernel<1><<<grid, kThreads, SMEM_BYTES, st>>>(mq, mkv, cu, kv_lens, O, H, window,
                                                         tiles, (int)items, nqt, B, err,
                                                         g_inject_timeout.load(), long_min,
                                                         TileList<1>{});
  return cudaGetLastError();
}

cudaError_t attn_tc_host_list(const bf16* qkv, const int32_t* cu, const int32_t* kv_lens, bf16* O,
                              int T, int H, int window, const int2* host_tiles, int n_tiles,
                              int B, int* err, cudaStream_t st) {
  static std::atomic<uint64_t> attr_done{0};  // per device ordinal
  if (cudaError_t rc = ensure_smem_attr(attn_tc_kernel<kAttnTcListMax>, SMEM_BYTES, attr_done))
    return rc;
  if (n_tiles < 0 || n_tiles > kAttnTcListMax) return cudaErrorInvalidValue;
  if (T <= 0 || n_tiles == 0) return cudaSuccess;
  CUtensorMap mq, mkv;
  const uint64_t cols = 3ull * H * DH;
  if (!make_map_bf16(&mq, qkv, cols, T, cols * 2, DH, QT) ||
      !make_map_bf16(&mkv, qkv, cols, T, cols * 2, DH, KT))
    return cudaErrorInvalidValue;
  const long long items = (long long)n_tiles * H;
  if (items > 0x7fffffff) return cudaErrorInvalidValue;
  static thread_local TileList<kAttnTcListMax> list;  // 16 KB: kept off the stack
  std::copy(host_tiles, host_tiles + n_tiles, list.t);
  const int grid = (int)std::min<long long>(items, (long long)kCtasPerSm * sm_count());
  attn_tc_kernel<kAttnTcListMax><<<grid, kThreads, SMEM_BYTES, st>>>(
      mq, mkv, cu, kv_lens, O, H, window, nullptr, (int)items, 0, B, err,
      g_inject_timeout.load(), 0x7fffffff, list);
  return cudaGetLastError();
}

}  // namespace sjb
