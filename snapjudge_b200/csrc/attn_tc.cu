// attn_tc.cu — tcgen05 flash attention for packed variable-length sequences (Dh = 64).
//
// Semantics of the reference attention (src/tensor.cpp:156-228): query i of
// segment b attends keys j in [max(0, i - w), min(kv_len, i + w + 1))
// (w = 0: all j < kv_len), scale 1/sqrt(64), max-subtracted softmax.  bf16
// q/k/v/o, fp32 scores and accumulation; P is rounded to bf16 for the P.V MMA
// (the row normaliser sums the fp32 probabilities).
//
// Persistent: 2 CTAs per SM walk a strided list of work items (128 queries of
// one segment x one head), longest segments first.  192 threads per CTA:
//   warps 0-3  softmax: thread = query row = TMEM lane.  Reads S_j from TMEM,
//              writes P_j (bf16) back to TMEM and moves on: the output is
//              accumulated in TMEM by the tensor core, so the softmax never
//              waits for a P.V product except to rescale it (below) and at the
//              end of an item
//   warp 4     TMA producer: Q of each item (2 buffers), then its K/V tiles of
//              64 keys through a 4-stage ring that runs on across items
//   warp 5     MMA issuer: S_j = Q K_j^T into TMEM S[g%2] (M=128, N=64, K=64,
//              both operands in shared memory); O += P_j V_j with P_j read from
//              TMEM (the A operand) and V from shared memory (MN-major); g
//              counts key tiles across items, so every phase runs on across items
// Rescaling: each row keeps a reference max m_ref for its exponentials and
// moves it only when a tile's max exceeds it by more than 2^8 (exponent 8 in
// log2 units); then the row's O (in TMEM) and running sum are multiplied by
// 2^(m_ref_old - m_ref_new) before the next P.V accumulates.  The result is the
// same softmax (every term uses the same reference), with P <= 2^8.
// Keys past kv_len and outside the window are masked with -inf (interior tiles
// skip the mask); key tiles wholly outside the window are skipped.  All mbarrier
// waits are bounded (error code, no trap).
#include <algorithm>

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
constexpr int STAGES = 4;
constexpr int kThreads = 192;
constexpr int Q_BYTES = QT * DH * 2;       // 16 KB
constexpr int KV_BYTES = KT * DH * 2;      // 8 KB each for K and V
constexpr int SMEM_BYTES = 2 * Q_BYTES + STAGES * 2 * KV_BYTES + 1024;
// TMEM columns: S[2] (fp32 64 each) | O (fp32 64) | P[2] (bf16 pairs, 32 each)
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t COL_S = 0, COL_O = 2 * KT, COL_P = 2 * KT + DH;
constexpr float kRescaleLog2 = 8.f;  // move the reference max when exceeded by 2^8
constexpr int RING = 4;              // decoded work items in flight (producer -> consumers)
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

// (2^a, 2^b) with one MUFU op: pack to f16 pairs, ex2.approx.f16x2, unpack.
__device__ __forceinline__ float2 ex2_pair(float a, float b) {
  uint32_t h;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(b), "f"(a));  // low half = a
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(h) : "r"(h));
  float2 r;
  asm("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
      "cvt.f32.f16 %0, lo;\n\tcvt.f32.f16 %1, hi;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "r"(h));
  return r;
}

struct Item {
  int b, q0, h, s0, n, nk, t_lo, n_kv;  // n_kv < 0 marks the end of this CTA's list
};

// Work item w: list form (tiles != null): tile w / H, head w % H; grid form:
// w = ((b * nqt) + qtile) * H + h.  False for idle grid-form items.
__device__ __forceinline__ bool decode(int w, const int2* tiles, int H, int nqt,
                                       const int32_t* cu, const int32_t* kv_lens, int window,
                                       Item& it) {
  it.h = w % H;
  const int rest = w / H;
  if (tiles) {
    const int2 t = tiles[rest];
    it.b = t.x;
    it.q0 = t.y;
  } else {
    it.b = rest / nqt;
    it.q0 = (rest % nqt) * QT;
  }
  it.s0 = cu[it.b];
  it.n = cu[it.b + 1] - it.s0;
  if (it.q0 >= it.n) return false;
  int nk = kv_lens ? kv_lens[it.b] : it.n;
  it.nk = min(nk, it.n);
  int k_lo = 0, k_hi = it.nk;
  if (window > 0) {
    k_lo = max(0, it.q0 - window);
    k_hi = min(it.nk, it.q0 + QT - 1 + window + 1);
  }
  it.t_lo = k_lo / KT;
  it.n_kv = k_hi > k_lo ? (k_hi - 1) / KT - it.t_lo + 1 : 0;
  return true;
}

__global__ void __launch_bounds__(kThreads, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapKV,
                   const int32_t* __restrict__ cu, const int32_t* __restrict__ kv_lens,
                   bf16* __restrict__ O, int H, int window, const int2* __restrict__ tiles,
                   int n_items, int nqt, int* err) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t q_full[2], q_empty[2], kv_full[STAGES], kv_empty[STAGES], s_full[2],
      s_empty[2], p_full[2], pv_done[2], drain, it_full[RING], it_empty[RING];
  __shared__ Item ring[RING];  // this CTA's work items, decoded once by the producer
  __shared__ uint32_t tmem_sh;
  __shared__ volatile int abort_sh;

  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem;                 // Q[2]
  uint8_t* sKV = smem + 2 * Q_BYTES;  // stage s: K at s*2*KV, V at +KV
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < RING; ++i) {
      mbar_init(&it_full[i], 1);
      mbar_init(&it_empty[i], 1 + 4);  // the MMA's P.V cursor + the 4 softmax warps
    }
    mbar_init(&drain, 1);
    abort_sh = 0;
    fence_barrier_init();
  }
  if (warp == 5) tmem_alloc(&tmem_sh, TMEM_COLS);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tmem = tmem_sh;

  if (warp == 4) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      // Decodes this CTA's items once (global loads off the consumers' paths),
      // publishes them in the ring, then loads each item's Q and K/V tiles.
      tma_prefetch(&mapQ);
      tma_prefetch(&mapKV);
      int stage = 0, issued = 0;
      uint32_t phase = 0, qi = 0, ri = 0;
      auto publish = [&](const Item& it) -> bool {
        const int slot = ri % RING;
        if (!mbar_wait(&it_empty[slot], ((ri / RING) & 1) ^ 1)) return false;
        ring[slot] = it;
        mbar_arrive(&it_full[slot]);  // release: the item is visible to its consumers
        ++ri;
        return true;
      };
      for (int w = blockIdx.x;; w += gridDim.x) {
        Item it;
        if (w >= n_items || abort_sh) {
          it.n_kv = -1;  // end of this CTA's list
          if (!publish(it)) record_err(err, 19);
          break;
        }
        if (!decode(w, tiles, H, nqt, cu, kv_lens, window, it)) continue;  // idle grid slot
        if (!publish(it)) {
          record_err(err, 19);
          abort_sh = 1;
          break;
        }
        if (it.n_kv == 0) continue;
        const int qb = qi & 1;
        if (!mbar_wait(&q_empty[qb], ((qi >> 1) & 1) ^ 1)) {
          record_err(err, 10);
          abort_sh = 1;
          break;
        }
        mbar_expect_tx(&q_full[qb], Q_BYTES);
        tma_load_2d(sQ + qb * Q_BYTES, &mapQ, &q_full[qb], it.h * DH, it.s0 + it.q0);
        ++qi;
        for (int j = 0; j < it.n_kv; ++j) {
          if (!mbar_wait(&kv_empty[stage], phase ^ 1)) {
            record_err(err, 11);
            abort_sh = 1;
            break;
          }
          const int row = it.s0 + (it.t_lo + j) * KT;
          uint8_t* dst = sKV + stage * 2 * KV_BYTES;
          mbar_expect_tx(&kv_full[stage], 2 * KV_BYTES);
          tma_load_2d(dst, &mapKV, &kv_full[stage], (H + it.h) * DH, row);
          tma_load_2d(dst + KV_BYTES, &mapKV, &kv_full[stage], (2 * H + it.h) * DH, row);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // drain: every issued copy has landed before the CTA can exit
      for (uint32_t k = qi > 2 ? qi - 2 : 0; k < qi; ++k)
        if (!mbar_wait(&q_full[k & 1], (k >> 1) & 1)) record_err(err, 12);
      for (int i = 0; i < STAGES && i < issued; ++i) {
        if (--stage < 0) { stage = STAGES - 1; phase ^= 1; }
        if (!mbar_wait(&kv_full[stage], phase)) record_err(err, 13);
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      // Two cursors walk the same sequence of key tiles: the S cursor runs
      // ahead as far as the two S buffers allow (it never waits behind a P.V),
      // the P.V cursor follows the softmax.  Each pass issues whatever is ready
      // (non-blocking tests); no progress for kWaitNs is an error.
      struct Cursor {
        uint32_t ri;  // ring index of the current item
        Item it;
        int j;
        uint32_t qi, g;
        int stage;
        uint32_t phase;
        bool have, done;
      };
      // Move to the next item with key tiles if the ring has it (non-blocking).
      // The P.V cursor (release = true) frees ring slots it is done with.
      auto seek = [&](Cursor& c, bool release) {
        while (!c.have && !c.done) {
          const int slot = c.ri % RING;
          if (!mbar_test(&it_full[slot], (c.ri / RING) & 1)) return;
          c.it = ring[slot];
          if (c.it.n_kv < 0) {
            c.done = true;
            return;
          }
          if (c.it.n_kv == 0) {
            if (release) mbar_arrive(&it_empty[slot]);
            ++c.ri;
            continue;
          }
          c.j = 0;
          c.have = true;
        }
      };
      auto advance = [&](Cursor& c, bool release) {
        ++c.g;
        if (++c.stage == STAGES) { c.stage = 0; c.phase ^= 1; }
        if (++c.j == c.it.n_kv) {
          if (release) mbar_arrive(&it_empty[c.ri % RING]);
          ++c.qi;
          ++c.ri;
          c.have = false;
        }
      };
      Cursor cs{0u, {}, 0, 0u, 0u, 0, 0u, false, false};
      Cursor cp = cs;
      uint64_t t_last = globaltimer();
      while (!cp.done && !abort_sh) {
        bool progressed = false;
        seek(cs, false);
        if (cs.have) {
          const int qb = cs.qi & 1;
          if ((cs.j > 0 || mbar_test(&q_full[qb], (cs.qi >> 1) & 1)) &&
              mbar_test(&kv_full[cs.stage], cs.phase) &&
              mbar_test(&s_empty[cs.g & 1], ((cs.g >> 1) & 1) ^ 1)) {
            fence_after_sync();
            const uint32_t q_addr = smem_u32(sQ + qb * Q_BYTES);
            const uint32_t k_addr = smem_u32(sKV + cs.stage * 2 * KV_BYTES);
#pragma unroll
            for (int kk = 0; kk < DH / 16; ++kk)
              mma_bf16(tmem + COL_S + (cs.g & 1) * KT, desc_kmajor_sw128(q_addr + kk * 32),
                       desc_kmajor_sw128(k_addr + kk * 32), IDESC_S, kk != 0);
            mma_commit(&s_full[cs.g & 1]);
            if (cs.j == cs.it.n_kv - 1) mma_commit(&q_empty[qb]);  // Q free after its last S
            advance(cs, false);
            progressed = true;
          }
        }
        seek(cp, true);
        if (cp.have && mbar_test(&p_full[cp.g & 1], (cp.g >> 1) & 1)) {
          fence_after_sync();
          const uint32_t v_addr = smem_u32(sKV + cp.stage * 2 * KV_BYTES + KV_BYTES);
#pragma unroll
          for (int kk = 0; kk < KT / 16; ++kk)
            mma_bf16_ts(tmem + COL_O, tmem + COL_P + (cp.g & 1) * (KT / 2) + kk * 8,
                        desc_mnmajor_sw128(v_addr + kk * 16 * 128), IDESC_O,
                        (cp.j > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&pv_done[cp.g & 1]);
          mma_commit(&kv_empty[cp.stage]);
          advance(cp, true);
          progressed = true;
        }
        if (progressed) {
          t_last = globaltimer();
        } else if (globaltimer() - t_last > kWaitNs) {
          record_err(err, 15);
          abort_sh = 1;
          break;
        } else {
          __nanosleep(20);
        }
      }
      mma_commit(&drain);
      if (!mbar_wait(&drain, 0)) record_err(err, 17);
    }
  } else {
    // ---------------- softmax warps 0-3 ----------------
    const int r = warp * 32 + lane;  // query row in the tile = TMEM lane
    const float scale = 0.125f * 1.4426950408889634f;  // log2(e) / sqrt(64)
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const uint32_t tS = tmem + COL_S + lane_off, tO = tmem + COL_O + lane_off,
                   tP = tmem + COL_P + lane_off;
    uint32_t g = 0;
    bool failed = false;
    // bounded wait by lane 0, result broadcast to the warp
    auto warp_wait = [&](uint64_t* bar, uint32_t parity) -> bool {
      int okw = 1;
      if (lane == 0) okw = mbar_wait(bar, parity) ? 1 : 0;
      return __shfl_sync(0xffffffffu, okw, 0) != 0;
    };
    for (uint32_t ri = 0; !failed && !abort_sh; ++ri) {
      const int slot = ri % RING;
      if (!warp_wait(&it_full[slot], (ri / RING) & 1)) { failed = true; break; }
      const Item it = ring[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&it_empty[slot]);
      if (it.n_kv < 0) break;  // end of this CTA's list
      const int i_q = it.q0 + r;
      const bool live = i_q < it.n;
      bf16* orow = O + (int64_t)(it.s0 + i_q) * H * DH + it.h * DH;
      if (it.n_kv == 0) {  // no visible key at all: the reference's empty sum gives 0
        if (live)
          for (int q = 0; q < 8; ++q) reinterpret_cast<uint4*>(orow)[q] = make_uint4(0, 0, 0, 0);
        continue;
      }
      int lo = 0, hi = it.nk;
      if (window > 0) {
        lo = max(0, i_q - window);
        hi = min(it.nk, i_q + window + 1);
      }
      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j < it.n_kv; ++j) {
        const uint32_t gj = g + j;
        if (!warp_wait(&s_full[gj & 1], (gj >> 1) & 1) || abort_sh) { failed = true; break; }
        fence_after_sync();
        uint32_t ra[32], rb[32];
        tmem_ld32(tS + (gj & 1) * KT, ra);
        tmem_ld32(tS + (gj & 1) * KT + 32, rb);
        tmem_ld_wait();
        fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[gj & 1]);
        const int kbase = (it.t_lo + j) * KT;
        float t4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        if (window == 0 && kbase + KT <= it.nk) {  // interior tile: every key visible
#pragma unroll
          for (int c = 0; c < KT; ++c)
            t4[c & 3] = fmaxf(t4[c & 3], __uint_as_float(c < 32 ? ra[c] : rb[c - 32]));
        } else {
#pragma unroll
          for (int c = 0; c < KT; ++c) {
            const int key = kbase + c;
            uint32_t& cell = c < 32 ? ra[c] : rb[c - 32];
            const float v = (key >= lo && key < hi) ? __uint_as_float(cell) : -INFINITY;
            cell = __float_as_uint(v);
            t4[c & 3] = fmaxf(t4[c & 3], v);
          }
        }
        const float m_tile = fmaxf(fmaxf(t4[0], t4[1]), fmaxf(t4[2], t4[3])) * scale;
        // move the reference max on the first visible tile, or when exceeded by 2^8
        const bool first = m_ref == -INFINITY;
        const bool grow = !first && m_tile > m_ref + kRescaleLog2;
        const float m_new = (first || grow) ? m_tile : m_ref;
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        if (__any_sync(0xffffffffu, grow) && j >= 1) {
          // O holds P_0..P_{j-1} V against m_ref: rescale this warp's rows
          if (!warp_wait(&pv_done[(gj - 1) & 1], ((gj - 1) >> 1) & 1)) { failed = true; break; }
          fence_after_sync();
          const float c = grow ? ex2(m_ref - m_new) : 1.f;
          uint32_t oa[32], ob[32];
          tmem_ld32(tO, oa);
          tmem_ld32(tO + 32, ob);
          tmem_ld_wait();
#pragma unroll
          for (int d = 0; d < 32; ++d) {
            oa[d] = __float_as_uint(__uint_as_float(oa[d]) * c);
            ob[d] = __float_as_uint(__uint_as_float(ob[d]) * c);
          }
          tmem_st32(tO, oa);
          tmem_st32(tO + 32, ob);
          tmem_st_wait();
        }
        if (grow) l *= ex2(m_ref - m_new);
        m_ref = m_new;
        // P_j = 2^(s * scale - m_use), two exponentials per MUFU op (ex2 on
        // f16 pairs: arguments <= 8, results <= 256; P is rounded to bf16
        // afterwards, below f16's precision); fp32 row sum
        float r4[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < KT; c += 2) {
          const float x0 = fmaf(__uint_as_float(c < 32 ? ra[c] : rb[c - 32]), scale, -m_use);
          const float x1 = fmaf(__uint_as_float(c + 1 < 32 ? ra[c + 1] : rb[c - 31]), scale, -m_use);
          const float2 p = ex2_pair(x0, x1);
          r4[(c >> 1) & 3] += p.x + p.y;
          __nv_bfloat162 pb = __floats2bfloat162_rn(p.x, p.y);
          pk[c >> 1] = *reinterpret_cast<uint32_t*>(&pb);
        }
        l += (r4[0] + r4[1]) + (r4[2] + r4[3]);
        // P[gj%2] was last read by the P.V of tile gj-2
        if (!warp_wait(&pv_done[gj & 1], ((gj >> 1) & 1) ^ 1)) { failed = true; break; }
        tmem_st32(tP + (gj & 1) * (KT / 2), pk);
        tmem_st_wait();
        fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[gj & 1]);
      }
      if (failed) break;
      // the item's output: wait for its last P.V, then O / l
      const uint32_t last = g + it.n_kv - 1;
      if (!warp_wait(&pv_done[last & 1], (last >> 1) & 1)) { failed = true; break; }
      fence_after_sync();
      uint32_t oa[32], ob[32];
      tmem_ld32(tO, oa);
      tmem_ld32(tO + 32, ob);
      tmem_ld_wait();
      fence_before_sync();
      g += it.n_kv;
      if (live) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          uint32_t wv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int d = q * 8 + 2 * e;
            const float a = __uint_as_float(d < 32 ? oa[d] : ob[d - 32]) * inv;
            const float b2 = __uint_as_float(d + 1 < 32 ? oa[d + 1] : ob[d - 31]) * inv;
            __nv_bfloat162 hb = __floats2bfloat162_rn(a, b2);
            wv[e] = *reinterpret_cast<uint32_t*>(&hb);
          }
          reinterpret_cast<uint4*>(orow)[q] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        }
      }
    }
    if (failed && lane == 0) {
      record_err(err, 18);
      abort_sh = 1;
    }
  }

  fence_before_sync();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    fence_after_sync();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

bool attn_tc_supported(int Dh) { return Dh == DH; }

cudaError_t attn_tc(const bf16* qkv, const int32_t* cu, const int32_t* kv_lens, bf16* O, int T,
                    int H, int window, const int2* tiles, int n_tiles, int B, int max_seqlen,
                    int* err, cudaStream_t st) {
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t rc = cudaFuncSetAttribute(attn_tc_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (rc != cudaSuccess) return rc;
    attr_set = true;
  }
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
  const int grid = (int)std::min<long long>(items, 2LL * sm_count());
  attn_tc_kernel<<<grid, kThreads, SMEM_BYTES, st>>>(mq, mkv, cu, kv_lens, O, H, window, tiles,
                                                      (int)items, nqt, err);
  return cudaGetLastError();
}

}  // namespace sjb
