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
//   warps 0-3  softmax: thread = query row = TMEM lane; online softmax in
//              registers; P (bf16) written to 128-byte-swizzled shared memory
//              once O_{j-1} has been folded (one P buffer); the output
//              accumulator o[64] lives in registers
//   warp 4     TMA producer: Q of each item (2 buffers, so the next item's Q
//              loads during the current one), then its K/V tiles of 64 keys
//              through a 3-stage ring that runs on across items
//   warp 5     MMA issuer: S_j = Q K_j^T into TMEM S[g%2] (M=128, N=64, K=64),
//              O_j = P_j V_j into TMEM O[g%2] (V is the MN-major operand);
//              g counts key tiles across items, so every buffer's phase runs
//              on across items as well
// The softmax warps fold O_{j-1} into o[] while the tensor core computes
// S_{j+1} and O_j.  Keys past kv_len and outside the window
// are masked with -inf (tiles wholly inside skip the mask); key tiles wholly
// outside the window are skipped.  All mbarrier waits are bounded (error code,
// no trap).
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
constexpr int STAGES = 3;
constexpr int kThreads = 192;
constexpr int Q_BYTES = QT * DH * 2;       // 16 KB
constexpr int KV_BYTES = KT * DH * 2;      // 8 KB each for K and V
constexpr int P_BYTES = QT * KT * 2;       // 16 KB
constexpr int SMEM_BYTES = 2 * Q_BYTES + STAGES * 2 * KV_BYTES + P_BYTES + 1024;
constexpr uint32_t TMEM_COLS = 256;        // S[2] x 64 + O[2] x 64
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

struct Item {
  int b, q0, h, s0, n, nk, t_lo, n_kv;
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
      s_empty[2], p_full[2], o_full[2], o_empty[2], drain;
  __shared__ uint32_t tmem_sh;
  __shared__ volatile int abort_sh;

  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sQ = smem;                                        // Q[2]
  uint8_t* sKV = smem + 2 * Q_BYTES;                         // stage s: K at s*2*KV, V at +KV
  uint8_t* sP = smem + 2 * Q_BYTES + STAGES * 2 * KV_BYTES;  // P
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 4);
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
  const uint32_t tS = tmem, tO = tmem + 2 * KT;  // S[i] at tS + i*64, O[i] at tO + i*64

  if (warp == 4) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      tma_prefetch(&mapQ);
      tma_prefetch(&mapKV);
      int stage = 0, issued = 0;
      uint32_t phase = 0, qi = 0;
      for (int w = blockIdx.x; w < n_items && !abort_sh; w += gridDim.x) {
        Item it;
        if (!decode(w, tiles, H, nqt, cu, kv_lens, window, it) || it.n_kv == 0) continue;
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
      int stage = 0;
      uint32_t phase = 0, qi = 0, g = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < n_items && ok && !abort_sh; w += gridDim.x) {
        Item it;
        if (!decode(w, tiles, H, nqt, cu, kv_lens, window, it) || it.n_kv == 0) continue;
        const int qb = qi & 1;
        if (!mbar_wait(&q_full[qb], (qi >> 1) & 1)) {
          record_err(err, 14);
          abort_sh = 1;
          break;
        }
        const uint32_t q_addr = smem_u32(sQ + qb * Q_BYTES);
        int prev_stage = 0;
        for (int j = 0; j <= it.n_kv; ++j) {
          if (j < it.n_kv) {
            const uint32_t gj = g + j;
            if (!mbar_wait(&kv_full[stage], phase) ||
                !mbar_wait(&s_empty[gj & 1], ((gj >> 1) & 1) ^ 1)) {
              record_err(err, 15);
              abort_sh = 1;
              ok = false;
              break;
            }
            fence_after_sync();
            const uint32_t k_addr = smem_u32(sKV + stage * 2 * KV_BYTES);
#pragma unroll
            for (int kk = 0; kk < DH / 16; ++kk)
              mma_bf16(tS + (gj & 1) * KT, desc_kmajor_sw128(q_addr + kk * 32),
                       desc_kmajor_sw128(k_addr + kk * 32), IDESC_S, kk != 0);
            mma_commit(&s_full[gj & 1]);
            if (j == it.n_kv - 1) mma_commit(&q_empty[qb]);  // Q free once its last S is done
          }
          if (j >= 1) {
            const uint32_t i = g + j - 1;
            if (!mbar_wait(&p_full[i & 1], (i >> 1) & 1) ||
                !mbar_wait(&o_empty[i & 1], ((i >> 1) & 1) ^ 1)) {
              record_err(err, 16);
              abort_sh = 1;
              ok = false;
              break;
            }
            fence_after_sync();
            const uint32_t p_addr = smem_u32(sP);
            const uint32_t v_addr = smem_u32(sKV + prev_stage * 2 * KV_BYTES + KV_BYTES);
#pragma unroll
            for (int kk = 0; kk < KT / 16; ++kk)
              mma_bf16(tO + (i & 1) * DH, desc_kmajor_sw128(p_addr + kk * 32),
                       desc_mnmajor_sw128(v_addr + kk * 16 * 128), IDESC_O, kk != 0);
            mma_commit(&o_full[i & 1]);
            mma_commit(&kv_empty[prev_stage]);
          }
          prev_stage = stage;
          if (j < it.n_kv && ++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        g += it.n_kv;
        ++qi;
      }
      mma_commit(&drain);
      if (!mbar_wait(&drain, 0)) record_err(err, 17);
    }
  } else {
    // ---------------- softmax warps 0-3 ----------------
    const int r = warp * 32 + lane;  // query row in the tile = TMEM lane
    const float scale = 0.125f * 1.4426950408889634f;  // log2(e) / sqrt(64)
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    uint32_t g = 0;
    bool failed = false;
    for (int w = blockIdx.x; w < n_items && !failed && !abort_sh; w += gridDim.x) {
      Item it;
      if (!decode(w, tiles, H, nqt, cu, kv_lens, window, it)) continue;
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
      float o[DH];
#pragma unroll
      for (int d = 0; d < DH; ++d) o[d] = 0.f;
      float m = -INFINITY, l = 0.f;
      float m_prev_tile = -INFINITY;  // running max used for P_{j-1}
      float m_acc = -INFINITY;        // scale o[] currently refers to

      auto fold = [&](uint32_t i, float m_i) -> bool {
        // o = o * 2^(m_acc - m_i) + O_i  (O_i was computed against m_i)
        int okw = 1;
        if (lane == 0) okw = mbar_wait(&o_full[i & 1], (i >> 1) & 1) ? 1 : 0;
        okw = __shfl_sync(0xffffffffu, okw, 0);
        if (!okw) return false;
        fence_after_sync();
        uint32_t ra[32], rb[32];
        tmem_ld32(tO + (i & 1) * DH + lane_off, ra);
        tmem_ld32(tO + (i & 1) * DH + 32 + lane_off, rb);
        tmem_ld_wait();
        const float c = (m_acc == -INFINITY) ? 0.f : ex2(m_acc - m_i);
#pragma unroll
        for (int d = 0; d < 32; ++d) {
          o[d] = o[d] * c + __uint_as_float(ra[d]);
          o[32 + d] = o[32 + d] * c + __uint_as_float(rb[d]);
        }
        m_acc = m_i;
        fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_empty[i & 1]);
        return true;
      };

      for (int j = 0; j < it.n_kv; ++j) {
        const uint32_t gj = g + j;
        int okw = 1;
        if (lane == 0) okw = mbar_wait(&s_full[gj & 1], (gj >> 1) & 1) ? 1 : 0;
        okw = __shfl_sync(0xffffffffu, okw, 0);
        if (!okw || abort_sh) { failed = true; break; }
        fence_after_sync();
        uint32_t ra[32], rb[32];
        tmem_ld32(tS + (gj & 1) * KT + lane_off, ra);
        tmem_ld32(tS + (gj & 1) * KT + 32 + lane_off, rb);
        tmem_ld_wait();
        fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[gj & 1]);
        const int kbase = (it.t_lo + j) * KT;
        // raw scores stay in ra/rb; masked keys become -inf
        float tmax = -INFINITY;
        if (window == 0 && kbase + KT <= it.nk) {  // interior tile: every key visible
#pragma unroll
          for (int c = 0; c < KT; ++c) tmax = fmaxf(tmax, __uint_as_float(c < 32 ? ra[c] : rb[c - 32]));
        } else {
#pragma unroll
          for (int c = 0; c < KT; ++c) {
            const int key = kbase + c;
            uint32_t& cell = c < 32 ? ra[c] : rb[c - 32];
            const float v = (key >= lo && key < hi) ? __uint_as_float(cell) : -INFINITY;
            cell = __float_as_uint(v);
            tmax = fmaxf(tmax, v);
          }
        }
        // running max in log2 units: m = max(m, tmax / sqrt(Dh) * log2 e)
        const float m_new = fmaxf(m, tmax * scale);
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const float corr = m == -INFINITY ? 0.f : ex2(m - m_use);
        // P_j = 2^(s * scale - m_use) packed to bf16 pairs; fp32 row sum
        float rs = 0.f;
        uint32_t pk[KT / 2];
#pragma unroll
        for (int c = 0; c < KT; c += 2) {
          const float p0 = ex2(fmaf(__uint_as_float(c < 32 ? ra[c] : rb[c - 32]), scale, -m_use));
          const float p1 =
              ex2(fmaf(__uint_as_float(c + 1 < 32 ? ra[c + 1] : rb[c - 31]), scale, -m_use));
          rs += p0 + p1;
          __nv_bfloat162 pb = __floats2bfloat162_rn(p0, p1);
          pk[c / 2] = *reinterpret_cast<uint32_t*>(&pb);
        }
        l = l * corr + rs;
        m = m_new;
        // O_{j-1} first: its completion also frees the single P buffer
        if (j >= 1 && !fold(gj - 1, m_prev_tile)) { failed = true; break; }
        uint8_t* prow = sP + r * 128;  // 128-byte-swizzled K-major row
#pragma unroll
        for (int ch = 0; ch < KT / 8; ++ch)
          *reinterpret_cast<uint4*>(prow + ((ch ^ (r & 7)) << 4)) =
              make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // P visible to the MMA
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[gj & 1]);
        m_prev_tile = m_use;
      }
      if (failed || !fold(g + it.n_kv - 1, m_prev_tile)) { failed = true; break; }
      g += it.n_kv;
      if (live) {
        // o is relative to m_acc (= the final running max); l to m
        const float c = (m_acc == -INFINITY || m == -INFINITY) ? 0.f : ex2(m_acc - m);
        const float inv = l > 0.f ? c / l : 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          uint32_t wv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __nv_bfloat162 hb =
                __floats2bfloat162_rn(o[q * 8 + 2 * e] * inv, o[q * 8 + 2 * e + 1] * inv);
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
