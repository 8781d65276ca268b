// capi.cu — kernel-level C entry points (include/snapjudge_b200.h, part 1).
//
// The five launchers of the reference's cuda/kernels.cu (sj_gemm :88,
// sj_gemm_geglu :168, sj_add_ln :243, sj_rope :282, sj_attn :351) with the
// same argument meaning, in packed varlen form, returning a status.  They
// allocate nothing: every buffer is the caller's.  Shapes the tcgen05 kernels
// take go to them; the rest run on the CUDA-core kernels (never on the host).
#include <algorithm>
#include <string>
#include <vector>

#include "../../include/snapjudge_b200.h"
#include "common.cuh"
#include "kernels.h"

using sjb::bf16;

namespace {
thread_local std::string g_err;

int fail(int code, const std::string& m) {
  g_err = m;
  return code;
}
int launched(cudaError_t rc, const char* what) {
  if (rc == cudaSuccess) return SJ_OK;
  g_err = std::string("snapjudge CUDA: ") + what + ": " + cudaGetErrorString(rc);
  return SJ_ERR_CUDA;
}
int check_cu(const int32_t* cu_host, int B, int* T, int* max_len, int* min_len = nullptr) {
  if (!cu_host) return fail(SJ_ERR_INVALID, "cu_seqlens_host is null");
  if (B < 0) return fail(SJ_ERR_INVALID, "negative batch");
  if (B > 0 && cu_host[0] != 0) return fail(SJ_ERR_INVALID, "cu_seqlens[0] must be 0");
  int ml = 0, mn = 0x7fffffff;
  for (int b = 0; b < B; ++b) {
    int n = cu_host[b + 1] - cu_host[b];
    if (n < 0) return fail(SJ_ERR_INVALID, "cu_seqlens must be non-decreasing");
    ml = n > ml ? n : ml;
    mn = n < mn ? n : mn;
  }
  *T = B > 0 ? cu_host[B] : 0;
  *max_len = ml;
  if (min_len) *min_len = mn;
  return SJ_OK;
}
}  // namespace

namespace sjb {
// Message returned by sj_last_error() on this thread (for entry points in other files).
void set_last_error(const std::string& m) { g_err = m; }
}  // namespace sjb

extern "C" {

int sj_b200_version(void) { return 100; }

const char* sj_last_error(void) { return g_err.c_str(); }

int sj_gemm(const sj_bf16* A, const sj_bf16* W, const float* bias, sj_bf16* C, int M, int N,
            int K, int has_bias, int act, void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(SJ_ERR_INVALID, "negative GEMM size");
  if (act < 0 || act > 2) return fail(SJ_ERR_INVALID, "act must be 0, 1 or 2");
  if ((M && K && !A) || (N && K && !W) || (M && N && !C) || (has_bias && !bias))
    return fail(SJ_ERR_INVALID, "null GEMM operand");
  auto st = static_cast<cudaStream_t>(stream);
  const bf16* a = reinterpret_cast<const bf16*>(A);
  const bf16* w = reinterpret_cast<const bf16*>(W);
  bf16* c = reinterpret_cast<bf16*>(C);
  const float* b = has_bias ? bias : nullptr;
  if (sjb::gemm_tc_supported(M, N, K, false))
    return launched(sjb::gemm_tc(a, w, b, c, nullptr, M, N, K, sjb::TC_STORE, act,
                                 sjb::TcRope{}, nullptr, st),
                    "gemm_tc");
  return launched(sjb::gemm_simt<bf16, bf16>(a, w, b, c, nullptr, M, N, K, act, false, st),
                  "gemm_simt");
}

int sj_gemm_geglu(const sj_bf16* A, const sj_bf16* Wi, sj_bf16* C, int M, int F, int K,
                  void* stream) {
  if (M < 0 || F < 0 || K < 0) return fail(SJ_ERR_INVALID, "negative GEMM size");
  if ((M && K && !A) || (F && K && !Wi) || (M && F && !C))
    return fail(SJ_ERR_INVALID, "null GEMM operand");
  auto st = static_cast<cudaStream_t>(stream);
  const bf16* a = reinterpret_cast<const bf16*>(A);
  const bf16* w = reinterpret_cast<const bf16*>(Wi);
  bf16* c = reinterpret_cast<bf16*>(C);
  if (sjb::gemm_tc_supported(M, F, K, true))
    return launched(sjb::gemm_tc(a, w, nullptr, c, nullptr, M, F, K, sjb::TC_GEGLU, 0,
                                 sjb::TcRope{}, nullptr, st),
                    "gemm_tc");
  return launched(sjb::gemm_simt<bf16, bf16>(a, w, nullptr, c, nullptr, M, F, K, 0, true, st),
                  "gemm_simt");
}

int sj_add_ln(float* X, const sj_bf16* R, const float* w, const float* b, sj_bf16* Y, int M,
              int D, float eps, int residual, int has_bias, void* stream) {
  if (M < 0 || D <= 0) return fail(SJ_ERR_INVALID, "bad LayerNorm size");
  if (M && (!X || !w || !Y || (residual && !R) || (has_bias && !b)))
    return fail(SJ_ERR_INVALID, "null LayerNorm operand");
  return launched(sjb::add_ln<bf16, bf16>(X, residual ? reinterpret_cast<const bf16*>(R) : nullptr,
                                          w, has_bias ? b : nullptr, reinterpret_cast<bf16*>(Y),
                                          M, D, eps, nullptr, static_cast<cudaStream_t>(stream)),
                  "add_ln");
}

int sj_rope(sj_bf16* qkv, const float* cos_t, const float* sin_t, const int32_t* cu_seqlens,
            const int32_t* cu_seqlens_host, int B, int H, int Dh, void* stream) {
  int T = 0, ml = 0, s;
  if ((s = check_cu(cu_seqlens_host, B, &T, &ml))) return s;
  if (H <= 0 || Dh <= 0 || Dh % 2) return fail(SJ_ERR_INVALID, "bad head shape");
  if (T && (!qkv || !cos_t || !sin_t || !cu_seqlens))
    return fail(SJ_ERR_INVALID, "null RoPE operand");
  return launched(sjb::rope_cu(reinterpret_cast<bf16*>(qkv), cos_t, sin_t, cu_seqlens, B, T, H,
                               Dh, static_cast<cudaStream_t>(stream)),
                  "rope");
}

int sj_attn(const sj_bf16* qkv, const int32_t* cu_seqlens, const int32_t* cu_seqlens_host,
            const int32_t* kv_lens, sj_bf16* O, int B, int H, int Dh, int window, void* stream) {
  int T = 0, ml = 0, mn = 0, s;
  if ((s = check_cu(cu_seqlens_host, B, &T, &ml, &mn))) return s;
  if (H <= 0 || window < 0) return fail(SJ_ERR_INVALID, "bad attention shape");
  if (T && (!qkv || !O || !cu_seqlens)) return fail(SJ_ERR_INVALID, "null attention operand");
  if (T == 0) return SJ_OK;
  auto st = static_cast<cudaStream_t>(stream);
  const bf16* q = reinterpret_cast<const bf16*>(qkv);
  bf16* o = reinterpret_cast<bf16*>(O);
  if (sjb::attn_tc_supported(Dh)) {
    // full attention: segments of kAttnLongMin tokens or more on the long-segment kernel
    const bool split = window == 0 && ml >= sjb::kAttnLongMin &&
                       sjb::attn_long_pays(cu_seqlens_host, B);
    if (split) {
      const int rc = launched(sjb::attn_long(q, cu_seqlens, kv_lens, o, T, H, nullptr, 0, B, ml,
                                             nullptr, st),
                              "attn_long");
      if (rc != SJ_OK) return rc;
      if (mn >= sjb::kAttnLongMin) return SJ_OK;  // no short segment left
    }
    // the remaining segments' 128-row query tiles, longest segment first (the
    // order of the engine's schedule), in the launch's parameter block when
    // they fit; otherwise the kernel's own grid order
    const int lmin = split ? sjb::kAttnLongMin : 0x7fffffff;
    long long nt = 0;
    for (int b = 0; b < B; ++b) {
      const int n = cu_seqlens_host[b + 1] - cu_seqlens_host[b];
      if (n < lmin) nt += (n + 127) / 128;
    }
    if (nt <= sjb::kAttnTcListMax) {
      static thread_local std::vector<int> segs;
      static thread_local std::vector<int2> tiles;
      segs.clear();
      tiles.clear();
      for (int b = 0; b < B; ++b) {
        const int n = cu_seqlens_host[b + 1] - cu_seqlens_host[b];
        if (n > 0 && n < lmin) segs.push_back(b);
      }
      std::stable_sort(segs.begin(), segs.end(), [&](int x, int y) {
        return cu_seqlens_host[x + 1] - cu_seqlens_host[x] >
               cu_seqlens_host[y + 1] - cu_seqlens_host[y];
      });
      for (int b : segs)
        for (int q0 = 0; q0 < cu_seqlens_host[b + 1] - cu_seqlens_host[b]; q0 += 128)
          tiles.push_back(make_int2(b, q0));
      return launched(sjb::attn_tc_host_list(q, cu_seqlens, kv_lens, o, T, H, window, tiles.data(),
                                             (int)tiles.size(), B, nullptr, st),
                      "attn_tc");
    }
    return launched(sjb::attn_tc(q, cu_seqlens, kv_lens, o, T, H, window, nullptr, 0, B, ml,
                                 nullptr, st, lmin),
                    "attn_tc");
  }
  if (Dh != 8 && Dh != 16 && Dh != 32 && Dh != 64 && Dh != 128)
    return fail(SJ_ERR_UNSUPPORTED, "head_dim must be 8, 16, 32, 64 or 128");
  return launched(sjb::attn_simt<bf16>(q, cu_seqlens, kv_lens, o, H, Dh, window, nullptr, 0, B, ml,
                                       st),
                  "attn_simt");
}

int sj_check_device_errors(void* stream) {
  auto st = static_cast<cudaStream_t>(stream);
  cudaError_t rc = cudaStreamSynchronize(st);
  if (rc != cudaSuccess) return launched(rc, "cudaStreamSynchronize");
  int a = 0, g = 0, sc = 0, al = 0;
  if ((rc = sjb::attn_tc_take_status(&a)) != cudaSuccess) return launched(rc, "attention status");
  if ((rc = sjb::attn_long_take_status(&al)) != cudaSuccess)
    return launched(rc, "attention status");
  if (!a) a = al;
  if ((rc = sjb::gemm_tc_take_status(&g)) != cudaSuccess) return launched(rc, "GEMM status");
  if ((rc = sjb::attn_noalloc_take_status(&sc)) != cudaSuccess)
    return launched(rc, "schedule status");
  if (sc)
    return fail(SJ_ERR_INVALID, "sj_attn_noalloc: the device cu_seqlens disagree with "
                                "cu_seqlens_host; the schedule was left idle and O not written");
  if (a || g)
    return fail(SJ_ERR_TIMEOUT, std::string("a bounded device wait ran out in the ") +
                                    (a ? "attention" : "GEMM") + " kernel (code " +
                                    std::to_string(a ? a : g) +
                                    "); the outputs of the calls since the last check are "
                                    "incomplete");
  return SJ_OK;
}

void sj_test_attn_wait_timeout(int enable) { sjb::attn_tc_inject_wait_timeout(enable != 0); }

int sj_quant_e4m3(const float* x, int64_t rows, int cols, uint8_t* q, float* scale,
                  void* stream) {
  if (rows < 0 || cols <= 0 || cols % 4 != 0)
    return fail(SJ_ERR_INVALID, "rows must be >= 0 and cols a positive multiple of 4");
  if (rows && (!x || !q || !scale)) return fail(SJ_ERR_INVALID, "null quantisation operand");
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(q) & 3))
    return fail(SJ_ERR_INVALID, "x must be 16-byte and q 4-byte aligned");
  return launched(sjb::quant_rows_e4m3<float>(x, rows, cols, q, scale,
                                              static_cast<cudaStream_t>(stream)),
                  "quant_rows_e4m3");
}

int sj_gemm_e4m3(const uint8_t* A, const uint8_t* W, const float* sa, const float* sw,
                 const float* bias, sj_bf16* C, int M, int N, int K, int has_bias, int act,
                 int geglu, void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(SJ_ERR_INVALID, "negative GEMM size");
  if (act < 0 || act > 2) return fail(SJ_ERR_INVALID, "act must be 0, 1 or 2");
  if (M == 0 || N == 0) return SJ_OK;
  const int epi = geglu ? sjb::TC_GEGLU : sjb::TC_STORE;
  if (!sjb::gemm_tc_f8_supported(M, N, K, epi))
    return fail(SJ_ERR_UNSUPPORTED, "the e4m3 GEMM needs K % 128 == 0 and N % 64 == 0");
  if (!A || !W || !sa || !sw || !C || (has_bias && !geglu && !bias))
    return fail(SJ_ERR_INVALID, "null GEMM operand");
  return launched(sjb::gemm_tc_f8(A, W, sa, sw, (has_bias && !geglu) ? bias : nullptr,
                                  reinterpret_cast<bf16*>(C), M, N, K, epi, geglu ? 0 : act,
                                  sjb::TcRope{}, nullptr, static_cast<cudaStream_t>(stream)),
                  "gemm_tc_f8");
}

}  // extern "C"
