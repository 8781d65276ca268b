// kernels.h — internal launchers of the snapjudge B200 kernels (C++ only).
//
// Every launcher is asynchronous on `st` and returns the launch status.  The
// C-ABI (capi.cu) and the encoder engine (engine.cu) are the only callers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace sjb {

// Set the message sj_last_error() returns on the calling thread (capi.cu).
void set_last_error(const std::string& m);

using bf16 = __nv_bfloat16;

enum Act { ACT_NONE = 0, ACT_GELU = 1, ACT_RELU = 2 };

// ---- norms (norm.cu) ------------------------------------------------------
// X[T, D] (fp32) = LN(emb[ids] (+ pos_emb[min(pos, max_pos - 1)])) * w (+ b);
// Y = cast(X) when Y != null.  Out-of-vocabulary ids produce a zero row and set
// *bad = 1.  Positions and bias need D <= 1024 (D % 4 == 0).
template <typename TY>
cudaError_t embed_ln(const int64_t* ids, int T, const float* emb, int V, int D,
                     const float* w, float eps, float* X, TY* Y, int* bad, cudaStream_t st,
                     const float* pos_emb = nullptr, const int32_t* pos = nullptr,
                     int max_pos = 0, const float* b = nullptr);

// Optional residual add (X += R), then Y = LN(X) * w (+ b).  With `rows`
// (length M), output row i normalises X[rows[i]] and no residual is applied.
template <typename TR, typename TY>
cudaError_t add_ln(float* X, const TR* R, const float* w, const float* b, TY* Y, int M, int D,
                   float eps, const int32_t* rows, cudaStream_t st);

// ---- GEMM on CUDA cores (gemm_simt.cu) --------------------------------------
// C[M, N] = act(A[M, K] W[N, K]^T + bias)           (resid == null, geglu == false)
// resid[M, N] += A W^T (+ bias)  (fp32 residual)     (resid != null)
// C[M, N] = gelu(A Wg^T) * (A Wu^T), W = [Wg; Wu]   (geglu == true, N = F)
template <typename TA, typename TC>
cudaError_t gemm_simt(const TA* A, const TA* W, const float* bias, TC* C, float* resid, int M,
                      int N, int K, int act, bool geglu, cudaStream_t st);

// ---- RoPE (rope.cu) -------------------------------------------------------------
// In-place rotate-half on the q and k parts of qkv [M, 3*H*Dh]; row r has
// position pos[r]; cos/sin tables [max_pos, Dh/2].
template <typename T>
cudaError_t rope(T* qkv, const float* cos_t, const float* sin_t, const int32_t* pos, int M, int H,
                 int Dh, cudaStream_t st);

// Same, with the position of row r found from cu_seqlens (no position array).
cudaError_t rope_cu(bf16* qkv, const float* cos_t, const float* sin_t, const int32_t* cu, int B,
                    int M, int H, int Dh, cudaStream_t st);

// pos[r] = r - cu[b] for the sequence b owning row r; seq[r] = b (seq may be null).
cudaError_t positions(const int32_t* cu, int B, int T, int32_t* pos, int32_t* seq, cudaStream_t st);

// ---- attention on CUDA cores (attn_simt.cu) ---------------------------------
// Packed varlen bidirectional attention over qkv [T, 3*H*Dh]; O [T, H*Dh].
// Segment b = rows [cu[b], cu[b+1]); its queries attend keys j < kv_len[b]
// (kv_lens null: the whole segment), |i - j| <= window when window > 0.
// tiles: list of (b, q0) query tiles of 64 rows, n_tiles entries; or null,
// then the grid covers B x ceil(max_seqlen / 64) tiles and idle ones exit.
template <typename T>
cudaError_t attn_simt(const T* qkv, const int32_t* cu, const int32_t* kv_lens, T* O, int H, int Dh,
                      int window, const int2* tiles, int n_tiles, int B, int max_seqlen,
                      cudaStream_t st);

// ---- decision heads on [CLS] (heads.cu) ---------------------------------------
struct HeadSpec {
  int n_heads;
  int off[8];   // first output column of head h in W/bias/probs
  int n_out[8];
  int kind[8];  // 0 softmax, 1 sigmoid
  int n_total;
};
// probs[b] = heads(Hc[b]) for already-normalised rows Hc [B, D].
cudaError_t dec_heads(const float* Hc, int B, int D, const float* W, const float* bias,
                      HeadSpec spec, float* probs, cudaStream_t st);

// Y[i] = bf16(X[i]) (identity attn_norm in bf16 mode).
cudaError_t cast_bf16(const float* X, bf16* Y, int64_t n, cudaStream_t st);

// decision-model tail (head.cu): h[r] += type_emb[qtype[segment of r]];
// marker rows m[b*K + k] = h[cu[b] + clamp(pos, 0, n_b - 1)]; the act head
// (masked logits, softmax statistics, act MLP and softmax), one block per segment
cudaError_t type_emb_add(float* h, const int32_t* cu, int B, const int64_t* qtype,
                         const float* te, int D, int T, cudaStream_t st);
cudaError_t gather_markers(const float* h, const int32_t* cu, const int64_t* pos, int B, int K,
                           int D, float* m, cudaStream_t st);
size_t act_head_smem(int K, int D, int n_act);
cudaError_t act_head(const float* h, const int32_t* cu, int B, const float* score,
                     const uint8_t* mask, int K, const float* w1, const float* b1,
                     const float* w2, const float* b2, int n_act, int D, float* logits,
                     float* act, bool top1_only, cudaStream_t st);
// pooled[b] = mean of h over segment b's rows (zeros for an empty segment)
cudaError_t mean_pool(const float* h, const int32_t* cu, int B, int D, float* pooled,
                      cudaStream_t st);

// ---- tcgen05 GEMM (gemm_tc.cu) ------------------------------------------------
// True when the tensor-core GEMM takes this shape (K % 64 == 0, N tiles of 256
// or, for geglu, F % 128 == 0, 16-byte aligned rows).
bool gemm_tc_supported(int M, int N, int K, bool geglu);

// TC_RESID: fp32 resid [M, N] += acc (+ bias).  TC_RESID16: the residual is
// bf16 and is C itself (SJ_PREC_FP8_TENSOR's residual stream): C += acc (+
// bias), rounded to bf16; N % 128 == 0.
enum TcEpi { TC_STORE = 0, TC_RESID = 1, TC_GEGLU = 2, TC_ROPE = 3, TC_RESID16 = 4 };
struct TcRope {
  const float* cos_t;
  const float* sin_t;
  const int32_t* pos;
  int H;  // q and k heads of 64 columns rotate; v columns pass through
};
// bf16 A[M, K], W[N, K] (for TC_GEGLU W = [Wg; Wu], 2N rows, N = F), fp32 accum.
// TC_STORE: C = acc (+bias, act); TC_RESID: resid += acc (+bias); TC_ROPE: C = rope(acc).
cudaError_t gemm_tc(const bf16* A, const bf16* W, const float* bias, bf16* C, float* resid,
                    int M, int N, int K, int epi, int act, TcRope rope, int* err,
                    cudaStream_t st);
// The FP8 variant (tcgen05 kind::f8f6f4): A [M, K] and W [N_w, K] are e4m3
// codes with a scale per A row (sa [M]) and per W row (sw [N_w], 16-byte
// aligned); acc = sa[m] sw[n] sum_k A[m, k] W[n, k] in fp32, then the epilogue
// as gemm_tc.  Epilogues TC_STORE, TC_GEGLU, TC_ROPE, TC_RESID; K % 128 == 0.
// As attn_tc_take_status, for the GEMM launches given no error flag.
cudaError_t gemm_tc_take_status(int* code);
bool gemm_tc_f8_supported(int M, int N, int K, int epi);
// SJ_PREC_FP8_TENSOR options.  C set: GEGLU output as e4m3 codes at one static
// scale, C gets e4m3(gelu(g) u / *scale) [M, N] bytes, rowscale[m] = *scale,
// bf16 C unused.  uniform: sa and sw hold one value each (per-tensor scales),
// so the epilogue multiplies by sa[0] * sw[0] without per-row or per-column
// scale loads.
struct TcQ8 {
  uint8_t* C = nullptr;
  const float* scale = nullptr;
  float* rowscale = nullptr;
  bool uniform = false;
};
// TC_RESID adds to the fp32 resid [M, N] (W the [N, K] output projection).
cudaError_t gemm_tc_f8(const uint8_t* A, const uint8_t* W, const float* sa, const float* sw,
                       const float* bias, bf16* C, int M, int N, int K, int epi, int act,
                       TcRope rope, int* err, cudaStream_t st, float* resid = nullptr,
                       TcQ8 q8 = TcQ8{});

// ---- e4m3 quantisation (quant.cu) --------------------------------------------
// Per row: scale = amax / 448 (1 for an all-zero row), q = e4m3(x * (448 / amax))
// rounded to nearest even, saturating.  T = float or bf16.
template <typename T>
cudaError_t quant_rows_e4m3(const T* x, int64_t rows, int cols, uint8_t* q, float* scale,
                            cudaStream_t st);
// Y = LN(X) * w (+ b) quantised as quant_rows_e4m3 (X fp32 [rows, D], D % 128 == 0,
// D <= 1024): the FP8 variant's attn_norm / mlp_norm.
cudaError_t ln_e4m3(const float* X, const float* w, const float* b, uint8_t* q, float* scale,
                    int64_t rows, int D, float eps, cudaStream_t st);
// SJ_PREC_FP8_TENSOR: one static scale per activation tensor, read from device
// memory (*s_t): LN(X) * w (+ b) (or, quant_rows_static, X itself) quantised as
// x / s_t, and sa[row] = s_t for the GEMM epilogue.  TX: float or bf16 (the
// per-tensor variant's bf16 residual stream).
template <typename TX>
cudaError_t ln_e4m3_static(const TX* X, const float* w, const float* b, uint8_t* q, float* sa,
                           const float* s_t, int64_t rows, int D, float eps, cudaStream_t st);
template <typename TX>
cudaError_t quant_rows_static(const TX* x, int64_t rows, int cols, uint8_t* q, float* sa,
                              const float* s_t, cudaStream_t st);
// Y = fp32(X), n % 4 == 0; widen_rows_f32: only rows[0..n) of [*, D] (D % 4 == 0)
cudaError_t widen_f32(const bf16* X, float* Y, int64_t n, cudaStream_t st);
cudaError_t widen_rows_f32(const bf16* X, float* Y, const int32_t* rows, int n, int D,
                           cudaStream_t st);
// *amax = max(*amax, max |x|) (float bits in an unsigned; calibration)
template <typename T>
cudaError_t amax_abs(const T* x, int64_t n, unsigned* amax, cudaStream_t st);
// s[i] = amax[i] * margin / 448, 1 where amax[i] == 0
cudaError_t scales_from_amax(const unsigned* amax, float* s, int n, float margin, cudaStream_t st);
// a weight with one scale per tensor: q = e4m3(x * 448 / amax), sw[0..rows) = amax / 448
cudaError_t quant_tensor_e4m3(const float* x, int64_t n, int rows, float amax, uint8_t* q,
                              float* sw, cudaStream_t st);

// ---- tcgen05 flash attention (attn_tc.cu) -----------------------------------
bool attn_tc_supported(int Dh);
// Launches given no error flag (err == null) record a wait that ran out in a
// status word of the library on their device.  *code = that word (0: none),
// which is then cleared; synchronous, on the current device, allocates nothing.
cudaError_t attn_tc_take_status(int* code);
// Failure-detection test hook: while enabled, attention launches of this
// process issue no TMA load, so their first bounded wait runs out (nothing is
// in flight) and they record a timeout and return.
void attn_tc_inject_wait_timeout(bool enable);
// sj_attn_noalloc's schedule check: *code != 0 when a schedule build found
// device cu_seqlens that disagree with the host mirror (then cleared).
cudaError_t attn_noalloc_take_status(int* code);
// tiles: list of (b, q0) query tiles of 128 rows (or null: B x ceil(max_seqlen/128)).
// In the grid form, segments of long_min tokens or more are skipped (they
// went to attn_long).
cudaError_t attn_tc(const bf16* qkv, const int32_t* cu, const int32_t* kv_lens, bf16* O, int T,
                    int H, int window, const int2* tiles, int n_tiles, int B, int max_seqlen,
                    int* err, cudaStream_t st, int long_min = 0x7fffffff);
// The same kernel on a query-tile list given in HOST memory (at most
// kAttnTcListMax tiles): the list travels in the launch's parameter block, so
// the call allocates nothing and concurrent calls share no state.
constexpr int kAttnTcListMax = 2048;
cudaError_t attn_tc_host_list(const bf16* qkv, const int32_t* cu, const int32_t* kv_lens, bf16* O,
                              int T, int H, int window, const int2* host_tiles, int n_tiles,
                              int B, int* err, cudaStream_t st);

// ---- tcgen05 flash attention for long segments (attn_long.cu) ----------------
// Full-attention layers (no window) at head_dim 64 send segments of at least
// kAttnLongMin tokens to attn_long (one CTA per SM, items of 256 queries,
// 128-key tiles) and the rest to attn_tc.  Measured per segment length (12
// heads, 65536 tokens, L2 flushed): attn_tc is faster up to 384 tokens, the
// two are even at 512, attn_long is 8-16 % faster from 768 to 2048.
constexpr int kAttnLongMin = 512;
// The split pays when the long segments carry at least half of the attention
// work (sum of n^2 over segments): otherwise the long kernel's launch, run
// before attn_tc on the same stream, costs more than it saves (C2's mixed
// lengths with one 512-token segment: 89 against 74 us).
inline bool attn_long_pays(const int32_t* cu_host, int B) {
  double all = 0.0, lng = 0.0;
  for (int b = 0; b < B; ++b) {
    const double n = (double)(cu_host[b + 1] - cu_host[b]);
    all += n * n;
    if (n >= kAttnLongMin) lng += n * n;
  }
  return lng > 0.0 && 2.0 * lng >= all;
}
// pairs: list of (b, q0) items of 256 query rows (q0 % 256 == 0), or null:
// the grid form over B x ceil(max_seqlen / 256) items per head, segments
// shorter than kAttnLongMin idle.
cudaError_t attn_long(const bf16* qkv, const int32_t* cu, const int32_t* kv_lens, bf16* O, int T,
                      int H, const int2* pairs, int n_pairs, int B, int max_seqlen, int* err,
                      cudaStream_t st);
// As attn_tc_take_status, for attn_long launches given no error flag.
cudaError_t attn_long_take_status(int* code);

}  // namespace sjb
