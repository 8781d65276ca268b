/*
 * snapjudge_b200.h — C ABI of the B200 (sm_100a) encoder forward for snapjudge.
 *
 * Two layers, both plain C: pointers, sizes, int status.
 *
 *  1. Kernel entry points — the five extern "C" launchers of the reference's
 *     cuda/kernels.cu, in packed variable-length form (cu_seqlens instead of a
 *     padded [B, L] batch) and returning a status instead of void.  Buffers are
 *     caller-owned DEVICE memory; the call is asynchronous on `stream`
 *     (a cudaStream_t passed as void*, NULL = legacy default stream).
 *
 *  2. The encoder engine (sj_fast_*) — what the reference's FastSnapjudge
 *     (include/snapjudge/fast.hpp:15-31, cuda/fast.cpp) does: weights resident
 *     on one GPU, the whole DecisionModel encoder (src/model.cpp:222-307) on
 *     device, results back in host memory.  One engine per GPU; an engine is
 *     not re-entrant (calls on one engine must not overlap; use one engine per
 *     host thread, or serialise).
 *
 * bf16 values cross the ABI as their 16-bit patterns (sj_bf16).
 * Status: SJ_OK (0) or a negative SJ_ERR_*; the message of the last failure on
 * the calling thread is returned by sj_last_error(), and the engine's own by
 * sj_fast_last_error(e).
 */
#ifndef SNAPJUDGE_B200_H
#define SNAPJUDGE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SJ_OK 0
#define SJ_ERR_INVALID (-1)     /* bad argument, shape or input (message says which) */
#define SJ_ERR_CUDA (-2)        /* a CUDA runtime call failed */
#define SJ_ERR_UNSUPPORTED (-3) /* shape or option this build does not implement */
#define SJ_ERR_TIMEOUT (-4)     /* a bounded device-side wait ran out (kernel returned early) */
#define SJ_ERR_STATE (-5)       /* call out of order (e.g. forward before sj_fast_commit) */

#define SJ_PREC_BF16 0 /* bf16 activations/weights, fp32 accumulation, fp32 residual stream */
#define SJ_PREC_FP32 1 /* fp32 everywhere (parity mode: 1e-4 relative to the CPU forward) */
#define SJ_PREC_FP8 2  /* SJ_PREC_BF16 with the QKV and Wi (GEGLU) projections on e4m3
                          operands: per-token activation scales, per-channel weight scales,
                          fp32 accumulation (DecisionModel encoder only; reported separately,
                          not held to the bf16 tolerances) */
#define SJ_PREC_FP8_TENSOR 3 /* SJ_PREC_FP8 with one scale per tensor: per-tensor weight scales,
                                static activation scales calibrated on the engine's first
                                forward (a bf16 pass recording each operand's amax, 2x
                                headroom), and the Wo2 projection on e4m3 too (the GEGLU
                                GEMM writes e4m3 codes); intermediate_size % 128 == 0 */

#define SJ_HEAD_SOFTMAX 0
#define SJ_HEAD_SIGMOID 1

typedef uint16_t sj_bf16;

/* Version of this ABI, major * 10000 + minor * 100 + patch. */
int sj_b200_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* sj_last_error(void);

/* ------------------------------------------------------------------------- */
/* 1. Kernel entry points (device pointers, async on `stream`).              */
/* ------------------------------------------------------------------------- */

/* C[M,N] = act(A[M,K] W[N,K]^T + bias); act 0 none, 1 erf-GELU, 2 ReLU.
 * bias (fp32 [N]) is read only when has_bias != 0.
 * Replaces sj_gemm (cuda/kernels.cu:88-108). */
int sj_gemm(const sj_bf16* A, const sj_bf16* W, const float* bias, sj_bf16* C, int M, int N,
            int K, int has_bias, int act, void* stream);

/* C[M,F] = gelu(A Wi[0:F]^T) * (A Wi[F:2F]^T), Wi [2F, K] in the checkpoint layout.
 * Replaces sj_gemm_geglu (cuda/kernels.cu:168-174). */
int sj_gemm_geglu(const sj_bf16* A, const sj_bf16* Wi, sj_bf16* C, int M, int F, int K,
                  void* stream);

/* X[M,D] (fp32) += R (bf16, when residual != 0); Y = LN(X) * w (+ b when has_bias).
 * Replaces sj_add_ln (cuda/kernels.cu:243-254). */
int sj_add_ln(float* X, const sj_bf16* R, const float* w, const float* b, sj_bf16* Y, int M,
              int D, float eps, int residual, int has_bias, void* stream);

/* In-place rotate-half RoPE on the q and k heads of packed qkv [T, 3*H*Dh];
 * row r of segment b has position r - cu_seqlens[b]; cos/sin are fp32
 * [max_pos, Dh/2] tables.  T = cu_seqlens[B] (read on the host from
 * cu_seqlens_host, which must equal the device array).
 * Replaces sj_rope (cuda/kernels.cu:282-288; position r % L there). */
int sj_rope(sj_bf16* qkv, const float* cos_t, const float* sin_t, const int32_t* cu_seqlens,
            const int32_t* cu_seqlens_host, int B, int H, int Dh, void* stream);

/* Bidirectional attention over packed qkv [T, 3*H*Dh] -> O [T, H*Dh].
 * Segment b = rows [cu_seqlens[b], cu_seqlens[b+1]); its queries attend keys
 * j < kv_lens[b] of the same segment (kv_lens NULL: the whole segment) and,
 * when window > 0, only |i - j| <= window.  softmax scale 1/sqrt(Dh), fp32
 * accumulation.  cu_seqlens_host mirrors cu_seqlens: the call orders the
 * query tiles longest segment first from it (up to 2,048 tiles, passed in the
 * launch's parameters; no allocation).
 * Replaces sj_attn (cuda/kernels.cu:351-357; lens + padded L there). */
int sj_attn(const sj_bf16* qkv, const int32_t* cu_seqlens, const int32_t* cu_seqlens_host,
            const int32_t* kv_lens, sj_bf16* O, int B, int H, int Dh, int window, void* stream);

/* sj_attn with the engine's longest-first query-tile schedule, for callers
 * that cannot allocate device memory (their device memory belongs to their own
 * pool allocator, or allocation is not allowed on their inference path).  No
 * counterpart in the reference.  The schedule lives in a static device array
 * of the library (512 KiB per GPU, resident until exit): at most 65536 query
 * tiles per call (tiles of 128 rows at head_dim 64, else 64 rows), larger
 * batches return SJ_ERR_INVALID.  The first call on a device looks the array
 * up (make it before any stream capture); calls whose launches overlap on the
 * GPU share the array and race.  Arguments as sj_attn. */
int sj_attn_noalloc(const sj_bf16* qkv, const int32_t* cu_seqlens, const int32_t* cu_seqlens_host,
                    const int32_t* kv_lens, sj_bf16* O, int B, int H, int Dh, int window,
                    void* stream);

/* Status of the kernel entry points above on the current device.  They are
 * asynchronous and return once their kernels are queued, so a failure inside
 * a kernel cannot be their return value: a bounded device-side wait that ran
 * out (the kernel stops issuing, waits for its own copies, frees its
 * resources and returns early, leaving its output incomplete) is recorded in
 * a status word of the library, one per device, shared by every call of
 * sj_gemm, sj_gemm_geglu, sj_attn, sj_attn_noalloc and sj_gemm_e4m3.  This
 * call waits for `stream`, returns SJ_ERR_TIMEOUT (message in sj_last_error)
 * if any of those calls recorded one since the last check, and clears the
 * word.  Call it where the reference would check cudaGetLastError after a
 * synchronisation (src/capi.cpp:89-93 reports failures the same way: a status
 * and a message).  The engine (sj_fast_*) keeps its own flags and reports in
 * sj_fast_sync and its synchronous calls. */
int sj_check_device_errors(void* stream);

/* Failure-detection test hook (no counterpart in the reference): while
 * enabled (enable != 0), tcgen05 attention launches in this process issue no
 * TMA load, so their first bounded wait (about 2 s) runs out with nothing in
 * flight; the kernel records SJ_ERR_TIMEOUT's code and returns.  For tests of
 * the timeout path only; disable it afterwards. */
void sj_test_attn_wait_timeout(int enable);

/* The FP8 variant's two kernels (no counterpart in the reference, which has
 * no FP8 path; SJ_PREC_FP8 runs them inside the engine).
 *
 * sj_quant_e4m3: per row of x (fp32 [rows, cols], cols % 4 == 0):
 * scale[r] = amax_r / 448 (1 for an all-zero row) and q[r, :] = e4m3 codes of
 * x * (448 / amax_r), rounded to nearest even, saturating. */
int sj_quant_e4m3(const float* x, int64_t rows, int cols, uint8_t* q, float* scale, void* stream);

/* C = act(sa[m] sw[n] sum_k A[m,k] W[n,k] + bias) on tcgen05 kind::f8f6f4:
 * A [M, K] and W [N, K] e4m3 codes with their row scales sa [M], sw [N]
 * (16-byte aligned), fp32 accumulation, bf16 C [M, N]; K % 128 == 0,
 * N % 64 == 0.  geglu != 0: W = [Wg; Wu] [2N, K], sw [2N] and
 * C = gelu(g) * u (act and bias ignored), as sj_gemm_geglu. */
int sj_gemm_e4m3(const uint8_t* A, const uint8_t* W, const float* sa, const float* sw,
                 const float* bias, sj_bf16* C, int M, int N, int K, int has_bias, int act,
                 int geglu, void* stream);

/* ------------------------------------------------------------------------- */
/* 2. Encoder engine (replaces FastSnapjudge, include/snapjudge/fast.hpp).    */
/* ------------------------------------------------------------------------- */
typedef struct sj_fast sj_fast;

typedef struct sj_fast_config {
  /* encoder/config.json, parsed as DecisionModel::load does (src/model.cpp:59-111) */
  int hidden_size;
  int num_hidden_layers;
  int num_attention_heads;
  int intermediate_size;
  int vocab_size;
  int max_position_embeddings;
  float norm_eps;
  int local_attention;          /* window = local_attention / 2 on sliding layers */
  const int* layer_sliding;     /* [num_hidden_layers] 1 = sliding_attention; NULL = all full */
  double rope_theta_full;
  double rope_theta_sliding;
  /* engine options */
  int precision;                /* SJ_PREC_BF16, SJ_PREC_FP32, SJ_PREC_FP8 or SJ_PREC_FP8_TENSOR */
  int device;                   /* CUDA device ordinal */
  int max_tokens;               /* tokens per device pass (workspace size); 0 = default */
  int arch;                     /* SJ_ARCH_MODERNBERT (0) or SJ_ARCH_SJMODEL (1) */
} sj_fast_config;

/* Model families the engine runs:
 * SJ_ARCH_MODERNBERT  the DecisionModel encoder (src/model.cpp), tensors
 *                     "encoder.*", "type_emb.weight", "head.layers.*", "scorer.*",
 *                     "act_head.*";
 * SJ_ARCH_SJMODEL     SjModel (src/sj_model.cpp:206-255): BERT-style pre-LN
 *                     encoder with learned positions (max_position_embeddings =
 *                     max_positions), biased q/k/v/o and GELU FFN, biased LNs;
 *                     tensors "sj.*" (sj_model.cpp:117-202); no RoPE or window;
 *                     sj_fast_forward gives act = [top1, 1 - top1]. */
#define SJ_ARCH_MODERNBERT 0
#define SJ_ARCH_SJMODEL 1

/* Create an engine on cfg->device.  Weights are then given by name with
 * sj_fast_set_tensor and uploaded by sj_fast_commit. */
int sj_fast_create(const sj_fast_config* cfg, sj_fast** out);

/* Stage one fp32 host tensor, named as in model.safetensors
 * ("encoder.layers.3.attn.Wqkv.weight", ...).  The shape is checked against
 * the config (the strict checks of src/model.cpp:17-33).  Decision heads on
 * [CLS] are named "task_heads.<i>.weight" [n_out, D] / ".bias" [n_out]. */
int sj_fast_set_tensor(sj_fast* e, const char* name, const float* host, const int64_t* shape,
                       int ndim);

/* Declare the [CLS] decision heads (n_heads <= 8, sum of n_out <= 64); kinds
 * SJ_HEAD_SOFTMAX / SJ_HEAD_SIGMOID.  Call before sj_fast_commit. */
int sj_fast_set_heads(sj_fast* e, int n_heads, const int* n_out, const int* kind);

/* Check that every required tensor is present, convert and upload. */
int sj_fast_commit(sj_fast* e);

/* Encoder forward on packed sequences, host buffers in and out (synchronous).
 * ids int64 [T], cu_seqlens int32 [B+1] (cu[0] = 0, non-decreasing,
 * T = cu[B]); kv_lens int32 [B] or NULL (see sj_attn).  hidden fp32 [T, D] =
 * final-norm hidden states, as DecisionModel::encode (src/model.cpp:222-307). */
int sj_fast_encode(sj_fast* e, const int64_t* ids, const int32_t* cu_seqlens,
                   const int32_t* kv_lens, int B, float* hidden);

/* Mean-pooled embeddings, host buffers (synchronous): pooled fp32 [B, D] =
 * the mean of segment b's final-norm hidden states over its rows (zeros for an
 * empty segment), summed in row order in fp32.  Replaces the encode + pooling
 * loop of Agent::embed (src/agent.cpp:315-357); tokenisation and truncation to
 * max_length stay with the caller.  Only [B, D] crosses back to the host. */
int sj_fast_embed(sj_fast* e, const int64_t* ids, const int32_t* cu_seqlens, int B,
                  float* pooled);

/* Encoder + [CLS] decision heads, host buffers (synchronous):
 * probs fp32 [B, sum n_out] (heads in declaration order). */
int sj_fast_decide(sj_fast* e, const int64_t* ids, const int32_t* cu_seqlens, int B,
                   float* probs);

/* The whole DecisionModel::forward (src/model.cpp:309-536) on the GPU, host
 * buffers (synchronous): the encoder, then the decision-model tail — type
 * embedding, the head TransformerEncoderLayers, the scorer on the marker rows
 * and the act head (:402-535).  Replaces the reference fast path's forward
 * (include/snapjudge/fast.hpp:24-30, cuda/fast.cpp:170-267) behind
 * FastSnapjudge::forward.  Needs the checkpoint's type_emb.weight,
 * head.layers.*, scorer.* and act_head.* tensors (set before commit).
 * Inputs as sj_fast_encode (a padded [B, L] batch is B segments of length L
 * with kv_lens = the attention-mask lengths); marker_pos int64 [B, K]
 * (clamped to the segment), marker_mask uint8 [B, K], qtype int64 [B] in
 * [0, 3).  Outputs: logits fp32 [B, K] (masked markers -1e4), act fp32
 * [B, n_act] (sj_fast_n_act). */
int sj_fast_forward(sj_fast* e, const int64_t* ids, const int32_t* cu_seqlens,
                    const int32_t* kv_lens, int B, const int64_t* marker_pos,
                    const uint8_t* marker_mask, int K, const int64_t* qtype, float* logits,
                    float* act);

/* Outputs of the act head (0 when the engine has no decision-model head). */
int sj_fast_n_act(const sj_fast* e);

/* Device-buffer variants, asynchronous on `stream` (NULL = the engine's
 * stream).  T = cu_seqlens_host[B] must not exceed the engine's max_tokens.
 * cu_seqlens_host mirrors the device array (it sizes the launches).
 * hidden / cls may be NULL; probs may be NULL when no heads are set. */
int sj_fast_encode_device(sj_fast* e, const int64_t* ids, const int32_t* cu_seqlens,
                          const int32_t* cu_seqlens_host, const int32_t* kv_lens, int B,
                          float* hidden, float* probs, void* stream);

/* Wait for the engine's device work; reports device-side errors (an
 * out-of-vocabulary id, a bounded wait that ran out) raised since the last
 * check. */
int sj_fast_sync(sj_fast* e, void* stream);

/* Number of device kernel launches issued by the last forward (for audits). */
int sj_fast_launch_count(const sj_fast* e);

/* Per-kernel timing with CUDA events recorded around every launch (off by
 * default; the reference has no tracing, bench/bench.cpp times whole calls).
 * Kernel classes, in this order: */
#define SJ_K_EMBED 0      /* embedding gather + LayerNorm */
#define SJ_K_LN 1         /* attn_norm / mlp_norm LayerNorm */
#define SJ_K_QKV 2        /* QKV projection (+ RoPE) */
#define SJ_K_ATTN 3       /* attention */
#define SJ_K_WO 4         /* attention output projection + residual */
#define SJ_K_GEGLU 5      /* Wi projection + GEGLU gate */
#define SJ_K_WO2 6        /* FFN output projection + residual */
#define SJ_K_FINAL 7      /* final norm, LoRA, decision heads, positions */
#define SJ_K_COUNT 8
int sj_fast_set_profiling(sj_fast* e, int enable);
/* SJ_PREC_FP8_TENSOR: forget the activation scales, so that the next forward
 * call calibrates them again on its own batch (a bf16 pass recording each e4m3
 * operand's amax, then the FP8 pass).  SJ_ERR_STATE for other precisions. */
int sj_fast_reset_calibration(sj_fast* e);
/* Accumulated since the last reset (synchronises the engine's work first):
 * ms[k] total milliseconds and launches[k] count of class k (arrays of
 * SJ_K_COUNT); reset != 0 clears the accumulators afterwards. */
int sj_fast_profile(sj_fast* e, double* ms, int64_t* launches, int reset);

const char* sj_fast_last_error(const sj_fast* e);
void sj_fast_destroy(sj_fast* e);

#ifdef __cplusplus
}
#endif

#endif /* SNAPJUDGE_B200_H */
