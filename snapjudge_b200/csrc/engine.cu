// engine.cu — the encoder engine behind sj_fast_* (include/snapjudge_b200.h).
//
// Device-resident replacement of the reference FastSnapjudge
// (include/snapjudge/fast.hpp:15-31, cuda/fast.cpp) running the encoder half
// of DecisionModel (src/model.cpp:222-307) on packed variable-length batches
// (and, with SJ_ARCH_SJMODEL, SjModel's encoder, src/sj_model.cpp:206-255:
// learned positions, biased LNs and q/k/v/o, GELU FFN, no RoPE):
//
//   pos  = position of each packed row (rope.cu)
//   X    = LN(emb[ids]) (fp32 residual stream), Y = act(X)       (norm.cu)
//   per layer:
//     Y    = LN(X) * attn_norm            (identity when absent, layer 0)
//     QKV  = Y Wqkv^T, RoPE on q,k        (tcgen05 GEMM, RoPE epilogue)
//     O    = attention(QKV)               (tcgen05 flash attention)
//     X   += O Wo^T                       (GEMM, fp32 residual epilogue)
//     Y    = LN(X) * mlp_norm
//     G    = gelu(Y Wg^T) * (Y Wu^T)      (GEMM, GEGLU epilogue)
//     X   += G Wo2^T
//   hidden = LN(X) * final_norm (+ LoRA); heads on the [CLS] rows
//
// bf16 mode: bf16 weights/activations, fp32 accumulation, fp32 residual and
// norms.  fp32 mode: every tensor fp32, CUDA-core GEMM and attention.
// Workspace is allocated once for `max_tokens` rows; host calls split larger
// batches into passes of whole sequences.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <type_traits>
#include <vector>

#include "../../include/snapjudge_b200.h"
#include "common.cuh"
#include "kernels.h"

using sjb::bf16;

namespace {

struct HostTensor {
  std::vector<float> data;
  std::vector<int64_t> shape;
};

std::string shape_str(const std::vector<int64_t>& s) {
  std::string o = "[";
  for (size_t i = 0; i < s.size(); ++i) o += (i ? "," : "") + std::to_string(s[i]);
  return o + "]";
}

struct LayerDev {
  float* attn_norm = nullptr;  // null: identity (reference layer 0)
  float* mlp_norm = nullptr;
  void* wqkv = nullptr;        // [3D, D]
  void* wo = nullptr;          // [D, D]
  void* wi = nullptr;          // [2F, D]  (gate rows, then up rows)
  void* wo2 = nullptr;         // [D, F]
  int window = 0;
  bool sliding = false;
  // SjModel (src/sj_model.cpp:127-151): LN biases, q/k/v concatenated into
  // wqkv with bias bqkv [3D], Wo bias, wi = ffn.w1 [F, D] + b1, wo2 = ffn.w2 + b2
  float *attn_norm_b = nullptr, *mlp_norm_b = nullptr;
  float *bqkv = nullptr, *bo = nullptr, *b1 = nullptr, *b2 = nullptr;
  // SJ_PREC_FP8: e4m3 copies of wqkv and wi with a scale per row;
  // SJ_PREC_FP8_TENSOR: wqkv, wi and wo2 with one scale per tensor (the scale
  // arrays then hold that one value in every row)
  uint8_t *wqkv8 = nullptr, *wi8 = nullptr, *wo2_8 = nullptr;
  float *sqkv = nullptr, *si = nullptr, *so2 = nullptr;
};

// One pre-norm TransformerEncoderLayer of the decision head (model.cpp:134-152):
// LN weights/biases and GEMM biases fp32, GEMM weights in the activation precision.
struct HeadLayerDev {
  float *n1w = nullptr, *n1b = nullptr, *n2w = nullptr, *n2b = nullptr;
  void *in_w = nullptr, *out_w = nullptr, *l1w = nullptr, *l2w = nullptr;  // [3D,D] [D,D] [4D,D] [D,4D]
  float *in_b = nullptr, *out_b = nullptr, *l1b = nullptr, *l2b = nullptr;
};

// Per-pass device inputs and outputs of the decision-model tail.
struct DmPass {
  const int64_t* qtype;   // [B]
  const int64_t* pos;     // [B, K]
  const uint8_t* mask;    // [B, K]
  int K;
  float* logits;          // [B, K]
  float* act;             // [B, n_act]
};

}  // namespace

struct sj_fast {
  sj_fast_config cfg{};
  int arch = SJ_ARCH_MODERNBERT;
  std::vector<int> sliding;
  int D = 0, H = 0, Dh = 0, F = 0, V = 0, NL = 0;
  int max_tokens = 0;
  bool bf16_mode = true;
  bool fp8 = false;  // SJ_PREC_FP8: QKV and Wi projections on e4m3 operands
  // SJ_PREC_FP8_TENSOR: QKV, Wi and Wo2 on e4m3 operands, one scale per tensor;
  // the activation scales are calibrated on the engine's first pass
  bool fp8_tensor = false;
  bool calibrated = false, calibrating = false;
  float* act_scale = nullptr;     // [3 * NL]: QKV input, Wi input, Wo2 input of each layer
  unsigned* act_amax = nullptr;   // [3 * NL] amax seen by the calibration pass (float bits)
  bool committed = false;
  cudaStream_t stream = nullptr;
  std::string err;
  int launches = 0;

  std::map<std::string, HostTensor> staged;
  std::vector<void*> allocs;

  // weights
  float* emb = nullptr;
  float* emb_norm = nullptr;
  float* final_norm = nullptr;
  std::vector<LayerDev> layers;
  float *cos_f = nullptr, *sin_f = nullptr, *cos_s = nullptr, *sin_s = nullptr;
  int lora_r = 0;
  float *lora_a = nullptr, *lora_b = nullptr;
  sjb::HeadSpec spec{};
  bool has_heads = false;
  float *head_w = nullptr, *head_b = nullptr;
  // SjModel: learned positions, biased embedding and final LNs
  float *pos_emb = nullptr, *emb_norm_b = nullptr, *final_norm_b = nullptr;
  // decision-model tail of DecisionModel::forward (model.cpp:402-535) or
  // SjModel::forward (sj_model.cpp:277-368)
  bool has_dm = false;
  int n_act = 0;
  int n_types = 3;    // rows of the type embedding
  int head_ffn = 0;   // FFN width of the head layers (4D, or SjModel's head_intermediate)
  std::vector<HeadLayerDev> hlayers;
  float* type_emb = nullptr;  // [3, D]
  float *sc_lnw = nullptr, *sc_lnb = nullptr, *sc_w1 = nullptr, *sc_b1 = nullptr,
        *sc_w2 = nullptr, *sc_b2 = nullptr;
  float *act_w1 = nullptr, *act_b1 = nullptr, *act_w2 = nullptr, *act_b2 = nullptr;
  // its per-call buffers, grown on demand: marker rows [BK, D] x 3, scores [BK],
  // logits [BK], act [B, n_act], and the inputs
  size_t dm_cap_bk = 0, dm_cap_b = 0;
  float *dm_m = nullptr, *dm_s = nullptr, *dm_s1 = nullptr, *dm_s2 = nullptr,
        *dm_logits = nullptr, *dm_act = nullptr;
  int64_t *dm_pos = nullptr, *dm_qt = nullptr;
  uint8_t* dm_mask = nullptr;

  // workspace
  float* X = nullptr;
  void *Y = nullptr, *QKV = nullptr, *O = nullptr, *G = nullptr;
  int32_t* pos = nullptr;
  int64_t* ids = nullptr;
  int32_t* cu = nullptr;
  int32_t* kvl = nullptr;
  int2* tiles = nullptr;
  int max_tiles = 0;
  float* Hc = nullptr;    // [max_tokens, D] normalised [CLS] rows
  float* probs = nullptr; // [max_tokens, n_total]
  float* hid = nullptr;   // [max_tokens, D] fp32 hidden (host-API staging)
  float* z = nullptr;     // LoRA [max_tokens, r]
  uint8_t* Y8 = nullptr;  // SJ_PREC_FP8: LN output as e4m3 [max_tokens, D]
  float* sa8 = nullptr;   //   and its row scales [max_tokens]
  uint8_t* G8 = nullptr;  // SJ_PREC_FP8_TENSOR: GEGLU output as e4m3 [max_tokens, F]
  bf16* Xh = nullptr;     //   its residual stream, bf16 [max_tokens, D]
  float* sg8 = nullptr;   //   and its row scales [max_tokens]
  int* dflags = nullptr;  // device error flags: [0] bad id, [1] gemm wait, [2] attn wait
  // pinned host staging
  int2* h_tiles = nullptr;
  int32_t* h_cu = nullptr;
  int32_t* h_kvl = nullptr;
  cudaEvent_t staged_ev = nullptr;
  // host_call: the last pass's h_cu / h_kvl have been copied to the device
  cudaEvent_t inputs_ev = nullptr;
  // per-kernel CUDA-event timing (sj_fast_set_profiling)
  bool profiling = false;
  struct Mark { int cls; cudaEvent_t a, b; };
  std::vector<Mark> marks;
  std::vector<cudaEvent_t> ev_pool;
  double prof_ms[SJ_K_COUNT] = {};
  int64_t prof_n[SJ_K_COUNT] = {};

  cudaEvent_t take_event() {
    if (!ev_pool.empty()) {
      cudaEvent_t e = ev_pool.back();
      ev_pool.pop_back();
      return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
  }
  // Record a start event before a launch of class `cls` (returns null when off).
  cudaEvent_t mark_begin(cudaStream_t st) {
    if (!profiling) return nullptr;
    cudaEvent_t a = take_event();
    cudaEventRecord(a, st);
    return a;
  }
  void mark_end(int cls, cudaEvent_t a, cudaStream_t st) {
    if (!a) return;
    cudaEvent_t b = take_event();
    cudaEventRecord(b, st);
    marks.push_back({cls, a, b});
  }
  int collect_profile() {
    for (const Mark& m : marks) {
      float ms = 0.f;
      cudaError_t rc = cudaEventSynchronize(m.b);
      if (rc == cudaSuccess) rc = cudaEventElapsedTime(&ms, m.a, m.b);
      if (rc != cudaSuccess) return cuda_fail(rc, "profile events");
      prof_ms[m.cls] += ms;
      prof_n[m.cls] += 1;
      ev_pool.push_back(m.a);
      ev_pool.push_back(m.b);
    }
    marks.clear();
    return SJ_OK;
  }

  int fail(int code, const std::string& m) {
    err = m;
    return code;
  }
  int cuda_fail(cudaError_t rc, const char* what) {
    err = std::string("snapjudge CUDA: ") + what + ": " + cudaGetErrorString(rc);
    return SJ_ERR_CUDA;
  }
  template <typename T>
  cudaError_t dalloc(T** p, size_t n) {
    void* q = nullptr;
    cudaError_t rc = cudaMalloc(&q, n * sizeof(T) > 0 ? n * sizeof(T) : 16);
    if (rc == cudaSuccess) allocs.push_back(q);
    *p = static_cast<T*>(q);
    return rc;
  }
  ~sj_fast() {
    cudaSetDevice(cfg.device);
    if (stream) cudaStreamSynchronize(stream);
    for (void* p : allocs) cudaFree(p);
    if (h_tiles) cudaFreeHost(h_tiles);
    if (h_cu) cudaFreeHost(h_cu);
    if (h_kvl) cudaFreeHost(h_kvl);
    if (staged_ev) cudaEventDestroy(staged_ev);
    if (inputs_ev) cudaEventDestroy(inputs_ev);
    for (const Mark& m : marks) {
      cudaEventDestroy(m.a);
      cudaEventDestroy(m.b);
    }
    for (cudaEvent_t e : ev_pool) cudaEventDestroy(e);
    if (stream) cudaStreamDestroy(stream);
  }

  const HostTensor* get(const std::string& n) const {
    auto it = staged.find(n);
    return it == staged.end() ? nullptr : &it->second;
  }
  int require(const std::string& n, std::vector<int64_t> want, const HostTensor** out) {
    const HostTensor* t = get(n);
    if (!t) return fail(SJ_ERR_INVALID, "Model weights incomplete: missing tensor " + n);
    if (t->shape != want)
      return fail(SJ_ERR_INVALID, "Model architecture mismatch: " + n + " expected " +
                                      shape_str(want) + " but checkpoint has " + shape_str(t->shape));
    *out = t;
    return SJ_OK;
  }
  int upload_f32(const HostTensor* t, float** dst) {
    cudaError_t rc = dalloc(dst, t->data.size());
    if (rc != cudaSuccess) return cuda_fail(rc, "cudaMalloc");
    rc = cudaMemcpy(*dst, t->data.data(), t->data.size() * sizeof(float), cudaMemcpyHostToDevice);
    return rc == cudaSuccess ? SJ_OK : cuda_fail(rc, "cudaMemcpy");
  }
  // GEMM weight in the activation precision (bf16 round-to-nearest-even or fp32)
  int upload_w(const HostTensor* t, void** dst) {
    if (!bf16_mode) return upload_f32(t, reinterpret_cast<float**>(dst));
    std::vector<bf16> tmp(t->data.size());
    for (size_t i = 0; i < tmp.size(); ++i) tmp[i] = __float2bfloat16_rn(t->data[i]);
    bf16* p = nullptr;
    cudaError_t rc = dalloc(&p, tmp.size());
    if (rc != cudaSuccess) return cuda_fail(rc, "cudaMalloc");
    rc = cudaMemcpy(p, tmp.data(), tmp.size() * sizeof(bf16), cudaMemcpyHostToDevice);
    *dst = p;
    return rc == cudaSuccess ? SJ_OK : cuda_fail(rc, "cudaMemcpy");
  }

  // e4m3 codes and row scales of a [rows, cols] weight (quantised on the device
  // from its fp32 values, as quant_rows_e4m3)
  int upload_e4m3(const HostTensor* t, uint8_t** q, float** scale) {
    const int64_t rows = t->shape[0], cols = t->shape[1];
    float* tmp = nullptr;
    cudaError_t rc = cudaMalloc(&tmp, t->data.size() * sizeof(float));
    if (rc != cudaSuccess) return cuda_fail(rc, "cudaMalloc");
    if ((rc = cudaMemcpy(tmp, t->data.data(), t->data.size() * sizeof(float),
                         cudaMemcpyHostToDevice)) == cudaSuccess &&
        (rc = dalloc(q, t->data.size())) == cudaSuccess && (rc = dalloc(scale, rows)) == cudaSuccess &&
        (rc = sjb::quant_rows_e4m3<float>(tmp, rows, (int)cols, *q, *scale, nullptr)) ==
            cudaSuccess)
      rc = cudaDeviceSynchronize();
    cudaFree(tmp);
    return rc == cudaSuccess ? SJ_OK : cuda_fail(rc, "e4m3 weight upload");
  }

  // e4m3 codes of a [rows, cols] weight with one scale for the whole tensor
  // (its amax / 448, taken on the host); the scale array holds it per row
  int upload_e4m3_tensor(const HostTensor* t, uint8_t** q, float** scale) {
    const int64_t rows = t->shape[0];
    float amax = 0.f;
    for (float v : t->data) amax = std::max(amax, std::fabs(v));
    float* tmp = nullptr;
    cudaError_t rc = cudaMalloc(&tmp, t->data.size() * sizeof(float));
    if (rc != cudaSuccess) return cuda_fail(rc, "cudaMalloc");
    if ((rc = cudaMemcpy(tmp, t->data.data(), t->data.size() * sizeof(float),
                         cudaMemcpyHostToDevice)) == cudaSuccess &&
        (rc = dalloc(q, t->data.size())) == cudaSuccess && (rc = dalloc(scale, rows)) == cudaSuccess &&
        (rc = sjb::quant_tensor_e4m3(tmp, (int64_t)t->data.size(), (int)rows, amax, *q, *scale,
                                     nullptr)) == cudaSuccess)
      rc = cudaDeviceSynchronize();
    cudaFree(tmp);
    return rc == cudaSuccess ? SJ_OK : cuda_fail(rc, "e4m3 weight upload");
  }

  int commit();
  int load_sjmodel();
  template <typename T>
  int forward(const int64_t* d_ids, const int32_t* d_cu, const int32_t* hcu,
              const int32_t* d_kvl, int B, int ntok, float* d_hidden, float* d_probs,
              const DmPass* dm, cudaStream_t st);
  template <typename T>
  int head_forward(const int32_t* d_cu, const int32_t* d_kvl, int B, int ntok, int nt,
                   float* h, const DmPass& dm, cudaStream_t st);
  template <typename T>
  int gemm_any(int cls, const T* A, const void* W, const float* bias, int act, T* C,
               float* resid, int M, int N, int K, int epi, const float* ct, const float* stb,
               cudaStream_t st);
  int run(const int64_t* d_ids, const int32_t* d_cu, const int32_t* hcu, const int32_t* d_kvl,
          int B, float* d_hidden, float* d_probs, const DmPass* dm, cudaStream_t st);
  int check_flags(cudaStream_t st);
  int host_call(const int64_t* ids_h, const int32_t* cu_h, const int32_t* kvl_h, int B,
                float* hidden_h, float* probs_h, float* pooled_h = nullptr);
  int dm_call(const int64_t* ids_h, const int32_t* cu_h, const int32_t* kvl_h, int B,
              const int64_t* pos_h, const uint8_t* mask_h, int K, const int64_t* qtype_h,
              float* logits_h, float* act_h);
  template <typename P>
  cudaError_t grow(P** p, size_t n) {  // replace *p by a buffer of n elements
    if (*p) {
      auto it = std::find(allocs.begin(), allocs.end(), static_cast<void*>(*p));
      if (it != allocs.end()) allocs.erase(it);
      cudaFree(*p);
      *p = nullptr;
    }
    return dalloc(p, n);
  }
};

// ------------------------------------------------------------------ commit
int sj_fast::commit() {
  if (committed) return fail(SJ_ERR_STATE, "sj_fast_commit: already committed");
  cudaError_t rc = cudaSetDevice(cfg.device);
  if (rc != cudaSuccess) return cuda_fail(rc, "cudaSetDevice");
  const HostTensor* t = nullptr;
  int s;
  if (arch == SJ_ARCH_SJMODEL) {
    if ((s = load_sjmodel())) return s;
  } else {
  if ((s = require("encoder.embeddings.tok_embeddings.weight", {V, D}, &t))) return s;
  if ((s = upload_f32(t, &emb))) return s;
  if ((s = require("encoder.embeddings.norm.weight", {D}, &t))) return s;
  if ((s = upload_f32(t, &emb_norm))) return s;
  if ((s = require("encoder.final_norm.weight", {D}, &t))) return s;
  if ((s = upload_f32(t, &final_norm))) return s;
  layers.resize(NL);
  const int win = cfg.local_attention > 0 ? cfg.local_attention / 2 : 0;
  for (int i = 0; i < NL; ++i) {
    LayerDev& ly = layers[i];
    std::string p = "encoder.layers." + std::to_string(i) + ".";
    ly.sliding = sliding[i] != 0;
    ly.window = ly.sliding ? win : 0;
    if (get(p + "attn_norm.weight")) {
      if ((s = require(p + "attn_norm.weight", {D}, &t))) return s;
      if ((s = upload_f32(t, &ly.attn_norm))) return s;
    }
    if ((s = require(p + "attn.Wqkv.weight", {3 * (int64_t)D, D}, &t))) return s;
    if ((s = upload_w(t, &ly.wqkv))) return s;
    if (fp8 && (s = fp8_tensor ? upload_e4m3_tensor(t, &ly.wqkv8, &ly.sqkv)
                               : upload_e4m3(t, &ly.wqkv8, &ly.sqkv)))
      return s;
    if ((s = require(p + "attn.Wo.weight", {D, D}, &t))) return s;
    if ((s = upload_w(t, &ly.wo))) return s;
    if ((s = require(p + "mlp_norm.weight", {D}, &t))) return s;
    if ((s = upload_f32(t, &ly.mlp_norm))) return s;
    if ((s = require(p + "mlp.Wi.weight", {2 * (int64_t)F, D}, &t))) return s;
    if ((s = upload_w(t, &ly.wi))) return s;
    if (fp8 && (s = fp8_tensor ? upload_e4m3_tensor(t, &ly.wi8, &ly.si)
                               : upload_e4m3(t, &ly.wi8, &ly.si)))
      return s;
    if ((s = require(p + "mlp.Wo.weight", {D, F}, &t))) return s;
    if ((s = upload_w(t, &ly.wo2))) return s;
    if (fp8_tensor && (s = upload_e4m3_tensor(t, &ly.wo2_8, &ly.so2))) return s;
  }
  // optional encoder-output LoRA (src/model.cpp:192-203)
  const HostTensor* la = get("lora_A.weight");
  const HostTensor* lb = get("lora_B.weight");
  if (la && lb) {
    if (la->shape.size() != 2 || lb->shape.size() != 2 || la->shape[0] != lb->shape[1] ||
        la->shape[1] != D || lb->shape[0] != D)
      return fail(SJ_ERR_INVALID, "Model 'lora_A.weight'/'lora_B.weight' must be [r,D] and [D,r]");
    lora_r = (int)la->shape[0];
    if ((s = upload_f32(la, &lora_a))) return s;
    if ((s = upload_f32(lb, &lora_b))) return s;
  }
  // RoPE tables: fp64 angles cast to fp32, as src/model.cpp:173-190
  {
    const int64_t half = Dh / 2, L = cfg.max_position_embeddings;
    HostTensor c, sn;
    c.data.resize(L * half);
    sn.data.resize(L * half);
    for (int which = 0; which < 2; ++which) {
      double theta = which == 0 ? cfg.rope_theta_full : cfg.rope_theta_sliding;
      for (int64_t p = 0; p < L; ++p)
        for (int64_t d = 0; d < half; ++d) {
          double inv = 1.0 / std::pow(theta, 2.0 * (double)d / Dh);
          double fr = (double)p * inv;
          c.data[p * half + d] = (float)std::cos(fr);
          sn.data[p * half + d] = (float)std::sin(fr);
        }
      if ((s = upload_f32(&c, which == 0 ? &cos_f : &cos_s))) return s;
      if ((s = upload_f32(&sn, which == 0 ? &sin_f : &sin_s))) return s;
    }
  }
  }  // SJ_ARCH_MODERNBERT
  // decision heads
  if (has_heads) {
    HostTensor w, b;
    for (int h = 0; h < spec.n_heads; ++h) {
      std::string p = "task_heads." + std::to_string(h) + ".";
      if ((s = require(p + "weight", {spec.n_out[h], D}, &t))) return s;
      w.data.insert(w.data.end(), t->data.begin(), t->data.end());
      if ((s = require(p + "bias", {spec.n_out[h]}, &t))) return s;
      b.data.insert(b.data.end(), t->data.begin(), t->data.end());
    }
    if ((s = upload_f32(&w, &head_w))) return s;
    if ((s = upload_f32(&b, &head_b))) return s;
  }
  // decision-model tail (model.cpp:130-176), when the checkpoint has one: the
  // type embedding, head TransformerEncoderLayers, scorer and act head
  if (arch == SJ_ARCH_MODERNBERT && get("type_emb.weight")) {
    head_ffn = 4 * D;
    if ((s = require("type_emb.weight", {3, D}, &t))) return s;
    if ((s = upload_f32(t, &type_emb))) return s;
    for (int i = 0; get("head.layers." + std::to_string(i) + ".norm1.weight"); ++i) {
      HeadLayerDev hl;
      const std::string p = "head.layers." + std::to_string(i) + ".";
      const int64_t d = D;
      struct {
        const char* name;
        std::vector<int64_t> shape;
        float** f32;
        void** w;
      } items[] = {{"norm1.weight", {d}, &hl.n1w, nullptr},
                   {"norm1.bias", {d}, &hl.n1b, nullptr},
                   {"norm2.weight", {d}, &hl.n2w, nullptr},
                   {"norm2.bias", {d}, &hl.n2b, nullptr},
                   {"self_attn.in_proj_weight", {3 * d, d}, nullptr, &hl.in_w},
                   {"self_attn.in_proj_bias", {3 * d}, &hl.in_b, nullptr},
                   {"self_attn.out_proj.weight", {d, d}, nullptr, &hl.out_w},
                   {"self_attn.out_proj.bias", {d}, &hl.out_b, nullptr},
                   {"linear1.weight", {4 * d, d}, nullptr, &hl.l1w},
                   {"linear1.bias", {4 * d}, &hl.l1b, nullptr},
                   {"linear2.weight", {d, 4 * d}, nullptr, &hl.l2w},
                   {"linear2.bias", {d}, &hl.l2b, nullptr}};
      for (auto& it : items) {
        if ((s = require(p + it.name, it.shape, &t))) return s;
        if ((s = it.f32 ? upload_f32(t, it.f32) : upload_w(t, it.w))) return s;
      }
      hlayers.push_back(hl);
    }
    // scorer: LayerNorm + Linear(D, D) + GELU + Linear(D, 1); its biases are optional
    if ((s = require("scorer.0.weight", {D}, &t)) || (s = upload_f32(t, &sc_lnw))) return s;
    if ((s = require("scorer.1.weight", {D, D}, &t)) || (s = upload_f32(t, &sc_w1))) return s;
    if ((s = require("scorer.3.weight", {1, D}, &t)) || (s = upload_f32(t, &sc_w2))) return s;
    if (get("scorer.0.bias") &&
        ((s = require("scorer.0.bias", {D}, &t)) || (s = upload_f32(t, &sc_lnb))))
      return s;
    if (get("scorer.1.bias") &&
        ((s = require("scorer.1.bias", {D}, &t)) || (s = upload_f32(t, &sc_b1))))
      return s;
    if (get("scorer.3.bias") &&
        ((s = require("scorer.3.bias", {1}, &t)) || (s = upload_f32(t, &sc_b2))))
      return s;
    // act head: Linear(D + 4, 256) + GELU + Linear(256, n_act)
    const HostTensor* a2 = get("act_head.2.weight");
    if (!a2 || a2->shape.size() != 2 || a2->shape[1] != 256 || a2->shape[0] < 1)
      return fail(SJ_ERR_INVALID, "Model 'act_head.2.weight' must be [n_act, 256]");
    n_act = (int)a2->shape[0];
    if ((s = require("act_head.0.weight", {256, (int64_t)D + 4}, &t)) ||
        (s = upload_f32(t, &act_w1)) || (s = require("act_head.0.bias", {256}, &t)) ||
        (s = upload_f32(t, &act_b1)) || (s = require("act_head.2.weight", {n_act, 256}, &t)) ||
        (s = upload_f32(t, &act_w2)) || (s = require("act_head.2.bias", {n_act}, &t)) ||
        (s = upload_f32(t, &act_b2)))
      return s;
    has_dm = true;
  }
  // workspace
  const size_t T = (size_t)max_tokens, es = bf16_mode ? 2 : 4;
  // 128-row (or 64-row) query tiles of every segment, then the 256-row items
  // of the long-segment attention
  max_tiles = max_tokens / 64 + max_tokens + 1 + max_tokens / 256 + max_tokens / sjb::kAttnLongMin + 1;
  if ((rc = dalloc(&X, T * D)) || (rc = dalloc((char**)&Y, T * D * es)) ||
      (rc = dalloc((char**)&QKV, T * 3 * D * es)) || (rc = dalloc((char**)&O, T * D * es)) ||
      (rc = dalloc((char**)&G, T * (hlayers.empty() ? F : std::max(F, head_ffn)) * es)) ||
      (rc = dalloc(&pos, T)) || (rc = dalloc(&ids, T)) ||
      (rc = dalloc(&cu, T + 1)) || (rc = dalloc(&kvl, T)) || (rc = dalloc(&tiles, max_tiles)) ||
      (rc = dalloc(&Hc, T * D)) || (rc = dalloc(&probs, T * (size_t)std::max(1, spec.n_total))) ||
      (rc = dalloc(&hid, T * D)) || (rc = dalloc(&z, T * (size_t)std::max(1, lora_r))) ||
      (rc = dalloc(&dflags, 8)) || (fp8 && ((rc = dalloc(&Y8, T * D)) || (rc = dalloc(&sa8, T)))) ||
      (fp8_tensor && ((rc = dalloc(&G8, T * F)) || (rc = dalloc(&sg8, T)) ||
                      (rc = dalloc(&Xh, T * D)) ||
                      (rc = dalloc(&act_scale, 3 * (size_t)NL)) ||
                      (rc = dalloc(&act_amax, 3 * (size_t)NL)))))
    return cuda_fail(rc, "cudaMalloc (workspace)");
  if ((rc = cudaMemset(dflags, 0, 8 * sizeof(int)))) return cuda_fail(rc, "cudaMemset");
  if ((rc = cudaMallocHost(&h_tiles, max_tiles * sizeof(int2))) ||
      (rc = cudaMallocHost(&h_cu, (T + 1) * sizeof(int32_t))) ||
      (rc = cudaMallocHost(&h_kvl, T * sizeof(int32_t))))
    return cuda_fail(rc, "cudaMallocHost");
  if ((rc = cudaEventCreateWithFlags(&staged_ev, cudaEventDisableTiming)) ||
      (rc = cudaEventCreateWithFlags(&inputs_ev, cudaEventDisableTiming)))
    return cuda_fail(rc, "cudaEventCreate");
  if ((rc = cudaEventRecord(staged_ev, stream)) || (rc = cudaEventRecord(inputs_ev, stream)))
    return cuda_fail(rc, "cudaEventRecord");
  staged.clear();
  committed = true;
  return SJ_OK;
}

// SjModel weights (src/sj_model.cpp:117-202), "sj.*" names and shapes; q/k/v
// are concatenated into one [3D, D] projection (bias [3D]) so that the QKV GEMM
// and the attention kernel are the DecisionModel encoder's.
int sj_fast::load_sjmodel() {
  const HostTensor* t = nullptr;
  int s;
  const int64_t d = D;
  auto f32 = [&](const std::string& n, std::vector<int64_t> shape, float** dst) -> int {
    int r = require(n, std::move(shape), &t);
    return r ? r : upload_f32(t, dst);
  };
  auto wgt = [&](const std::string& n, std::vector<int64_t> shape, void** dst) -> int {
    int r = require(n, std::move(shape), &t);
    return r ? r : upload_w(t, dst);
  };
  // q, k, v of one attention block -> [3D, D] weight + [3D] bias
  auto qkv = [&](const std::string& p, void** w, float** b) -> int {
    HostTensor cw, cb;
    cw.shape = {3 * d, d};
    cb.shape = {3 * d};
    for (const char* x : {"q", "k", "v"}) {
      int r = require(p + "attn." + x + ".weight", {d, d}, &t);
      if (r) return r;
      cw.data.insert(cw.data.end(), t->data.begin(), t->data.end());
      if ((r = require(p + "attn." + x + ".bias", {d}, &t))) return r;
      cb.data.insert(cb.data.end(), t->data.begin(), t->data.end());
    }
    int r = upload_w(&cw, w);
    return r ? r : upload_f32(&cb, b);
  };
  if ((s = f32("sj.embeddings.word.weight", {V, d}, &emb)) ||
      (s = f32("sj.embeddings.position.weight", {cfg.max_position_embeddings, d}, &pos_emb)) ||
      (s = f32("sj.embeddings.norm.weight", {d}, &emb_norm)) ||
      (s = f32("sj.embeddings.norm.bias", {d}, &emb_norm_b)))
    return s;
  layers.resize(NL);
  for (int i = 0; i < NL; ++i) {
    LayerDev& ly = layers[i];
    const std::string p = "sj.encoder.layers." + std::to_string(i) + ".";
    if ((s = f32(p + "attn_norm.weight", {d}, &ly.attn_norm)) ||
        (s = f32(p + "attn_norm.bias", {d}, &ly.attn_norm_b)) ||
        (s = qkv(p, &ly.wqkv, &ly.bqkv)) || (s = wgt(p + "attn.o.weight", {d, d}, &ly.wo)) ||
        (s = f32(p + "attn.o.bias", {d}, &ly.bo)) ||
        (s = f32(p + "ffn_norm.weight", {d}, &ly.mlp_norm)) ||
        (s = f32(p + "ffn_norm.bias", {d}, &ly.mlp_norm_b)) ||
        (s = wgt(p + "ffn.w1.weight", {F, d}, &ly.wi)) || (s = f32(p + "ffn.w1.bias", {F}, &ly.b1)) ||
        (s = wgt(p + "ffn.w2.weight", {d, F}, &ly.wo2)) || (s = f32(p + "ffn.w2.bias", {d}, &ly.b2)))
      return s;
  }
  if ((s = f32("sj.encoder.final_norm.weight", {d}, &final_norm)) ||
      (s = f32("sj.encoder.final_norm.bias", {d}, &final_norm_b)))
    return s;
  // the forward tail (sj_model.cpp:293-368), when present
  const HostTensor* te = get("sj.type_emb.weight");
  if (te) {
    if (te->shape.size() != 2 || te->shape[1] != d || te->shape[0] < 1)
      return fail(SJ_ERR_INVALID, "Model 'sj.type_emb.weight' must be [n_types, D]");
    n_types = (int)te->shape[0];
    if ((s = upload_f32(te, &type_emb))) return s;
    for (int i = 0; get("sj.head.layers." + std::to_string(i) + ".norm1.weight"); ++i) {
      HeadLayerDev hl;
      const std::string p = "sj.head.layers." + std::to_string(i) + ".";
      const HostTensor* w1 = get(p + "ffn.w1.weight");
      if (!w1 || w1->shape.size() != 2 || w1->shape[1] != d)
        return fail(SJ_ERR_INVALID, "Model '" + p + "ffn.w1.weight' must be [head_intermediate, D]");
      const int64_t fh = w1->shape[0];
      if (i == 0) head_ffn = (int)fh;
      if (fh != head_ffn) return fail(SJ_ERR_INVALID, "head layers of different FFN widths");
      if ((s = f32(p + "norm1.weight", {d}, &hl.n1w)) || (s = f32(p + "norm1.bias", {d}, &hl.n1b)) ||
          (s = f32(p + "norm2.weight", {d}, &hl.n2w)) || (s = f32(p + "norm2.bias", {d}, &hl.n2b)) ||
          (s = qkv(p, &hl.in_w, &hl.in_b)) || (s = wgt(p + "attn.o.weight", {d, d}, &hl.out_w)) ||
          (s = f32(p + "attn.o.bias", {d}, &hl.out_b)) ||
          (s = wgt(p + "ffn.w1.weight", {fh, d}, &hl.l1w)) || (s = f32(p + "ffn.w1.bias", {fh}, &hl.l1b)) ||
          (s = wgt(p + "ffn.w2.weight", {d, fh}, &hl.l2w)) || (s = f32(p + "ffn.w2.bias", {d}, &hl.l2b)))
        return s;
      hlayers.push_back(hl);
    }
    if ((s = f32("sj.scorer.norm.weight", {d}, &sc_lnw)) ||
        (s = f32("sj.scorer.norm.bias", {d}, &sc_lnb)) ||
        (s = f32("sj.scorer.w1.weight", {d, d}, &sc_w1)) ||
        (s = f32("sj.scorer.w1.bias", {d}, &sc_b1)) ||
        (s = f32("sj.scorer.w2.weight", {1, d}, &sc_w2)) ||
        (s = f32("sj.scorer.w2.bias", {1}, &sc_b2)))
      return s;
    n_act = 2;
    has_dm = true;
  }
  return SJ_OK;
}

// ------------------------------------------------------------------ forward
#define SJ_LAUNCH(cls, expr)                               \
  do {                                                     \
    cudaEvent_t ev_ = mark_begin(st);                      \
    cudaError_t rc_ = (expr);                              \
    mark_end(cls, ev_, st);                                \
    ++launches;                                            \
    if (rc_ != cudaSuccess) return cuda_fail(rc_, #expr);  \
  } while (0)

// C = act(A W^T + bias) (epi STORE), resid += A W^T (+ bias) (RESID), GEGLU or
// QKV + RoPE: the tcgen05 GEMM in bf16 mode when it takes the shape, the
// CUDA-core GEMM otherwise (fp32 mode, odd shapes).
template <typename T>
int sj_fast::gemm_any(int cls, const T* A, const void* W, const float* bias, int act, T* C,
                      float* resid, int M, int N, int K, int epi, const float* ct,
                      const float* stb, cudaStream_t st) {
  if constexpr (std::is_same<T, bf16>::value) {
    const bool geglu = epi == sjb::TC_GEGLU;
    if (sjb::gemm_tc_supported(M, N, K, geglu) && (epi != sjb::TC_ROPE || Dh == 64)) {
      sjb::TcRope rp{ct, stb, pos, H};
      SJ_LAUNCH(cls, sjb::gemm_tc(A, static_cast<const bf16*>(W), bias, C, resid, M, N, K, epi, act,
                                  rp, dflags + 1, st));
      return SJ_OK;
    }
  }
  SJ_LAUNCH(cls, (sjb::gemm_simt<T, T>(A, static_cast<const T*>(W), bias, C, resid, M, N, K, act,
                                       epi == sjb::TC_GEGLU, st)));
  if (epi == sjb::TC_ROPE) SJ_LAUNCH(cls, sjb::rope<T>(C, ct, stb, pos, M, H, Dh, st));
  return SJ_OK;
}

template <typename T>
int sj_fast::forward(const int64_t* d_ids, const int32_t* d_cu, const int32_t* hcu,
                     const int32_t* d_kvl, int B, int ntok, float* d_hidden, float* d_probs,
                     const DmPass* dm, cudaStream_t st) {
  constexpr bool kBf16 = std::is_same<T, bf16>::value;
  const bool tc_attn = kBf16 && sjb::attn_tc_supported(Dh);
  const int qt = tc_attn ? 128 : 64;
  // query-tile schedule, longest segments first (they take the longest)
  cudaError_t rc = cudaEventSynchronize(staged_ev);  // previous upload of h_tiles done
  if (rc != cudaSuccess) return cuda_fail(rc, "cudaEventSynchronize");
  std::vector<int> order(B);
  for (int b = 0; b < B; ++b) order[b] = b;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) {
    return hcu[a + 1] - hcu[a] > hcu[b + 1] - hcu[b];
  });
  // h_tiles = [query tiles of every segment, longest first: those of the
  // segments of kAttnLongMin tokens or more (n_long_tiles) come first]
  //           [256-row items of those long segments (n_pairs)]
  // Full-attention layers at head_dim 64 run the long items on attn_long and
  // the remaining tiles on attn_tc; windowed layers run every tile on attn_tc.
  int nt = 0, n_long_tiles = 0, n_pairs = 0;
  const bool split = tc_attn && sjb::attn_long_pays(hcu, B);
  for (int b : order) {
    const int n = hcu[b + 1] - hcu[b];
    for (int q0 = 0; q0 < n; q0 += qt) {
      if (nt >= max_tiles) return fail(SJ_ERR_INVALID, "too many query tiles");
      h_tiles[nt++] = make_int2(b, q0);
    }
    if (split && n >= sjb::kAttnLongMin) n_long_tiles = nt;
  }
  if (n_long_tiles > 0) {
    for (int b : order) {
      const int n = hcu[b + 1] - hcu[b];
      if (n < sjb::kAttnLongMin) break;
      for (int q0 = 0; q0 < n; q0 += 256) {
        if (nt + n_pairs >= max_tiles) return fail(SJ_ERR_INVALID, "too many query tiles");
        h_tiles[nt + n_pairs++] = make_int2(b, q0);
      }
    }
  }
  if (nt + n_pairs > 0) {
    rc = cudaMemcpyAsync(tiles, h_tiles, (nt + n_pairs) * sizeof(int2), cudaMemcpyHostToDevice,
                         st);
    if (rc != cudaSuccess) return cuda_fail(rc, "cudaMemcpyAsync (tiles)");
  }
  if ((rc = cudaEventRecord(staged_ev, st))) return cuda_fail(rc, "cudaEventRecord");

  T* Yt = static_cast<T*>(Y);
  T* Qt = static_cast<T*>(QKV);
  T* Ot = static_cast<T*>(O);
  T* Gt = static_cast<T*>(G);
  const float eps = cfg.norm_eps;
  SJ_LAUNCH(SJ_K_FINAL, sjb::positions(d_cu, B, ntok, pos, nullptr, st));
  const bool sjm = arch == SJ_ARCH_SJMODEL;
  // SJ_PREC_FP8: the attn_norm and mlp_norm outputs are e4m3 rows with their
  // scales (Y8, sa8), the QKV and Wi GEMMs run on the e4m3 weights.
  // SJ_PREC_FP8_TENSOR: the same with one static scale per activation tensor
  // (act_scale); the GEGLU GEMM writes e4m3 codes (G8) for an e4m3 Wo2, and
  // the residual stream is bf16 (Xh: written by the embedding, updated by the
  // Wo and Wo2 epilogues, widened to fp32 X for the final norm).  Its
  // calibration pass runs the bf16 path and records each e4m3 operand's amax
  // (act_amax).
  const bool f8 = kBf16 && fp8 && !sjm && !calibrating;
  const bool f8t = f8 && fp8_tensor;
  const bool y0 = !layers.empty() && !layers[0].attn_norm;
  T* y_emb = f8t ? reinterpret_cast<T*>(Xh) : (y0 ? Yt : nullptr);
  SJ_LAUNCH(SJ_K_EMBED, sjb::embed_ln<T>(d_ids, ntok, emb, V, D, emb_norm, eps, X, y_emb, dflags,
                                         st, pos_emb, pos, cfg.max_position_embeddings,
                                         emb_norm_b));

  auto gemm = [&](int cls, const T* A, const void* W, T* C, float* resid, int N, int K, int epi,
                  const float* ct, const float* stb, const float* bias = nullptr,
                  int act = 0) -> int {
    return gemm_any<T>(cls, A, W, bias, act, C, resid, ntok, N, K, epi, ct, stb, st);
  };

  int s;
  for (int li = 0; li < NL; ++li) {
    const LayerDev& ly = layers[li];
    const T* Yin = Yt;
    if (f8t) {
      if (ly.attn_norm)
        SJ_LAUNCH(SJ_K_LN, sjb::ln_e4m3_static<bf16>(Xh, ly.attn_norm, ly.attn_norm_b, Y8, sa8,
                                                     act_scale + 3 * li, ntok, D, eps, st));
      else
        SJ_LAUNCH(SJ_K_LN,
                  sjb::quant_rows_static<bf16>(Xh, ntok, D, Y8, sa8, act_scale + 3 * li, st));
    } else if (f8) {
      if (ly.attn_norm)
        SJ_LAUNCH(SJ_K_LN, sjb::ln_e4m3(X, ly.attn_norm, ly.attn_norm_b, Y8, sa8, ntok, D, eps, st));
      else
        SJ_LAUNCH(SJ_K_LN, sjb::quant_rows_e4m3<float>(X, ntok, D, Y8, sa8, st));
    } else if (ly.attn_norm) {
      SJ_LAUNCH(SJ_K_LN, (sjb::add_ln<T, T>(X, nullptr, ly.attn_norm, ly.attn_norm_b, Yt, ntok, D, eps,
                                          nullptr, st)));
    } else if (li > 0) {
      if constexpr (kBf16) SJ_LAUNCH(SJ_K_LN, sjb::cast_bf16(X, Yt, (int64_t)ntok * D, st));
      else Yin = reinterpret_cast<const T*>(X);
    }
    if (calibrating) {  // the QKV input (layer 0's identity norm: X itself)
      if constexpr (kBf16) {
        if (ly.attn_norm || li > 0)
          SJ_LAUNCH(SJ_K_LN, sjb::amax_abs<bf16>(Yt, (int64_t)ntok * D, act_amax + 3 * li, st));
        else
          SJ_LAUNCH(SJ_K_LN, sjb::amax_abs<float>(X, (int64_t)ntok * D, act_amax + 3 * li, st));
      }
    }
    const float* ct = ly.sliding ? cos_s : cos_f;
    const float* stb = ly.sliding ? sin_s : sin_f;
    if (sjm) {  // SjModel: biased q/k/v, no RoPE
      if ((s = gemm(SJ_K_QKV, Yin, ly.wqkv, Qt, nullptr, 3 * D, D, sjb::TC_STORE, nullptr, nullptr,
                    ly.bqkv)))
        return s;
    } else if (f8) {
      if constexpr (kBf16) {
        sjb::TcRope rp{ct, stb, pos, H};
        sjb::TcQ8 uq;
        uq.uniform = f8t;
        SJ_LAUNCH(SJ_K_QKV, sjb::gemm_tc_f8(Y8, ly.wqkv8, sa8, ly.sqkv, nullptr, Qt, ntok, 3 * D, D,
                                            sjb::TC_ROPE, 0, rp, dflags + 1, st, nullptr, uq));
      }
    } else if ((s = gemm(SJ_K_QKV, Yin, ly.wqkv, Qt, nullptr, 3 * D, D, sjb::TC_ROPE, ct, stb))) {
      return s;
    }
    if (tc_attn) {
      if constexpr (kBf16) {
        if (ly.window == 0 && n_pairs > 0) {
          SJ_LAUNCH(SJ_K_ATTN, sjb::attn_long(Qt, d_cu, d_kvl, Ot, ntok, H, tiles + nt, n_pairs, B,
                                              0, dflags + 2, st));
          if (nt > n_long_tiles)
            SJ_LAUNCH(SJ_K_ATTN, sjb::attn_tc(Qt, d_cu, d_kvl, Ot, ntok, H, 0, tiles + n_long_tiles,
                                              nt - n_long_tiles, B, 0, dflags + 2, st));
        } else {
          SJ_LAUNCH(SJ_K_ATTN, sjb::attn_tc(Qt, d_cu, d_kvl, Ot, ntok, H, ly.window, tiles, nt, B, 0,
                                            dflags + 2, st));
        }
      }
    } else {
      SJ_LAUNCH(SJ_K_ATTN, sjb::attn_simt<T>(Qt, d_cu, d_kvl, Ot, H, Dh, ly.window, tiles, nt, B, 0, st));
    }
    if (f8t) {
      if constexpr (kBf16)
        SJ_LAUNCH(SJ_K_WO, sjb::gemm_tc(Ot, static_cast<const bf16*>(ly.wo), ly.bo, Xh, nullptr, ntok, D,
                                        D, sjb::TC_RESID16, 0,
                                        sjb::TcRope{}, dflags + 1, st));
    } else if ((s = gemm(SJ_K_WO, Ot, ly.wo, nullptr, X, D, D, sjb::TC_RESID, nullptr, nullptr,
                         ly.bo))) {
      return s;
    }
    if (f8t)
      SJ_LAUNCH(SJ_K_LN, sjb::ln_e4m3_static<bf16>(Xh, ly.mlp_norm, ly.mlp_norm_b, Y8, sa8,
                                                   act_scale + 3 * li + 1, ntok, D, eps, st));
    else if (f8)
      SJ_LAUNCH(SJ_K_LN, sjb::ln_e4m3(X, ly.mlp_norm, ly.mlp_norm_b, Y8, sa8, ntok, D, eps, st));
    else
      SJ_LAUNCH(SJ_K_LN, (sjb::add_ln<T, T>(X, nullptr, ly.mlp_norm, ly.mlp_norm_b, Yt, ntok, D, eps,
                                            nullptr, st)));
    if (calibrating) {
      if constexpr (kBf16)
        SJ_LAUNCH(SJ_K_LN, sjb::amax_abs<bf16>(Yt, (int64_t)ntok * D, act_amax + 3 * li + 1, st));
    }
    if (sjm) {  // SjModel: G = gelu(Y W1^T + b1), X += G W2^T + b2
      if ((s = gemm(SJ_K_GEGLU, Yt, ly.wi, Gt, nullptr, F, D, sjb::TC_STORE, nullptr, nullptr, ly.b1,
                    sjb::ACT_GELU)))
        return s;
    } else if (f8t) {
      if constexpr (kBf16) {
        sjb::TcQ8 q8;
        q8.C = G8;
        q8.scale = act_scale + 3 * li + 2;
        q8.rowscale = sg8;
        q8.uniform = true;
        SJ_LAUNCH(SJ_K_GEGLU, sjb::gemm_tc_f8(Y8, ly.wi8, sa8, ly.si, nullptr, nullptr, ntok, F, D,
                                              sjb::TC_GEGLU, 0, sjb::TcRope{}, dflags + 1, st,
                                              nullptr, q8));
      }
    } else if (f8) {
      if constexpr (kBf16)
        SJ_LAUNCH(SJ_K_GEGLU, sjb::gemm_tc_f8(Y8, ly.wi8, sa8, ly.si, nullptr, Gt, ntok, F, D,
                                              sjb::TC_GEGLU, 0, sjb::TcRope{}, dflags + 1, st));
    } else if ((s = gemm(SJ_K_GEGLU, Yt, ly.wi, Gt, nullptr, F, D, sjb::TC_GEGLU, nullptr, nullptr))) {
      return s;
    }
    if (calibrating) {
      if constexpr (kBf16)
        SJ_LAUNCH(SJ_K_GEGLU, sjb::amax_abs<bf16>(Gt, (int64_t)ntok * F, act_amax + 3 * li + 2, st));
    }
    if (f8t) {
      if constexpr (kBf16) {
        sjb::TcQ8 uq;
        uq.uniform = true;
        SJ_LAUNCH(SJ_K_WO2, sjb::gemm_tc_f8(G8, ly.wo2_8, sg8, ly.so2, ly.b2, Xh, ntok, D, F,
                                            sjb::TC_RESID16, 0, sjb::TcRope{}, dflags + 1, st,
                                            nullptr, uq));
      }
    } else if ((s = gemm(SJ_K_WO2, Gt, ly.wo2, nullptr, X, D, F, sjb::TC_RESID, nullptr, nullptr,
                         ly.b2))) {
      return s;
    }
  }
  // final norm (+ LoRA): all rows -> d_hidden, [CLS] rows -> heads
  if (f8t) {  // the bf16 residual stream to fp32: every row, or only the [CLS] rows
    if (d_hidden) SJ_LAUNCH(SJ_K_FINAL, sjb::widen_f32(Xh, X, (int64_t)ntok * D, st));
    else if (d_probs && has_heads) SJ_LAUNCH(SJ_K_FINAL, sjb::widen_rows_f32(Xh, X, d_cu, B, D, st));
  }
  if (d_hidden) {
    SJ_LAUNCH(SJ_K_FINAL, (sjb::add_ln<float, float>(X, nullptr, final_norm, final_norm_b, d_hidden, ntok,
                                                     D, eps, nullptr, st)));
    if (lora_r > 0) {
      SJ_LAUNCH(SJ_K_FINAL, (sjb::gemm_simt<float, float>(d_hidden, lora_a, nullptr, z, nullptr, ntok, lora_r, D,
                                              0, false, st)));
      SJ_LAUNCH(SJ_K_FINAL, (sjb::gemm_simt<float, float>(z, lora_b, nullptr, nullptr, d_hidden, ntok, D,
                                              lora_r, 0, false, st)));
    }
    if (dm && (s = head_forward<T>(d_cu, d_kvl, B, ntok, nt, d_hidden, *dm, st))) return s;
  }
  if (d_probs && has_heads) {
    SJ_LAUNCH(SJ_K_FINAL, (sjb::add_ln<float, float>(X, nullptr, final_norm, final_norm_b, Hc, B, D, eps,
                                                     d_cu, st)));
    if (lora_r > 0) {
      SJ_LAUNCH(SJ_K_FINAL, (sjb::gemm_simt<float, float>(Hc, lora_a, nullptr, z, nullptr, B, lora_r, D, 0,
                                              false, st)));
      SJ_LAUNCH(SJ_K_FINAL, (sjb::gemm_simt<float, float>(z, lora_b, nullptr, nullptr, Hc, B, D, lora_r, 0,
                                              false, st)));
    }
    SJ_LAUNCH(SJ_K_FINAL, sjb::dec_heads(Hc, B, D, head_w, head_b, spec, d_probs, st));
  }
  return SJ_OK;
}

// The decision-model tail on the final-norm hidden states h [ntok, D] (fp32,
// the head's residual stream), DecisionModel::forward model.cpp:402-535:
//   h += type_emb[qtype]
//   per head layer: h += out_proj(attn(LN1(h) in_proj^T + b)) + b   (no RoPE, keys < kv_len)
//                   h += linear2(relu(linear1(LN2(h)))) (+ biases)  (LN eps 1e-5)
//   scorer on the marker rows: LN -> Linear + GELU -> Linear(1); masked logits
//   act head per segment (head.cu)
// The head layers run in the activation precision on the encoder's kernels;
// the scorer and act head in fp32.
template <typename T>
int sj_fast::head_forward(const int32_t* d_cu, const int32_t* d_kvl, int B, int ntok, int nt,
                          float* h, const DmPass& dm, cudaStream_t st) {
  constexpr bool kBf16 = std::is_same<T, bf16>::value;
  const bool tc_attn = kBf16 && sjb::attn_tc_supported(Dh);
  T* Yt = static_cast<T*>(Y);
  T* Qt = static_cast<T*>(QKV);
  T* Ot = static_cast<T*>(O);
  T* Ft = static_cast<T*>(G);
  int s;
  // DecisionModel's head: LN eps 1e-5, ReLU FFN of 4D (model.cpp:419-459);
  // SjModel's: the config eps, GELU FFN of head_intermediate (sj_model.cpp:303-321)
  const bool sjm = arch == SJ_ARCH_SJMODEL;
  const float heps = sjm ? cfg.norm_eps : 1e-5f;
  const int ffn_act = sjm ? sjb::ACT_GELU : sjb::ACT_RELU;
  SJ_LAUNCH(SJ_K_FINAL, sjb::type_emb_add(h, d_cu, B, dm.qtype, type_emb, D, ntok, st));
  for (const HeadLayerDev& hl : hlayers) {
    SJ_LAUNCH(SJ_K_LN, (sjb::add_ln<T, T>(h, nullptr, hl.n1w, hl.n1b, Yt, ntok, D, heps, nullptr, st)));
    if ((s = gemm_any<T>(SJ_K_QKV, Yt, hl.in_w, hl.in_b, 0, Qt, nullptr, ntok, 3 * D, D,
                         sjb::TC_STORE, nullptr, nullptr, st)))
      return s;
    if (tc_attn) {
      if constexpr (kBf16)
        SJ_LAUNCH(SJ_K_ATTN, sjb::attn_tc(Qt, d_cu, d_kvl, Ot, ntok, H, 0, tiles, nt, B, 0,
                                         dflags + 2, st));
    } else {
      SJ_LAUNCH(SJ_K_ATTN, sjb::attn_simt<T>(Qt, d_cu, d_kvl, Ot, H, Dh, 0, tiles, nt, B, 0, st));
    }
    if ((s = gemm_any<T>(SJ_K_WO, Ot, hl.out_w, hl.out_b, 0, nullptr, h, ntok, D, D, sjb::TC_RESID,
                         nullptr, nullptr, st)))
      return s;
    SJ_LAUNCH(SJ_K_LN, (sjb::add_ln<T, T>(h, nullptr, hl.n2w, hl.n2b, Yt, ntok, D, heps, nullptr, st)));
    if ((s = gemm_any<T>(SJ_K_GEGLU, Yt, hl.l1w, hl.l1b, ffn_act, Ft, nullptr, ntok, head_ffn, D,
                         sjb::TC_STORE, nullptr, nullptr, st)))
      return s;
    if ((s = gemm_any<T>(SJ_K_WO2, Ft, hl.l2w, hl.l2b, 0, nullptr, h, ntok, D, head_ffn, sjb::TC_RESID,
                         nullptr, nullptr, st)))
      return s;
  }
  // scorer (model.cpp:462-487) and act head (:489-533), fp32
  const int BK = B * dm.K;
  SJ_LAUNCH(SJ_K_FINAL, sjb::gather_markers(h, d_cu, dm.pos, B, dm.K, D, dm_m, st));
  SJ_LAUNCH(SJ_K_FINAL, (sjb::add_ln<float, float>(dm_m, nullptr, sc_lnw, sc_lnb, dm_s, BK, D,
                                                   cfg.norm_eps, nullptr, st)));
  SJ_LAUNCH(SJ_K_FINAL, (sjb::gemm_simt<float, float>(dm_s, sc_w1, sc_b1, dm_s1, nullptr, BK, D, D,
                                                      sjb::ACT_GELU, false, st)));
  SJ_LAUNCH(SJ_K_FINAL, (sjb::gemm_simt<float, float>(dm_s1, sc_w2, sc_b2, dm_s2, nullptr, BK, 1, D,
                                                      0, false, st)));
  SJ_LAUNCH(SJ_K_FINAL, sjb::act_head(h, d_cu, B, dm_s2, dm.mask, dm.K, act_w1, act_b1, act_w2,
                                      act_b2, n_act, D, dm.logits, dm.act, sjm, st));
  return SJ_OK;
}

int sj_fast::run(const int64_t* d_ids, const int32_t* d_cu, const int32_t* hcu,
                 const int32_t* d_kvl, int B, float* d_hidden, float* d_probs, const DmPass* dm,
                 cudaStream_t st) {
  if (!committed) return fail(SJ_ERR_STATE, "forward before sj_fast_commit");
  if (B < 0) return fail(SJ_ERR_INVALID, "negative batch");
  if (B == 0) return SJ_OK;
  if (hcu[0] != 0) return fail(SJ_ERR_INVALID, "cu_seqlens[0] must be 0");
  for (int b = 0; b < B; ++b) {
    const int n = hcu[b + 1] - hcu[b];
    if (n < 0) return fail(SJ_ERR_INVALID, "cu_seqlens must be non-decreasing");
    // RoPE tables end at max_position_embeddings; SjModel clamps its learned
    // positions to the last row instead (sj_model.cpp:228-230)
    if (arch == SJ_ARCH_MODERNBERT && n > cfg.max_position_embeddings)
      return fail(SJ_ERR_INVALID, "sequence " + std::to_string(b) + " has " + std::to_string(n) +
                                      " tokens > max_position_embeddings " +
                                      std::to_string(cfg.max_position_embeddings));
    if (d_probs && has_heads && n == 0)
      return fail(SJ_ERR_INVALID, "sequence " + std::to_string(b) + " is empty (no [CLS] row)");
  }
  const int T = hcu[B];
  if (T > max_tokens)
    return fail(SJ_ERR_INVALID, "batch of " + std::to_string(T) + " tokens exceeds max_tokens " +
                                    std::to_string(max_tokens));
  if (T == 0) return SJ_OK;
  launches = 0;
  cudaError_t rc = cudaSetDevice(cfg.device);
  if (rc != cudaSuccess) return cuda_fail(rc, "cudaSetDevice");
  if (fp8_tensor && !calibrated) {
    // calibration: this first pass runs in bf16 and records the amax of every
    // tensor that becomes an e4m3 operand; the scales are amax * 2 / 448 (a
    // binade of headroom for later batches, whose larger values saturate at
    // 448), fixed from then on; the pass then runs again in FP8
    rc = cudaMemsetAsync(act_amax, 0, 3 * (size_t)NL * sizeof(unsigned), st);
    if (rc != cudaSuccess) return cuda_fail(rc, "cudaMemsetAsync");
    calibrating = true;
    const int cs = forward<bf16>(d_ids, d_cu, hcu, d_kvl, B, T, d_hidden, d_probs, dm, st);
    calibrating = false;
    if (cs) return cs;
    rc = sjb::scales_from_amax(act_amax, act_scale, 3 * NL, 2.f, st);
    if (rc != cudaSuccess) return cuda_fail(rc, "scales_from_amax");
    calibrated = true;
    launches = 0;
  }
  return bf16_mode ? forward<bf16>(d_ids, d_cu, hcu, d_kvl, B, T, d_hidden, d_probs, dm, st)
                   : forward<float>(d_ids, d_cu, hcu, d_kvl, B, T, d_hidden, d_probs, dm, st);
}

int sj_fast::check_flags(cudaStream_t st) {
  int h[8];
  cudaError_t rc = cudaMemcpyAsync(h, dflags, sizeof(h), cudaMemcpyDeviceToHost, st);
  if (rc == cudaSuccess) rc = cudaStreamSynchronize(st);
  if (rc != cudaSuccess) return cuda_fail(rc, "device sync");
  if (h[0] || h[1] || h[2]) {
    cudaMemsetAsync(dflags, 0, sizeof(h), st);
    cudaStreamSynchronize(st);
    if (h[0]) return fail(SJ_ERR_INVALID, "input id out of vocabulary range");
    return fail(SJ_ERR_TIMEOUT, std::string("a bounded device wait ran out in the ") +
                                    (h[1] ? "GEMM" : "attention") + " kernel (code " +
                                    std::to_string(h[1] ? h[1] : h[2]) + ")");
  }
  return SJ_OK;
}

int sj_fast::host_call(const int64_t* ids_h, const int32_t* cu_h, const int32_t* kvl_h, int B,
                       float* hidden_h, float* probs_h, float* pooled_h) {
  if (!committed) return fail(SJ_ERR_STATE, "forward before sj_fast_commit");
  if (B <= 0) return B == 0 ? SJ_OK : fail(SJ_ERR_INVALID, "negative batch");
  if (!cu_h || (!ids_h && cu_h[B] > 0)) return fail(SJ_ERR_INVALID, "null input");
  if (probs_h && !has_heads) return fail(SJ_ERR_STATE, "no decision heads set");
  if (cu_h[0] != 0) return fail(SJ_ERR_INVALID, "cu_seqlens[0] must be 0");
  for (int b = 0; b < B; ++b) {
    if (cu_h[b + 1] < cu_h[b]) return fail(SJ_ERR_INVALID, "cu_seqlens must be non-decreasing");
    if (kvl_h && (kvl_h[b] < 0 || kvl_h[b] > cu_h[b + 1] - cu_h[b]))
      return fail(SJ_ERR_INVALID, "kv_lens[b] must lie in [0, length of segment b]");
  }
  for (int64_t r = 0; r < cu_h[B]; ++r)
    if (ids_h[r] < 0 || ids_h[r] >= V)
      return fail(SJ_ERR_INVALID, "input id " + std::to_string(ids_h[r]) + " at row " +
                                      std::to_string(r) + " outside the vocabulary [0, vocab_size)");
  cudaError_t rc = cudaSetDevice(cfg.device);
  if (rc != cudaSuccess) return cuda_fail(rc, "cudaSetDevice");
  const int nout = std::max(1, spec.n_total);
  int b0 = 0;
  while (b0 < B) {
    // largest run of whole sequences that fits the workspace (at most
    // max_tokens rows and max_tokens sequences: empty ones take no rows)
    int b1 = b0;
    while (b1 < B && b1 - b0 < max_tokens && cu_h[b1 + 1] - cu_h[b0] <= max_tokens) ++b1;
    if (b1 == b0)
      return fail(SJ_ERR_INVALID, "sequence longer than max_tokens");
    const int nb = b1 - b0, base = cu_h[b0], T = cu_h[b1] - base;
    // the host runs one pass ahead: it waits only until the previous pass's
    // h_cu / h_kvl have reached the device (the device buffers are reused in
    // stream order; forward() guards its own schedule upload)
    rc = cudaEventSynchronize(inputs_ev);
    if (rc != cudaSuccess) return cuda_fail(rc, "cudaEventSynchronize");
    for (int b = 0; b <= nb; ++b) h_cu[b] = cu_h[b0 + b] - base;
    if (kvl_h) for (int b = 0; b < nb; ++b) h_kvl[b] = kvl_h[b0 + b];
    if ((rc = cudaMemcpyAsync(ids, ids_h + base, T * sizeof(int64_t), cudaMemcpyHostToDevice,
                              stream)) ||
        (rc = cudaMemcpyAsync(cu, h_cu, (nb + 1) * sizeof(int32_t), cudaMemcpyHostToDevice,
                              stream)) ||
        (kvl_h && (rc = cudaMemcpyAsync(kvl, h_kvl, nb * sizeof(int32_t),
                                        cudaMemcpyHostToDevice, stream))))
      return cuda_fail(rc, "cudaMemcpyAsync (inputs)");
    if ((rc = cudaEventRecord(inputs_ev, stream))) return cuda_fail(rc, "cudaEventRecord");
    // h_cu is read by run() for the schedule; it is pinned host memory that
    // stays untouched until the next pass's event wait above.
    int s = run(ids, cu, h_cu, kvl_h ? kvl : nullptr, nb, (hidden_h || pooled_h) ? hid : nullptr,
                probs_h ? probs : nullptr, nullptr, stream);
    if (s) return s;
    if (pooled_h) {  // per-segment means into Hc ([nb, D] <= [max_tokens, D])
      cudaStream_t st = stream;
      SJ_LAUNCH(SJ_K_FINAL, sjb::mean_pool(hid, cu, nb, D, Hc, stream));
      if ((rc = cudaMemcpyAsync(pooled_h + (int64_t)b0 * D, Hc, (size_t)nb * D * sizeof(float),
                                cudaMemcpyDeviceToHost, stream)))
        return cuda_fail(rc, "cudaMemcpyAsync (pooled)");
    }
    if (hidden_h && (rc = cudaMemcpyAsync(hidden_h + (int64_t)base * D, hid,
                                          (size_t)T * D * sizeof(float), cudaMemcpyDeviceToHost,
                                          stream)))
      return cuda_fail(rc, "cudaMemcpyAsync (hidden)");
    if (probs_h && (rc = cudaMemcpyAsync(probs_h + (int64_t)b0 * nout, probs,
                                         (size_t)nb * nout * sizeof(float),
                                         cudaMemcpyDeviceToHost, stream)))
      return cuda_fail(rc, "cudaMemcpyAsync (probs)");
    b0 = b1;
  }
  return check_flags(stream);
}

int sj_fast::dm_call(const int64_t* ids_h, const int32_t* cu_h, const int32_t* kvl_h, int B,
                     const int64_t* pos_h, const uint8_t* mask_h, int K, const int64_t* qtype_h,
                     float* logits_h, float* act_h) {
  if (!committed) return fail(SJ_ERR_STATE, "forward before sj_fast_commit");
  if (!has_dm)
    return fail(SJ_ERR_STATE, "the checkpoint has no decision-model head (type_emb, head, scorer"
                              "; act_head for DecisionModel)");
  if (B <= 0) return B == 0 ? SJ_OK : fail(SJ_ERR_INVALID, "negative batch");
  if (K < 1 || K > 4096) return fail(SJ_ERR_INVALID, "K (markers per sequence) must be in [1, 4096]");
  if (!cu_h || !ids_h || !pos_h || !mask_h || !qtype_h || !logits_h || !act_h)
    return fail(SJ_ERR_INVALID, "null input or output");
  if (cu_h[0] != 0) return fail(SJ_ERR_INVALID, "cu_seqlens[0] must be 0");
  for (int b = 0; b < B; ++b) {
    const int n = cu_h[b + 1] - cu_h[b];
    if (n < 1) return fail(SJ_ERR_INVALID, "every sequence needs at least one row ([CLS])");
    if (n > max_tokens) return fail(SJ_ERR_INVALID, "sequence longer than max_tokens");
    if (kvl_h && (kvl_h[b] < 0 || kvl_h[b] > n))
      return fail(SJ_ERR_INVALID, "kv_lens[b] must lie in [0, length of segment b]");
    if (qtype_h[b] < 0 || qtype_h[b] >= n_types)
      return fail(SJ_ERR_INVALID, "qtype " + std::to_string(qtype_h[b]) + " outside [0, " +
                                      std::to_string(n_types) + ")");
  }
  for (int64_t r = 0; r < cu_h[B]; ++r)
    if (ids_h[r] < 0 || ids_h[r] >= V)
      return fail(SJ_ERR_INVALID, "input id " + std::to_string(ids_h[r]) + " at row " +
                                      std::to_string(r) + " outside the vocabulary [0, vocab_size)");
  cudaError_t rc = cudaSetDevice(cfg.device);
  if (rc != cudaSuccess) return cuda_fail(rc, "cudaSetDevice");
  // passes of whole sequences; per-call buffers sized for the largest pass
  std::vector<std::pair<int, int>> passes;
  size_t max_nb = 0;
  for (int b0 = 0; b0 < B;) {
    int b1 = b0;
    while (b1 < B && cu_h[b1 + 1] - cu_h[b0] <= max_tokens) ++b1;
    passes.emplace_back(b0, b1);
    max_nb = std::max(max_nb, (size_t)(b1 - b0));
    b0 = b1;
  }
  if ((rc = cudaStreamSynchronize(stream))) return cuda_fail(rc, "cudaStreamSynchronize");
  const size_t bk = max_nb * (size_t)K;
  if (bk > dm_cap_bk) {
    if ((rc = grow(&dm_m, bk * D)) || (rc = grow(&dm_s, bk * D)) || (rc = grow(&dm_s1, bk * D)) ||
        (rc = grow(&dm_s2, bk)) || (rc = grow(&dm_logits, bk)) || (rc = grow(&dm_pos, bk)) ||
        (rc = grow(&dm_mask, bk)))
      return cuda_fail(rc, "cudaMalloc (marker rows)");
    dm_cap_bk = bk;
  }
  if (max_nb > dm_cap_b) {
    if ((rc = grow(&dm_qt, max_nb)) || (rc = grow(&dm_act, max_nb * (size_t)n_act)))
      return cuda_fail(rc, "cudaMalloc (act)");
    dm_cap_b = max_nb;
  }
  for (const auto& p : passes) {
    const int b0 = p.first, b1 = p.second, nb = b1 - b0, base = cu_h[b0], T = cu_h[b1] - base;
    rc = cudaEventSynchronize(staged_ev);
    if (rc != cudaSuccess) return cuda_fail(rc, "cudaEventSynchronize");
    for (int b = 0; b <= nb; ++b) h_cu[b] = cu_h[b0 + b] - base;
    if (kvl_h) for (int b = 0; b < nb; ++b) h_kvl[b] = kvl_h[b0 + b];
    const size_t nbk = (size_t)nb * K;
    if ((rc = cudaMemcpyAsync(ids, ids_h + base, T * sizeof(int64_t), cudaMemcpyHostToDevice,
                              stream)) ||
        (rc = cudaMemcpyAsync(cu, h_cu, (nb + 1) * sizeof(int32_t), cudaMemcpyHostToDevice,
                              stream)) ||
        (kvl_h && (rc = cudaMemcpyAsync(kvl, h_kvl, nb * sizeof(int32_t), cudaMemcpyHostToDevice,
                                        stream))) ||
        (rc = cudaMemcpyAsync(dm_qt, qtype_h + b0, nb * sizeof(int64_t), cudaMemcpyHostToDevice,
                              stream)) ||
        (rc = cudaMemcpyAsync(dm_pos, pos_h + (size_t)b0 * K, nbk * sizeof(int64_t),
                              cudaMemcpyHostToDevice, stream)) ||
        (rc = cudaMemcpyAsync(dm_mask, mask_h + (size_t)b0 * K, nbk, cudaMemcpyHostToDevice,
                              stream)))
      return cuda_fail(rc, "cudaMemcpyAsync (inputs)");
    DmPass dm{dm_qt, dm_pos, dm_mask, K, dm_logits, dm_act};
    int s = run(ids, cu, h_cu, kvl_h ? kvl : nullptr, nb, hid, nullptr, &dm, stream);
    if (s) return s;
    if ((rc = cudaMemcpyAsync(logits_h + (size_t)b0 * K, dm_logits, nbk * sizeof(float),
                              cudaMemcpyDeviceToHost, stream)) ||
        (rc = cudaMemcpyAsync(act_h + (size_t)b0 * n_act, dm_act,
                              (size_t)nb * n_act * sizeof(float), cudaMemcpyDeviceToHost, stream)))
      return cuda_fail(rc, "cudaMemcpyAsync (outputs)");
    if ((rc = cudaEventRecord(staged_ev, stream))) return cuda_fail(rc, "cudaEventRecord");
    // the next pass overwrites dm_* and the inputs: let this one finish reading them
    if ((rc = cudaStreamSynchronize(stream))) return cuda_fail(rc, "cudaStreamSynchronize");
  }
  return check_flags(stream);
}

// ------------------------------------------------------------------ C ABI
extern "C" {

int sj_fast_create(const sj_fast_config* cfg, sj_fast** out) {
  // failures leave their message in sj_last_error() (there is no engine yet)
  auto bad = [](int code, const std::string& m) {
    sjb::set_last_error("sj_fast_create: " + m);
    return code;
  };
  if (!cfg || !out) return bad(SJ_ERR_INVALID, "null argument");
  *out = nullptr;
  std::unique_ptr<sj_fast> e(new sj_fast());
  e->cfg = *cfg;
  const sj_fast_config& c = *cfg;
  if (c.hidden_size <= 0 || c.num_attention_heads <= 0 || c.num_hidden_layers < 0 ||
      c.intermediate_size <= 0 || c.vocab_size <= 0 || c.max_position_embeddings <= 0 ||
      c.hidden_size % c.num_attention_heads != 0 ||
      (c.hidden_size / c.num_attention_heads) % 2 != 0)
    return bad(SJ_ERR_INVALID, "bad model shape (sizes must be positive, hidden_size a multiple "
                               "of num_attention_heads, head_dim even)");
  if (c.precision != SJ_PREC_BF16 && c.precision != SJ_PREC_FP32 && c.precision != SJ_PREC_FP8 &&
      c.precision != SJ_PREC_FP8_TENSOR)
    return bad(SJ_ERR_UNSUPPORTED, "unknown precision");
  // the FP8 variant: the DecisionModel encoder, e4m3 GEMMs need K = D % 128 == 0,
  // the quantising LN D <= 1024, the attention head_dim 64 and N % 64 == 0
  if ((c.precision == SJ_PREC_FP8 || c.precision == SJ_PREC_FP8_TENSOR) &&
      (c.arch != SJ_ARCH_MODERNBERT || c.hidden_size % 128 != 0 || c.hidden_size > 1024 ||
       c.hidden_size / c.num_attention_heads != 64 ||
       c.intermediate_size % (c.precision == SJ_PREC_FP8_TENSOR ? 128 : 64) != 0))
    return bad(SJ_ERR_UNSUPPORTED, "the FP8 variant needs the DecisionModel encoder with "
                                   "hidden_size % 128 == 0, <= 1024, head_dim 64");
  if (c.arch != SJ_ARCH_MODERNBERT && c.arch != SJ_ARCH_SJMODEL)
    return bad(SJ_ERR_UNSUPPORTED, "unknown arch");
  // SjModel's learned positions are added in the warp-per-row embedding kernel
  if (c.arch == SJ_ARCH_SJMODEL && (c.hidden_size > 1024 || c.hidden_size % 4 != 0))
    return bad(SJ_ERR_UNSUPPORTED, "SjModel needs hidden_size <= 1024 and % 4 == 0");
  e->D = c.hidden_size;
  e->H = c.num_attention_heads;
  e->Dh = e->D / e->H;
  e->F = c.intermediate_size;
  e->V = c.vocab_size;
  e->NL = c.num_hidden_layers;
  e->bf16_mode = c.precision == SJ_PREC_BF16 || c.precision == SJ_PREC_FP8 ||
                 c.precision == SJ_PREC_FP8_TENSOR;
  e->fp8 = c.precision == SJ_PREC_FP8 || c.precision == SJ_PREC_FP8_TENSOR;
  e->fp8_tensor = c.precision == SJ_PREC_FP8_TENSOR;
  e->max_tokens = c.max_tokens > 0 ? c.max_tokens : (e->bf16_mode ? 262144 : 65536);
  e->max_tokens = std::max(e->max_tokens, 128);
  e->arch = c.arch;
  e->sliding.assign(e->NL, 0);
  if (c.layer_sliding && c.arch == SJ_ARCH_MODERNBERT)
    for (int i = 0; i < e->NL; ++i) e->sliding[i] = c.layer_sliding[i];
  e->cfg.layer_sliding = nullptr;  // not retained
  if (e->bf16_mode && (e->D % 8 != 0 || e->F % 8 != 0))
    return bad(SJ_ERR_UNSUPPORTED, "bf16 mode needs hidden_size and intermediate_size % 8 == 0");
  cudaError_t rc = cudaSetDevice(c.device);
  if (rc == cudaSuccess) rc = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
  if (rc != cudaSuccess)
    return bad(SJ_ERR_CUDA, std::string("device ") + std::to_string(c.device) + ": " +
                                cudaGetErrorString(rc));
  *out = e.release();
  return SJ_OK;
}

int sj_fast_set_tensor(sj_fast* e, const char* name, const float* host, const int64_t* shape,
                       int ndim) {
  if (!e || !name || !host || (ndim > 0 && !shape) || ndim < 0 || ndim > 8)
    return SJ_ERR_INVALID;
  if (e->committed) return e->fail(SJ_ERR_STATE, "sj_fast_set_tensor after sj_fast_commit");
  HostTensor t;
  int64_t n = 1;
  for (int i = 0; i < ndim; ++i) {
    if (shape[i] < 0) return e->fail(SJ_ERR_INVALID, std::string("negative dim in ") + name);
    t.shape.push_back(shape[i]);
    n *= shape[i];
  }
  t.data.assign(host, host + n);
  e->staged[name] = std::move(t);
  return SJ_OK;
}

int sj_fast_set_heads(sj_fast* e, int n_heads, const int* n_out, const int* kind) {
  if (!e) return SJ_ERR_INVALID;
  if (e->committed) return e->fail(SJ_ERR_STATE, "sj_fast_set_heads after sj_fast_commit");
  if (n_heads < 0 || n_heads > 8 || (n_heads > 0 && (!n_out || !kind)))
    return e->fail(SJ_ERR_INVALID, "n_heads must be in [0, 8]");
  sjb::HeadSpec s{};
  s.n_heads = n_heads;
  int off = 0;
  for (int h = 0; h < n_heads; ++h) {
    if (n_out[h] <= 0 || (kind[h] != SJ_HEAD_SOFTMAX && kind[h] != SJ_HEAD_SIGMOID))
      return e->fail(SJ_ERR_INVALID, "bad head " + std::to_string(h));
    s.off[h] = off;
    s.n_out[h] = n_out[h];
    s.kind[h] = kind[h];
    off += n_out[h];
  }
  if (off > 64) return e->fail(SJ_ERR_INVALID, "at most 64 head outputs in total");
  s.n_total = off;
  e->spec = s;
  e->has_heads = n_heads > 0;
  return SJ_OK;
}

int sj_fast_commit(sj_fast* e) { return e ? e->commit() : SJ_ERR_INVALID; }

int sj_fast_encode(sj_fast* e, const int64_t* ids, const int32_t* cu_seqlens,
                   const int32_t* kv_lens, int B, float* hidden) {
  if (!e) return SJ_ERR_INVALID;
  if (!hidden && B > 0) return e->fail(SJ_ERR_INVALID, "null hidden output");
  return e->host_call(ids, cu_seqlens, kv_lens, B, hidden, nullptr);
}

int sj_fast_embed(sj_fast* e, const int64_t* ids, const int32_t* cu_seqlens, int B,
                  float* pooled) {
  if (!e) return SJ_ERR_INVALID;
  if (!pooled && B > 0) return e->fail(SJ_ERR_INVALID, "null pooled output");
  return e->host_call(ids, cu_seqlens, nullptr, B, nullptr, nullptr, pooled);
}

int sj_fast_decide(sj_fast* e, const int64_t* ids, const int32_t* cu_seqlens, int B,
                   float* probs) {
  if (!e) return SJ_ERR_INVALID;
  if (!probs && B > 0) return e->fail(SJ_ERR_INVALID, "null probs output");
  return e->host_call(ids, cu_seqlens, nullptr, B, nullptr, probs);
}

int sj_fast_forward(sj_fast* e, const int64_t* ids, const int32_t* cu_seqlens,
                    const int32_t* kv_lens, int B, const int64_t* marker_pos,
                    const uint8_t* marker_mask, int K, const int64_t* qtype, float* logits,
                    float* act) {
  if (!e) return SJ_ERR_INVALID;
  return e->dm_call(ids, cu_seqlens, kv_lens, B, marker_pos, marker_mask, K, qtype, logits, act);
}

int sj_fast_n_act(const sj_fast* e) { return e && e->has_dm ? e->n_act : 0; }

int sj_fast_encode_device(sj_fast* e, const int64_t* ids, const int32_t* cu_seqlens,
                          const int32_t* cu_seqlens_host, const int32_t* kv_lens, int B,
                          float* hidden, float* probs, void* stream) {
  if (!e) return SJ_ERR_INVALID;
  if (!cu_seqlens_host || (B > 0 && (!ids || !cu_seqlens)))
    return e->fail(SJ_ERR_INVALID, "null input");
  if (probs && !e->has_heads) return e->fail(SJ_ERR_STATE, "no decision heads set");
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : e->stream;
  return e->run(ids, cu_seqlens, cu_seqlens_host, kv_lens, B, hidden, probs, nullptr, st);
}

int sj_fast_sync(sj_fast* e, void* stream) {
  if (!e) return SJ_ERR_INVALID;
  cudaError_t rc = cudaSetDevice(e->cfg.device);
  if (rc != cudaSuccess) return e->cuda_fail(rc, "cudaSetDevice");
  return e->check_flags(stream ? static_cast<cudaStream_t>(stream) : e->stream);
}

int sj_fast_launch_count(const sj_fast* e) { return e ? e->launches : 0; }

int sj_fast_reset_calibration(sj_fast* e) {
  if (!e) return SJ_ERR_INVALID;
  if (!e->fp8_tensor) return e->fail(SJ_ERR_STATE, "sj_fast_reset_calibration: not SJ_PREC_FP8_TENSOR");
  e->calibrated = false;
  return SJ_OK;
}

int sj_fast_set_profiling(sj_fast* e, int enable) {
  if (!e) return SJ_ERR_INVALID;
  e->profiling = enable != 0;
  return SJ_OK;
}

int sj_fast_profile(sj_fast* e, double* ms, int64_t* launches, int reset) {
  if (!e) return SJ_ERR_INVALID;
  cudaError_t rc = cudaSetDevice(e->cfg.device);
  if (rc != cudaSuccess) return e->cuda_fail(rc, "cudaSetDevice");
  int s = e->collect_profile();
  if (s) return s;
  for (int k = 0; k < SJ_K_COUNT; ++k) {
    if (ms) ms[k] = e->prof_ms[k];
    if (launches) launches[k] = e->prof_n[k];
    if (reset) {
      e->prof_ms[k] = 0;
      e->prof_n[k] = 0;
    }
  }
  return SJ_OK;
}

const char* sj_fast_last_error(const sj_fast* e) { return e ? e->err.c_str() : "null engine"; }

void sj_fast_destroy(sj_fast* e) { delete e; }

}  // extern "C"
