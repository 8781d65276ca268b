// fast.cpp — snapjudge::FastSnapjudge on libsnapjudge_b200 (drop-in for the
// reference's cuda/fast.cpp).
//
// Compiled inside the snapjudge tree: it implements include/snapjudge/fast.hpp
// (FastSnapjudge(DecisionModel*, int max_len, bool use_graphs) + forward with
// the signature of DecisionModel::forward, model.hpp:64-70) and reads the
// model's weights through the `friend class FastSnapjudge` access the
// reference grants (model.hpp:128-129), as its own fast path does.
//
//  * the encoder (model.cpp:333-400) runs on the GPU through the C ABI
//    (sj_fast_*): every padded row is computed, keys masked by the row's
//    attention-mask length, so padded rows match the CPU forward too;
//  * the decision-model tail (model.cpp:409-535: type embedding, head
//    TransformerEncoderLayers, scorer, act head) runs on the host in fp32 with
//    the reference's own tensor ops, as the reference fast path intended
//    (cuda/fast.cpp:1-6: "fp32 scorer/act-head tail").
// Failures throw std::runtime_error("snapjudge CUDA: ..."), as cuda/fast.cpp:54-58.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "snapjudge/fast.hpp"
#include "snapjudge/model.hpp"
#include "snapjudge/tensor.hpp"
#include "snapjudge_b200.h"

namespace snapjudge {

namespace {

[[noreturn]] void fail(const sj_fast* e, int rc, const std::string& what) {
  throw std::runtime_error("snapjudge CUDA: " + what + ": " +
                           (e ? sj_fast_last_error(e) : sj_last_error()) + " (status " +
                           std::to_string(rc) + ")");
}

Tensor view(const float* p, std::vector<int64_t> shape) {
  return Tensor::wrap(std::move(shape),
                      std::shared_ptr<float[]>(const_cast<float*>(p), [](float*) {}));
}

// [M, D] rows of (b, i, head h) -> [B, H, L, Dh] and back
void split_heads(const float* src, int64_t B, int64_t L, int64_t H, int64_t Dh, int64_t ld,
                 int64_t off, float* dst) {
  for (int64_t b = 0; b < B; ++b)
    for (int64_t i = 0; i < L; ++i)
      for (int64_t h = 0; h < H; ++h)
        std::memcpy(dst + ((b * H + h) * L + i) * Dh, src + (b * L + i) * ld + off + h * Dh,
                    sizeof(float) * static_cast<size_t>(Dh));
}
void merge_heads(const float* src, int64_t B, int64_t L, int64_t H, int64_t Dh, float* dst) {
  for (int64_t b = 0; b < B; ++b)
    for (int64_t i = 0; i < L; ++i)
      for (int64_t h = 0; h < H; ++h)
        std::memcpy(dst + (b * L + i) * H * Dh + h * Dh, src + ((b * H + h) * L + i) * Dh,
                    sizeof(float) * static_cast<size_t>(Dh));
}

}  // namespace

struct FastSnapjudge::Impl {
  DecisionModel* m = nullptr;
  sj_fast* e = nullptr;
  int max_len = 512;
  ~Impl() {
    if (e) sj_fast_destroy(e);
  }
};

FastSnapjudge::FastSnapjudge(DecisionModel* model, int max_len, bool /*use_graphs*/)
    : impl_(std::make_unique<Impl>()) {
  Impl& im = *impl_;
  im.m = model;
  im.max_len = max_len;
  const ModelConfig& c = model->cfg_;
  std::vector<int> sliding(static_cast<size_t>(c.num_hidden_layers));
  for (int i = 0; i < c.num_hidden_layers; ++i)
    sliding[static_cast<size_t>(i)] = model->layers_[static_cast<size_t>(i)].attention_type ==
                                      "sliding_attention";
  sj_fast_config fc{};
  fc.hidden_size = c.hidden_size;
  fc.num_hidden_layers = c.num_hidden_layers;
  fc.num_attention_heads = c.num_attention_heads;
  fc.intermediate_size = c.intermediate_size;
  fc.vocab_size = c.vocab_size;
  fc.max_position_embeddings = c.max_position_embeddings;
  fc.norm_eps = c.norm_eps;
  fc.local_attention = c.local_attention;
  fc.layer_sliding = sliding.data();
  fc.rope_theta_full = c.rope_theta_full;
  fc.rope_theta_sliding = c.rope_theta_sliding;
  fc.precision = SJ_PREC_BF16;
  fc.device = 0;
  fc.max_tokens = 0;
  int rc = sj_fast_create(&fc, &im.e);
  if (rc) fail(nullptr, rc, "sj_fast_create");
  auto put = [&](const std::string& name, const float* p, std::vector<int64_t> shape) {
    int r = sj_fast_set_tensor(im.e, name.c_str(), p, shape.data(), static_cast<int>(shape.size()));
    if (r) fail(im.e, r, "sj_fast_set_tensor " + name);
  };
  const int64_t D = model->D_, F = model->F_, V = c.vocab_size;
  put("encoder.embeddings.tok_embeddings.weight", model->emb_w_.get(), {V, D});
  put("encoder.embeddings.norm.weight", model->emb_norm_.get(), {D});
  put("encoder.final_norm.weight", model->final_norm_.get(), {D});
  for (size_t i = 0; i < model->layers_.size(); ++i) {
    const LayerWeights& ly = model->layers_[i];
    const std::string p = "encoder.layers." + std::to_string(i) + ".";
    if (ly.has_attn_norm) put(p + "attn_norm.weight", ly.attn_norm.d.get(), {D});
    put(p + "attn.Wqkv.weight", ly.wqkv.d.get(), {3 * D, D});
    put(p + "attn.Wo.weight", ly.wo.d.get(), {D, D});
    put(p + "mlp_norm.weight", ly.mlp_norm.d.get(), {D});
    put(p + "mlp.Wi.weight", ly.wi.d.get(), {2 * F, D});
    put(p + "mlp.Wo.weight", ly.wo2.d.get(), {D, F});
  }
  if (model->lora_r_ > 0) {
    put("lora_A.weight", model->lora_a_.get(), {model->lora_r_, D});
    put("lora_B.weight", model->lora_b_.get(), {D, model->lora_r_});
  }
  rc = sj_fast_commit(im.e);
  if (rc) fail(im.e, rc, "sj_fast_commit");
}

FastSnapjudge::~FastSnapjudge() = default;

void FastSnapjudge::forward(const std::vector<std::vector<int64_t>>& input_ids,
                            const std::vector<std::vector<int64_t>>& attention_mask,
                            const std::vector<std::vector<int64_t>>& marker_pos,
                            const std::vector<std::vector<uint8_t>>& marker_mask,
                            const std::vector<int64_t>& qtype,
                            std::vector<std::vector<float>>& logits_out,
                            std::vector<std::vector<float>>& act_out) {
  const DecisionModel& md = *impl_->m;
  const int64_t B = static_cast<int64_t>(input_ids.size());
  if (B == 0) return;
  const int64_t L = static_cast<int64_t>(input_ids[0].size());
  const int64_t K = static_cast<int64_t>(marker_pos[0].size());
  const int64_t M = B * L, D = md.D_, H = md.H_, Dh = md.Dh_;

  // ---- encoder on the GPU: each padded row is a segment of length L whose
  // queries attend the first lens[b] keys (the padded-batch semantics)
  std::vector<int64_t> flat(static_cast<size_t>(M));
  std::vector<int32_t> cu(static_cast<size_t>(B + 1)), kvl(static_cast<size_t>(B));
  std::vector<int64_t> lens(static_cast<size_t>(B));
  for (int64_t b = 0; b < B; ++b) {
    std::copy(input_ids[b].begin(), input_ids[b].end(), flat.begin() + b * L);
    int64_t s = 0;
    for (int64_t v : attention_mask[b]) s += v;
    lens[b] = s;
    kvl[b] = static_cast<int32_t>(s);
    cu[b] = static_cast<int32_t>(b * L);
  }
  cu[B] = static_cast<int32_t>(M);
  Tensor h({M, D});
  int rc = sj_fast_encode(impl_->e, flat.data(), cu.data(), kvl.data(), static_cast<int>(B),
                          h.mutable_data());
  if (rc) fail(impl_->e, rc, "sj_fast_encode");

  // ---- decision-model tail on the host (model.cpp:409-535), fp32
  for (int64_t b = 0; b < B; ++b) {
    const float* te = md.type_emb_.get() + qtype[b] * D;
    for (int64_t i = 0; i < L; ++i) {
      float* row = h.mutable_data() + (b * L + i) * D;
      for (int64_t j = 0; j < D; ++j) row[j] += te[j];
    }
  }
  Tensor Q({B, H, L, Dh}), Kt({B, H, L, Dh}), V({B, H, L, Dh}), AO({M, D});
  for (const auto& hl : md.head_) {
    Tensor ln = layer_norm(h, hl.n1w.get(), hl.n1b.get(), 1e-5f);
    Tensor qkv = gemm_nt(ln, view(hl.in_w.get(), {3 * D, D}), hl.in_b.get(), 0);
    split_heads(qkv.data_ptr(), B, L, H, Dh, 3 * D, 0, Q.mutable_data());
    split_heads(qkv.data_ptr(), B, L, H, Dh, 3 * D, D, Kt.mutable_data());
    split_heads(qkv.data_ptr(), B, L, H, Dh, 3 * D, 2 * D, V.mutable_data());
    Tensor at = attention(Q, Kt, V, lens, 0);
    merge_heads(at.data_ptr(), B, L, H, Dh, AO.mutable_data());
    add_(h, gemm_nt(AO, view(hl.out_w.get(), {D, D}), hl.out_b.get(), 0));
    ln = layer_norm(h, hl.n2w.get(), hl.n2b.get(), 1e-5f);
    Tensor f1 = gemm_nt(ln, view(hl.l1w.get(), {4 * D, D}), hl.l1b.get(), 2);
    add_(h, gemm_nt(f1, view(hl.l2w.get(), {D, 4 * D}), hl.l2b.get(), 0));
  }
  // scorer on the marker rows (positions clamped to [0, L))
  Tensor mk({B * K, D});
  for (int64_t b = 0; b < B; ++b)
    for (int64_t k = 0; k < K; ++k) {
      const int64_t p = std::min(std::max<int64_t>(marker_pos[b][k], 0), L - 1);
      std::memcpy(mk.mutable_data() + (b * K + k) * D, h.data_ptr() + (b * L + p) * D,
                  sizeof(float) * static_cast<size_t>(D));
    }
  Tensor s = layer_norm(mk, md.scorer_ln_w_.get(), md.scorer_ln_b_.get(), md.cfg_.norm_eps);
  s = gemm_nt(s, view(md.scorer_w1_.get(), {D, D}), md.scorer_b1_.get(), 1);
  s = gemm_nt(s, view(md.scorer_w2_.get(), {1, D}), md.scorer_b2_.get(), 0);
  logits_out.assign(static_cast<size_t>(B), std::vector<float>(static_cast<size_t>(K)));
  for (int64_t b = 0; b < B; ++b)
    for (int64_t k = 0; k < K; ++k)
      logits_out[b][k] = marker_mask[b][k] ? s.data_ptr()[b * K + k] : -1e4f;
  // act head: [CLS row, top1, top1 - top2, normalised entropy, k / 255]
  const int n_act = md.cfg_.n_act;
  act_out.assign(static_cast<size_t>(B), std::vector<float>(static_cast<size_t>(n_act)));
  for (int64_t b = 0; b < B; ++b) {
    const std::vector<float>& lg = logits_out[b];
    const float mx = *std::max_element(lg.begin(), lg.end());
    std::vector<double> p(lg.size());
    double z = 0;
    for (size_t j = 0; j < lg.size(); ++j) z += (p[j] = std::exp(lg[j] - mx));
    double top1 = 0, top2 = 0, ent = 0, ks = 0;
    for (double& v : p) {
      v /= z;
      if (v > top1) { top2 = top1; top1 = v; } else if (v > top2) { top2 = v; }
      ent -= v * std::log(std::max(v, 1e-9));
    }
    for (int64_t k = 0; k < K; ++k) ks += marker_mask[b][k];
    const double kf = std::max(2.0, ks);
    ent /= std::log(kf);
    std::vector<float> feats(static_cast<size_t>(D + 4));
    std::memcpy(feats.data(), h.data_ptr() + b * L * D, sizeof(float) * static_cast<size_t>(D));
    feats[D] = static_cast<float>(top1);
    feats[D + 1] = static_cast<float>(top1 - top2);
    feats[D + 2] = static_cast<float>(ent);
    feats[D + 3] = static_cast<float>(kf / 255.0);
    Tensor a1 = gemm_nt(view(feats.data(), {1, D + 4}), view(md.act_w1_.get(), {256, D + 4}),
                        md.act_b1_.get(), 1);
    Tensor a2 = gemm_nt(a1, view(md.act_w2_.get(), {n_act, 256}), md.act_b2_.get(), 0);
    float amx = a2.data_ptr()[0];
    for (int j = 1; j < n_act; ++j) amx = std::max(amx, a2.data_ptr()[j]);
    double as = 0;
    std::vector<float> ex(static_cast<size_t>(n_act));
    for (int j = 0; j < n_act; ++j) as += (ex[j] = std::exp(a2.data_ptr()[j] - amx));
    for (int j = 0; j < n_act; ++j) act_out[b][j] = static_cast<float>(ex[j] / as);
  }
}

}  // namespace snapjudge
