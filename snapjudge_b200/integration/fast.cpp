// fast.cpp — snapjudge::FastSnapjudge on libsnapjudge_b200 (drop-in for the
// reference's cuda/fast.cpp).
//
// Compiled inside the snapjudge tree: it implements include/snapjudge/fast.hpp
// (FastSnapjudge(DecisionModel*, int max_len, bool use_graphs) + forward with
// the signature of DecisionModel::forward, model.hpp:64-70) and reads the
// model's weights through the `friend class FastSnapjudge` access the
// reference grants (model.hpp:128-129), as its own fast path does.
//
// The whole forward (model.cpp:309-536) runs on the GPU through the C ABI
// (sj_fast_forward): the encoder, then the decision-model tail (type embedding,
// head TransformerEncoderLayers, scorer on the marker rows, act head).  A
// padded batch is packed to its valid rows unless a live marker points into
// the padding; then every padded row is computed, keys masked by the row's
// attention-mask length, as the CPU forward does.
// Failures throw std::runtime_error("snapjudge CUDA: ..."), as cuda/fast.cpp:54-58.
// Precision: bf16 (the reference fast path's contract, cuda/fast.cpp:1-6) unless
// SNAPJUDGE_FAST_PRECISION=fp32 selects the fp32 parity mode (1e-4 relative to
// the CPU forward), e.g. to reproduce CPU outputs that sit on a tie.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "snapjudge/fast.hpp"
#include "snapjudge/model.hpp"
#include "snapjudge_b200.h"

namespace snapjudge {

namespace {

[[noreturn]] void fail(const sj_fast* e, int rc, const std::string& what) {
  throw std::runtime_error("snapjudge CUDA: " + what + ": " +
                           (e ? sj_fast_last_error(e) : sj_last_error()) + " (status " +
                           std::to_string(rc) + ")");
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
  const char* prec = std::getenv("SNAPJUDGE_FAST_PRECISION");
  fc.precision = (prec && std::string(prec) == "fp32") ? SJ_PREC_FP32 : SJ_PREC_BF16;
  fc.device = 0;
  fc.max_tokens = 0;
  int rc = sj_fast_create(&fc, &im.e);
  if (rc) fail(nullptr, rc, "sj_fast_create");
  auto put = [&](const std::string& name, const float* p, std::vector<int64_t> shape) {
    if (!p) return;  // optional tensor absent
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
  // decision-model tail (model.cpp:130-176 names and shapes)
  put("type_emb.weight", model->type_emb_.get(), {3, D});
  for (size_t i = 0; i < model->head_.size(); ++i) {
    const auto& hl = model->head_[i];
    const std::string p = "head.layers." + std::to_string(i) + ".";
    put(p + "norm1.weight", hl.n1w.get(), {D});
    put(p + "norm1.bias", hl.n1b.get(), {D});
    put(p + "norm2.weight", hl.n2w.get(), {D});
    put(p + "norm2.bias", hl.n2b.get(), {D});
    put(p + "self_attn.in_proj_weight", hl.in_w.get(), {3 * D, D});
    put(p + "self_attn.in_proj_bias", hl.in_b.get(), {3 * D});
    put(p + "self_attn.out_proj.weight", hl.out_w.get(), {D, D});
    put(p + "self_attn.out_proj.bias", hl.out_b.get(), {D});
    put(p + "linear1.weight", hl.l1w.get(), {4 * D, D});
    put(p + "linear1.bias", hl.l1b.get(), {4 * D});
    put(p + "linear2.weight", hl.l2w.get(), {D, 4 * D});
    put(p + "linear2.bias", hl.l2b.get(), {D});
  }
  put("scorer.0.weight", model->scorer_ln_w_.get(), {D});
  put("scorer.0.bias", model->scorer_ln_b_.get(), {D});
  put("scorer.1.weight", model->scorer_w1_.get(), {D, D});
  put("scorer.1.bias", model->scorer_b1_.get(), {D});
  put("scorer.3.weight", model->scorer_w2_.get(), {1, D});
  put("scorer.3.bias", model->scorer_b2_.get(), {1});
  put("act_head.0.weight", model->act_w1_.get(), {256, D + 4});
  put("act_head.0.bias", model->act_b1_.get(), {256});
  put("act_head.2.weight", model->act_w2_.get(), {c.n_act, 256});
  put("act_head.2.bias", model->act_b2_.get(), {c.n_act});
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
  const int64_t B = static_cast<int64_t>(input_ids.size());
  if (B == 0) return;
  const int64_t L = static_cast<int64_t>(input_ids[0].size());
  const int64_t K = static_cast<int64_t>(marker_pos[0].size());
  const int64_t M = B * L;
  const int n_act = sj_fast_n_act(impl_->e);

  std::vector<int64_t> pos(static_cast<size_t>(B * K));
  std::vector<uint8_t> mm(static_cast<size_t>(B * K));
  std::vector<int32_t> kvl(static_cast<size_t>(B));
  // The outputs depend on padded rows only through a live marker that points
  // past its row's length (model.cpp:463-474 gathers that padded row).  Without
  // one, only the valid rows are computed (packed segments); otherwise each
  // padded row is a segment of length L whose queries attend the first lens[b]
  // keys (the padded-batch semantics).
  bool pack = true;
  for (int64_t b = 0; b < B; ++b) {
    std::copy(marker_pos[b].begin(), marker_pos[b].end(), pos.begin() + b * K);
    std::copy(marker_mask[b].begin(), marker_mask[b].end(), mm.begin() + b * K);
    int64_t s = 0;
    for (int64_t v : attention_mask[b]) s += v;
    kvl[b] = static_cast<int32_t>(s);
    if (s < 1) pack = false;
    for (int64_t k = 0; k < K; ++k) {
      const int64_t p = std::min(std::max<int64_t>(marker_pos[b][k], 0), L - 1);
      if (marker_mask[b][k] && p >= s) pack = false;
    }
  }
  std::vector<int64_t> flat;
  std::vector<int32_t> cu(static_cast<size_t>(B + 1), 0);
  flat.reserve(static_cast<size_t>(M));
  for (int64_t b = 0; b < B; ++b) {
    const int64_t n = pack ? kvl[b] : L;
    flat.insert(flat.end(), input_ids[b].begin(), input_ids[b].begin() + n);
    cu[b + 1] = cu[b] + static_cast<int32_t>(n);
  }
  std::vector<float> lg(static_cast<size_t>(B * K)), ac(static_cast<size_t>(B * n_act));
  int rc = sj_fast_forward(impl_->e, flat.data(), cu.data(), pack ? nullptr : kvl.data(),
                           static_cast<int>(B), pos.data(), mm.data(), static_cast<int>(K),
                           qtype.data(), lg.data(), ac.data());
  if (rc) fail(impl_->e, rc, "sj_fast_forward");
  logits_out.assign(static_cast<size_t>(B), std::vector<float>(static_cast<size_t>(K)));
  act_out.assign(static_cast<size_t>(B), std::vector<float>(static_cast<size_t>(n_act)));
  for (int64_t b = 0; b < B; ++b) {
    std::copy(lg.begin() + b * K, lg.begin() + (b + 1) * K, logits_out[b].begin());
    std::copy(ac.begin() + b * n_act, ac.begin() + (b + 1) * n_act, act_out[b].begin());
  }
}

}  // namespace snapjudge
