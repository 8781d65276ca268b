// ref_driver.cpp — C-ABI shim over the snapjudge reference's own CPU forward.
//
// TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile together with the
// reference's unchanged src/model.cpp, src/tensor.cpp and src/safetensors.cpp
// (compiled where they lie, output only into oracle/_ref/).  Tests use it to
// pin the C restatement (sj_oracle.c) and the CUDA path; the benchmark's
// reference arm times it.  The product library never links it.
//
// Entry points wrap, one to one:
//   sjref_sj_*     SjModel (src/sj_model.cpp): load from sj_config.json +
//                  model.safetensors (:88-204), encode (:257-275), forward (:277-368)
//   sjref_load     Agent::Agent's loading steps (src/agent.cpp:40-85):
//                  rl_agent_config.json + encoder/config.json + model.safetensors
//                  -> DecisionModel::load (src/model.cpp:35-205)
//   sjref_encode   DecisionModel::encode  (src/model.cpp:222-307)
//   sjref_forward  DecisionModel::forward (src/model.cpp:309-536)
//   sjref_*        the tensor ops of src/tensor.cpp
#include <cstdint>
#include <cstring>
#include <fstream>
#include <memory>
#include <string>
#include <vector>

#include "nlohmann/json.hpp"
#include "snapjudge/model.hpp"
#include "snapjudge/safetensors.hpp"
#include "snapjudge/sj_model.hpp"
#include "snapjudge/tensor.hpp"

using nlohmann::json;
using namespace snapjudge;

namespace {
thread_local std::string g_err;

json read_json(const std::string& p) {
  std::ifstream f(p);
  if (!f.good()) throw std::runtime_error("cannot open " + p);
  json j;
  f >> j;
  return j;
}

Tensor wrap(const float* p, std::vector<int64_t> shape) {
  return Tensor::wrap(std::move(shape),
                      std::shared_ptr<float[]>(const_cast<float*>(p), [](float*) {}));
}

void copy_out(const Tensor& t, float* out) {
  std::memcpy(out, t.data_ptr(), sizeof(float) * static_cast<size_t>(t.numel()));
}
}  // namespace

extern "C" {

const char* sjref_last_error() { return g_err.c_str(); }

void* sjref_load(const char* dir) {
  try {
    std::string d(dir);
    json rl = read_json(d + "/rl_agent_config.json");
    json enc = read_json(d + "/encoder/config.json");
    SafeTensors w = SafeTensors::load(d + "/model.safetensors");
    auto m = DecisionModel::load(rl, enc, w, d);
    return m.release();
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}

void sjref_free(void* h) { delete static_cast<DecisionModel*>(h); }

int sjref_n_act(void* h) { return static_cast<DecisionModel*>(h)->cfg().n_act; }

// ids/mask [B, L] row-major; out [B, L, D].
int sjref_encode(void* h, const int64_t* ids, const int64_t* mask, int64_t B, int64_t L,
                 float* out) {
  try {
    auto* m = static_cast<DecisionModel*>(h);
    std::vector<std::vector<int64_t>> vi(static_cast<size_t>(B)), vm(static_cast<size_t>(B));
    for (int64_t b = 0; b < B; ++b) {
      vi[b].assign(ids + b * L, ids + (b + 1) * L);
      vm[b].assign(mask + b * L, mask + (b + 1) * L);
    }
    auto hs = m->encode(vi, vm);
    const int D = m->D();
    for (int64_t b = 0; b < B; ++b)
      for (int64_t i = 0; i < L; ++i)
        std::memcpy(out + (b * L + i) * D, hs[b][i].data(), sizeof(float) * D);
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}

int sjref_forward(void* h, const int64_t* ids, const int64_t* mask, int64_t B, int64_t L,
                  const int64_t* marker_pos, const uint8_t* marker_mask, int64_t K,
                  const int64_t* qtype, float* logits, float* act) {
  try {
    auto* m = static_cast<DecisionModel*>(h);
    std::vector<std::vector<int64_t>> vi(B), vm(B), mp(B);
    std::vector<std::vector<uint8_t>> mm(B);
    for (int64_t b = 0; b < B; ++b) {
      vi[b].assign(ids + b * L, ids + (b + 1) * L);
      vm[b].assign(mask + b * L, mask + (b + 1) * L);
      mp[b].assign(marker_pos + b * K, marker_pos + (b + 1) * K);
      mm[b].assign(marker_mask + b * K, marker_mask + (b + 1) * K);
    }
    std::vector<int64_t> qt(qtype, qtype + B);
    std::vector<std::vector<float>> lo, ao;
    m->forward(vi, vm, mp, mm, qt, lo, ao);
    const int na = m->cfg().n_act;
    for (int64_t b = 0; b < B; ++b) {
      std::memcpy(logits + b * K, lo[b].data(), sizeof(float) * K);
      std::memcpy(act + b * na, ao[b].data(), sizeof(float) * na);
    }
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}

// ---- SjModel (src/sj_model.cpp) ----
void* sjref_sj_load(const char* dir) {
  try {
    std::string d(dir);
    json cfg = read_json(d + "/sj_config.json");
    SafeTensors w = SafeTensors::load(d + "/model.safetensors");
    return SjModel::load(cfg, w, d).release();
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}

void sjref_sj_free(void* h) { delete static_cast<SjModel*>(h); }

int sjref_sj_encode(void* h, const int64_t* ids, const int64_t* mask, int64_t B, int64_t L,
                    int64_t D, float* out) {
  try {
    auto* m = static_cast<SjModel*>(h);
    std::vector<std::vector<int64_t>> vi(static_cast<size_t>(B)), vm(static_cast<size_t>(B));
    for (int64_t b = 0; b < B; ++b) {
      vi[b].assign(ids + b * L, ids + (b + 1) * L);
      vm[b].assign(mask + b * L, mask + (b + 1) * L);
    }
    auto hs = m->encode(vi, vm);
    for (int64_t b = 0; b < B; ++b)
      for (int64_t i = 0; i < L; ++i)
        std::memcpy(out + (b * L + i) * D, hs[b][i].data(), sizeof(float) * D);
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}

// act [B, 2]
int sjref_sj_forward(void* h, const int64_t* ids, const int64_t* mask, int64_t B, int64_t L,
                     const int64_t* marker_pos, const uint8_t* marker_mask, int64_t K,
                     const int64_t* qtype, float* logits, float* act) {
  try {
    auto* m = static_cast<SjModel*>(h);
    std::vector<std::vector<int64_t>> vi(B), vm(B), mp(B);
    std::vector<std::vector<uint8_t>> mm(B);
    for (int64_t b = 0; b < B; ++b) {
      vi[b].assign(ids + b * L, ids + (b + 1) * L);
      vm[b].assign(mask + b * L, mask + (b + 1) * L);
      mp[b].assign(marker_pos + b * K, marker_pos + (b + 1) * K);
      mm[b].assign(marker_mask + b * K, marker_mask + (b + 1) * K);
    }
    std::vector<int64_t> qt(qtype, qtype + B);
    std::vector<std::vector<float>> lo, ao;
    m->forward(vi, vm, mp, mm, qt, lo, ao);
    for (int64_t b = 0; b < B; ++b) {
      std::memcpy(logits + b * K, lo[b].data(), sizeof(float) * K);
      std::memcpy(act + b * 2, ao[b].data(), sizeof(float) * 2);
    }
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}

// ---- tensor ops (src/tensor.cpp) ----
int sjref_layer_norm(const float* x, int64_t rows, int64_t D, const float* w, const float* b,
                     float eps, float* out) {
  copy_out(layer_norm(wrap(x, {rows, D}), w, b, eps), out);
  return 0;
}

int sjref_gemm_nt(const float* a, int64_t M, int64_t K, const float* w, int64_t N,
                  const float* bias, int act, float* out) {
  copy_out(gemm_nt(wrap(a, {M, K}), wrap(w, {N, K}), bias, act), out);
  return 0;
}

int sjref_geglu(const float* a, int64_t M, int64_t K, const float* wi, int64_t F, float* out) {
  copy_out(gemm_geglu(wrap(a, {M, K}), wrap(wi, {2 * F, K})), out);
  return 0;
}

int sjref_attention(const float* q, const float* k, const float* v, int64_t B, int64_t H,
                    int64_t L, int64_t Dh, const int64_t* lens, int window, float* out) {
  std::vector<int64_t> vl;
  if (lens) vl.assign(lens, lens + B);
  copy_out(attention(wrap(q, {B, H, L, Dh}), wrap(k, {B, H, L, Dh}), wrap(v, {B, H, L, Dh}),
                     vl, window),
           out);
  return 0;
}

int sjref_rope(float* qkv, int64_t M, const float* cos_t, const float* sin_t, int64_t L,
               int64_t H, int64_t Dh) {
  Tensor t = wrap(qkv, {M, 3 * H * Dh});
  rope_inplace(t, cos_t, sin_t, L, H, Dh);
  return 0;
}

}  // extern "C"
