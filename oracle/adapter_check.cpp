// adapter_check.cpp — the reference's DecisionModel::forward (CPU, fp32) against
// snapjudge::FastSnapjudge::forward (snapjudge_b200/integration/fast.cpp, the
// whole forward on the GPU through the C ABI) on one checkpoint and a ragged
// padded batch, once packed to its valid rows and once with a live marker on a
// padded row (the padding computed).  TEST INFRASTRUCTURE ONLY (built by oracle/Makefile into oracle/_ref/).
//
// usage: adapter_check <checkpoint dir>  -> prints one JSON line of max diffs;
// exit 0 when the bf16 tolerances hold (logits 2e-2, act probabilities 5e-3).
#include <cmath>
#include <cstdio>
#include <fstream>
#include <random>
#include <string>
#include <vector>

#include "nlohmann/json.hpp"
#include "snapjudge/fast.hpp"
#include "snapjudge/model.hpp"
#include "snapjudge/safetensors.hpp"

using namespace snapjudge;

int main(int argc, char** argv) {
  if (argc < 2) return 2;
  std::string d = argv[1];
  nlohmann::json rl, enc;
  std::ifstream(d + "/rl_agent_config.json") >> rl;
  std::ifstream(d + "/encoder/config.json") >> enc;
  SafeTensors w = SafeTensors::load(d + "/model.safetensors");
  auto model = DecisionModel::load(rl, enc, w, d);
  const int V = model->cfg().vocab_size;
  std::mt19937 rng(11);
  const int B = 4, L = 37, K = 4;
  const int lens[B] = {37, 20, 1, 9};
  std::vector<std::vector<int64_t>> ids(B, std::vector<int64_t>(L, 0)), mask(B, std::vector<int64_t>(L, 0));
  std::vector<std::vector<int64_t>> mp(B, std::vector<int64_t>(K, 0));
  std::vector<std::vector<uint8_t>> mm(B, std::vector<uint8_t>(K, 0));
  std::vector<int64_t> qt(B);
  for (int b = 0; b < B; ++b) {
    for (int i = 0; i < lens[b]; ++i) {
      ids[b][i] = static_cast<int64_t>(rng() % V);
      mask[b][i] = 1;
    }
    const int k = 1 + static_cast<int>(rng() % K);
    for (int j = 0; j < k; ++j) {
      mp[b][j] = static_cast<int64_t>(rng() % lens[b]);
      mm[b][j] = 1;
    }
    qt[b] = static_cast<int64_t>(rng() % 3);
  }
  FastSnapjudge fast(model.get(), 512, true);
  double dl = 0, da = 0;
  // batch 1: markers on valid rows (the adapter packs the batch to its valid
  // rows); batch 2: one live marker on a padded row (it computes the padding)
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1) {
      mp[3][0] = lens[3] + 5;  // a padded position of row 3
      mm[3][0] = 1;
    }
    std::vector<std::vector<float>> lg_ref, act_ref, lg, act;
    model->forward(ids, mask, mp, mm, qt, lg_ref, act_ref);
    fast.forward(ids, mask, mp, mm, qt, lg, act);
    for (int b = 0; b < B; ++b) {
      for (int k = 0; k < K; ++k) dl = std::max(dl, (double)std::fabs(lg[b][k] - lg_ref[b][k]));
      for (size_t j = 0; j < act[b].size(); ++j)
        da = std::max(da, (double)std::fabs(act[b][j] - act_ref[b][j]));
    }
  }
  std::printf("{\"logits_max_abs\": %.3g, \"act_max_abs\": %.3g}\n", dl, da);
  return (dl <= 2e-2 && da <= 5e-3) ? 0 : 1;
}
