// cache_policy.cu — the expert cache's decision functions (host code, no device work).
//
// Reference: src/moe/cached_layer.rs — fill_candidate (:344-355), top_k_ids (:358-363),
// union_by_votes (:367-379), streamed_misses (:385-398), lru_victim (:401-410). Same ordering keys as
// the reference, so the same inputs pick the same experts; tests/test_policy.py checks them against
// the reference's own known-answer cases and against randomised cases.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <numeric>
#include <vector>

#include "moe_b200.h"

namespace {

// IEEE-754 total order of f32 as an unsigned key (what Rust's f32::total_cmp compares).
inline uint32_t total_key(float f) {
  uint32_t b;
  std::memcpy(&b, &f, 4);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

}  // namespace

extern "C" {

int moe_policy_top_k_ids(const float* logits, int n, int k, int32_t* out) {
  if (n < 0 || k < 0 || (n && !logits) || (k && !out)) return -1;
  std::vector<int> idx(n);
  std::iota(idx.begin(), idx.end(), 0);
  const int take = std::min(k, n);
  std::partial_sort(idx.begin(), idx.begin() + take, idx.end(), [&](int a, int b) {
    const uint32_t ka = total_key(logits[a]), kb = total_key(logits[b]);
    return ka != kb ? ka > kb : a < b;
  });
  for (int i = 0; i < take; ++i) out[i] = idx[i];
  return take;
}

int moe_policy_union_by_votes(const int32_t* const* rankings, const int32_t* lens, int n_rankings, int32_t* out) {
  if (n_rankings < 0 || (n_rankings && (!rankings || !lens))) return -1;
  std::map<int, std::pair<int, int>> seen;  // expert -> (votes, best rank)
  for (int r = 0; r < n_rankings; ++r)
    for (int i = 0; i < lens[r]; ++i) {
      auto it = seen.find(rankings[r][i]);
      if (it == seen.end()) seen.emplace(rankings[r][i], std::make_pair(1, i));
      else {
        it->second.first += 1;
        it->second.second = std::min(it->second.second, i);
      }
    }
  std::vector<std::pair<int, std::pair<int, int>>> v(seen.begin(), seen.end());
  std::sort(v.begin(), v.end(), [](const auto& a, const auto& b) {
    if (a.second.first != b.second.first) return a.second.first > b.second.first;
    if (a.second.second != b.second.second) return a.second.second < b.second.second;
    return a.first < b.first;
  });
  for (size_t i = 0; i < v.size(); ++i) out[i] = v[i].first;
  return (int)v.size();
}

int moe_policy_streamed_misses(const uint32_t* ids, const float* weights, const int32_t* row_lens, int rows,
                               float frac, int cap, uint32_t* out) {
  if (rows < 0 || (rows && (!row_lens || !ids || !weights))) return -1;
  if (frac <= 0.0f || cap <= 0) return 0;
  std::map<uint32_t, float> total;  // distinct missed expert -> routed weight
  int p = 0;
  for (int r = 0; r < rows; ++r)
    for (int j = 0; j < row_lens[r]; ++j, ++p) total[ids[p]] += weights[p];
  const int take = std::min((int)std::ceil(frac * (float)total.size()), cap);
  std::vector<std::pair<uint32_t, float>> v(total.begin(), total.end());
  std::sort(v.begin(), v.end(), [](const auto& a, const auto& b) {
    const uint32_t ka = total_key(a.second), kb = total_key(b.second);
    return ka != kb ? ka > kb : a.first < b.first;
  });
  const int n = std::min<int>(take, (int)v.size());
  for (int i = 0; i < n; ++i) out[i] = v[i].first;
  return n;
}

int moe_policy_lru_victim(const int32_t* slot_expert, const int32_t* slot_published, const uint64_t* last_use,
                          int n_slots, const int32_t* protect, int n_protect, int32_t* expert_out) {
  int best = -1;
  for (int s = 0; s < n_slots; ++s) {
    const int e = slot_expert[s];
    if (e < 0 || !slot_published[s]) continue;
    bool prot = false;
    for (int i = 0; i < n_protect && !prot; ++i) prot = protect[i] == e;
    if (prot) continue;
    if (best < 0 || last_use[s] < last_use[best] || (last_use[s] == last_use[best] && e < slot_expert[best])) best = s;
  }
  if (best >= 0 && expert_out) *expert_out = slot_expert[best];
  return best;
}

int moe_policy_fill_candidate(const int32_t* slot_expert, int n_slots, const uint64_t* hit_counts, int n_experts) {
  bool any_free = false;
  std::vector<char> taken(n_experts > 0 ? n_experts : 0, 0);
  for (int s = 0; s < n_slots; ++s) {
    if (slot_expert[s] < 0) any_free = true;
    else if (slot_expert[s] < n_experts) taken[slot_expert[s]] = 1;
  }
  if (!any_free) return -1;
  int best = -1;
  for (int e = 0; e < n_experts; ++e) {
    if (taken[e]) continue;
    if (best < 0 || hit_counts[e] > hit_counts[best]) best = e;  // ties keep the lowest id
  }
  return best;
}

}  // extern "C"
