// Choosing a node's split across features and across ranks: the ordering key
// of a candidate, the feature range each rank evaluates, and the merge of the
// ranks' best candidates. The CUDA kernels (eval_kernel, merge_best_kernel)
// and the host (learner.cpp) use these, and a CPU harness runs the same
// functions against the oracle's selection.
//
// The order is the reference's selection (select_splits,
// kernels/boost.metal:1245-1302): the largest gain, and among equal gains the
// smallest feature.
#pragma once
#include <cstdint>
#include <cstring>

#include "exec.h"

namespace xgbb {

// Order-preserving map of a float gain to uint32 (-0 folded onto +0), so that
// a 64-bit max over (gain << 32 | ~feature) picks the largest gain and, among
// equal gains, the smallest feature.
XGBB_HD inline uint32_t gain_order(float g) {
  const float z = g == 0.0f ? 0.0f : g;
  uint32_t b;
  std::memcpy(&b, &z, 4);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

XGBB_HD inline unsigned long long split_key(float gain, uint32_t feature) {
  return ((unsigned long long)gain_order(gain) << 32) | (0xffffffffu - feature);
}

XGBB_HD inline uint32_t key_feature(unsigned long long key) { return 0xffffffffu - uint32_t(key & 0xffffffffu); }

// Rank `rank` of `world` evaluates features [*lo, *hi). The feature count is
// padded to a multiple of the ranks (*pad) so that a reduce-scatter of the
// feature-major histograms hands every rank whole features; ranks past the
// last real feature get an empty range.
XGBB_HD inline void rank_features(uint32_t cols, uint32_t world, uint32_t rank, uint32_t* pad, uint32_t* lo,
                                  uint32_t* hi) {
  const uint32_t p = (cols + world - 1) / world * world;
  const uint32_t per = p / world;
  *pad = p;
  *lo = rank * per < cols ? rank * per : cols;
  *hi = (rank + 1) * per < cols ? (rank + 1) * per : cols;
}

// The best of every rank's key for one slot (`key_of(r)` for r < ranks).
// Returns the winning rank; *key receives its key.
template <class KeyOf>
XGBB_HD uint32_t merge_rank_keys(uint32_t ranks, KeyOf key_of, unsigned long long* key) {
  uint32_t best = 0;
  unsigned long long k0 = key_of(0u);
  for (uint32_t r = 1; r < ranks; ++r) {
    const unsigned long long k = key_of(r);
    if (k > k0) {
      k0 = k;
      best = r;
    }
  }
  *key = k0;
  return best;
}

}  // namespace xgbb
