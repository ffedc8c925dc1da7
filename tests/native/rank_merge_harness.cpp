// Test harness: the product's choice of a node's split when its features are
// spread over ranks (csrc/split_select.h), run on the CPU: every rank keeps
// the largest key of its own feature range, as eval_kernel's atomicMax does,
// and the ranks' keys are merged as merge_best_kernel merges them. Test
// infrastructure only.
#include <cstdint>
#include <vector>

#include "split_select.h"

using namespace xgbb;

// gains [nodes][cols]: each (node, feature)'s best candidate gain. Writes the
// chosen feature (-1 when no rank had a key) and its gain per node.
extern "C" int rank_merge(const float* gains, uint32_t nodes, uint32_t cols, uint32_t world, int32_t* feature,
                          float* gain) {
  std::vector<unsigned long long> keys(size_t(world) * nodes, 0);
  uint32_t pad = 0;
  for (uint32_t r = 0; r < world; ++r) {
    uint32_t lo, hi;
    rank_features(cols, world, r, &pad, &lo, &hi);
    if (pad % world || lo > hi || hi > cols) return -1;
    for (uint32_t n = 0; n < nodes; ++n)
      for (uint32_t f = lo; f < hi; ++f) {
        const unsigned long long k = split_key(gains[size_t(n) * cols + f], f);
        if (k > keys[size_t(r) * nodes + n]) keys[size_t(r) * nodes + n] = k;
      }
  }
  for (uint32_t n = 0; n < nodes; ++n) {
    unsigned long long key;
    merge_rank_keys(world, [&](uint32_t r) { return keys[size_t(r) * nodes + n]; }, &key);
    const uint32_t f = key_feature(key);
    feature[n] = key && f < cols ? int32_t(f) : -1;
    gain[n] = key && f < cols ? gains[size_t(n) * cols + f] : 0.0f;
  }
  return 0;
}
