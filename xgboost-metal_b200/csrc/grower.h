// Host-driven tree growth: the reference's fallback driver for loss-guided
// trees, leaf budgets (max_leaves) and depths beyond the device driver's ten
// levels (src/tree.cpp:291-349, 1031-1120). The host keeps a priority queue
// of evaluated leaves and pops them in batches; a backend builds the
// histograms, evaluates the splits and partitions the rows of each batch.
//
// The control logic here has no device code: the CUDA backend lives in
// queue.cu, and any backend that evaluates splits with the same semantics
// grows the same tree.
#pragma once
#include <cstdint>
#include <vector>

#include "common.h"

namespace xgbb {

// Leaves popped per depth-wise batch (src/tree.cpp:1031-1050); a batch has
// at most twice as many children.
constexpr uint32_t kQueueBatch = 256;

// Rows [begin, begin + count) of the backend's row order belong to one node.
struct Segment {
  uint32_t begin, count;
};

// One leaf of a batch whose rows are split between its two children: rows
// with bin <= split_bin go left, missing values follow default_left.
struct PartitionItem {
  uint32_t begin, count;
  int32_t feature, split_bin;
  uint32_t default_left;
};

class GrowerBackend {
 public:
  virtual ~GrowerBackend() = default;
  // The best split of each node over its segment. The root totals its own
  // histogram; other nodes take their exact (g, h) totals from `sums` ([n][2],
  // the parent split's child sums) so the missing bin is total - present.
  virtual void evaluate(const std::vector<Segment>& nodes, bool root, const std::vector<long long>& sums,
                        std::vector<DevSplit>& out) = 0;
  // Reorders each item's segment so that its left rows come first; returns the
  // left row count of each item.
  virtual void partition(const std::vector<PartitionItem>& items, std::vector<uint32_t>& left) = 0;
};

struct GrowerParams {
  TreeParams tree;  // max_depth 0 = unlimited
  bool lossguide = false;
  uint32_t max_leaves = 0;  // 0 = unlimited
  // The group's power-of-two gradient scales (g, h): integer sums are in
  // units of 1/scale.
  float scale_g = 1.0f, scale_h = 1.0f;
};

// Grows one tree over `rows` rows; returns the node table (node id = index)
// with the device driver's field conventions.
std::vector<DevNode> grow_tree_host_driven(GrowerBackend& backend, uint32_t rows, const GrowerParams& p);

// The parent weight and Hessian an applied split records on its node, from
// the exact child sums (the device driver's control step,
// kernels/split_statistics.metal.h:1-38).
void applied_parent_stats(const DevSplit& s, const GrowerParams& p, float* weight, float* hessian);

}  // namespace xgbb
