// Host-driven tree growth (src/tree.cpp:291-349, 1031-1120 in the reference):
// a priority queue of evaluated leaves, popped one at a time by largest gain
// (loss-guided) or in batches of up to 256 leaves of one depth in node-id
// order (depth-wise); each popped batch is applied, its leaves' rows are
// partitioned and the children are evaluated together.
#include "grower.h"

#include <cmath>
#include <queue>

namespace xgbb {

namespace {

struct QueuedLeaf {
  uint32_t id, depth;
  Segment rows;
  DevSplit split;
};

// std::priority_queue pops the largest element: loss-guided trees pop the
// largest gain first, ties and depth-wise trees the smallest node id
// (src/tree.cpp:63-69). Node ids are unique, so the order is total.
struct PopsLater {
  bool lossguide;
  bool operator()(const QueuedLeaf& a, const QueuedLeaf& b) const {
    if (lossguide && a.split.gain != b.split.gain) return a.split.gain < b.split.gain;
    return a.id > b.id;
  }
};

DevNode leaf_node(int32_t parent, float leaf, float cover) {
  DevNode n{};
  n.left = n.right = n.feature = -1;
  n.split_bin = -1;
  n.parent = parent;
  n.leaf = leaf;
  n.cover = cover;
  n.base_weight = leaf;
  return n;
}

}  // namespace

void applied_parent_stats(const DevSplit& s, const GrowerParams& p, float* weight, float* hessian) {
  int eg = 0, eh = 0;
  std::frexp(p.scale_g, &eg);
  std::frexp(p.scale_h, &eh);
  const double inv_g = std::ldexp(1.0, -(eg - 1)), inv_h = std::ldexp(1.0, -(eh - 1));
  auto value_of = [](long long v, double inv) { return v == 0 ? 0.0 : double(v) * inv; };
  const double G = value_of(s.left_g, inv_g) + value_of(s.right_g, inv_g);
  const double H = value_of(s.left_hs, inv_h) + value_of(s.right_hs, inv_h);
  double value = 0.0;
  if (H > 0.0) {
    const double alpha = std::fabs(double(p.tree.reg_alpha));
    const double t = std::fabs(G) <= alpha ? 0.0 : (G < 0.0 ? G + alpha : G - alpha);
    value = -t / (H + double(p.tree.reg_lambda));
    const double limit = std::fabs(double(p.tree.max_delta_step));
    if (limit != 0.0 && std::fabs(value) > limit) value = std::copysign(limit, value);
  }
  *weight = float(value);
  *hessian = float(H);
}

std::vector<DevNode> grow_tree_host_driven(GrowerBackend& backend, uint32_t rows, const GrowerParams& p) {
  const TreeParams& tp = p.tree;
  const uint32_t max_depth = tp.max_depth, max_leaves = p.max_leaves;
  const float eta = tp.eta;
  std::vector<DevNode> nodes;
  std::priority_queue<QueuedLeaf, std::vector<QueuedLeaf>, PopsLater> queue(PopsLater{p.lossguide});
  uint32_t leaves = 1;  // the root counts as one leaf

  {
    std::vector<DevSplit> out;
    backend.evaluate({Segment{0, rows}}, true, {}, out);
    require(out.size() == 1, "grower backend returned no root split");
    const DevSplit& s = out[0];
    DevNode root = leaf_node(-1, s.parent_weight * eta, s.total_h);
    root.base_weight = s.parent_weight;
    root.flags = 1u;
    nodes.push_back(root);
    queue.push(QueuedLeaf{0, 0, Segment{0, rows}, s});
  }

  std::vector<QueuedLeaf> batch, kids;
  std::vector<PartitionItem> items;
  std::vector<uint32_t> left_rows;
  std::vector<Segment> kid_rows;
  std::vector<long long> kid_sums;
  std::vector<DevSplit> kid_splits;
  for (;;) {
    // Pop a batch: the leaves whose split is usable within the depth and leaf
    // limits, each counted as one more leaf.
    batch.clear();
    if (queue.empty()) break;
    const uint32_t depth = queue.top().depth;
    do {
      QueuedLeaf leaf = queue.top();
      queue.pop();
      const DevSplit& s = leaf.split;
      if (s.feature >= 0 && s.gain > 1.0e-6f && s.gain >= tp.min_split_loss &&
          (!max_depth || leaf.depth < max_depth) && (!max_leaves || leaves < max_leaves)) {
        ++leaves;
        batch.push_back(leaf);
      }
      if (p.lossguide) break;
    } while (!queue.empty() && queue.top().depth == depth && batch.size() < kQueueBatch);
    if (batch.empty()) break;

    // Apply: children numbered in pop order; the leaves that may grow further
    // have their rows partitioned.
    kids.clear();
    items.clear();
    for (QueuedLeaf& leaf : batch) {
      DevSplit& s = leaf.split;
      require(nodes.size() + 2 <= size_t(INT32_MAX), "tree exceeds the node index range");
      const uint32_t left = uint32_t(nodes.size());
      applied_parent_stats(s, p, &s.applied_parent_weight, &s.applied_parent_hessian);
      nodes.push_back(leaf_node(int32_t(leaf.id), s.left_weight * eta, s.left_h));
      nodes.push_back(leaf_node(int32_t(leaf.id), s.right_weight * eta, s.right_h));
      DevNode& nd = nodes[leaf.id];
      nd.left = int32_t(left);
      nd.right = int32_t(left + 1);
      nd.feature = s.feature;
      nd.split_bin = s.split_bin;
      nd.default_left = s.default_left;
      nd.threshold = s.threshold;
      nd.gain = s.gain;
      nd.cover = s.applied_parent_hessian;
      nd.base_weight = s.applied_parent_weight;
      nd.flags |= 2u;
      if ((!max_depth || leaf.depth + 1 < max_depth) && (!max_leaves || leaves < max_leaves)) {
        items.push_back(PartitionItem{leaf.rows.begin, leaf.rows.count, s.feature, s.split_bin, s.default_left});
        kids.push_back(QueuedLeaf{left, leaf.depth + 1, leaf.rows, s});
        kids.push_back(QueuedLeaf{left + 1, leaf.depth + 1, leaf.rows, s});
      }
    }
    if (kids.empty()) continue;
    backend.partition(items, left_rows);
    require(left_rows.size() == items.size(), "grower backend returned no partition counts");
    kid_rows.clear();
    kid_sums.clear();
    for (size_t i = 0; i < items.size(); ++i) {
      const uint32_t nl = left_rows[i];
      require(nl <= items[i].count, "grower backend returned an invalid partition");
      const DevSplit& s = kids[2 * i].split;
      kid_rows.push_back(Segment{items[i].begin, nl});
      kid_rows.push_back(Segment{items[i].begin + nl, items[i].count - nl});
      kid_sums.insert(kid_sums.end(), {s.left_g, s.left_hs, s.right_g, s.right_hs});
    }
    backend.evaluate(kid_rows, false, kid_sums, kid_splits);
    require(kid_splits.size() == kids.size(), "grower backend returned too few splits");
    for (size_t i = 0; i < kids.size(); ++i) {
      QueuedLeaf& k = kids[i];
      k.rows = kid_rows[i];
      k.split = kid_splits[i];
      nodes[k.id].cover = k.split.total_h;
      nodes[k.id].flags |= 1u;
      if (k.split.gain > 1.0e-6f) queue.push(k);
    }
  }
  return nodes;
}

}  // namespace xgbb
