// Test harness: the product's host-driven grower (csrc/grower.cpp) driven by
// a backend that evaluates and partitions with the CPU oracle, so that the
// grower's control logic (queue order, batches, limits, node numbering and
// fields, applied parent statistics) can be checked against the oracle's own
// host-driven grower without a GPU. Test infrastructure only.
#include <cstring>
#include <vector>

#include "grower.h"
extern "C" {
#include "oracle.h"
}

namespace {

struct OracleBackend : xgbb::GrowerBackend {
  const uint32_t* bins;
  uint32_t rows, cols, stride;
  const int64_t* q;
  const float* scale;
  const float* cuts;
  const uint32_t* counts;
  const float* minima;
  orc_tree_params tp;
  std::vector<uint32_t> order;

  void evaluate(const std::vector<xgbb::Segment>& nodes, bool root, const std::vector<long long>& sums,
                std::vector<xgbb::DevSplit>& out) override {
    out.assign(nodes.size(), xgbb::DevSplit{});
    std::vector<int64_t> hist(size_t(cols) * (stride + 1) * 2);
    std::vector<orc_split> cand(cols);
    for (size_t i = 0; i < nodes.size(); ++i) {
      std::fill(hist.begin(), hist.end(), 0);
      orc_histogram(bins, cols, stride, q, order.data() + nodes[i].begin, nodes[i].count, hist.data());
      int64_t s[2] = {root ? 0 : sums[2 * i], root ? 0 : sums[2 * i + 1]};
      orc_evaluate_splits(hist.data(), 1, cols, stride, scale, cuts, counts, minima, tp.reg_lambda, tp.reg_alpha,
                          tp.min_child_weight, tp.max_delta_step, root ? 0u : 1u, s, cand.data());
      orc_split b;
      orc_select_splits(cand.data(), 1, cols, scale, tp.reg_lambda, tp.reg_alpha, tp.max_delta_step, &b);
      xgbb::DevSplit& d = out[i];
      d.gain = b.gain;
      d.threshold = b.threshold;
      d.feature = b.feature;
      d.split_bin = -1;
      if (b.feature >= 0) {
        const uint32_t f = uint32_t(b.feature);
        for (uint32_t k = 0; k < counts[f]; ++k)
          if (std::memcmp(&cuts[size_t(f) * stride + k], &b.threshold, 4) == 0) d.split_bin = int32_t(k);
      }
      d.default_left = b.default_left;
      d.left_weight = b.left_weight;
      d.right_weight = b.right_weight;
      d.parent_weight = b.parent_weight;
      d.left_h = b.left_h;
      d.right_h = b.right_h;
      d.total_g = b.total_g;
      d.total_h = b.total_h;
      // Left zero: the grower derives them from the child sums.
      d.applied_parent_weight = 0.0f;
      d.applied_parent_hessian = 0.0f;
      d.left_g = b.left_sum_g;
      d.left_hs = b.left_sum_h;
      d.right_g = b.right_sum_g;
      d.right_hs = b.right_sum_h;
    }
  }

  void partition(const std::vector<xgbb::PartitionItem>& items, std::vector<uint32_t>& left) override {
    left.assign(items.size(), 0);
    std::vector<uint32_t> right;
    for (size_t i = 0; i < items.size(); ++i) {
      const xgbb::PartitionItem& it = items[i];
      uint32_t* seg = order.data() + it.begin;
      uint32_t nl = 0;
      right.clear();
      for (uint32_t j = 0; j < it.count; ++j) {
        const uint32_t b = bins[size_t(seg[j]) * cols + uint32_t(it.feature)];
        const bool go_left = b == ORC_MISSING ? it.default_left != 0 : int32_t(b) <= it.split_bin;
        if (go_left) seg[nl++] = seg[j];
        else right.push_back(seg[j]);
      }
      std::copy(right.begin(), right.end(), seg + nl);
      left[i] = nl;
    }
  }
};

}  // namespace

extern "C" int grower_harness(const uint32_t* bins, uint32_t rows, uint32_t cols, const int64_t* q,
                              const float* scale, const float* cuts, uint32_t stride, const uint32_t* counts,
                              const float* minima, const orc_tree_params* tp, uint32_t lossguide,
                              uint32_t max_leaves, xgbb::DevNode* nodes, uint32_t capacity) {
  try {
    OracleBackend be;
    be.bins = bins;
    be.rows = rows;
    be.cols = cols;
    be.stride = stride;
    be.q = q;
    be.scale = scale;
    be.cuts = cuts;
    be.counts = counts;
    be.minima = minima;
    be.tp = *tp;
    be.order.resize(rows);
    for (uint32_t r = 0; r < rows; ++r) be.order[r] = r;
    xgbb::GrowerParams p;
    p.tree = xgbb::TreeParams{tp->max_depth, tp->eta, tp->reg_lambda, tp->reg_alpha, tp->min_child_weight,
                              tp->max_delta_step, tp->min_split_loss};
    p.lossguide = lossguide != 0;
    p.max_leaves = max_leaves;
    p.scale_g = scale[0];
    p.scale_h = scale[1];
    const std::vector<xgbb::DevNode> out = xgbb::grow_tree_host_driven(be, rows, p);
    if (out.size() > capacity) return -1;
    std::copy(out.begin(), out.end(), nodes);
    return int(out.size());
  } catch (const std::exception&) {
    return -2;
  }
}
