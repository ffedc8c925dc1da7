// Reference cross-check harness: the reference's own serial Metal kernel
// functions, compiled for the host through refshim/metal_shim.hpp, behind a
// plain C ABI. TEST INFRASTRUCTURE ONLY: it pins the C oracle (oracle.c)
// against the reference code it restates. Nothing in the product links it.
//
// The reference sources are included from their own location (the kernels/ directory named by
// the REF variable of oracle/Makefile); nothing is copied into this repository. Only
// data-movement glue lives here (buffer set-up, run detection, the level loop,
// row bookkeeping); every numeric decision is made by a reference function:
//   quantize                 kernels/boost.metal:461-499
//   sketch_summarize_ordered kernels/quantile.metal.h:216-240
//   sketch_reduce_serial     kernels/quantile.metal.h:317-352
//   sketch_cuts              kernels/quantile.metal.h:354-411
//   mass_atomic_bits         kernels/objectives.metal.h:59-67
//   quantize_gradients       kernels/boost.metal:605-657
//   evaluate_splits          kernels/boost.metal:921-1020
//   select_splits            kernels/boost.metal:1245-1265
//   tree_driver_apply        kernels/tree_driver.metal.h:28-94
//   split_left               kernels/boost.metal:1325-1329
//   predict                  kernels/boost.metal:1738-1765
#include <thread>  // before the shim, whose `thread` address-space macro it must not see
using host_thread = std::thread;

#include "metal_shim.hpp"
#include "metalgb/shared.h"
using namespace metalgb;
#include "boost.metal"

#include <cstdio>
#include <vector>

namespace {

// Host-side work sizing from src/quantile.cpp:11-20 (not a kernel; restated).
u32 sketch_budget(u32 bins, u32 count) {
  if (!count) return 1;
  double epsilon = 1.0 / std::min(bins, count);
  for (u32 level = 1; level < 32; ++level) {
    auto limit = std::min<std::uint64_t>(
        count, static_cast<std::uint64_t>(std::ceil(level / (epsilon / 2.0))) + 1);
    if ((std::uint64_t{1} << level) * limit >= count) return static_cast<u32>(limit);
  }
  return count;
}

u32 round_up(u32 v, u32 m) { return (v + m - 1) / m * m; }

// Runs body(i) for i in [0, n) on every host thread. The reference runs these
// loops as independent GPU threads (one per (node, feature) or per row tile),
// so their order does not matter; the bench's CPU arm uses all host cores.
template <class F>
void parallel_for(u32 n, F body) {
  u32 threads = std::max(1u, host_thread::hardware_concurrency());
  threads = std::min(threads, std::max(1u, n));
  if (threads == 1) {
    for (u32 i = 0; i < n; ++i) body(i);
    return;
  }
  std::vector<host_thread> pool;
  for (u32 t = 0; t < threads; ++t)
    pool.emplace_back([=, &body] {
      for (u32 i = t; i < n; i += threads) body(i);
    });
  for (auto& th : pool) th.join();
}

// Cuts for one numeric feature, following Matrix::make_quantile_cuts
// (src/quantile.cpp:22-213) with the serial summary, reduction and cut
// kernels. Input runs follow sketch_input_blocks/offsets/compact/runs
// (kernels/quantile.metal.h:19-140): valid entries are non-NaN with a nonzero
// weight, consecutive fp32_equal values form one run whose value is its first
// entry and whose weight is its length (unit weights, capped at 2^24) or the
// sketch_add sum of its weights in row order.
void feature_cuts(const float* X, u32 rows, u32 cols, u32 f, const float* weights, u32 max_bin,
                  u32 hist_bins, float* cuts, u32* count, float* minimum) {
  bool unit = weights == nullptr;
  std::vector<float2> queue;
  u32 elements = 0, nonmissing = 0;
  bool have_previous = false;
  float previous = 0;
  for (u32 r = 0; r < rows; ++r) {
    float v = X[std::size_t(r) * cols + f];
    float w = unit ? 1.0f : weights[r];
    nonmissing += !isnan(v);
    bool valid = !isnan(v) && (as_type<uint>(w) & 0x7fffffffu) != 0;
    if (!valid) continue;
    ++elements;
    if (!have_previous || !fp32_equal(v, previous)) {
      queue.push_back(float2(v, unit ? 1.0f : w));
    } else if (unit) {
      queue.back().y = float(std::min<u32>(u32(queue.back().y) + 1, 1u << 24));
    } else {
      queue.back().y = sketch_add(queue.back().y, w);
    }
    have_previous = true;
    previous = v;
  }
  u32 runs = u32(queue.size());
  u32 limit = sketch_budget(max_bin, nonmissing);
  u32 budget = sketch_budget(max_bin, elements);
  std::vector<SketchBatch> batches;
  std::uint64_t capacity = std::uint64_t{2} * limit;
  std::size_t slots = 0;
  for (std::uint64_t begin = 0; begin < runs; begin += capacity) {
    u32 size = u32(std::min<std::uint64_t>(capacity, runs - begin));
    u32 stride = round_up(size, 256);
    u32 exact = unit && elements <= (1u << 24);
    batches.push_back({begin, slots, size, stride, limit, exact});
    slots += stride;
  }
  u32 nbatch = u32(batches.size());
  std::vector<float2> sorted(std::max<std::size_t>(slots, 1));
  std::vector<float4> summaries(std::max<std::size_t>(slots, 1));
  std::vector<u32> sizes(std::max<u32>(nbatch, 1));
  for (u32 b = 0; b < nbatch; ++b) {
    auto& t = batches[b];
    float2* dst = sorted.data() + t.offset;
    for (u32 i = 0; i < t.size; ++i) dst[i] = queue[t.input + i];
    // Any ascending order works here: entries that compare equal either are
    // interchangeable or trigger the reference's own order repair.
    std::stable_sort(dst, dst + t.size, [](float2 a, float2 b) { return fp32_less(a.x, b.x); });
    sizes[b] = sketch_summarize_ordered(dst, t, summaries.data() + t.offset, queue.data());
  }
  u32 levels = u32(std::bit_width(std::max(1u, nbatch))) + 1;
  SketchFeature feature{0, 0, limit, budget, 0, nbatch, levels, 0};
  std::vector<float4> level_store(std::size_t(limit) * levels);
  std::vector<float4> workspace(std::size_t(limit) * 4);
  SketchStats stats{nonmissing, elements, runs, 0};
  SketchParams sp{nbatch, 0, 1, 0};
  sketch_reduce_serial<>(summaries.data(), sizes.data(), batches.data(), &feature, level_store.data(),
                         workspace.data(), &stats, sp, 0u);
  MatrixParams mp{rows, 1, round_up(rows, 256), hist_bins, max_bin};
  uchar categorical = 0;
  sketch_cuts<>(workspace.data(), &feature, &stats, cuts, count, minimum, &categorical, mp, 0u);
}

}  // namespace

extern "C" {

// Returns the cut stride (histogram_bins = max(1, min(max_bin, rows)),
// src/data.cpp:1232) and fills cuts[f*stride + i], counts[f], minima[f].
// `cuts` must hold cols * min(max_bin, max(rows,1)) floats.
int xgbref_sketch_cuts(const float* X, uint32_t rows, uint32_t cols, const float* weights,
                       uint32_t max_bin, float* cuts, uint32_t* counts, float* minima) {
  u32 hist_bins = std::max(1u, std::min(max_bin, rows));
  // Features are independent (one summary per feature): one task each.
  parallel_for(cols, [&](u32 f) {
    std::fill(cuts + std::size_t(f) * hist_bins, cuts + std::size_t(f + 1) * hist_bins, 0.0f);
    feature_cuts(X, rows, cols, f, weights, max_bin, hist_bins, cuts + std::size_t(f) * hist_bins,
                 counts + f, minima + f);
  });
  return int(hist_bins);
}

// Row-major bin indices, 0xffffffff for missing, via the quantize kernel.
void xgbref_quantize(const float* X, uint32_t rows, uint32_t cols, const float* cuts,
                     uint32_t cut_stride, const uint32_t* counts, uint32_t* bins_out) {
  MatrixParams p{rows, cols, round_up(rows, 256), cut_stride, cut_stride};
  std::vector<uchar> categorical(cols, 0);
  bool wide = cut_stride > 65534;
  std::vector<u32> storage(std::size_t(rows) * cols);
  auto* bins16 = reinterpret_cast<ushort*>(storage.data());
  atomic_uint missing = 0;
  for (u32 r = 0; r < rows; ++r)
    for (u32 c = 0; c < cols; ++c)
      quantize<>(X, cuts, counts, bins16, categorical.data(), &missing, p, uint2(r, c));
  for (u32 r = 0; r < rows; ++r)
    for (u32 c = 0; c < cols; ++c) {
      std::size_t fm = std::size_t(c) * rows + r;
      bins_out[std::size_t(r) * cols + c] =
          wide ? storage[fm] : load_bin(bins16, fm, cut_stride);
    }
}

// The reference's own feature-major uint16 bins (bins[f * rows + row],
// 0xffff = missing; Matrix::quantize, src/data.cpp:1210-1306) via the
// quantize kernel, rows in parallel. Only for cut strides up to 65534.
void xgbref_quantize_fm(const float* X, uint32_t rows, uint32_t cols, const float* cuts,
                        uint32_t cut_stride, const uint32_t* counts, uint16_t* fm_out) {
  MatrixParams p{rows, cols, rows, cut_stride, cut_stride};
  std::vector<uchar> categorical(cols, 0);
  atomic_uint missing = 0;
  const u32 chunk = 4096;
  parallel_for((rows + chunk - 1) / chunk, [&](u32 t) {
    for (u32 r = t * chunk; r < std::min(rows, (t + 1) * chunk); ++r)
      for (u32 c = 0; c < cols; ++c)
        quantize<>(X, cuts, counts, reinterpret_cast<ushort*>(fm_out), categorical.data(), &missing, p,
                   uint2(r, c));
  });
}

// Gradient pairs [rows][groups] from the reference's gradients kernel
// (kernels/boost.metal:553-601), rows in parallel.
void xgbref_gradients(int objective, const float* margins, const float* labels, const float* weights,
                      uint32_t rows, uint32_t groups, float scale_pos_weight, float* pairs) {
  GradientParams p{rows, groups, 1, uint(objective), weights ? 1u : 0u, 0, 0, 0, scale_pos_weight, 1, 0, 0};
  const u32 chunk = 4096;
  parallel_for((rows + chunk - 1) / chunk, [&](u32 t) {
    for (u32 r = t * chunk; r < std::min(rows, (t + 1) * chunk); ++r)
      for (u32 g = 0; g < groups; ++g)
        gradients<>(margins, labels, weights, reinterpret_cast<Pair*>(pairs), p, uint2(r, g));
  });
}

// Per-group power-of-two scales (float pairs: g-scale, h-scale). The exact
// magnitude sums use the reference's mass_atomic_bits; the exponent rule is
// gradient_scales (kernels/gradient_quantization.metal.h:49-63), restated
// because that kernel's reduction is cooperative.
void xgbref_gradient_scales(const float* pairs, uint32_t rows, uint32_t groups, float* scales) {
  for (u32 g = 0; g < groups; ++g) {
    for (u32 part = 0; part < 2; ++part) {
      uint mass[kObjectiveMassWords] = {};
      for (u32 r = 0; r < rows; ++r) {
        float v = pairs[(std::size_t(r) * groups + g) * 2 + part];
        mass_atomic_bits(mass, as_type<uint>(v) & 0x7fffffffu);
      }
      int exponent = 0;
      for (uint word = kObjectiveMassWords; word-- > 0;)
        if (mass[word]) {
          exponent = max(0, int(word * 32 + 32 - clz(mass[word])) - 149);
          break;
        }
      scales[g * 2 + part] = as_type<float>(uint(62 - exponent + 127) << 23);
    }
  }
}

void xgbref_quantize_gradients(const float* pairs, uint32_t rows, uint32_t groups,
                               const float* scales, int64_t* out) {
  // scales buffer layout of the kernel: float2[groups] then GradCert[groups].
  std::vector<uint> buffer(std::size_t(groups) * (2 + 8), 0);
  std::memcpy(buffer.data(), scales, groups * 8);
  GradientParams p{rows, groups, 1, 0, 0, 0, 0, 0, 1, 1, 0, 0};
  for (u32 g = 0; g < groups; ++g)
    for (u32 r = 0; r < rows; ++r)
      quantize_gradients<>(reinterpret_cast<const Pair*>(pairs),
                           reinterpret_cast<const float2*>(buffer.data()),
                           reinterpret_cast<long2*>(out), p, uint2(r / 256, g), r % 256);
}

// Split candidates, one Split record (96 bytes, include/metalgb/shared.h:124)
// per (node, feature). hist is int64 (g, h) pairs [nodes][cols][bins + 1].
void xgbref_evaluate_splits(const int64_t* hist, uint32_t nodes, uint32_t cols, uint32_t bins,
                            const float* scale, const float* cuts, const uint32_t* counts,
                            const float* minima, float reg_lambda, float reg_alpha,
                            float min_child_weight, float max_delta_step, uint32_t use_parent_sums,
                            const int64_t* node_sums, void* out) {
  std::vector<int> monotone(cols, 0);
  std::vector<float2> bounds(std::max<u32>(nodes, 1), float2(-INFINITY, INFINITY));
  std::vector<uchar> allowed(std::max<std::size_t>(std::size_t(nodes) * cols, 1), 1);
  std::vector<uchar> categorical(cols, 0);
  float2 dummy2[1] = {float2(0)};
  uint dummy_u[1] = {0};
  uint dummy_cat[1] = {0};
  SplitParams p{};
  p.nodes = nodes; p.cols = cols; p.bins = bins; p.group = 0;
  p.reg_lambda = reg_lambda; p.reg_alpha = reg_alpha;
  p.min_child_weight = min_child_weight; p.max_delta_step = max_delta_step;
  p.max_cat_to_onehot = 4; p.max_cat_threshold = 64; p.sort_stride = 1; p.has_categorical = 0;
  p.use_parent_sums = use_parent_sums;
  float2 s(scale[0], scale[1]);
  parallel_for(nodes * cols, [&](u32 i) {
    const u32 n = i / cols, f = i % cols;
    float2 local_dummy[1] = {float2(0)};
    uint local_u[1] = {0}, local_cat[1] = {0};
    evaluate_splits<>(reinterpret_cast<const uint*>(hist), &s, cuts, counts, minima, monotone.data(),
                      bounds.data(), allowed.data(), reinterpret_cast<Split*>(out), categorical.data(),
                      local_dummy, local_u, local_cat, reinterpret_cast<const long2*>(node_sums), p,
                      uint2(f, n));
  });
  (void)dummy2;
  (void)dummy_u;
  (void)dummy_cat;
}

void xgbref_select_splits(const void* candidates, uint32_t nodes, uint32_t cols, const float* scale,
                          float reg_lambda, float reg_alpha, float max_delta_step, void* best) {
  SplitParams p{};
  p.nodes = nodes; p.cols = cols; p.reg_lambda = reg_lambda; p.reg_alpha = reg_alpha;
  p.max_delta_step = max_delta_step;
  std::vector<float2> bounds(std::max<u32>(nodes, 1), float2(-INFINITY, INFINITY));
  float2 s(scale[0], scale[1]);
  for (u32 n = 0; n < nodes; ++n)
    select_splits<>(reinterpret_cast<const Split*>(candidates), reinterpret_cast<Split*>(best), &s,
                    bounds.data(), p, n);
}

// Output node record of xgbref_grow_tree (mirrors metalgb::Node plus the
// split's bin index, which the bin-form partition uses).
struct RefNode {
  int32_t left, right, feature, parent;
  float threshold, leaf, cover, gain;
  uint32_t default_left, split_bin;
};

// One depthwise tree from quantised gradients q (int64 pairs per row) and
// their scale, using the reference's split evaluation, selection and tree
// driver. bins: row-major, 0xffffffff = missing. Writes at most node_capacity
// RefNode records and, per row, the leaf value the tree assigns (the margin
// increment), traversed by the predict kernel over bin lower bounds as the
// reference's training-margin update does (src/learner.cpp:933-976). Returns
// the node count, or -1 on a driver error.
int xgbref_grow_tree(const uint32_t* bins, uint32_t rows, uint32_t cols, const int64_t* q,
                     const float* scale, const float* cuts, uint32_t cut_stride,
                     const uint32_t* counts, const float* minima, uint32_t max_depth, float eta,
                     float reg_lambda, float reg_alpha, float min_child_weight, float max_delta_step,
                     float min_split_loss, RefNode* out_nodes, uint32_t node_capacity,
                     float* row_leaf) {
  const u32 B = cut_stride;
  TreeDriverParams tp{};
  tp.split.cols = cols; tp.split.bins = B;
  tp.split.reg_lambda = reg_lambda; tp.split.reg_alpha = reg_alpha;
  tp.split.min_child_weight = min_child_weight; tp.split.max_delta_step = max_delta_step;
  tp.partition.rows = rows;
  tp.max_depth = max_depth;
  u32 capacity = (max_depth >= 31) ? 0xffffffffu : ((2u << max_depth) - 1);
  tp.node_capacity = capacity;
  tp.min_gain = min_split_loss;
  TreeDriverState state{1, 1, 0, 0};
  std::vector<Split> history(capacity);
  std::vector<uint> flags(capacity, 0);
  std::vector<uint> ids{0};
  std::vector<IntPair> sums{IntPair{0, 0}};
  std::vector<std::vector<u32>> segments(1);
  segments[0].resize(rows);
  for (u32 r = 0; r < rows; ++r) segments[0][r] = r;
  // Decoded bin lower bounds (quantile_values, kernels/boost.metal:503-531).
  auto decoded = [&](u32 r, u32 f) -> float {
    u32 b = bins[std::size_t(r) * cols + f];
    if (b == 0xffffffffu) return NAN;
    return b ? cuts[std::size_t(f) * B + b - 1] : -INFINITY;
  };
  for (u32 depth = 0; depth < max_depth && state.frontier_count; ++depth) {
    u32 nodes = state.frontier_count;
    std::vector<int64_t> hist(std::size_t(nodes) * cols * (B + 1) * 2, 0);
    std::vector<u32> seg_count(nodes), seg_offset(nodes);
    u32 offset = 0;
    for (u32 s = 0; s < nodes; ++s) {
      seg_count[s] = u32(segments[s].size());
      seg_offset[s] = offset;
      offset += seg_count[s];
    }
    // Exact int64 sums, one feature per task.
    parallel_for(cols, [&](u32 f) {
      for (u32 s = 0; s < nodes; ++s)
        for (u32 r : segments[s]) {
          u32 b = bins[std::size_t(r) * cols + f];
          std::size_t cell = ((std::size_t(s) * cols + f) * (B + 1) + (b == 0xffffffffu ? B : b)) * 2;
          hist[cell] = int64_t(uint64_t(hist[cell]) + uint64_t(q[std::size_t(r) * 2]));
          hist[cell + 1] = int64_t(uint64_t(hist[cell + 1]) + uint64_t(q[std::size_t(r) * 2 + 1]));
        }
    });
    std::vector<Split> candidates(std::size_t(nodes) * cols), best(nodes);
    xgbref_evaluate_splits(hist.data(), nodes, cols, B, scale, cuts, counts, minima, reg_lambda,
                           reg_alpha, min_child_weight, max_delta_step, depth != 0,
                           reinterpret_cast<const int64_t*>(sums.data()), candidates.data());
    xgbref_select_splits(candidates.data(), nodes, cols, scale, reg_lambda, reg_alpha,
                         max_delta_step, best.data());
    std::vector<uint> next_ids(2 * nodes), selected_counts(nodes), selected_offsets(nodes),
        parent_hist(nodes);
    std::vector<IntPair> next_sums(2 * nodes);
    std::vector<Split> selected(nodes);
    std::vector<int2> children(nodes);
    tree_driver_apply<>(&state, ids.data(), best.data(), seg_count.data(), seg_offset.data(),
                        history.data(), flags.data(), next_ids.data(), next_sums.data(),
                        selected.data(), selected_counts.data(), selected_offsets.data(),
                        children.data(), parent_hist.data(), tp, 0u);
    if (state.error) return -1;
    u32 next = state.frontier_count;
    std::vector<std::vector<u32>> next_segments(next);
    for (u32 s = 0; s < next / 2; ++s) {
      u32 slot = parent_hist[s];
      const Split& sp = selected[s];
      for (u32 r : segments[slot]) {
        bool left = split_left(decoded(r, u32(sp.feature)), sp.threshold, sp.default_left, 0, 0, 0,
                               nullptr);
        next_segments[2 * s + (left ? 0 : 1)].push_back(r);
      }
    }
    ids.assign(next_ids.begin(), next_ids.begin() + next);
    sums.assign(next_sums.begin(), next_sums.begin() + next);
    segments = std::move(next_segments);
  }
  // Host replay (src/tree.cpp:1663-1717), scalar numeric leaves only.
  u32 count = state.node_count;
  if (count > node_capacity) return -1;
  std::vector<Node> tree(1);
  std::vector<u32> split_bin(1, 0);
  for (u32 id = 0; id < count; ++id) {
    if (id >= tree.size()) return -1;
    uint status = flags[id];
    if (!(status & kTreeDriverEvaluated)) continue;
    const Split& split = history[id];
    tree[id].cover = split.total_h;
    if (!id) tree[0].leaf = split.parent_weight * eta;
    if (!(status & kTreeDriverExpanded)) continue;
    int left = int(tree.size());
    tree[id].left = left; tree[id].right = left + 1; tree[id].feature = split.feature;
    tree[id].threshold = split.threshold; tree[id].default_left = split.default_left;
    tree[id].gain = split.gain;
    tree[id].cover = split.applied_parent_hessian;
    // Bin index k with left iff bin <= k; k = -1 sends every present row right.
    u32 f = u32(split.feature);
    int k = -1;
    for (u32 b = 0; b < counts[f]; ++b)
      if (as_type<uint>(cuts[std::size_t(f) * B + b]) == as_type<uint>(split.threshold)) k = int(b);
    split_bin[id] = u32(k);
    Node l, r;
    l.parent = int(id); r.parent = int(id);
    l.leaf = split.left_weight * eta; l.cover = split.left_h;
    r.leaf = split.right_weight * eta; r.cover = split.right_h;
    tree.push_back(l); tree.push_back(r);
    split_bin.push_back(0); split_bin.push_back(0);
  }
  if (tree.size() != count) return -1;
  for (u32 i = 0; i < count; ++i) {
    const Node& n = tree[i];
    out_nodes[i] = RefNode{n.left, n.right, n.feature, n.parent, n.threshold, n.leaf, n.cover, n.gain,
                           n.default_left, split_bin[i]};
  }
  // Margin increments through the predict kernel: base margin 0, one tree.
  if (row_leaf) {
    TreeMeta meta{0, count, 0, 0, 0, 1, 0};
    std::vector<float> row(cols);
    float zero = 0, base = 0;
    uint no_categories = 0;
    PredictParams pp{1, cols, 1, 1, 0, 1, 0, 0, 1, 1, 0, 0, 0};
    for (u32 r = 0; r < rows; ++r) {
      for (u32 f = 0; f < cols; ++f) row[f] = decoded(r, f);
      predict<>(row.data(), tree.data(), &meta, &base, &zero, row_leaf + r, &no_categories, nullptr,
                nullptr, nullptr, pp, uint2(0, 0));
    }
  }
  return int(count);
}

// The same tree over the reference's feature-major uint16 bins (as
// xgbref_quantize_fm writes them), built the way the reference's level loop
// builds it: at each level only the smaller child of every node pair gets a
// histogram (a tie builds the left one; plan_histograms,
// kernels/boost.metal:661-698) and its sibling is the parent minus it
// (subtract_histograms, :780-794). Histograms are built per (node, feature)
// task over all host threads; partitions per node pair and the margin
// increments per row block run in parallel as well. Splits, selection, the
// driver and prediction are the reference's functions as in xgbref_grow_tree.
int xgbref_grow_tree_fm(const uint16_t* fm, uint32_t rows, uint32_t cols, const int64_t* q,
                        const float* scale, const float* cuts, uint32_t cut_stride,
                        const uint32_t* counts, const float* minima, uint32_t max_depth, float eta,
                        float reg_lambda, float reg_alpha, float min_child_weight, float max_delta_step,
                        float min_split_loss, RefNode* out_nodes, uint32_t node_capacity,
                        float* row_leaf) {
  const u32 B = cut_stride;
  if (B > 65534) return -1;
  const std::size_t per_node = std::size_t(cols) * (B + 1) * 2;
  TreeDriverParams tp{};
  tp.split.cols = cols; tp.split.bins = B;
  tp.split.reg_lambda = reg_lambda; tp.split.reg_alpha = reg_alpha;
  tp.split.min_child_weight = min_child_weight; tp.split.max_delta_step = max_delta_step;
  tp.partition.rows = rows;
  tp.max_depth = max_depth;
  u32 capacity = (max_depth >= 31) ? 0xffffffffu : ((2u << max_depth) - 1);
  tp.node_capacity = capacity;
  tp.min_gain = min_split_loss;
  TreeDriverState state{1, 1, 0, 0};
  std::vector<Split> history(capacity);
  std::vector<uint> flags(capacity, 0);
  std::vector<uint> ids{0};
  std::vector<IntPair> sums{IntPair{0, 0}};
  std::vector<std::vector<u32>> segments(1);
  segments[0].resize(rows);
  for (u32 r = 0; r < rows; ++r) segments[0][r] = r;
  auto bin_of = [&](u32 r, u32 f) -> u32 { return load_bin(fm, std::size_t(f) * rows + r, B); };
  auto decoded = [&](u32 r, u32 f) -> float {
    u32 b = bin_of(r, f);
    if (b == 0xffffffffu) return NAN;
    return b ? cuts[std::size_t(f) * B + b - 1] : -INFINITY;
  };
  std::vector<int64_t> prev;     // the previous level's histograms [nodes][cols][B + 1][2]
  std::vector<uint> parent_hist;  // previous-level slot of each pair's parent
  for (u32 depth = 0; depth < max_depth && state.frontier_count; ++depth) {
    u32 nodes = state.frontier_count;
    std::vector<int64_t> hist(std::size_t(nodes) * per_node, 0);
    std::vector<u32> seg_count(nodes), seg_offset(nodes), built;
    u32 offset = 0;
    for (u32 s = 0; s < nodes; ++s) {
      seg_count[s] = u32(segments[s].size());
      seg_offset[s] = offset;
      offset += seg_count[s];
    }
    if (depth == 0) built.push_back(0);
    else
      for (u32 s = 0; s + 1 < nodes; s += 2) built.push_back(seg_count[s] <= seg_count[s + 1] ? s : s + 1);
    parallel_for(u32(built.size()) * cols, [&](u32 i) {
      const u32 s = built[i / cols], f = i % cols;
      int64_t* h = hist.data() + std::size_t(s) * per_node + std::size_t(f) * (B + 1) * 2;
      const uint16_t* col = fm + std::size_t(f) * rows;
      for (u32 r : segments[s]) {
        u32 b = col[r];
        b = b == 65535 ? B : b;
        h[2 * b] = int64_t(uint64_t(h[2 * b]) + uint64_t(q[std::size_t(r) * 2]));
        h[2 * b + 1] = int64_t(uint64_t(h[2 * b + 1]) + uint64_t(q[std::size_t(r) * 2 + 1]));
      }
    });
    if (depth) {
      parallel_for(u32(built.size()) * cols, [&](u32 i) {
        const u32 pair = i / cols, f = i % cols, small = built[pair], other = small ^ 1u;
        const int64_t* par = prev.data() + std::size_t(parent_hist[pair]) * per_node + std::size_t(f) * (B + 1) * 2;
        const int64_t* got = hist.data() + std::size_t(small) * per_node + std::size_t(f) * (B + 1) * 2;
        int64_t* out = hist.data() + std::size_t(other) * per_node + std::size_t(f) * (B + 1) * 2;
        for (u32 k = 0; k < (B + 1) * 2; ++k) out[k] = int64_t(uint64_t(par[k]) - uint64_t(got[k]));
      });
    }
    std::vector<Split> candidates(std::size_t(nodes) * cols), best(nodes);
    xgbref_evaluate_splits(hist.data(), nodes, cols, B, scale, cuts, counts, minima, reg_lambda,
                           reg_alpha, min_child_weight, max_delta_step, depth != 0,
                           reinterpret_cast<const int64_t*>(sums.data()), candidates.data());
    xgbref_select_splits(candidates.data(), nodes, cols, scale, reg_lambda, reg_alpha,
                         max_delta_step, best.data());
    std::vector<uint> next_ids(2 * nodes), selected_counts(nodes), selected_offsets(nodes);
    parent_hist.assign(nodes, 0);
    std::vector<IntPair> next_sums(2 * nodes);
    std::vector<Split> selected(nodes);
    std::vector<int2> children(nodes);
    tree_driver_apply<>(&state, ids.data(), best.data(), seg_count.data(), seg_offset.data(),
                        history.data(), flags.data(), next_ids.data(), next_sums.data(),
                        selected.data(), selected_counts.data(), selected_offsets.data(),
                        children.data(), parent_hist.data(), tp, 0u);
    if (state.error) return -1;
    u32 next = state.frontier_count;
    std::vector<std::vector<u32>> next_segments(next);
    parallel_for(next / 2, [&](u32 s) {
      u32 slot = parent_hist[s];
      const Split& sp = selected[s];
      for (u32 r : segments[slot]) {
        bool left = split_left(decoded(r, u32(sp.feature)), sp.threshold, sp.default_left, 0, 0, 0,
                               nullptr);
        next_segments[2 * s + (left ? 0 : 1)].push_back(r);
      }
    });
    ids.assign(next_ids.begin(), next_ids.begin() + next);
    sums.assign(next_sums.begin(), next_sums.begin() + next);
    segments = std::move(next_segments);
    prev = std::move(hist);
  }
  // Host replay (src/tree.cpp:1663-1717), scalar numeric leaves only.
  u32 count = state.node_count;
  if (count > node_capacity) return -1;
  std::vector<Node> tree(1);
  std::vector<u32> split_bin(1, 0);
  for (u32 id = 0; id < count; ++id) {
    if (id >= tree.size()) return -1;
    uint status = flags[id];
    if (!(status & kTreeDriverEvaluated)) continue;
    const Split& split = history[id];
    tree[id].cover = split.total_h;
    if (!id) tree[0].leaf = split.parent_weight * eta;
    if (!(status & kTreeDriverExpanded)) continue;
    int left = int(tree.size());
    tree[id].left = left; tree[id].right = left + 1; tree[id].feature = split.feature;
    tree[id].threshold = split.threshold; tree[id].default_left = split.default_left;
    tree[id].gain = split.gain;
    tree[id].cover = split.applied_parent_hessian;
    u32 f = u32(split.feature);
    int k = -1;
    for (u32 b = 0; b < counts[f]; ++b)
      if (as_type<uint>(cuts[std::size_t(f) * B + b]) == as_type<uint>(split.threshold)) k = int(b);
    split_bin[id] = u32(k);
    Node l, r;
    l.parent = int(id); r.parent = int(id);
    l.leaf = split.left_weight * eta; l.cover = split.left_h;
    r.leaf = split.right_weight * eta; r.cover = split.right_h;
    tree.push_back(l); tree.push_back(r);
    split_bin.push_back(0); split_bin.push_back(0);
  }
  if (tree.size() != count) return -1;
  for (u32 i = 0; i < count; ++i) {
    const Node& n = tree[i];
    out_nodes[i] = RefNode{n.left, n.right, n.feature, n.parent, n.threshold, n.leaf, n.cover, n.gain,
                           n.default_left, split_bin[i]};
  }
  if (row_leaf) {
    TreeMeta meta{0, count, 0, 0, 0, 1, 0};
    PredictParams pp{1, cols, 1, 1, 0, 1, 0, 0, 1, 1, 0, 0, 0};
    const u32 chunk = 4096;
    parallel_for((rows + chunk - 1) / chunk, [&](u32 t) {
      std::vector<float> row(cols);
      float zero = 0, base = 0;
      uint no_categories = 0;
      for (u32 r = t * chunk; r < std::min(rows, (t + 1) * chunk); ++r) {
        for (u32 f = 0; f < cols; ++f) row[f] = decoded(r, f);
        predict<>(row.data(), tree.data(), &meta, &base, &zero, row_leaf + r, &no_categories, nullptr,
                  nullptr, nullptr, pp, uint2(0, 0));
      }
    });
  }
  return int(count);
}

}  // extern "C"
