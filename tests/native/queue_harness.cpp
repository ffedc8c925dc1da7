// Test harness: host-driven growth (csrc/grower.cpp) with the GPU backend's
// block functions (csrc/queue_par.h: node histograms, row partitions, margin
// walk) run on the CPU by the serial executor, and split evaluation by the
// oracle on the histograms those functions build. Each histogram is also
// compared with the oracle's histogram of the same rows. Test infrastructure
// only.
#include <algorithm>
#include <cstring>
#include <vector>

#include "grower.h"
#include "queue_par.h"
extern "C" {
#include "oracle.h"
}

using namespace xgbb;

namespace {

struct EmuBackend : GrowerBackend {
  Ellpack e;
  const float2* pairs;
  float2 sc;
  const uint32_t* bins;  // oracle bins [rows][cols]
  const int64_t* q;      // oracle quantised gradients [rows][2]
  const float* scale;
  const float* cuts;
  const uint32_t* counts;
  const float* minima;
  orc_tree_params tp;
  std::vector<uint32_t> order, scratch;
  uint64_t hist_mismatches = 0, evaluations = 0;
  // Sparse rows (used when `sparse`): row_ptr [rows + 1], entries.
  bool sparse = false;
  std::vector<unsigned long long> row_ptr;
  std::vector<uint32_t> entries;

  template <class CodeT>
  void make_sparse_rows() {
    row_ptr.assign(size_t(e.rows) + 1, 0);
    for (uint32_t r = 0; r < e.rows; ++r) row_ptr[r + 1] = row_ptr[r] + csr_row_count<CodeT>(e, r);
    entries.assign(std::max<size_t>(row_ptr[e.rows], 1), 0);
    for (uint32_t r = 0; r < e.rows; ++r) csr_row_fill<CodeT>(e, r, row_ptr[r], entries.data());
  }

  void build_sparse(const std::vector<Segment>& nodes, std::vector<longlong2>& built) {
    const uint32_t n = uint32_t(nodes.size()), C = e.cols, B1 = e.bins + 1;
    std::vector<uint32_t> seg(2 * n), tiles(n + 1);
    uint32_t total = 0;
    for (uint32_t s = 0; s < n; ++s) {
      seg[2 * s] = nodes[s].begin;
      seg[2 * s + 1] = nodes[s].count;
      tiles[s] = total;
      total += (nodes[s].count + kQueueTileRows - 1) / kQueueTileRows;
    }
    tiles[n] = total;
    built.assign(size_t(C) * n * B1, longlong2{0, 0});
    std::vector<unsigned long long> totals(2 * size_t(n), 0), tot(2);
    HostExec ex;
    for (uint32_t t = 0; t < total; ++t)
      queue_hist_csr_tile(ex, e.bins, C, row_ptr.data(), entries.data(), order.data(), pairs, sc, seg.data(),
                          tiles.data(), n, t, tot.data(), totals.data(), built.data());
    for (uint32_t f = 0; f < C; ++f)
      for (uint32_t s = 0; s < n; ++s) queue_fill_missing(e.bins, n, totals.data(), built.data(), f, s);
  }

  template <class CodeT>
  void build(const std::vector<Segment>& nodes, std::vector<longlong2>& built) {
    const uint32_t n = uint32_t(nodes.size()), C = e.cols, B1 = e.bins + 1;
    std::vector<uint32_t> seg(2 * n), tiles(n + 1);
    uint32_t total = 0;
    for (uint32_t s = 0; s < n; ++s) {
      seg[2 * s] = nodes[s].begin;
      seg[2 * s + 1] = nodes[s].count;
      tiles[s] = total;
      total += (nodes[s].count + kQueueTileRows - 1) / kQueueTileRows;
    }
    tiles[n] = total;
    built.assign(size_t(C) * n * B1, longlong2{0, 0});
    std::vector<unsigned long long> sg(kQueueFeatures * kQueueBins), sh(kQueueFeatures * kQueueBins);
    HostExec ex;
    const uint64_t items = uint64_t(total) * ((C + kQueueFeatures - 1) / kQueueFeatures);
    for (uint64_t item = 0; item < items; ++item)
      queue_hist_item<CodeT>(ex, e, order.data(), pairs, sc, seg.data(), tiles.data(), n, item, sg.data(), sh.data(),
                             built.data());
  }

  void evaluate(const std::vector<Segment>& nodes, bool root, const std::vector<long long>& sums,
                std::vector<DevSplit>& out) override {
    const uint32_t n = uint32_t(nodes.size()), C = e.cols, B = e.bins, B1 = B + 1;
    std::vector<longlong2> built;
    if (sparse) build_sparse(nodes, built);
    else if (e.bytes_per_code == 1) build<uint8_t>(nodes, built);
    else build<uint16_t>(nodes, built);
    out.assign(n, DevSplit{});
    std::vector<int64_t> hist(size_t(C) * B1 * 2), want(hist.size());
    std::vector<orc_split> cand(C);
    for (uint32_t s = 0; s < n; ++s) {
      ++evaluations;
      for (uint32_t f = 0; f < C; ++f)
        for (uint32_t b = 0; b < B1; ++b) {
          const longlong2 v = built[(size_t(f) * n + s) * B1 + b];
          hist[(size_t(f) * B1 + b) * 2] = v.x;
          hist[(size_t(f) * B1 + b) * 2 + 1] = v.y;
        }
      std::fill(want.begin(), want.end(), 0);
      orc_histogram(bins, C, B, q, order.data() + nodes[s].begin, nodes[s].count, want.data());
      if (want != hist) ++hist_mismatches;
      int64_t ps[2] = {root ? 0 : sums[2 * s], root ? 0 : sums[2 * s + 1]};
      orc_evaluate_splits(hist.data(), 1, C, B, scale, cuts, counts, minima, tp.reg_lambda, tp.reg_alpha,
                          tp.min_child_weight, tp.max_delta_step, root ? 0u : 1u, ps, cand.data());
      orc_split b;
      orc_select_splits(cand.data(), 1, C, scale, tp.reg_lambda, tp.reg_alpha, tp.max_delta_step, &b);
      DevSplit& d = out[s];
      d.gain = b.gain;
      d.threshold = b.threshold;
      d.feature = b.feature;
      d.split_bin = -1;
      if (b.feature >= 0)
        for (uint32_t k = 0; k < counts[b.feature]; ++k)
          if (std::memcmp(&cuts[size_t(b.feature) * B + k], &b.threshold, 4) == 0) d.split_bin = int32_t(k);
      d.default_left = b.default_left;
      d.left_weight = b.left_weight;
      d.right_weight = b.right_weight;
      d.parent_weight = b.parent_weight;
      d.left_h = b.left_h;
      d.right_h = b.right_h;
      d.total_g = b.total_g;
      d.total_h = b.total_h;
      d.left_g = b.left_sum_g;
      d.left_hs = b.left_sum_h;
      d.right_g = b.right_sum_g;
      d.right_hs = b.right_sum_h;
    }
  }

  template <class CodeT>
  void run_partition(const std::vector<PartitionItem>& items, std::vector<uint32_t>& left) {
    const uint32_t m = uint32_t(items.size());
    std::vector<uint32_t> desc(5 * size_t(m)), tiles(m + 1), cursor(2 * size_t(m));
    uint32_t total = 0;
    for (uint32_t i = 0; i < m; ++i) {
      desc[5 * i] = items[i].begin;
      desc[5 * i + 1] = items[i].count;
      desc[5 * i + 2] = uint32_t(items[i].feature);
      desc[5 * i + 3] = uint32_t(items[i].split_bin);
      desc[5 * i + 4] = items[i].default_left;
      tiles[i] = total;
      total += (items[i].count + kQueuePartRows - 1) / kQueuePartRows;
      cursor[2 * i] = items[i].begin;
      cursor[2 * i + 1] = items[i].begin + items[i].count;
    }
    tiles[m] = total;
    std::vector<uint32_t> flags(kQueuePartRows), rank(kQueuePartRows), base(2);
    HostExec ex;
    // Tiles in reverse order: the result must not depend on which tile
    // claims its room first.
    for (uint32_t t = total; t-- > 0;)
      queue_partition_tile<CodeT>(ex, e, order.data(), scratch.data(), desc.data(), tiles.data(), m, t,
                                  cursor.data(), flags.data(), rank.data(), base.data());
    left.assign(m, 0);
    for (uint32_t i = 0; i < m; ++i) {
      std::copy(scratch.begin() + items[i].begin, scratch.begin() + items[i].begin + items[i].count,
                order.begin() + items[i].begin);
      if (cursor[2 * i] != cursor[2 * i + 1]) throw Error("partition cursors disagree");
      left[i] = cursor[2 * i] - items[i].begin;
    }
  }

  void partition(const std::vector<PartitionItem>& items, std::vector<uint32_t>& left) override {
    if (e.bytes_per_code == 1) run_partition<uint8_t>(items, left);
    else run_partition<uint16_t>(items, left);
  }
};

}  // namespace

// ELLPACK codes are built from the oracle bins with the library's layout
// rules (uint8 when every feature's codes, missing included, fit 256
// symbols; `wide` forces uint16); `sparse` builds the node histograms from
// the rows' present codes. margins[rows] start at `base` and receive
// the tree's leaves through the margin walk. stats[0] = histogram mismatches
// against the oracle, stats[1] = evaluated nodes. Returns the node count.
extern "C" int queue_harness(const uint32_t* bins, uint32_t rows, uint32_t cols, const int64_t* q, const float* pairs,
                             const float* scale, const float* cuts, uint32_t stride, const uint32_t* counts,
                             const float* minima, const orc_tree_params* tp, uint32_t lossguide, uint32_t max_leaves,
                             int wide, int sparse, float base, DevNode* nodes, uint32_t capacity, float* margins,
                             uint64_t* stats) {
  try {
    uint32_t max_count = 0;
    bool has_missing = false;
    for (uint32_t f = 0; f < cols; ++f) max_count = std::max(max_count, counts[f]);
    for (size_t i = 0; i < size_t(rows) * cols; ++i) has_missing = has_missing || bins[i] == ORC_MISSING;
    Ellpack e{};
    e.rows = rows;
    e.cols = cols;
    e.bins = stride;
    const bool narrow = !wide && (max_count <= 255 || (!has_missing && max_count <= 256));
    e.bytes_per_code = narrow ? 1 : 2;
    e.missing = !narrow ? stride : (stride <= 255 ? stride : (max_count <= 255 ? 0xffu : 0x100u));
    const uint32_t align = 16 / e.bytes_per_code;
    e.stride = std::max(align, (cols + align - 1) / align * align);
    std::vector<uint8_t> c8;
    std::vector<uint16_t> c16;
    if (narrow) c8.assign(size_t(rows) * e.stride, 0);
    else c16.assign(size_t(rows) * e.stride, 0);
    for (uint32_t r = 0; r < rows; ++r)
      for (uint32_t f = 0; f < cols; ++f) {
        const uint32_t b = bins[size_t(r) * cols + f];
        const uint32_t code = b == ORC_MISSING ? e.missing : b;
        if (narrow) c8[size_t(r) * e.stride + f] = uint8_t(code);
        else c16[size_t(r) * e.stride + f] = uint16_t(code);
      }
    e.codes = narrow ? static_cast<const void*>(c8.data()) : static_cast<const void*>(c16.data());
    EmuBackend be;
    be.e = e;
    be.pairs = reinterpret_cast<const float2*>(pairs);
    be.sc = float2{scale[0], scale[1]};
    be.bins = bins;
    be.q = q;
    be.scale = scale;
    be.cuts = cuts;
    be.counts = counts;
    be.minima = minima;
    be.tp = *tp;
    be.sparse = sparse != 0;
    if (be.sparse) {
      if (narrow) be.make_sparse_rows<uint8_t>();
      else be.make_sparse_rows<uint16_t>();
    }
    be.order.resize(rows);
    be.scratch.resize(rows);
    for (uint32_t r = 0; r < rows; ++r) be.order[r] = r;
    GrowerParams p;
    p.tree = TreeParams{tp->max_depth, tp->eta, tp->reg_lambda, tp->reg_alpha, tp->min_child_weight,
                        tp->max_delta_step, tp->min_split_loss};
    p.lossguide = lossguide != 0;
    p.max_leaves = max_leaves;
    p.scale_g = scale[0];
    p.scale_h = scale[1];
    const std::vector<DevNode> out = grow_tree_host_driven(be, rows, p);
    if (out.size() > capacity) return -1;
    std::copy(out.begin(), out.end(), nodes);
    for (uint32_t r = 0; r < rows; ++r) margins[r] = base;
    for (uint32_t r = 0; r < rows; ++r) {
      if (narrow) queue_margin_row<uint8_t>(e, out.data(), uint32_t(out.size()), margins, 1, 0, r);
      else queue_margin_row<uint16_t>(e, out.data(), uint32_t(out.size()), margins, 1, 0, r);
    }
    stats[0] = be.hist_mismatches;
    stats[1] = be.evaluations;
    return int(out.size());
  } catch (const std::exception&) {
    return -2;
  }
}
