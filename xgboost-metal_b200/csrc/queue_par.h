// The per-block work of host-driven trees (queue.cu), written against the
// executors of exec.h so the tests run the same code on the CPU:
//
//   queue_hist_item       one (row tile of a node, group of features) item of
//                         the node histograms
//   queue_partition_tile  one row tile of a leaf whose rows are split between
//                         its children
//   queue_margin_row      one row's leaf value added to its margin
//
// Reference semantics: histograms are the exact int64 sums of the quantised
// gradients per (node, feature, bin), missing values in bin B
// (kernels/boost.metal:700-733, kernels/histogram_missing.metal.h:13-60); a
// present row goes left iff its bin <= split_bin and a missing one follows
// default_left (kernels/boost.metal:1325-1329, 1497-1499); leaves add
// weight * eta to the margins (src/tree.cpp:1663-1717).
#pragma once
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "common.h"
#include "exec.h"
#include "tree.h"

namespace xgbb {

constexpr uint32_t kQueueFeatures = 8;  // features per histogram work item
constexpr uint32_t kQueueBins = kMaxBins + 1;

// q = round-half-even(v * scale) with the product rounded to float first
// (kernels/boost.metal:605-657).
XGBB_HD inline long long quantize_value(float v, float scale) {
#if defined(__CUDA_ARCH__)
  return __float2ll_rn(__fmul_rn(v, scale));
#else
  const float p = v * scale;
  return (long long)std::nearbyint(p);
#endif
}

// The node (or item) whose tiles contain tile t: the last s with tiles[s] <= t.
XGBB_HD inline uint32_t owner_of(const uint32_t* tiles, uint32_t n, uint32_t t) {
  uint32_t lo = 0, hi = n;  // tiles[lo] <= t < tiles[hi]
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) / 2;
    if (tiles[mid] <= t) lo = mid;
    else hi = mid;
  }
  return lo;
}

template <class CodeT>
XGBB_HD inline uint32_t code_at(const Ellpack& e, uint32_t row, uint32_t f) {
  return static_cast<const CodeT*>(e.codes)[size_t(row) * e.stride + f];
}

// Item `item` of the histograms of `slots` nodes: node s owns
// order[seg[2s], seg[2s] + seg[2s + 1]); tiles[s] is the exclusive scan of
// the nodes' tiles of kQueueTileRows rows. Items are tile-major: the
// kQueueFeatures-feature groups of one tile are consecutive. The item's sums
// collect in sg/sh ([kQueueFeatures][bins + 1], 64-bit, exact mod 2^64) and
// are added once per bin to built ([cols][slots][bins + 1]).
template <class CodeT, class Ex>
XGBB_HD void queue_hist_item(Ex& ex, const Ellpack& e, const uint32_t* order, const float2* pairs, float2 sc,
                             const uint32_t* seg, const uint32_t* tiles, uint32_t slots, uint64_t item,
                             unsigned long long* sg, unsigned long long* sh, longlong2* built) {
  const uint32_t C = e.cols, B = e.bins, B1 = B + 1;
  const uint32_t groups = (C + kQueueFeatures - 1) / kQueueFeatures;
  const uint32_t t = uint32_t(item / groups), fg = uint32_t(item % groups);
  const uint32_t s = owner_of(tiles, slots, t);
  const uint32_t begin = seg[2 * s] + (t - tiles[s]) * kQueueTileRows;
  const uint32_t seg_end = seg[2 * s] + seg[2 * s + 1];
  const uint32_t end = seg_end < begin + kQueueTileRows ? seg_end : begin + kQueueTileRows;
  ex.for_each(kQueueFeatures * B1, [&](uint32_t i) {
    sg[i] = 0;
    sh[i] = 0;
  });
  // Index k = (row, feature in the group): consecutive indices read one
  // row's consecutive codes.
  ex.for_each((end - begin) * kQueueFeatures, [&](uint32_t k) {
    const uint32_t fl = k % kQueueFeatures, f = fg * kQueueFeatures + fl;
    if (f >= C) return;
    const uint32_t row = order[begin + k / kQueueFeatures];
    const uint32_t code = code_at<CodeT>(e, row, f);
    const uint32_t bin = code == e.missing ? B : code;
    if (bin > B) return;  // not a code of this matrix
    const float2 p = pairs[row];
    ex.add_u64(&sg[fl * B1 + bin], (unsigned long long)quantize_value(p.x, sc.x));
    ex.add_u64(&sh[fl * B1 + bin], (unsigned long long)quantize_value(p.y, sc.y));
  });
  ex.for_each(kQueueFeatures * B1, [&](uint32_t i) {
    const uint32_t f = fg * kQueueFeatures + i / B1, b = i % B1;
    const unsigned long long g = sg[i], h = sh[i];
    if (f < C && (g | h)) {
      longlong2* dst = built + (size_t(f) * slots + s) * B1 + b;
      ex.add_u64(reinterpret_cast<unsigned long long*>(&dst->x), g);
      ex.add_u64(reinterpret_cast<unsigned long long*>(&dst->y), h);
    }
  });
}

// Tile t (kQueuePartRows rows) of the partition items: items[i] = (begin,
// count, feature, split_bin, default_left), tiles[i] the exclusive scan of
// their tiles. The tile claims room for its left rows at cursor[2i] (counting
// up from begin) and for its right rows at cursor[2i + 1] (counting down from
// begin + count) and writes its rows to `scratch` there, in row order within
// each side. flags/rank hold kQueuePartRows words; base two.
template <class CodeT, class Ex>
XGBB_HD void queue_partition_tile(Ex& ex, const Ellpack& e, const uint32_t* order, uint32_t* scratch,
                                  const uint32_t* items, const uint32_t* tiles, uint32_t nitems, uint32_t t,
                                  uint32_t* cursor, uint32_t* flags, uint32_t* rank, uint32_t* base) {
  const uint32_t it = owner_of(tiles, nitems, t);
  const uint32_t* d = items + 5 * size_t(it);
  const uint32_t seg_end = d[0] + d[1];
  const uint32_t f = d[2];
  const int32_t split_bin = int32_t(d[3]);
  const bool default_left = d[4] != 0;
  const uint32_t tile_begin = d[0] + (t - tiles[it]) * kQueuePartRows;
  const uint32_t n = seg_end - tile_begin < kQueuePartRows ? seg_end - tile_begin : kQueuePartRows;
  ex.for_each(n, [&](uint32_t i) {
    const uint32_t row = order[tile_begin + i];
    const uint32_t code = f < e.cols ? code_at<CodeT>(e, row, f) : e.missing;
    const bool left = code == e.missing ? default_left : int32_t(code) <= split_bin;
    flags[i] = left ? 1u : 0u;
    rank[i] = flags[i];
  });
  const uint32_t lefts = ex.scan_exclusive(rank, n, Add32{});
  ex.for_each(1, [&](uint32_t) {
    base[0] = ex.add_u32(cursor + 2 * it, lefts);
    base[1] = ex.sub_u32(cursor + 2 * it + 1, n - lefts) - (n - lefts);
  });
  ex.for_each(n, [&](uint32_t i) {
    const uint32_t row = order[tile_begin + i];
    if (flags[i]) scratch[base[0] + rank[i]] = row;
    else scratch[base[1] + (i - rank[i])] = row;
  });
}

// ---------------------------------------------------------------------------
// Sparse rows (kernels/histogram_csr.metal.h:22-152 in the reference): each
// row's present codes as (feature << 16 | code) entries in feature order,
// row_ptr[r] .. row_ptr[r + 1]. A node histogram then costs work in
// proportion to the present values; each node's exact total is summed
// alongside, and its missing bin is the total minus the present bins.
// ---------------------------------------------------------------------------
template <class CodeT>
XGBB_HD inline uint32_t csr_row_count(const Ellpack& e, uint32_t r) {
  uint32_t n = 0;
  for (uint32_t f = 0; f < e.cols; ++f) n += code_at<CodeT>(e, r, f) != e.missing;
  return n;
}

template <class CodeT>
XGBB_HD inline void csr_row_fill(const Ellpack& e, uint32_t r, unsigned long long at, uint32_t* entries) {
  for (uint32_t f = 0; f < e.cols; ++f) {
    const uint32_t code = code_at<CodeT>(e, r, f);
    if (code != e.missing) entries[at++] = (f << 16) | code;
  }
}

// Tile t of the sparse histograms of `slots` nodes (segments and tiles as
// for queue_hist_item): every present entry of the tile's rows is added to
// built[feature][slot][code]; tot[2] (block scratch) collects the rows'
// exact (g, h) sums, added to node_totals[slot][2] once per tile.
template <class Ex>
XGBB_HD void queue_hist_csr_tile(Ex& ex, uint32_t bins, uint32_t cols, const unsigned long long* row_ptr,
                                 const uint32_t* entries, const uint32_t* order, const float2* pairs, float2 sc,
                                 const uint32_t* seg, const uint32_t* tiles, uint32_t slots, uint32_t t,
                                 unsigned long long* tot, unsigned long long* node_totals, longlong2* built) {
  const uint32_t B1 = bins + 1;
  const uint32_t s = owner_of(tiles, slots, t);
  const uint32_t begin = seg[2 * s] + (t - tiles[s]) * kQueueTileRows;
  const uint32_t seg_end = seg[2 * s] + seg[2 * s + 1];
  const uint32_t end = seg_end < begin + kQueueTileRows ? seg_end : begin + kQueueTileRows;
  ex.for_each(1, [&](uint32_t) {
    tot[0] = 0;
    tot[1] = 0;
  });
  ex.for_each(end - begin, [&](uint32_t i) {
    const uint32_t row = order[begin + i];
    const float2 p = pairs[row];
    const unsigned long long qg = (unsigned long long)quantize_value(p.x, sc.x);
    const unsigned long long qh = (unsigned long long)quantize_value(p.y, sc.y);
    ex.add_u64(&tot[0], qg);
    ex.add_u64(&tot[1], qh);
    for (unsigned long long k = row_ptr[row]; k < row_ptr[row + 1]; ++k) {
      const uint32_t f = entries[k] >> 16, code = entries[k] & 0xffffu;
      if (f >= cols || code >= bins) continue;
      longlong2* dst = built + (size_t(f) * slots + s) * B1 + code;
      ex.add_u64(reinterpret_cast<unsigned long long*>(&dst->x), qg);
      ex.add_u64(reinterpret_cast<unsigned long long*>(&dst->y), qh);
    }
  });
  ex.for_each(1, [&](uint32_t) {
    ex.add_u64(&node_totals[2 * s], tot[0]);
    ex.add_u64(&node_totals[2 * s + 1], tot[1]);
  });
}

// The missing bin of (feature f, slot s): the node total minus the present
// bins, mod 2^64.
XGBB_HD inline void queue_fill_missing(uint32_t bins, uint32_t slots, const unsigned long long* node_totals,
                                       longlong2* built, uint32_t f, uint32_t s) {
  longlong2* h = built + (size_t(f) * slots + s) * (bins + 1);
  unsigned long long g = node_totals[2 * s], hh = node_totals[2 * s + 1];
  for (uint32_t b = 0; b < bins; ++b) {
    g -= (unsigned long long)h[b].x;
    hh -= (unsigned long long)h[b].y;
  }
  h[bins].x = (long long)g;
  h[bins].y = (long long)hh;
}

// margins[row][group] += the leaf `row` reaches in `nodes`, walking its
// codes (at most node_count steps).
template <class CodeT>
XGBB_HD inline void queue_margin_row(const Ellpack& e, const DevNode* nodes, uint32_t node_count, float* margins,
                                     uint32_t groups, uint32_t group, uint32_t r) {
  uint32_t n = 0;
  for (uint32_t step = 0; step < node_count; ++step) {
    const DevNode nd = nodes[n];
    if (nd.left < 0 || uint32_t(nd.feature) >= e.cols) break;
    const uint32_t code = code_at<CodeT>(e, r, uint32_t(nd.feature));
    const bool left = code == e.missing ? nd.default_left != 0u : int32_t(code) <= nd.split_bin;
    const int32_t next = left ? nd.left : nd.right;
    if (next < 0 || uint32_t(next) >= node_count) break;
    n = uint32_t(next);
  }
  float* m = margins + size_t(r) * groups + group;
#if defined(__CUDA_ARCH__)
  *m = __fadd_rn(*m, nodes[n].leaf);
#else
  *m = *m + nodes[n].leaf;
#endif
}

}  // namespace xgbb
