// Test harness: the GPU sketch's data-parallel algorithms (csrc/sketch_par.h)
// run on the CPU with the serial executor, chunk by chunk and batch by batch
// as the kernels run them, so the tests can compare their cuts bit for bit
// with the host sketch. Test infrastructure only.
#include <algorithm>
#include <cmath>
#include <vector>

#include "sketch_par.h"

using namespace xgbb;
using namespace xgbb::sketch;

namespace {

template <class T>
T* grab(std::vector<T>& v, size_t n) {
  v.assign(n, T{});
  return v.data();
}

}  // namespace

// X row-major [rows][cols]; cuts [cols][stride]. `chunk` is the rows per run
// extraction step (small values exercise runs that cross chunks); with
// `segments` > 1 each feature's rows are split into that many segments whose
// runs are counted, linked and written as the GPU's segment passes do. The
// batch and reduction steps follow the kernels' plan (plan_group) and scratch
// layouts; with `tree` the reduction is the merge tree (plan_tree), regular
// features finishing from its nodes and irregular ones through
// reduce_feature. serial[0..2] count the hand-overs to serial forms,
// serial[3] and serial[4] the regular and irregular features of the tree.
extern "C" int sketch_harness(const float* X, uint32_t rows, uint32_t cols, const float* weights, uint32_t max_bin,
                              uint32_t chunk, uint32_t segments, uint32_t tree, float* cuts, uint32_t* counts,
                              float* minima, uint64_t* serial) {
  const uint32_t stride = std::max(1u, std::min(max_bin, rows));
  std::fill(cuts, cuts + size_t(cols) * stride, 0.0f);
  HostExec ex;
  // Runs of every feature: runs[f * rows ...].
  std::vector<Run> runs(size_t(std::max(rows, 1u)) * std::max(cols, 1u));
  std::vector<uint32_t> stats(size_t(cols) * 3);
  std::vector<float> cv, cw, lw(1);
  std::vector<uint32_t> c0, c1, c2, c3, c4;
  const bool unit = weights == nullptr;
  for (uint32_t f = 0; f < cols; ++f) {
    ChunkWork c{grab(cv, chunk), grab(cw, chunk), grab(c0, chunk), grab(c1, chunk), grab(c2, chunk),
                grab(c3, chunk), grab(c4, chunk), lw.data()};
    auto pass = [&](uint32_t lo, uint32_t hi, RunCarry& carry, RunOut out) {
      for (uint32_t r0 = lo; r0 < hi; r0 += chunk) {
        const uint32_t n = std::min(chunk, hi - r0);
        runs_chunk(
            ex,
            [&](uint32_t i, float& v, float& w) {
              v = X[size_t(r0 + i) * cols + f];
              w = weights ? weights[r0 + i] : 1.0f;
            },
            n, unit, carry, out, c);
      }
    };
    Run* fr = runs.data() + size_t(f) * rows;
    if (segments <= 1) {
      RunCarry carry{0, 0, 0, 0, 0.0f, 0.0f, 0.0f};
      pass(0, rows, carry, RunOut{fr, true, 0u, nullptr});
      stats[3 * f] = carry.runs;
      stats[3 * f + 1] = carry.elements;
      stats[3 * f + 2] = carry.nonmissing;
    } else {
      const uint32_t seg_rows = (rows + segments - 1) / segments;
      std::vector<RunCarry> p1(segments);
      std::vector<SegmentLink> link(segments);
      for (uint32_t s = 0; s < segments; ++s) {
        p1[s] = RunCarry{0, 0, 0, 0, 0.0f, 0.0f, 0.0f};
        pass(std::min(rows, s * seg_rows), std::min(rows, (s + 1) * seg_rows), p1[s], RunOut{nullptr, false, 0u, nullptr});
      }
      link_segments(
          p1.data(), segments, unit, link.data(),
          [&](uint32_t s, uint32_t k, float& v, float& w) {
            const size_t r = size_t(s) * seg_rows + k;
            v = X[r * cols + f];
            w = weights ? weights[r] : 1.0f;
          },
          [&](uint32_t s) { return std::min(rows, (s + 1) * seg_rows) - std::min(rows, s * seg_rows); },
          stats.data() + 3 * f);
      for (uint32_t s = 0; s < segments; ++s) {
        RunCarry carry = link[s].in;
        pass(std::min(rows, s * seg_rows), std::min(rows, (s + 1) * seg_rows), carry,
             RunOut{fr, true, link[s].in.runs, &link[s].cont_w});
      }
      finish_links(link.data(), segments, fr);
    }
    minima[f] = -INFINITY;
  }
  const GroupPlan plan = plan_group(stats.data(), cols, 0, rows, max_bin);
  const TreePlan tp = plan_tree(plan);
  std::vector<Entry> summaries(std::max<uint64_t>(tree ? tp.entries : plan.summary_entries, 1));
  std::vector<uint32_t> sizes(std::max(tree ? tp.sizes : plan.sizes, 1u));
  std::vector<unsigned char> scratch(batch_scratch_bytes(plan.cap)), work(std::max<uint64_t>(plan.work_bytes, 1));
  // Every other batch takes the radix form of the sort (the GPU kernel's
  // path), the others the bitonic form: both must give the host sketch's cuts.
  std::vector<unsigned char> radix(radix_sort_bytes(plan.cap, 32));
  size_t task_index = 0;
  for (const BatchTask& t : plan.tasks) {
    const BatchWork bw = batch_work_at(scratch.data(), plan.cap);
    sizes[t.size_slot] = summarize_par(ex, runs.data() + t.run_begin, t.size, t.limit, bw.keys, bw.sorted, bw.entries,
                                       summaries.data() + t.summary_at, bw.w,
                                       (task_index++ & 1) ? radix.data() : nullptr);
  }
  std::vector<uint32_t> irregular(std::max<size_t>(plan.reduce.size(), 1), tree ? 0u : 1u);
  if (tree) {
    uint32_t big = 2;
    for (const ReduceTask& rt : plan.reduce) big = std::max(big, reduce_big(rt.limit, rt.budget));
    std::vector<unsigned char> mscratch(merge_scratch_bytes(big));
    for (const auto& level : tp.levels)
      for (const MergeTask& t : level)
        merge_node(ex, t, summaries.data(), sizes.data(), irregular.data(), merge_work_at(mscratch.data(), big));
    for (const FinishTask& t : tp.finish) {
      if (irregular[t.local]) continue;
      const ReduceWork r = reduce_work_at(work.data() + t.work_at, t.limit, t.budget, t.levels);
      counts[t.feature] = finish_tree(ex, t, tp.res.data(), summaries.data(), sizes.data(), max_bin, r,
                                      cuts + size_t(t.feature) * stride);
      ++serial[3];
    }
  }
  for (uint32_t j = 0; j < plan.reduce.size(); ++j) {
    const ReduceTask& t = plan.reduce[j];
    if (!irregular[j]) continue;
    const ReduceWork r = reduce_work_at(work.data() + t.work_at, t.limit, t.budget, t.levels);
    counts[t.feature] = reduce_feature(ex, summaries.data() + t.summary_at, sizes.data() + t.first_size, t.nbatch,
                                       t.limit, t.budget, t.levels, max_bin, r, cuts + size_t(t.feature) * stride);
    if (tree) ++serial[4];
  }
  for (int k = 0; k < 3; ++k) serial[k] = ex.notes[k];
  return 0;
}
