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
// extraction step (small values exercise runs that cross chunks). The batch
// and reduction steps follow the kernels' plan (plan_group) and scratch
// layouts (batch_work_at, reduce_work_at) exactly.
extern "C" int sketch_harness(const float* X, uint32_t rows, uint32_t cols, const float* weights, uint32_t max_bin,
                              uint32_t chunk, float* cuts, uint32_t* counts, float* minima, uint64_t* serial) {
  const uint32_t stride = std::max(1u, std::min(max_bin, rows));
  std::fill(cuts, cuts + size_t(cols) * stride, 0.0f);
  HostExec ex;
  // Runs of every feature, chunk by chunk: runs[f * rows ...].
  std::vector<Run> runs(size_t(std::max(rows, 1u)) * std::max(cols, 1u));
  std::vector<uint32_t> stats(size_t(cols) * 3);
  std::vector<float> cv, cw, lw(1);
  std::vector<uint32_t> c0, c1, c2, c3, c4;
  for (uint32_t f = 0; f < cols; ++f) {
    RunCarry carry{0, 0, 0, 0, 0.0f, 0.0f};
    ChunkWork c{grab(cv, chunk), grab(cw, chunk), grab(c0, chunk), grab(c1, chunk), grab(c2, chunk),
                grab(c3, chunk), grab(c4, chunk), lw.data()};
    for (uint32_t r0 = 0; r0 < rows; r0 += chunk) {
      const uint32_t n = std::min(chunk, rows - r0);
      runs_chunk(
          ex,
          [&](uint32_t i, float& v, float& w) {
            v = X[size_t(r0 + i) * cols + f];
            w = weights ? weights[r0 + i] : 1.0f;
          },
          n, weights == nullptr, carry, runs.data() + size_t(f) * rows, c);
    }
    stats[3 * f] = carry.runs;
    stats[3 * f + 1] = carry.elements;
    stats[3 * f + 2] = carry.nonmissing;
    minima[f] = -INFINITY;
  }
  const GroupPlan plan = plan_group(stats.data(), cols, 0, rows, max_bin);
  std::vector<Entry> summaries(std::max<uint64_t>(plan.summary_entries, 1));
  std::vector<uint32_t> sizes(std::max(plan.sizes, 1u));
  std::vector<unsigned char> scratch(batch_scratch_bytes(plan.cap)), work(std::max<uint64_t>(plan.work_bytes, 1));
  for (const BatchTask& t : plan.tasks) {
    const BatchWork bw = batch_work_at(scratch.data(), plan.cap);
    sizes[t.size_slot] = summarize_par(ex, runs.data() + t.run_begin, t.size, t.limit, bw.keys, bw.sorted, bw.entries,
                                       summaries.data() + t.summary_at, bw.w);
  }
  for (const ReduceTask& t : plan.reduce) {
    const ReduceWork r = reduce_work_at(work.data() + t.work_at, t.limit, t.budget, t.levels);
    counts[t.feature] = reduce_feature(ex, summaries.data() + t.summary_at, sizes.data() + t.first_size, t.nbatch,
                                       t.limit, t.budget, t.levels, max_bin, r, cuts + size_t(t.feature) * stride);
  }
  for (int k = 0; k < 3; ++k) serial[k] = ex.notes[k];
  return 0;
}
