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
// extraction step (small values exercise runs that cross chunks).
// serial[3] receives how often the data-parallel forms handed over to the
// serial definitions (prune, combine, batch prefix sums).
extern "C" int sketch_harness(const float* X, uint32_t rows, uint32_t cols, const float* weights, uint32_t max_bin,
                              uint32_t chunk, float* cuts, uint32_t* counts, float* minima, uint64_t* serial) {
  const uint32_t stride = std::max(1u, std::min(max_bin, rows));
  std::fill(cuts, cuts + size_t(cols) * stride, 0.0f);
  HostExec ex;
  std::vector<Run> runs(std::max(rows, 1u));
  std::vector<float> cv, cw, lw(1);
  std::vector<uint32_t> c0, c1, c2, c3, c4;
  for (uint32_t f = 0; f < cols; ++f) {
    // Runs, chunk by chunk.
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
          n, weights == nullptr, carry, runs.data(), c);
    }
    const FeaturePlan p = plan_feature(max_bin, carry.runs, carry.elements, carry.nonmissing);
    // Batch summaries.
    std::vector<Entry> summaries(size_t(std::max(p.nbatch, 1u)) * p.limit);
    std::vector<uint32_t> sizes(std::max(p.nbatch, 1u));
    std::vector<unsigned long long> keys;
    std::vector<Run> sorted;
    std::vector<Entry> entries;
    std::vector<uint32_t> wu, wv;
    std::vector<float> wf;
    const uint32_t cap = p.capacity;
    BatchWork bw{grab(keys, pow2_ceil(cap)), grab(sorted, cap), grab(entries, cap),
                 Work{grab(wu, cap + 2), grab(wv, cap + 2), grab(wf, cap + 2)}};
    for (uint32_t k = 0; k < p.nbatch; ++k) {
      const uint64_t begin = uint64_t(k) * cap;
      const uint32_t size = uint32_t(std::min<uint64_t>(cap, p.runs - begin));
      sizes[k] = summarize_par(ex, runs.data() + begin, size, p.limit, bw.keys, bw.sorted, bw.entries,
                               summaries.data() + size_t(k) * p.limit, bw.w);
    }
    // Levels and cuts.
    const uint32_t big = 2 * std::max(p.limit, p.budget) + 2;
    std::vector<Entry> resident(size_t(p.limit) * p.levels), a, b, s;
    std::vector<uint32_t> lc(p.levels), ru, rv, size(1);
    std::vector<float> rf;
    ReduceWork rw{resident.data(), lc.data(), grab(a, big), grab(b, big), grab(s, big),
                  Work{grab(ru, big), grab(rv, big), grab(rf, big)}, size.data()};
    counts[f] = reduce_feature(ex, summaries.data(), sizes.data(), p.nbatch, p.limit, p.budget, p.levels, max_bin,
                               rw, cuts + size_t(f) * stride);
    minima[f] = -INFINITY;
  }
  for (int k = 0; k < 3; ++k) serial[k] = ex.notes[k];
  return 0;
}
