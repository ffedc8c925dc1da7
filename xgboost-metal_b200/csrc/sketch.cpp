// Quantile cuts for dense float32 features: weighted quantile summaries over
// runs of equal values, pruned and combined level by level, then at most
// max_bin cut values per feature.
//
// Semantics follow the reference's summary kernels (tabulai/xgboost-metal
// kernels/quantile.metal.h:19-411 and src/quantile.cpp:11-213): runs in row
// order, batches of 2*limit runs sorted and summarised into (rmin, rmax, wmin,
// value) entries, sketch_prune / sketch_combine / the per-level reduction, and
// the cut rule (distinct values when the summary is small, binary64 rank
// queries otherwise, then max + (|max| + 1e-5)). Entries are plain IEEE
// binary32 with gradual underflow; -0 is read as +0, and ties keep row order.
//
// It runs on the host. Workers take blocks of features: one sequential pass
// over the rows copies a block's columns into contiguous buffers (each cache
// line of the row-major matrix is read once per block, not once per
// feature), then each column is summarised. The cuts decide every bin, so
// they are compared exactly against the checker in the tests.
#include "sketch.h"

#include "sketch_par.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

namespace xgbb {
namespace {

using sketch::budget_for;
using sketch::Entry;
using sketch::Run;

// Stable sort of runs by value: an LSD radix sort on order-preserving keys
// (the sign bit flipped for positives, all bits for negatives), which orders
// every non-NaN float as `<` does (-0 never occurs: it is read as +0) and
// keeps equal values in their input order, as std::stable_sort would. Each
// run travels as one 64-bit word, key above weight; the three digit
// histograms (11, 11 and 10 bits) come from one counting pass, and a pass in
// which every key has the same digit is skipped.
inline float key_value(uint32_t k) {
  const uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  float v;
  std::memcpy(&v, &b, 4);
  return v;
}
void sort_runs(Run* a, size_t n, std::vector<uint64_t>& buf, std::vector<uint64_t>& tmp) {
  if (n < 2) return;
  buf.resize(n);
  tmp.resize(n);
  static constexpr int kShift[3] = {0, 11, 22};
  static constexpr uint32_t kMask[3] = {0x7ffu, 0x7ffu, 0x3ffu};
  uint32_t hist[3][2048] = {};
  for (size_t i = 0; i < n; ++i) {
    const uint32_t k = sketch::order_key(a[i].v);
    buf[i] = (uint64_t(k) << 32) | sketch::float_bits(a[i].w);
    ++hist[0][k & 0x7ffu];
    ++hist[1][(k >> 11) & 0x7ffu];
    ++hist[2][k >> 22];
  }
  uint64_t* src = buf.data();
  uint64_t* dst = tmp.data();
  for (int p = 0; p < 3; ++p) {
    uint32_t* h = hist[p];
    const int shift = 32 + kShift[p];
    const uint32_t mask = kMask[p];
    if (h[(src[0] >> shift) & mask] == n) continue;  // one digit: order unchanged
    uint32_t sum = 0;
    for (uint32_t d = 0; d <= mask; ++d) {
      const uint32_t c = h[d];
      h[d] = sum;
      sum += c;
    }
    for (size_t i = 0; i < n; ++i) dst[h[(src[i] >> shift) & mask]++] = src[i];
    std::swap(src, dst);
  }
  for (size_t i = 0; i < n; ++i) {
    const uint32_t wb = uint32_t(src[i]);
    float w;
    std::memcpy(&w, &wb, 4);
    a[i] = Run{key_value(uint32_t(src[i] >> 32)), w};
  }
}

// One feature's cuts from its column `col` (contiguous, `rows` values).
void one_feature(const float* col, uint32_t rows, const float* weights, uint32_t max_bin, float* out,
                 uint32_t* count_out, float* minimum) {
  const bool unit = weights == nullptr;
  std::vector<Run> runs;
  runs.reserve(rows);
  uint32_t elements = 0, nonmissing = 0;
  float previous = 0;
  for (uint32_t r = 0; r < rows; ++r) {
    float v = col[r];
    const float w = unit ? 1.0f : weights[r];
    nonmissing += !std::isnan(v);
    uint32_t wb;
    std::memcpy(&wb, &w, 4);
    if (std::isnan(v) || (wb & 0x7fffffffu) == 0) continue;
    if (v == 0.0f) v = 0.0f;  // -0 reads as +0
    ++elements;
    if (runs.empty() || !(v == previous)) {
      runs.push_back({v, unit ? 1.0f : w});
    } else if (unit) {
      runs.back().w = std::min(runs.back().w + 1.0f, 16777216.0f);
    } else {
      runs.back().w = runs.back().w + w;
    }
    previous = v;
  }
  *minimum = -INFINITY;
  const uint32_t nruns = uint32_t(runs.size());
  const uint32_t limit = budget_for(max_bin, nonmissing);
  const uint32_t budget = budget_for(max_bin, elements);
  const uint64_t capacity = 2ull * limit;
  const uint32_t nbatch = uint32_t((nruns + capacity - 1) / capacity);
  uint32_t levels = 1;
  for (uint32_t c = std::max(1u, nbatch); c; c >>= 1) ++levels;
  std::vector<Entry> resident(size_t(limit) * levels), current(2 * size_t(limit) + 1),
      scratch(2 * size_t(limit) + 1), summary(capacity + 1);
  uint32_t counts[64] = {0};
  std::vector<uint64_t> sort_buf, sort_tmp;
  const auto prune = sketch::prune_serial;
  const auto combine = sketch::combine_serial;
  for (uint32_t batch = 0; batch < nbatch; ++batch) {
    const uint64_t begin = batch * capacity;
    const uint32_t size = uint32_t(std::min<uint64_t>(capacity, nruns - begin));
    Run* src = runs.data() + begin;
    sort_runs(src, size, sort_buf, sort_tmp);
    uint32_t n = 0;
    float total = 0;
    for (uint32_t i = 0; i < size;) {
      Run value = src[i];
      uint32_t j = i + 1;
      while (j < size && src[j].v == value.v) value.w = value.w + src[j++].w;
      summary[n++] = {total, total + value.w, value.w, value.v};
      total = total + value.w;
      i = j;
    }
    n = prune(summary.data(), n, limit);
    std::copy(summary.begin(), summary.begin() + n, current.begin());
    uint32_t level = 0;
    for (;;) {
      n = prune(current.data(), n, limit);
      n = combine(current.data(), n, resident.data() + size_t(level) * limit, counts[level],
                  scratch.data());
      counts[level] = 0;
      if (n <= limit) break;
      ++level;
    }
    counts[level] = n;
    std::copy(current.begin(), current.begin() + n, resident.begin() + size_t(level) * limit);
  }
  uint32_t n = 0;
  for (uint32_t level = 0; level < levels; ++level) {
    n = combine(current.data(), n, resident.data() + size_t(level) * limit, counts[level],
                scratch.data());
    n = prune(current.data(), n, std::max(budget, limit));
  }
  const uint32_t size = prune(current.data(), n, budget);
  *count_out = sketch::select_cuts(current.data(), size, max_bin, out);
}

}  // namespace

uint32_t cut_stride(uint32_t rows, uint32_t max_bin) { return std::max(1u, std::min(max_bin, rows)); }

void sketch_cuts(const float* X, uint32_t rows, uint32_t cols, const float* weights,
                 uint32_t max_bin, float* cuts, uint32_t* counts, float* minima, int threads) {
  const uint32_t stride = cut_stride(rows, max_bin);
  std::fill(cuts, cuts + size_t(cols) * stride, 0.0f);
  if (threads <= 0) threads = int(std::max(1u, std::thread::hardware_concurrency()));
  threads = int(std::min<uint32_t>(uint32_t(threads), std::max(1u, cols)));
  // Blocks of up to 16 features (one 64-byte line of a row), fewer when there
  // are few features per worker, handed out by a shared counter.
  const uint32_t block = std::max(1u, std::min(16u, cols / uint32_t(threads)));
  const uint32_t nblocks = (cols + block - 1) / block;
  std::atomic<uint32_t> next{0};
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t)
    pool.emplace_back([&] {
      std::vector<float> buf(size_t(block) * rows);
      for (uint32_t b = next++; b < nblocks; b = next++) {
        const uint32_t f0 = b * block, nf = std::min(block, cols - f0);
        for (uint32_t r = 0; r < rows; ++r) {
          const float* row = X + size_t(r) * cols + f0;
          for (uint32_t j = 0; j < nf; ++j) buf[size_t(j) * rows + r] = row[j];
        }
        for (uint32_t j = 0; j < nf; ++j) {
          const uint32_t f = f0 + j;
          one_feature(buf.data() + size_t(j) * rows, rows, weights, max_bin, cuts + size_t(f) * stride,
                      counts + f, minima + f);
        }
      }
    });
  for (auto& th : pool) th.join();
}

}  // namespace xgbb
