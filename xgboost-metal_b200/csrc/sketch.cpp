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
// This first version runs on the host, one feature per worker thread; the
// cuts it produces decide every bin, so they are compared exactly against the
// checker in the tests.
#include "sketch.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

namespace xgbb {
namespace {

struct Run {
  float v, w;
};
struct Entry {
  float rmin, rmax, wmin, value;
};

uint32_t budget_for(uint32_t bins, uint32_t count) {
  if (!count) return 1;
  const double epsilon = 1.0 / double(std::min(bins, count));
  for (uint32_t level = 1; level < 32; ++level) {
    uint64_t limit = uint64_t(std::ceil(level / (epsilon / 2.0))) + 1;
    limit = std::min<uint64_t>(limit, count);
    if ((uint64_t{1} << level) * limit >= count) return uint32_t(limit);
  }
  return count;
}

inline float lower_next(const Entry& e) { return e.rmin + e.wmin; }
inline float upper_prev(const Entry& e) { return e.rmax - e.wmin; }

uint32_t prune(Entry* e, uint32_t size, uint32_t capacity) {
  if (size <= capacity) return size;
  if (capacity == 0) return 0;
  if (capacity == 1) return 1;
  const float begin = e[0].rmax, range = e[size - 1].rmin - begin;
  const uint32_t n = capacity - 1;
  uint32_t count = 1, i = 1, last = 0;
  const Entry tail = e[size - 1];
  Entry left = e[1], right = e[2];
  for (uint32_t k = 1; k < n; ++k) {
    const float rank = 2.0f * (float(k) * range / float(n) + begin);
    while (i < size - 1 && rank >= right.rmax + right.rmin) {
      ++i;
      left = right;
      if (i < size - 1) right = e[i + 1];
    }
    if (i == size - 1) break;
    if (rank < lower_next(left) + upper_prev(right)) {
      if (i != last) {
        e[count++] = left;
        last = i;
      }
    } else if (i + 1 != last) {
      e[count++] = right;
      last = i + 1;
    }
  }
  if (last != size - 1) e[count++] = tail;
  return count;
}

uint32_t combine(Entry* cur, uint32_t n, const Entry* other, uint32_t m, Entry* scratch) {
  if (!m) return n;
  if (!n) {
    std::copy(other, other + m, cur);
    return m;
  }
  uint32_t a = 0, b = 0, count = 0;
  float prev_a = 0, prev_b = 0;
  while (a < n && b < m) {
    const Entry x = cur[a], y = other[b];
    Entry r;
    if (x.value == y.value) {
      r = {x.rmin + y.rmin, x.rmax + y.rmax, x.wmin + y.wmin, x.value};
      prev_a = lower_next(x);
      prev_b = lower_next(y);
      ++a;
      ++b;
    } else if (x.value < y.value) {
      r = {x.rmin + prev_b, x.rmax + upper_prev(y), x.wmin, x.value};
      prev_a = lower_next(x);
      ++a;
    } else {
      r = {y.rmin + prev_a, y.rmax + upper_prev(x), y.wmin, y.value};
      prev_b = lower_next(y);
      ++b;
    }
    scratch[count++] = r;
  }
  const float tail_a = cur[n - 1].rmax, tail_b = other[m - 1].rmax;
  while (a < n) {
    Entry x = cur[a++];
    x.rmin = x.rmin + prev_b;
    x.rmax = x.rmax + tail_b;
    scratch[count++] = x;
  }
  while (b < m) {
    Entry y = other[b++];
    y.rmin = y.rmin + prev_a;
    y.rmax = y.rmax + tail_a;
    scratch[count++] = y;
  }
  float prev_min = 0, prev_max = 0;
  for (uint32_t i = 0; i < count; ++i) {
    Entry e = scratch[i];
    if (e.rmin < prev_min) e.rmin = prev_min;
    else prev_min = e.rmin;
    if (e.rmax < prev_max) e.rmax = prev_max;
    if (e.rmax < lower_next(e)) e.rmax = lower_next(e);
    prev_max = e.rmax;
    cur[i] = e;
  }
  return count;
}

uint64_t bits64(double v) {
  uint64_t b;
  std::memcpy(&b, &v, 8);
  return b;
}

void one_feature(const float* X, uint32_t rows, uint32_t cols, uint32_t f, const float* weights,
                 uint32_t max_bin, float* out, uint32_t* count_out, float* minimum) {
  const bool unit = weights == nullptr;
  std::vector<Run> runs;
  runs.reserve(rows);
  uint32_t elements = 0, nonmissing = 0;
  float previous = 0;
  for (uint32_t r = 0; r < rows; ++r) {
    float v = X[size_t(r) * cols + f];
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
  for (uint32_t batch = 0; batch < nbatch; ++batch) {
    const uint64_t begin = batch * capacity;
    const uint32_t size = uint32_t(std::min<uint64_t>(capacity, nruns - begin));
    Run* src = runs.data() + begin;
    std::stable_sort(src, src + size, [](const Run& a, const Run& b) { return a.v < b.v; });
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
  uint32_t count = 0;
  if (!size) {
    out[0] = 1e-5f;
    *count_out = 1;
    return;
  }
  const Entry* e = current.data();
  if (size <= max_bin) {
    float last = e[0].value;
    for (uint32_t i = 1; i < size; ++i)
      if (last < e[i].value) {
        out[count++] = e[i].value;
        last = e[i].value;
      }
  } else {
    float last = e[0].value;
    uint32_t next = 1, cursor = 0;
    const double total = double(e[size - 1].rmax);
    for (uint32_t i = 1; i < max_bin; ++i) {
      const uint64_t rank = bits64(double(i) * total / double(max_bin) * 2.0);
      while (cursor < size - 2 && rank >= bits64(double(e[cursor + 1].rmin + e[cursor + 1].rmax)))
        ++cursor;
      const float boundary = lower_next(e[cursor]) + upper_prev(e[cursor + 1]);
      float value = e[cursor + ((std::isnan(boundary) || rank >= bits64(double(boundary))) ? 1 : 0)].value;
      if (value <= last) {
        while (next < size && e[next].value <= last) ++next;
        if (next == size) break;
        value = e[next].value;
      } else if (next < size && e[next].value <= value) {
        do {
          ++next;
        } while (next < size && e[next].value <= value);
      }
      out[count++] = value;
      last = value;
    }
  }
  const float tail = e[size - 1].value;
  out[count++] = tail + (std::fabs(tail) + 1e-5f);
  *count_out = count;
}

}  // namespace

uint32_t cut_stride(uint32_t rows, uint32_t max_bin) { return std::max(1u, std::min(max_bin, rows)); }

void sketch_cuts(const float* X, uint32_t rows, uint32_t cols, const float* weights,
                 uint32_t max_bin, float* cuts, uint32_t* counts, float* minima, int threads) {
  const uint32_t stride = cut_stride(rows, max_bin);
  std::fill(cuts, cuts + size_t(cols) * stride, 0.0f);
  if (threads <= 0) threads = int(std::max(1u, std::thread::hardware_concurrency()));
  threads = int(std::min<uint32_t>(uint32_t(threads), std::max(1u, cols)));
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t)
    pool.emplace_back([=] {
      for (uint32_t f = uint32_t(t); f < cols; f += uint32_t(threads))
        one_feature(X, rows, cols, f, weights, max_bin, cuts + size_t(f) * stride, counts + f,
                    minima + f);
    });
  for (auto& th : pool) th.join();
}

}  // namespace xgbb
