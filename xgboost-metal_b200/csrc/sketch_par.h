// Weighted quantile sketch in a data-parallel form (the GPU sketch), and the
// serial summary operations it shares with the host sketch (sketch.cpp).
//
// The reference computes cuts on its GPU (kernels/quantile.metal.h:19-411,
// src/quantile.cpp:22-213): per feature, runs of equal values in row order;
// batches of 2 * limit runs, each sorted and summarised into (rmin, rmax,
// wmin, value) entries and pruned to `limit`; the batch summaries combined
// and pruned level by level; then at most max_bin cuts. Every float
// operation below happens in the order of the serial definition, so the
// data-parallel forms give the serial results bit for bit:
//   - prune: each output index is found by binary search, which equals the
//     serial scan whenever the entries' rank sums and the query ranks are
//     non-decreasing (checked; otherwise the serial form runs);
//   - combine: each entry's place and neighbours are found by binary search
//     in the other summary, and the serial clamp of ranks is a running
//     maximum (an associative selection, no rounding);
//   - summaries: a stable sort (sort keys carry the input position), and the
//     prefix sums of the weights as exact integers when they are (otherwise
//     serial).
//
// The algorithms are written against an executor `Ex` that runs a loop body
// for every index with a barrier after it, and block-wide scans: the CUDA
// kernels (sketch_gpu.cu) run them with one thread block per task, and the
// tests run the same code with HostExec on the CPU.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "exec.h"

namespace xgbb {
namespace sketch {

struct Run {
  float v, w;
};
struct Entry {
  float rmin, rmax, wmin, value;
};

XGBB_HD inline float lower_next(const Entry& e) { return e.rmin + e.wmin; }
XGBB_HD inline float upper_prev(const Entry& e) { return e.rmax - e.wmin; }

XGBB_HD inline uint32_t float_bits(float v) {
  uint32_t b;
  std::memcpy(&b, &v, 4);
  return b;
}
XGBB_HD inline uint64_t double_bits(double v) {
  uint64_t b;
  std::memcpy(&b, &v, 8);
  return b;
}
// Order-preserving key of a non-NaN float (-0 never occurs: it is read as +0).
XGBB_HD inline uint32_t order_key(float v) {
  const uint32_t b = float_bits(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Summary size budget of `count` values for `bins` bins (src/quantile.cpp:11-20).
inline uint32_t budget_for(uint32_t bins, uint32_t count) {
  if (!count) return 1;
  const double epsilon = 1.0 / double(bins < count ? bins : count);
  for (uint32_t level = 1; level < 32; ++level) {
    uint64_t limit = uint64_t(std::ceil(level / (epsilon / 2.0))) + 1;
    if (limit > count) limit = count;
    if ((uint64_t{1} << level) * limit >= count) return uint32_t(limit);
  }
  return count;
}

// ---------------------------------------------------------------------------
// Serial definitions (kernels/quantile.metal.h:192-352).
// ---------------------------------------------------------------------------

// Keeps at most `capacity` entries of e[0, size) in place: the first, the
// entries nearest the evenly spaced ranks, and the last.
XGBB_HD inline uint32_t prune_serial(Entry* e, uint32_t size, uint32_t capacity) {
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

// Merges `other` (m entries) into `cur` (n entries, room for n + m); scratch
// holds n + m entries. Returns the merged size. Each merged entry's ranks are
// clamped to be non-decreasing as it is produced: rmin to the running rmin,
// rmax to the running rmax and to rmin + wmin.
XGBB_HD inline uint32_t combine_serial(Entry* cur, uint32_t n, const Entry* other, uint32_t m, Entry* scratch) {
  if (!m) return n;
  if (!n) {
    for (uint32_t i = 0; i < m; ++i) cur[i] = other[i];
    return m;
  }
  uint32_t a = 0, b = 0, count = 0;
  float prev_a = 0, prev_b = 0, prev_min = 0, prev_max = 0;
  auto emit = [&](Entry e) {
    if (e.rmin < prev_min) e.rmin = prev_min;
    else prev_min = e.rmin;
    if (e.rmax < prev_max) e.rmax = prev_max;
    if (e.rmax < lower_next(e)) e.rmax = lower_next(e);
    prev_max = e.rmax;
    scratch[count++] = e;
  };
  while (a < n && b < m) {
    const Entry x = cur[a], y = other[b];
    if (x.value == y.value) {
      emit({x.rmin + y.rmin, x.rmax + y.rmax, x.wmin + y.wmin, x.value});
      prev_a = lower_next(x);
      prev_b = lower_next(y);
      ++a;
      ++b;
    } else if (x.value < y.value) {
      emit({x.rmin + prev_b, x.rmax + upper_prev(y), x.wmin, x.value});
      prev_a = lower_next(x);
      ++a;
    } else {
      emit({y.rmin + prev_a, y.rmax + upper_prev(x), y.wmin, y.value});
      prev_b = lower_next(y);
      ++b;
    }
  }
  const float tail_a = cur[n - 1].rmax, tail_b = other[m - 1].rmax;
  while (a < n) {
    const Entry x = cur[a++];
    emit({x.rmin + prev_b, x.rmax + tail_b, x.wmin, x.value});
  }
  while (b < m) {
    const Entry y = other[b++];
    emit({y.rmin + prev_a, y.rmax + tail_a, y.wmin, y.value});
  }
  for (uint32_t i = 0; i < count; ++i) cur[i] = scratch[i];
  return count;
}

// At most max_bin cuts from a final summary of `size` entries
// (kernels/quantile.metal.h:354-400): the distinct values after the first
// when the summary is small, else binary64 rank queries with the boundary
// rule and strictly increasing values; then max + (|max| + 1e-5). An empty
// summary gives the single cut 1e-5. Returns the cut count.
XGBB_HD inline uint32_t select_cuts(const Entry* e, uint32_t size, uint32_t max_bin, float* out) {
  uint32_t count = 0;
  if (!size) {
    out[0] = 1e-5f;
    return 1;
  }
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
      const uint64_t rank = double_bits(double(i) * total / double(max_bin) * 2.0);
      while (cursor < size - 2 && rank >= double_bits(double(e[cursor + 1].rmin + e[cursor + 1].rmax))) ++cursor;
      const float boundary = lower_next(e[cursor]) + upper_prev(e[cursor + 1]);
      float value = e[cursor + ((boundary != boundary || rank >= double_bits(double(boundary))) ? 1 : 0)].value;
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
  out[count++] = tail + (fabsf(tail) + 1e-5f);
  return count;
}

// ---------------------------------------------------------------------------
// Data-parallel forms.
// ---------------------------------------------------------------------------

// Where a data-parallel form hands over to the serial definition (counted
// by the test executor).
enum SerialPath : uint32_t { kPruneSerial = 0, kCombineSerial = 1, kPrefixSerial = 2 };

// First index j in [lo, hi) with key(j) > x (hi when none), for
// non-decreasing keys.
template <class Key>
XGBB_HD inline uint32_t upper_bound_by(uint32_t lo, uint32_t hi, float x, Key key) {
  while (lo < hi) {
    const uint32_t mid = lo + (hi - lo) / 2;
    if (x < key(mid)) hi = mid;
    else lo = mid + 1;
  }
  return lo;
}

// Scratch of the parallel operations on up to `cap` entries. `fa` and `fb`
// hold the keys the binary searches probe (rank sums, entry values); the
// kernels place them in shared memory.
struct Work {
  uint32_t* u;  // [cap + 1] per-index words
  uint32_t* v;  // [cap + 1]
  float* f;     // [cap + 1]
  float* fa;    // [cap + 1]
  float* fb;    // [cap + 1]
};

// First index j in [0, n) with v[j] >= x.
XGBB_HD inline uint32_t lower_bound_f(const float* v, uint32_t n, float x) {
  uint32_t lo = 0, hi = n;
  while (lo < hi) {
    const uint32_t mid = lo + (hi - lo) / 2;
    if (v[mid] < x) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

// prune_serial(in, size, capacity) written to `out` (may not alias `in`).
template <class Ex>
XGBB_HD uint32_t prune_par(Ex& ex, const Entry* in, uint32_t size, uint32_t capacity, Entry* out, Work w) {
  if (size <= capacity || capacity <= 1) {
    const uint32_t keep = size <= capacity ? size : capacity;
    ex.for_each(keep, [&](uint32_t i) { out[i] = in[i]; });
    return keep;
  }
  const float begin = in[0].rmax, range = in[size - 1].rmin - begin;
  const uint32_t n = capacity - 1;
  // The binary searches need non-decreasing rank sums s_j = rmax + rmin
  // (j >= 2) and query ranks (range >= 0); otherwise run the serial form.
  uint32_t* bad = w.v;
  float* sums = w.fa;  // s_j, probed by the searches below
  ex.for_each(1, [&](uint32_t) { bad[0] = !(range >= 0.0f); });
  ex.for_each(size, [&](uint32_t j) {
    const float s = in[j].rmax + in[j].rmin;
    sums[j] = s;
    if (s != s || (j >= 3 && s < in[j - 1].rmax + in[j - 1].rmin)) bad[0] = 1;
  });
  if (bad[0]) {
    ex.note(kPruneSerial);
    ex.for_each(size, [&](uint32_t j) { out[j] = in[j]; });
    uint32_t* result = w.v;
    ex.for_each(1, [&](uint32_t) { result[0] = prune_serial(out, size, capacity); });
    return result[0];
  }
  // c_k: the entry chosen for rank k (size when rank k ends the scan).
  uint32_t* chosen = w.u;
  ex.for_each(n, [&](uint32_t k) {
    if (k == 0) {
      chosen[0] = 0;
      return;
    }
    const float rank = 2.0f * (float(k) * range / float(n) + begin);
    const uint32_t j = upper_bound_by(2, size, rank, [&](uint32_t t) { return sums[t]; });
    const uint32_t i = j - 1;  // in [1, size - 1]
    if (i == size - 1) {
      chosen[k] = size;
      return;
    }
    chosen[k] = rank < lower_next(in[i]) + upper_prev(in[i + 1]) ? i : i + 1;
  });
  // Appended: ranks before the end whose choice differs from the previous one.
  uint32_t* pos = w.v;
  ex.for_each(n, [&](uint32_t k) { pos[k] = (k > 0 && chosen[k] < size && chosen[k] != chosen[k - 1]) ? 1u : 0u; });
  const uint32_t appended = ex.scan_exclusive(pos, n, Add32{});
  ex.for_each(n, [&](uint32_t k) {
    if (k == 0) out[0] = in[0];
    else if (chosen[k] < size && chosen[k] != chosen[k - 1]) out[1 + pos[k]] = in[chosen[k]];
  });
  // The last appended entry: the largest choice before the end (choices are
  // non-decreasing), or the first entry.
  uint32_t* last = w.v + n;
  ex.for_each(1, [&](uint32_t) { last[0] = 0; });
  ex.for_each(n, [&](uint32_t k) {
    if (k > 0 && chosen[k] < size && (k + 1 == n || chosen[k + 1] >= size)) last[0] = chosen[k];
  });
  uint32_t count = 1 + appended;
  if (last[0] != size - 1) {
    ex.for_each(1, [&](uint32_t) { out[count] = in[size - 1]; });
    ++count;
  }
  return count;
}

// combine_serial(cur, n, other, m) written to `out` (no aliasing); values in
// each input are strictly increasing (checked; otherwise the serial form).
template <class Ex>
XGBB_HD uint32_t combine_par(Ex& ex, const Entry* cur, uint32_t n, const Entry* other, uint32_t m, Entry* out,
                             Entry* scratch, Work w) {
  if (!m || !n) {
    const Entry* src = m ? other : cur;
    const uint32_t k = m ? m : n;
    ex.for_each(k, [&](uint32_t i) { out[i] = src[i]; });
    return k;
  }
  uint32_t* bad = w.v;
  ex.for_each(1, [&](uint32_t) { bad[0] = 0; });
  ex.for_each(n + m, [&](uint32_t i) {
    const Entry* e = i < n ? cur : other;
    const uint32_t j = i < n ? i : i - n;
    const Entry x = e[j];
    // NaN or a sign bit (negative or -0) anywhere: ties of the running
    // maxima below could then differ in their bits; use the serial form.
    if (x.value != x.value || ((float_bits(x.rmin) | float_bits(x.rmax) | float_bits(x.wmin)) >> 31) ||
        x.rmin != x.rmin || x.rmax != x.rmax || x.wmin != x.wmin)
      bad[0] = 1;
    if (j > 0 && !(e[j - 1].value < x.value)) bad[0] = 1;
  });
  if (bad[0]) {
    ex.note(kCombineSerial);
    ex.for_each(n, [&](uint32_t i) { out[i] = cur[i]; });
    uint32_t* result = w.v;
    ex.for_each(1, [&](uint32_t) { result[0] = combine_serial(out, n, other, m, scratch); });
    return result[0];
  }
  // The values both sides' searches probe.
  float* va = w.fa;
  float* vb = w.fb;
  ex.for_each(n + m, [&](uint32_t i) {
    if (i < n) va[i] = cur[i].value;
    else vb[i - n] = other[i - n].value;
  });
  // Matches: cur[a] equals other[lower_bound(a)].
  uint32_t* match_a = w.u;      // [n] 1 when cur[a] has an equal in other
  uint32_t* match_b = w.u + n;  // [m]
  ex.for_each(n + m, [&](uint32_t i) {
    if (i < n) {
      const uint32_t b = lower_bound_f(vb, m, va[i]);
      match_a[i] = b < m && vb[b] == va[i];
    } else {
      const uint32_t b = i - n;
      const uint32_t a = lower_bound_f(va, n, vb[b]);
      match_b[b] = a < n && va[a] == vb[b];
    }
  });
  ex.scan_exclusive(match_a, n, Add32{});
  const uint32_t pairs = ex.scan_exclusive(match_b, m, Add32{});
  const uint32_t count = n + m - pairs;
  const float tail_a = cur[n - 1].rmax, tail_b = other[m - 1].rmax;
  ex.for_each(n + m, [&](uint32_t i) {
    if (i < n) {
      const uint32_t a = i;
      const Entry x = cur[a];
      const uint32_t b = lower_bound_f(vb, m, x.value);
      const uint32_t at = a + b - match_a[a];
      if (b < m && vb[b] == x.value) {
        const Entry y = other[b];
        scratch[at] = {x.rmin + y.rmin, x.rmax + y.rmax, x.wmin + y.wmin, x.value};
      } else {
        const float prev_b = b ? lower_next(other[b - 1]) : 0.0f;
        const float up = b < m ? upper_prev(other[b]) : tail_b;
        scratch[at] = {x.rmin + prev_b, x.rmax + up, x.wmin, x.value};
      }
    } else {
      const uint32_t b = i - n;
      const Entry y = other[b];
      const uint32_t a = lower_bound_f(va, n, y.value);
      if (a < n && va[a] == y.value) return;  // written by its match
      const uint32_t at = b + a - match_b[b];
      const float prev_a = a ? lower_next(cur[a - 1]) : 0.0f;
      const float up = a < n ? upper_prev(cur[a]) : tail_a;
      scratch[at] = {y.rmin + prev_a, y.rmax + up, y.wmin, y.value};
    }
  });
  // Ranks clamped to be non-decreasing: rmin by a running maximum from 0,
  // rmax by a running maximum (from 0) of max(rmax, rmin + wmin).
  float* f = w.f;
  ex.for_each(count, [&](uint32_t i) { f[i] = scratch[i].rmin; });
  ex.scan_inclusive(f, count, 0.0f, KeepMax{});
  ex.for_each(count, [&](uint32_t i) {
    Entry e = scratch[i];
    e.rmin = f[i];
    out[i] = e;
  });
  ex.for_each(count, [&](uint32_t i) { f[i] = KeepMax{}(out[i].rmax, lower_next(out[i])); });
  ex.scan_inclusive(f, count, 0.0f, KeepMax{});
  ex.for_each(count, [&](uint32_t i) { out[i].rmax = f[i]; });
  return count;
}

// One batch of runs (in row order, `size` of them) to its summary pruned to
// `limit` entries: a stable sort by value, equal values merged (weights added
// in sorted order), prefix sums of the weights. `keys` holds
// pow2_ceil(size) words, `sorted` and `entries` size entries.
XGBB_HD inline uint32_t pow2_ceil(uint32_t x) {
  uint32_t p = 1;
  while (p < x) p <<= 1;
  return p;
}

// Scratch of the radix form of the sort: two key and two 16-bit order
// arrays of `size` entries, then 256 * (warps + 1) counters.
XGBB_HD inline size_t radix_sort_bytes(uint32_t size, uint32_t warps) {
  return size_t(size) * 12 + size_t(256) * (warps + 1) * 4;
}

template <class Ex>
XGBB_HD uint32_t summarize_par(Ex& ex, const Run* runs, uint32_t size, uint32_t limit, unsigned long long* keys,
                               Run* sorted, Entry* entries, Entry* out, Work w, unsigned char* radix = nullptr) {
  if (!size) return 0;
  if (radix && size < 65536) {
    // Stable radix sort of the order-preserving value keys.
    uint32_t* k32 = reinterpret_cast<uint32_t*>(radix);
    uint16_t* o16 = reinterpret_cast<uint16_t*>(k32 + 2 * size);
    uint32_t* cnt = reinterpret_cast<uint32_t*>(radix + size_t(size) * 12);
    ex.for_each(size, [&](uint32_t i) { k32[i] = order_key(runs[i].v); });
    ex.stable_order(k32, o16, size, k32 + size, o16 + size, cnt);
    ex.for_each(size, [&](uint32_t i) { sorted[i] = runs[o16[i]]; });
  } else {
    const uint32_t p = pow2_ceil(size);
    ex.for_each(p, [&](uint32_t i) {
      keys[i] = i < size ? ((unsigned long long)order_key(runs[i].v) << 32) | i : ~0ull;
    });
    // Bitonic sort, ascending; keys are distinct, so the order is the stable
    // order by value.
    for (uint32_t k = 2; k <= p; k <<= 1)
      for (uint32_t j = k >> 1; j > 0; j >>= 1)
        ex.for_each(p / 2, [&](uint32_t t) {
          // Pair (i, l), i < l: 2j * (t / j) + t % j, with j a power of two.
          const uint32_t i = ((t & ~(j - 1)) << 1) | (t & (j - 1)), l = i + j;
          const bool up = (i & k) == 0;
          const unsigned long long a = keys[i], b = keys[l];
          if ((a > b) == up) {
            keys[i] = b;
            keys[l] = a;
          }
        });
    ex.for_each(size, [&](uint32_t i) { sorted[i] = runs[uint32_t(keys[i] & 0xffffffffu)]; });
  }
  // Groups of equal values: head flags, group ids, weights summed in order.
  uint32_t* head = w.u;
  ex.for_each(size, [&](uint32_t i) { head[i] = (i == 0 || !(sorted[i].v == sorted[i - 1].v)) ? 1u : 0u; });
  float* gw = w.f;
  uint32_t* exact = w.v + size;  // 1 while every group weight is an integer in [0, 2^24]
  ex.for_each(1, [&](uint32_t) { exact[0] = 1; });
  ex.for_each(size, [&](uint32_t i) {
    if (!head[i]) return;
    float s = sorted[i].w;
    for (uint32_t j = i + 1; j < size && sorted[j].v == sorted[i].v; ++j) s = s + sorted[j].w;
    gw[i] = s;
    if (!(s >= 0.0f && s <= 16777216.0f && s == floorf(s))) exact[0] = 0;
  });
  const uint32_t groups = ex.scan_exclusive(head, size, Add32{});  // head[i] = group index of i
  // Compact the group weights and values: entries[g].wmin, .value.
  ex.for_each(size, [&](uint32_t i) {
    if (i == 0 || !(sorted[i].v == sorted[i - 1].v)) {
      entries[head[i]].wmin = gw[i];
      entries[head[i]].value = sorted[i].v;
    }
  });
  // Prefix sums of the group weights: exact integers when the weights are
  // integers summing to at most 2^24 (every float partial sum is then exact),
  // else the serial float sum.
  uint32_t* iw = w.u;
  bool integer = exact[0] != 0;
  if (integer) {
    ex.for_each(groups, [&](uint32_t g) { iw[g] = uint32_t(entries[g].wmin); });
    integer = ex.scan_exclusive(iw, groups, SatAdd24{}) <= (1u << 24);
  }
  if (integer) {
    ex.for_each(groups, [&](uint32_t g) {
      const float total = float(iw[g]);
      entries[g].rmin = total;
      entries[g].rmax = total + entries[g].wmin;
    });
  } else {
    ex.note(kPrefixSerial);
    ex.for_each(1, [&](uint32_t) {
      float total = 0.0f;
      for (uint32_t g = 0; g < groups; ++g) {
        entries[g].rmin = total;
        entries[g].rmax = total + entries[g].wmin;
        total = total + entries[g].wmin;
      }
    });
  }
  return prune_par(ex, entries, groups, limit, out, w);
}

// ---------------------------------------------------------------------------
// Runs of one feature, a chunk of rows at a time (sketch_input_*,
// kernels/quantile.metal.h:19-140): values with a non-zero weight, NaN
// skipped, -0 read as +0; consecutive equal values (skipping the rows in
// between that are not used) form one run whose weight is the row count
// capped at 2^24, or the float sum of the weights in row order.
// ---------------------------------------------------------------------------
struct RunCarry {
  uint32_t has_prev, runs, elements, nonmissing;
  float prev, w;  // value and weight so far of the last run
  float first;    // value of the first used row (set with has_prev)
};

// How runs_chunk writes a chunk's runs: `write` false only counts them (the
// first pass over a segment of rows); run indices below `own_from` belong to
// an earlier segment, and a weight for such a run goes to *cont_w instead.
struct RunOut {
  Run* runs;
  bool write;
  uint32_t own_from;
  float* cont_w;
};

// Per-row scratch of a chunk of up to `cap` rows.
struct ChunkWork {
  float* v;
  float* w;
  uint32_t* valid;
  uint32_t* last;   // 1 + index of the last used row at or before i (0: none)
  uint32_t* start;  // 1 when row i starts a run
  uint32_t* rank;   // runs started before row i in the chunk
  uint32_t* count;  // row counts (scratch for sums)
  float* last_w;    // [1] weight of the chunk's last run
};

// `load(i)` gives the (value, weight) of row i of the chunk; runs go to
// runs[carry.runs ...]; `carry` is updated for the next chunk.
template <class Ex, class Load>
XGBB_HD void runs_chunk(Ex& ex, Load load, uint32_t n, bool unit, RunCarry& carry, RunOut out, ChunkWork c) {
  if (!n) return;
  Run* runs = out.runs;
  ex.for_each(n, [&](uint32_t i) {
    float v, w;
    load(i, v, w);
    const bool nonmissing = !(v != v);
    const bool used = nonmissing && (float_bits(w) & 0x7fffffffu) != 0;
    if (used && v == 0.0f) v = 0.0f;
    c.v[i] = v;
    c.w[i] = w;
    c.valid[i] = used;
    c.last[i] = used ? i + 1 : 0u;
    c.count[i] = nonmissing;
  });
  const uint32_t nonmissing = ex.scan_exclusive(c.count, n, Add32{});
  ex.scan_inclusive(c.last, n, 0u, MaxU32{});
  const uint32_t has_prev = carry.has_prev, runs0 = carry.runs;
  const float prev0 = carry.prev, w0 = carry.w;
  ex.for_each(n, [&](uint32_t i) {
    uint32_t s = 0;
    if (c.valid[i]) {
      const uint32_t j = i ? c.last[i - 1] : 0u;
      const bool has = j ? true : has_prev != 0;
      const float prev = j ? c.v[j - 1] : prev0;
      s = (!has || !(c.v[i] == prev)) ? 1u : 0u;
    }
    c.start[i] = s;
    c.rank[i] = s;
    c.count[i] = c.valid[i];
  });
  const uint32_t started = ex.scan_exclusive(c.rank, n, Add32{});
  const uint32_t used = ex.scan_exclusive(c.count, n, Add32{});
  // Each run's rows are summed in order by the thread of its first row in
  // the chunk (a run continued from the previous chunk starts from the
  // carried weight).
  ex.for_each(n, [&](uint32_t i) {
    if (!c.valid[i]) return;
    const bool continues = !c.start[i] && (i ? c.last[i - 1] : 0u) == 0;
    if (!c.start[i] && !continues) return;
    float acc;
    if (c.start[i]) acc = unit ? 1.0f : c.w[i];
    else acc = unit ? fminf(w0 + 1.0f, 16777216.0f) : w0 + c.w[i];
    uint32_t j = i + 1;
    for (; j < n; ++j) {
      if (!c.valid[j]) continue;
      if (c.start[j]) break;
      acc = unit ? fminf(acc + 1.0f, 16777216.0f) : acc + c.w[j];
    }
    const uint32_t run = c.start[i] ? runs0 + c.rank[i] : runs0 - 1;
    if (out.write) {
      if (run < out.own_from) {
        out.cont_w[0] = acc;
      } else {
        if (c.start[i]) runs[run].v = c.v[i];
        runs[run].w = acc;
      }
    }
    if (j == n) c.last_w[0] = acc;
  });
  const uint32_t last = c.last[n - 1];
  if (!has_prev && last) {
    // The first used row of the chunk is the first of the rows so far.
    ex.for_each(n, [&](uint32_t i) {
      if (c.valid[i] && (i == 0 || c.last[i - 1] == 0)) carry.first = c.v[i];
    });
  }
  ex.for_each(1, [&](uint32_t) {
    carry.nonmissing += nonmissing;
    carry.elements += used;
    if (last) {
      carry.has_prev = 1;
      carry.prev = c.v[last - 1];
      carry.runs = runs0 + started;
      carry.w = c.last_w[0];
    }
  });
}

template <class Ex, class Load>
XGBB_HD void runs_chunk(Ex& ex, Load load, uint32_t n, bool unit, RunCarry& carry, Run* runs, ChunkWork c) {
  runs_chunk(ex, load, n, unit, carry, RunOut{runs, true, 0u, nullptr}, c);
}

// ---------------------------------------------------------------------------
// A feature's runs from segments of rows processed at the same time. Pass 1
// counts each segment's runs from an empty carry (runs_chunk with write
// false), keeping its RunCarry. link_segments then walks the segments in
// order: it gives each segment the carry the single pass would reach at its
// first row (the run count so far, the last used value and the weight of the
// run still open there) and notes which segments continue the previous
// segment's last run. Pass 2 writes every segment's runs from that carry; a
// continuing run's weight lands in cont_w, and finish_links stores those
// weights in segment order, so a run spanning several segments keeps the
// weight of its last segment. The runs are those of the single pass.
//
// A continuation's weight is min(prev + count, 2^24) with unit weights. With
// weights, a segment whose used rows all continue the previous run passes on
// a float sum that the single pass forms row by row, so link_segments forms
// it the same way from the segment's rows (`load_w(s, k, v, w)`: row k of
// segment s; `rows_of(s)`: its row count).
// ---------------------------------------------------------------------------
struct SegmentLink {
  RunCarry in;    // the carry at the segment's first row
  uint32_t cont;  // 1 when the segment's first run continues the previous one
  float cont_w;   // that run's weight after this segment (written by pass 2)
};

template <class LoadW, class RowsOf>
XGBB_HD void link_segments(const RunCarry* pass1, uint32_t nseg, bool unit, SegmentLink* link, LoadW load_w,
                           RowsOf rows_of, uint32_t* stats) {
  RunCarry cur{0, 0, 0, 0, 0.0f, 0.0f, 0.0f};
  for (uint32_t s = 0; s < nseg; ++s) {
    const RunCarry& p = pass1[s];
    link[s].in = cur;
    link[s].cont = 0;
    link[s].cont_w = 0.0f;
    cur.elements += p.elements;
    cur.nonmissing += p.nonmissing;
    if (!p.has_prev) continue;  // no used row: the open run carries over
    const bool cont = cur.has_prev && p.first == cur.prev;
    link[s].cont = cont;
    cur.runs += p.runs - (cont ? 1u : 0u);
    if (cont && p.runs == 1) {
      // Every used row of the segment extends the open run.
      if (unit) {
        cur.w = fminf(cur.w + p.w, 16777216.0f);
      } else {
        float acc = cur.w;
        for (uint32_t k = 0, n = rows_of(s); k < n; ++k) {
          float v, w;
          load_w(s, k, v, w);
          if (v == v && (float_bits(w) & 0x7fffffffu) != 0) acc = acc + w;
        }
        cur.w = acc;
      }
    } else {
      cur.w = p.w;
    }
    cur.has_prev = 1;
    cur.prev = p.prev;
  }
  stats[0] = cur.runs;
  stats[1] = cur.elements;
  stats[2] = cur.nonmissing;
}

XGBB_HD inline void finish_links(const SegmentLink* link, uint32_t nseg, Run* runs) {
  for (uint32_t s = 0; s < nseg; ++s)
    if (link[s].cont) runs[link[s].in.runs - 1].w = link[s].cont_w;
}

// ---------------------------------------------------------------------------
// One feature's batch summaries reduced level by level, then its cuts
// (sketch_reduce_*, kernels/quantile.metal.h:317-352, and src/quantile.cpp).
// ---------------------------------------------------------------------------
struct ReduceWork {
  Entry* resident;   // [levels][limit]
  uint32_t* counts;  // [levels]
  Entry* a;          // three buffers of 2 * limit + 1 entries
  Entry* b;
  Entry* scratch;
  Work w;            // 2 * limit + 2 words each
  uint32_t* size;    // [1]
};

// The end of a feature's reduction: the resident summary of every level
// (`resident(level, count)`, count 0 when the level holds none) merged from
// the lowest level up, each merge pruned to max(budget, limit), then pruned
// to `budget` and turned into cuts; returns the cut count.
template <class Ex, class Resident>
XGBB_HD uint32_t finish_reduce(Ex& ex, uint32_t levels, uint32_t limit, uint32_t budget, uint32_t max_bin,
                               ReduceWork r, Resident resident, float* cuts) {
  uint32_t n = 0;
  const uint32_t keep = budget > limit ? budget : limit;
  for (uint32_t level = 0; level < levels; ++level) {
    uint32_t m = 0;
    const Entry* res = resident(level, m);
    n = combine_par(ex, r.a, n, res, m, r.b, r.scratch, r.w);
    n = prune_par(ex, r.b, n, keep, r.a, r.w);
  }
  n = prune_par(ex, r.a, n, budget, r.b, r.w);
  ex.for_each(1, [&](uint32_t) { r.size[0] = select_cuts(r.b, n, max_bin, cuts); });
  return r.size[0];
}

// summaries[k * limit ...] holds batch k's sizes[k] entries. Writes at most
// max_bin cuts to `cuts` and returns their count.
template <class Ex>
XGBB_HD uint32_t reduce_feature(Ex& ex, const Entry* summaries, const uint32_t* sizes, uint32_t nbatch,
                                uint32_t limit, uint32_t budget, uint32_t levels, uint32_t max_bin, ReduceWork r,
                                float* cuts) {
  ex.for_each(levels, [&](uint32_t l) { r.counts[l] = 0; });
  for (uint32_t k = 0; k < nbatch; ++k) {
    const uint32_t size = sizes[k];
    // The batch summary is pruned already; from level to level the current
    // summary is pruned, then merged with that level's resident summary.
    uint32_t n = prune_par(ex, summaries + size_t(k) * limit, size, limit, r.a, r.w);
    uint32_t level = 0;
    for (;;) {
      n = prune_par(ex, r.a, n, limit, r.b, r.w);
      n = combine_par(ex, r.b, n, r.resident + size_t(level) * limit, r.counts[level], r.a, r.scratch, r.w);
      ex.for_each(1, [&](uint32_t) { r.counts[level] = 0; });
      if (n <= limit) break;
      ++level;
    }
    Entry* dst = r.resident + size_t(level) * limit;
    ex.for_each(n, [&](uint32_t i) { dst[i] = r.a[i]; });
    ex.for_each(1, [&](uint32_t) { r.counts[level] = n; });
  }
  return finish_reduce(
      ex, levels, limit, budget, max_bin, r,
      [&](uint32_t level, uint32_t& count) {
        count = r.counts[level];
        return static_cast<const Entry*>(r.resident + size_t(level) * limit);
      },
      cuts);
}

// Batches and levels of one feature (src/quantile.cpp:98-127): batches of
// 2 * limit runs; `levels` resident summaries of `limit` entries.
struct FeaturePlan {
  uint32_t runs, limit, budget, capacity, nbatch, levels;
};
inline FeaturePlan plan_feature(uint32_t max_bin, uint32_t runs, uint32_t elements, uint32_t nonmissing) {
  FeaturePlan p;
  p.runs = runs;
  p.limit = budget_for(max_bin, nonmissing);
  p.budget = budget_for(max_bin, elements);
  p.capacity = 2 * p.limit;
  p.nbatch = uint32_t((uint64_t(runs) + p.capacity - 1) / p.capacity);
  p.levels = 1;
  for (uint32_t c = p.nbatch > 1 ? p.nbatch : 1u; c; c >>= 1) ++p.levels;
  return p;
}

// Scratch of one batch summary of at most `capacity` runs.
struct BatchWork {
  unsigned long long* keys;  // [pow2_ceil(capacity)]
  Run* sorted;               // [capacity]
  Entry* entries;            // [capacity]
  Work w;                    // capacity + 2 words each
};

// ---------------------------------------------------------------------------
// The GPU sketch's plan for a group of features and the layouts of its
// scratch (sketch_gpu.cu), shared with the tests.
// ---------------------------------------------------------------------------

// One batch: runs[run_begin, run_begin + size) of a feature, summarised into
// `limit` entries at summaries[summary_at]; its size lands in sizes[size_slot].
struct BatchTask {
  unsigned long long run_begin, summary_at;
  uint32_t size, limit, size_slot, pad;
};
// One feature's reduction: its batch summaries from summaries[summary_at]
// (sizes from sizes[first_size]) and its work area at work + work_at.
struct ReduceTask {
  unsigned long long summary_at, work_at;
  uint32_t first_size, nbatch, limit, budget, levels, feature;
};

// Entries of the largest summary a reduction step holds.
XGBB_HD inline uint32_t reduce_big(uint32_t limit, uint32_t budget) {
  return 2 * (limit > budget ? limit : budget) + 2;
}

inline size_t reduce_work_bytes(uint32_t limit, uint32_t budget, uint32_t levels) {
  const size_t big = reduce_big(limit, budget);
  const size_t bytes = (size_t(limit) * levels + 3 * big) * sizeof(Entry) + 5 * big * 4 + (size_t(levels) + 1) * 4;
  return (bytes + 255) / 256 * 256;
}

XGBB_HD inline ReduceWork reduce_work_at(unsigned char* base, uint32_t limit, uint32_t budget, uint32_t levels) {
  const uint32_t big = reduce_big(limit, budget);
  ReduceWork r;
  r.resident = reinterpret_cast<Entry*>(base);
  r.a = r.resident + size_t(limit) * levels;
  r.b = r.a + big;
  r.scratch = r.b + big;
  r.w.u = reinterpret_cast<uint32_t*>(r.scratch + big);
  r.w.v = r.w.u + big;
  r.w.f = reinterpret_cast<float*>(r.w.v + big);
  r.w.fa = r.w.f + big;
  r.w.fb = r.w.fa + big;
  r.counts = reinterpret_cast<uint32_t*>(r.w.fb + big);
  r.size = r.counts + levels;
  return r;
}

// Bytes of one batch's scratch for batches of at most `cap` runs.
inline size_t batch_scratch_bytes(uint32_t cap) {
  const size_t bytes = size_t(pow2_ceil(cap)) * 8 + size_t(cap) * (sizeof(Run) + sizeof(Entry)) + 5 * (size_t(cap) + 2) * 4;
  return (bytes + 255) / 256 * 256;
}

XGBB_HD inline BatchWork batch_work_at(unsigned char* base, uint32_t cap) {
  BatchWork bw;
  bw.keys = reinterpret_cast<unsigned long long*>(base);
  bw.sorted = reinterpret_cast<Run*>(bw.keys + pow2_ceil(cap));
  bw.entries = reinterpret_cast<Entry*>(bw.sorted + cap);
  bw.w.u = reinterpret_cast<uint32_t*>(bw.entries + cap);
  bw.w.v = bw.w.u + cap + 2;
  bw.w.f = reinterpret_cast<float*>(bw.w.v + cap + 2);
  bw.w.fa = bw.w.f + cap + 2;
  bw.w.fb = bw.w.fa + cap + 2;
  return bw;
}

// Tasks of `nf` features (feature f0 + j has its runs at runs[j * rows]) from
// their (runs, elements, nonmissing) statistics.
struct GroupPlan {
  std::vector<BatchTask> tasks;
  std::vector<ReduceTask> reduce;
  uint64_t summary_entries = 0, work_bytes = 0;
  uint32_t sizes = 0, cap = 2;
};
inline GroupPlan plan_group(const uint32_t* stats, uint32_t nf, uint32_t f0, uint32_t rows, uint32_t max_bin) {
  GroupPlan g;
  for (uint32_t j = 0; j < nf; ++j) {
    const FeaturePlan p = plan_feature(max_bin, stats[3 * j], stats[3 * j + 1], stats[3 * j + 2]);
    g.reduce.push_back(ReduceTask{g.summary_entries, g.work_bytes, g.sizes, p.nbatch, p.limit, p.budget, p.levels,
                                  f0 + j});
    for (uint32_t k = 0; k < p.nbatch; ++k) {
      const uint64_t begin = uint64_t(k) * p.capacity;
      const uint32_t size = uint32_t(p.runs - begin < p.capacity ? p.runs - begin : p.capacity);
      g.tasks.push_back(BatchTask{uint64_t(j) * rows + begin, g.summary_entries + uint64_t(k) * p.limit, size,
                                  p.limit, g.sizes + k, 0});
      if (size > g.cap) g.cap = size;
    }
    g.summary_entries += uint64_t(p.nbatch > 1 ? p.nbatch : 1u) * p.limit;
    g.sizes += p.nbatch > 1 ? p.nbatch : 1u;
    g.work_bytes += reduce_work_bytes(p.limit, p.budget, p.levels);
  }
  return g;
}

// ---------------------------------------------------------------------------
// The reduction as a tree of merges. reduce_feature inserts batch summaries
// one by one: each is merged with the summary held at level 0, the result
// (pruned to `limit`) with the one held at level 1, and so on, a binary
// counter. Whenever every such merge yields more than `limit` entries, node
// i of level l + 1 is prune(combine(node 2i + 1, node 2i), limit) over the
// nodes of level l (node 2i + 1 the newer), the nodes left over at odd
// counts are the summaries the counter holds at the end, and finish_reduce
// over them gives the same cuts. All merges of a level run at once, across
// features. A merge that yields `limit` entries or fewer marks its feature
// irregular (the counter would have kept that result at its level); such a
// feature takes reduce_feature instead, whose steps are then cheap.
// ---------------------------------------------------------------------------
struct MergeTask {
  unsigned long long older_at, newer_at, out_at;  // entry offsets
  uint32_t older_size, newer_size, out_size;       // size slots
  uint32_t limit, local;                           // local: feature index within the group
};
struct FinishRes {
  unsigned long long at;
  uint32_t size_slot, present;
};
struct FinishTask {
  uint32_t feature, local, limit, budget, levels, res_begin;
  unsigned long long work_at;
};
struct TreePlan {
  std::vector<std::vector<MergeTask>> levels;  // the merges of level 1, 2, ...
  std::vector<FinishTask> finish;
  std::vector<FinishRes> res;
  uint64_t entries = 0;  // summary entries including the tree's nodes
  uint32_t sizes = 0;    // size slots including the tree's nodes
};

inline TreePlan plan_tree(const GroupPlan& g) {
  TreePlan t;
  t.entries = g.summary_entries;
  t.sizes = g.sizes;
  for (uint32_t j = 0; j < g.reduce.size(); ++j) {
    const ReduceTask& rt = g.reduce[j];
    struct Node {
      unsigned long long at;
      uint32_t slot;
    };
    std::vector<Node> prev;
    for (uint32_t k = 0; k < rt.nbatch; ++k)
      prev.push_back({rt.summary_at + uint64_t(k) * rt.limit, rt.first_size + k});
    std::vector<FinishRes> res(rt.levels, FinishRes{0, 0, 0});
    uint32_t level = 0;
    while (prev.size() >= 2) {
      if (prev.size() & 1) res[level] = FinishRes{prev.back().at, prev.back().slot, 1};
      if (t.levels.size() <= level) t.levels.resize(level + 1);
      std::vector<Node> cur;
      for (size_t i = 0; i + 1 < prev.size(); i += 2) {
        const Node out{t.entries, t.sizes};
        t.entries += rt.limit;
        t.sizes += 1;
        t.levels[level].push_back(MergeTask{prev[i].at, prev[i + 1].at, out.at, prev[i].slot, prev[i + 1].slot,
                                            out.slot, rt.limit, j});
        cur.push_back(out);
      }
      prev.swap(cur);
      ++level;
    }
    if (prev.size() == 1) res[level] = FinishRes{prev[0].at, prev[0].slot, 1};
    t.finish.push_back(FinishTask{rt.feature, j, rt.limit, rt.budget, rt.levels, uint32_t(t.res.size()), rt.work_at});
    t.res.insert(t.res.end(), res.begin(), res.end());
  }
  return t;
}

// Scratch of one merge: the merged summary, the combine's unclamped
// entries, and the per-index words (the searched keys come separately).
struct MergeWork {
  Entry* merged;
  Entry* scratch;
  Work w;
};
inline size_t merge_scratch_bytes(uint32_t big) {
  return (size_t(big) * 2 * sizeof(Entry) + size_t(big) * 5 * 4 + 255) / 256 * 256;
}
XGBB_HD inline MergeWork merge_work_at(unsigned char* base, uint32_t big) {
  MergeWork m;
  m.merged = reinterpret_cast<Entry*>(base);
  m.scratch = m.merged + big;
  m.w.u = reinterpret_cast<uint32_t*>(m.scratch + big);
  m.w.v = m.w.u + big;
  m.w.f = reinterpret_cast<float*>(m.w.v + big);
  m.w.fa = m.w.f + big;
  m.w.fb = m.w.fa + big;
  return m;
}

// One tree merge; sets irregular[task.local] when the combine keeps `limit`
// entries or fewer.
template <class Ex>
XGBB_HD void merge_node(Ex& ex, const MergeTask& t, Entry* entries, uint32_t* sizes, uint32_t* irregular,
                        MergeWork m) {
  const uint32_t n = combine_par(ex, entries + t.newer_at, sizes[t.newer_size], entries + t.older_at,
                                 sizes[t.older_size], m.merged, m.scratch, m.w);
  const uint32_t kept = prune_par(ex, m.merged, n, t.limit, entries + t.out_at, m.w);
  ex.for_each(1, [&](uint32_t) {
    sizes[t.out_size] = kept;
    if (n <= t.limit) irregular[t.local] = 1;
  });
}

// A regular feature's cuts from the tree's left-over nodes.
template <class Ex>
XGBB_HD uint32_t finish_tree(Ex& ex, const FinishTask& t, const FinishRes* res, const Entry* entries,
                             const uint32_t* sizes, uint32_t max_bin, ReduceWork r, float* cuts) {
  return finish_reduce(
      ex, t.levels, t.limit, t.budget, max_bin, r,
      [&](uint32_t level, uint32_t& count) {
        const FinishRes& x = res[t.res_begin + level];
        count = x.present ? sizes[x.size_slot] : 0u;
        return entries + x.at;
      },
      cuts);
}

}  // namespace sketch
}  // namespace xgbb
