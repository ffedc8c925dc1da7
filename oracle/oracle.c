/* CPU oracle for histogram tree training -- see oracle.h.
 *
 * TEST INFRASTRUCTURE ONLY: the bit-exact checker for the CUDA product, never
 * part of it. Single-threaded, IEEE-754 binary32/binary64 arithmetic with no
 * contraction (built with -ffp-contract=off) and gradual underflow.
 *
 * Reference semantics restated here (paths inside tabulai/xgboost-metal):
 *   cuts        kernels/quantile.metal.h:19-411, src/quantile.cpp:11-213
 *   bins        kernels/boost.metal:461-499, kernels/float_order.metal.h:1-33
 *   gradients   kernels/boost.metal:553-601
 *   quantise    kernels/gradient_quantization.metal.h:1-67,
 *               kernels/objectives.metal.h:59-67, kernels/boost.metal:605-657
 *   histograms  kernels/boost.metal:700-733, kernels/histogram_missing.metal.h
 *   split scan  kernels/boost.metal:902-1005, kernels/scalar_gain.metal.h:1-103,
 *               kernels/split_statistics.metal.h:1-38
 *   selection   kernels/boost.metal:1245-1265
 *   driver      kernels/tree_driver.metal.h:28-94, src/tree.cpp:1663-1717
 *   partition   kernels/boost.metal:1325-1329 (bin form :1383-1389)
 *   margins     kernels/boost.metal:1738-1765, src/learner.cpp:933-976
 *   base score  kernels/boost.metal:356-420, src/objectives.cpp:17-41
 *
 * The reference evaluates binary64 in software (kernels/cox_arithmetic.metal.h)
 * because Metal has no fp64; every such operation is an IEEE binary64 add,
 * multiply, divide or fma with round-to-nearest-even, so native double
 * arithmetic in the same order gives the same bits. Comparisons the reference
 * makes through an order key for subnormals (kernels/float_order.metal.h) are
 * plain IEEE comparisons here, which agree because nothing flushes to zero.
 *
 * Where this oracle defines its own semantics (the reference's output depends
 * on Metal-specific transcendentals or on an unstable sort), it says [ours].
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "det_math.h"

static uint32_t f32_bits(float v) {
  uint32_t b;
  memcpy(&b, &v, 4);
  return b;
}
static uint64_t f64_bits(double v) {
  uint64_t b;
  memcpy(&b, &v, 8);
  return b;
}
static float f32_from(uint32_t b) {
  float v;
  memcpy(&v, &b, 4);
  return v;
}

/* ------------------------------------------------------------------------ */
/* Cuts: weighted quantile summaries (kernels/quantile.metal.h).             */
/* ------------------------------------------------------------------------ */

typedef struct { float v, w; } orc_run;
typedef struct { float rmin, rmax, wmin, value; } orc_entry;

/* src/quantile.cpp:11-20 */
static uint32_t sketch_budget(uint32_t bins, uint32_t count) {
  if (!count) return 1;
  double epsilon = 1.0 / (double)(bins < count ? bins : count);
  for (uint32_t level = 1; level < 32; ++level) {
    uint64_t limit = (uint64_t)ceil(level / (epsilon / 2.0)) + 1;
    if (limit > count) limit = count;
    if (((uint64_t)1 << level) * limit >= count) return (uint32_t)limit;
  }
  return count;
}

static float min_next(orc_entry e) { return e.rmin + e.wmin; }
static float max_previous(orc_entry e) { return e.rmax - e.wmin; }

/* sketch_prune_serial, kernels/quantile.metal.h:192-214 */
static uint32_t sketch_prune(orc_entry* e, uint32_t size, uint32_t capacity) {
  if (size <= capacity) return size;
  if (!capacity) return 0;
  if (capacity == 1) return 1;
  float begin = e[0].rmax, range = e[size - 1].rmin - begin;
  uint32_t n = capacity - 1, count = 1, i = 1, last = 0;
  orc_entry tail = e[size - 1], left = e[1], right = e[2];
  for (uint32_t k = 1; k < n; ++k) {
    float rank = 2.0f * ((float)k * range / (float)n + begin);
    while (i < size - 1 && rank >= right.rmax + right.rmin) {
      ++i;
      left = right;
      if (i < size - 1) right = e[i + 1];
    }
    if (i == size - 1) break;
    if (rank < min_next(left) + max_previous(right)) {
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

/* sketch_combine_serial, kernels/quantile.metal.h:266-315 */
static uint32_t sketch_combine(orc_entry* cur, uint32_t n, const orc_entry* other, uint32_t m,
                               orc_entry* scratch) {
  if (!m) return n;
  if (!n) {
    memcpy(cur, other, m * sizeof(orc_entry));
    return m;
  }
  uint32_t a = 0, b = 0, count = 0;
  float prev_a = 0, prev_b = 0;
  while (a < n && b < m) {
    orc_entry x = cur[a], y = other[b], r;
    if (x.value == y.value) {
      r.rmin = x.rmin + y.rmin; r.rmax = x.rmax + y.rmax; r.wmin = x.wmin + y.wmin; r.value = x.value;
      prev_a = min_next(x);
      prev_b = min_next(y);
      ++a;
      ++b;
    } else if (x.value < y.value) {
      r.rmin = x.rmin + prev_b; r.rmax = x.rmax + max_previous(y); r.wmin = x.wmin; r.value = x.value;
      prev_a = min_next(x);
      ++a;
    } else {
      r.rmin = y.rmin + prev_a; r.rmax = y.rmax + max_previous(x); r.wmin = y.wmin; r.value = y.value;
      prev_b = min_next(y);
      ++b;
    }
    scratch[count++] = r;
  }
  float tail_a = cur[n - 1].rmax, tail_b = other[m - 1].rmax;
  while (a < n) {
    orc_entry x = cur[a++];
    x.rmin = x.rmin + prev_b;
    x.rmax = x.rmax + tail_b;
    scratch[count++] = x;
  }
  while (b < m) {
    orc_entry y = other[b++];
    y.rmin = y.rmin + prev_a;
    y.rmax = y.rmax + tail_a;
    scratch[count++] = y;
  }
  float prev_min = 0, prev_max = 0;
  for (uint32_t i = 0; i < count; ++i) {
    orc_entry e = scratch[i];
    if (e.rmin < prev_min) e.rmin = prev_min;
    else prev_min = e.rmin;
    if (e.rmax < prev_max) e.rmax = prev_max;
    if (e.rmax < min_next(e)) e.rmax = min_next(e);
    prev_max = e.rmax;
    cur[i] = e;
  }
  return count;
}

/* Stable merge sort of runs by value. [ours] Ties keep input (row) order;
 * the reference re-sorts ties of unequal bits (+0/-0) or, with user weights,
 * unequal weights with a libc++-style introsort (kernels/sketch_sort.metal.h:124)
 * -- only those inputs can give a different summary. */
static void sort_runs(orc_run* v, orc_run* tmp, uint32_t n) {
  for (uint32_t width = 1; width < n; width *= 2) {
    for (uint32_t lo = 0; lo < n; lo += 2 * width) {
      uint32_t mid = lo + width < n ? lo + width : n;
      uint32_t hi = lo + 2 * width < n ? lo + 2 * width : n;
      uint32_t i = lo, j = mid, k = lo;
      while (i < mid && j < hi) tmp[k++] = (v[j].v < v[i].v) ? v[j++] : v[i++];
      while (i < mid) tmp[k++] = v[i++];
      while (j < hi) tmp[k++] = v[j++];
    }
    memcpy(v, tmp, n * sizeof(orc_run));
  }
}

uint32_t orc_cut_stride(uint32_t rows, uint32_t max_bin) {
  /* histogram_bins, src/data.cpp:1232 */
  uint32_t b = max_bin < rows ? max_bin : rows;
  return b ? b : 1;
}

static void feature_cuts(const float* X, uint32_t rows, uint32_t cols, uint32_t f,
                         const float* weights, uint32_t max_bin, float* out, uint32_t* count_out,
                         float* minimum) {
  int unit = weights == NULL;
  orc_run* runs = (orc_run*)malloc(((size_t)rows + 1) * sizeof(orc_run));
  uint32_t nruns = 0, elements = 0, nonmissing = 0;
  float previous = 0;
  /* Runs of equal consecutive valid values in row order
   * (sketch_input_blocks..sketch_input_runs, kernels/quantile.metal.h:19-140). */
  for (uint32_t r = 0; r < rows; ++r) {
    float v = X[(size_t)r * cols + f];
    float w = unit ? 1.0f : weights[r];
    nonmissing += !isnan(v);
    if (isnan(v) || (f32_bits(w) & 0x7fffffffu) == 0) continue;
    /* [ours] -0 reads as +0, so a summary never depends on which signed zero
     * came first (the reference keeps the first one's sign). */
    if (v == 0.0f) v = 0.0f;
    ++elements;
    if (!nruns || !(v == previous)) {
      runs[nruns].v = v;
      runs[nruns].w = unit ? 1.0f : w;
      ++nruns;
    } else if (unit) {
      float c = runs[nruns - 1].w + 1.0f;
      runs[nruns - 1].w = c > 16777216.0f ? 16777216.0f : c;
    } else {
      runs[nruns - 1].w = runs[nruns - 1].w + w;
    }
    previous = v;
  }
  *minimum = -INFINITY;
  uint32_t limit = sketch_budget(max_bin, nonmissing);
  uint32_t budget = sketch_budget(max_bin, elements);
  uint64_t capacity = 2ull * limit;
  uint32_t nbatch = (uint32_t)((nruns + capacity - 1) / capacity);
  uint32_t levels = 1;
  {
    uint32_t c = nbatch ? nbatch : 1;
    while (c) {
      ++levels;
      c >>= 1;
    }
  }
  orc_entry* resident = (orc_entry*)calloc((size_t)limit * levels, sizeof(orc_entry));
  orc_entry* current = (orc_entry*)calloc(2 * (size_t)limit + 1, sizeof(orc_entry));
  orc_entry* scratch = (orc_entry*)calloc(2 * (size_t)limit + 1, sizeof(orc_entry));
  orc_entry* summary = (orc_entry*)calloc(capacity + 1, sizeof(orc_entry));
  orc_run* tmp = (orc_run*)malloc((capacity + 1) * sizeof(orc_run));
  uint32_t counts[64] = {0};
  /* sketch_summarize_ordered per batch, then sketch_reduce_serial
   * (kernels/quantile.metal.h:216-240, 317-352). */
  for (uint32_t batch = 0; batch < nbatch; ++batch) {
    uint32_t begin = (uint32_t)(batch * capacity);
    uint32_t size = (uint32_t)((nruns - begin) < capacity ? (nruns - begin) : capacity);
    orc_run* src = runs + begin;
    sort_runs(src, tmp, size);
    uint32_t n = 0;
    float total = 0;
    for (uint32_t i = 0; i < size;) {
      orc_run value = src[i];
      uint32_t j = i + 1;
      while (j < size && src[j].v == value.v) value.w = value.w + src[j++].w;
      summary[n].rmin = total;
      summary[n].rmax = total + value.w;
      summary[n].wmin = value.w;
      summary[n].value = value.v;
      ++n;
      total = total + value.w;
      i = j;
    }
    n = sketch_prune(summary, n, limit);
    memcpy(current, summary, n * sizeof(orc_entry));
    uint32_t level = 0;
    for (;;) {
      n = sketch_prune(current, n, limit);
      n = sketch_combine(current, n, resident + (size_t)level * limit, counts[level], scratch);
      counts[level] = 0;
      if (n <= limit) break;
      ++level;
    }
    counts[level] = n;
    memcpy(resident + (size_t)level * limit, current, n * sizeof(orc_entry));
  }
  uint32_t n = 0;
  for (uint32_t level = 0; level < levels; ++level) {
    n = sketch_combine(current, n, resident + (size_t)level * limit, counts[level], scratch);
    n = sketch_prune(current, n, budget > limit ? budget : limit);
  }
  uint32_t size = sketch_prune(current, n, budget);
  /* sketch_cuts_serial, kernels/quantile.metal.h:354-400 */
  uint32_t count = 0;
  if (!size) {
    out[0] = 1e-5f;
    *count_out = 1;
  } else {
    orc_entry* e = current;
    if (size <= max_bin) {
      float last = e[0].value;
      for (uint32_t i = 1; i < size; ++i) {
        float value = e[i].value;
        if (last < value) {
          out[count++] = value;
          last = value;
        }
      }
    } else {
      float last = e[0].value;
      uint32_t next = 1, cursor = 0;
      double total = (double)e[size - 1].rmax;
      for (uint32_t i = 1; i < max_bin; ++i) {
        /* Rank i*total/max_bin*2 in binary64; ranks and cumulative weights
         * are nonnegative, so the reference's bitwise comparison of their
         * binary64 encodings is kept as is. */
        uint64_t rank = f64_bits((double)i * total / (double)max_bin * 2.0);
        while (cursor < size - 2 &&
               rank >= f64_bits((double)(e[cursor + 1].rmin + e[cursor + 1].rmax)))
          ++cursor;
        float boundary = min_next(e[cursor]) + max_previous(e[cursor + 1]);
        float value = e[cursor + (isnan(boundary) || rank >= f64_bits((double)boundary))].value;
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
    float tail = e[size - 1].value;
    out[count++] = tail + (fabsf(tail) + 1e-5f);
    *count_out = count;
  }
  free(runs);
  free(resident);
  free(current);
  free(scratch);
  free(summary);
  free(tmp);
}

uint32_t orc_sketch_cuts(const float* X, uint32_t rows, uint32_t cols, const float* weights,
                         uint32_t max_bin, float* cuts, uint32_t* counts, float* minima) {
  uint32_t stride = orc_cut_stride(rows, max_bin);
  for (uint32_t f = 0; f < cols; ++f) {
    float* out = cuts + (size_t)f * stride;
    memset(out, 0, stride * sizeof(float));
    feature_cuts(X, rows, cols, f, weights, max_bin, out, counts + f, minima + f);
  }
  return stride;
}

/* quantize, kernels/boost.metal:461-499 (numeric features) */
void orc_quantize(const float* X, uint32_t rows, uint32_t cols, const float* cuts,
                  uint32_t stride, const uint32_t* counts, uint32_t* bins) {
  for (uint32_t r = 0; r < rows; ++r)
    for (uint32_t c = 0; c < cols; ++c) {
      float v = X[(size_t)r * cols + c];
      uint32_t count = counts[c];
      if (isnan(v) || !count) {
        bins[(size_t)r * cols + c] = ORC_MISSING;
        continue;
      }
      uint32_t lo = 0, hi = count;
      while (lo < hi) {
        uint32_t mid = lo + (hi - lo) / 2;
        if (v >= cuts[(size_t)c * stride + mid]) lo = mid + 1;
        else hi = mid;
      }
      bins[(size_t)r * cols + c] = lo < count - 1 ? lo : count - 1;
    }
}

/* ------------------------------------------------------------------------ */
/* Gradients and their fixed-point quantisation.                            */
/* ------------------------------------------------------------------------ */

float orc_expf(float x) { return det_expf(x); }

/* gradients, kernels/boost.metal:553-601, for objectives 0 (squared error),
 * 1 (logistic) and 3 (softprob). [ours] exp is det_expf, and the softmax
 * denominator is a binary64 sum in class order, where the reference uses
 * Metal's exp and an extended-precision sum. */
void orc_gradients(int objective, const float* margins, const float* labels,
                   const float* weights, uint32_t rows, uint32_t groups, float scale_pos_weight,
                   float* pairs) {
  for (uint32_t r = 0; r < rows; ++r) {
    float label = labels[r];
    for (uint32_t k = 0; k < groups; ++k) {
      size_t idx = (size_t)r * groups + k;
      float pred = margins[idx];
      float w = weights ? weights[r] : 1.0f;
      float g = pred - label, h = 1.0f;
      if (objective == ORC_LOGISTIC) {
        float prob = 1.0f / (1.0f + det_expf(-pred));
        w = w * (label == 1.0f ? scale_pos_weight : 1.0f);
        g = prob - label;
        h = fmaxf(prob * (1.0f - prob), 1.0e-16f);
      } else if (objective == ORC_SOFTPROB) {
        float mx = 0x1p-126f;
        for (uint32_t j = 0; j < groups; ++j) mx = fmaxf(mx, margins[(size_t)r * groups + j]);
        double denom = 0;
        for (uint32_t j = 0; j < groups; ++j)
          denom += (double)det_expf(margins[(size_t)r * groups + j] - mx);
        float prob = (float)((double)det_expf(pred - mx) / denom);
        g = prob - ((uint32_t)label == k ? 1.0f : 0.0f);
        pairs[idx * 2] = g * w;
        pairs[idx * 2 + 1] = fmaxf(fabsf(g) * w, 1.0e-16f);
        continue;
      }
      pairs[idx * 2] = g * w;
      pairs[idx * 2 + 1] = h * w;
    }
  }
}

/* Exact sum of float magnitudes in units of 2^-149 (mass_atomic_bits,
 * kernels/objectives.metal.h:59-67) and the scale 2^(62 - e) with 2^e the
 * smallest power of two above it, at least 1
 * (kernels/gradient_quantization.metal.h:49-63). */
void orc_gradient_scales(const float* pairs, uint32_t rows, uint32_t groups, float* scales) {
  for (uint32_t k = 0; k < groups; ++k)
    for (uint32_t part = 0; part < 2; ++part) {
      uint32_t mass[10] = {0};
      for (uint32_t r = 0; r < rows; ++r) {
        uint32_t bits = f32_bits(pairs[((size_t)r * groups + k) * 2 + part]) & 0x7fffffffu;
        uint32_t exponent = (bits >> 23) & 255;
        uint64_t mantissa = (bits & 0x7fffffu) | (exponent ? 0x800000u : 0u);
        uint32_t shift = exponent ? exponent - 1 : 0;
        /* add mantissa * 2^shift into the 320-bit integer */
        uint32_t word = shift / 32, bit = shift % 32;
        uint64_t wide = mantissa << bit; /* at most 56 bits */
        uint64_t carry = 0;
        for (uint32_t i = word; i < 10; ++i) {
          uint64_t add = (i == word) ? (wide & 0xffffffffu) : (i == word + 1) ? (wide >> 32) : 0;
          uint64_t s = (uint64_t)mass[i] + add + carry;
          mass[i] = (uint32_t)s;
          carry = s >> 32;
          if (!carry && i > word) break;
        }
      }
      int e = 0;
      for (int w = 9; w >= 0; --w)
        if (mass[w]) {
          int bitlen = w * 32 + 32 - __builtin_clz(mass[w]);
          e = bitlen - 149 > 0 ? bitlen - 149 : 0;
          break;
        }
      scales[k * 2 + part] = f32_from((uint32_t)(62 - e + 127) << 23);
    }
}

/* q = round-half-even(v * scale) as int64 (kernels/boost.metal:616-618). */
void orc_quantize_gradients(const float* pairs, uint32_t rows, uint32_t groups,
                            const float* scales, int64_t* q) {
  for (uint32_t r = 0; r < rows; ++r)
    for (uint32_t k = 0; k < groups; ++k) {
      size_t idx = (size_t)r * groups + k;
      q[idx * 2] = (int64_t)nearbyintf(pairs[idx * 2] * scales[k * 2]);
      q[idx * 2 + 1] = (int64_t)nearbyintf(pairs[idx * 2 + 1] * scales[k * 2 + 1]);
    }
}

/* ------------------------------------------------------------------------ */
/* Histograms, split scan, selection.                                        */
/* ------------------------------------------------------------------------ */

/* hist[f][bin] += q over the given rows, int64 wrap-around, missing at
 * index stride (kernels/boost.metal:700-733). */
void orc_histogram(const uint32_t* bins, uint32_t cols, uint32_t stride, const int64_t* q,
                   const uint32_t* rows, uint32_t nrows, int64_t* hist) {
  for (uint32_t i = 0; i < nrows; ++i) {
    uint32_t r = rows[i];
    for (uint32_t f = 0; f < cols; ++f) {
      uint32_t b = bins[(size_t)r * cols + f];
      size_t cell = ((size_t)f * (stride + 1) + (b == ORC_MISSING ? stride : b)) * 2;
      hist[cell] = (int64_t)((uint64_t)hist[cell] + (uint64_t)q[(size_t)r * 2]);
      hist[cell + 1] = (int64_t)((uint64_t)hist[cell + 1] + (uint64_t)q[(size_t)r * 2 + 1]);
    }
  }
}

/* An exact integer sum in units of 1/scale as binary64: one rounding of the
 * integer, then an exact power-of-two scaling (split_stat_value_bits,
 * kernels/split_statistics.metal.h:4-16). */
static double stat_value(int64_t v, float scale) {
  if (!v) return 0.0;
  int exponent;
  frexpf(scale, &exponent);
  return ldexp((double)v, -(exponent - 1));
}

typedef struct {
  float reg_lambda, reg_alpha, min_child_weight, max_delta_step;
} split_params;

/* scalar_weight, kernels/scalar_gain.metal.h:56-82: RN32(RN64(-T(G)/(H+lambda)))
 * with T the L1 soft threshold, clamped to +-max_delta_step; 0 when H <= 0. */
static float leaf_weight(double G, double H, const split_params* p) {
  if (!(H > 0)) return 0.0f;
  double alpha = fabs((double)p->reg_alpha);
  double t = fabs(G) <= alpha ? 0.0 : (G < 0 ? G + alpha : G - alpha);
  double den = H + (double)p->reg_lambda;
  float w = (float)(-t / den);
  float limit = fabsf(p->max_delta_step);
  if (limit != 0 && fabsf(w) > limit) w = copysignf(limit, w);
  return w;
}

/* scalar_gain, kernels/scalar_gain.metal.h:91-103. */
static float node_gain(double G, double H, float w, const split_params* p) {
  if (!(H > 0)) return 0.0f;
  double wd = (double)w;
  double square = (double)(float)(wd * wd);
  double quadratic = (H + (double)p->reg_lambda) * square;
  double sum = fma(G + G, wd, quadratic);
  double alpha = (double)p->reg_alpha;
  sum = fma(alpha + alpha, fabs(wd), sum);
  return (float)(-sum);
}

static int valid_hessian(double H, float min_child_weight) {
  return H > 0 && H >= (double)fabsf(min_child_weight);
}

/* consider_split, kernels/boost.metal:902-920 */
static void consider(orc_split* best, int64_t lg, int64_t lh, int64_t rg, int64_t rh,
                     const float* scale, float threshold, uint32_t default_left, uint32_t feature,
                     float parent_gain, const split_params* p) {
  double LG = stat_value(lg, scale[0]), LH = stat_value(lh, scale[1]);
  double RG = stat_value(rg, scale[0]), RH = stat_value(rh, scale[1]);
  if (!valid_hessian(LH, p->min_child_weight) || !valid_hessian(RH, p->min_child_weight)) return;
  float lw = leaf_weight(LG, LH, p), rw = leaf_weight(RG, RH, p);
  float gain = (node_gain(LG, LH, lw, p) + node_gain(RG, RH, rw, p)) - parent_gain;
  if (gain > best->gain) {
    best->gain = gain;
    best->threshold = threshold;
    best->feature = (int32_t)feature;
    best->default_left = default_left;
    best->left_h = (float)LH;
    best->right_h = (float)RH;
    best->left_weight = lw;
    best->right_weight = rw;
    best->left_sum_g = lg;
    best->left_sum_h = lh;
    best->right_sum_g = rg;
    best->right_sum_h = rh;
  }
}

/* evaluate_feature, kernels/boost.metal:921-1005 (numeric features). */
void orc_evaluate_splits(const int64_t* hist, uint32_t nodes, uint32_t cols, uint32_t stride,
                         const float* scale, const float* cuts, const uint32_t* counts,
                         const float* minima, float reg_lambda, float reg_alpha,
                         float min_child_weight, float max_delta_step, uint32_t use_parent_sums,
                         const int64_t* node_sums, orc_split* out) {
  split_params p = {reg_lambda, reg_alpha, min_child_weight, max_delta_step};
  for (uint32_t node = 0; node < nodes; ++node)
    for (uint32_t f = 0; f < cols; ++f) {
      const int64_t* h = hist + ((size_t)node * cols + f) * (stride + 1) * 2;
      uint32_t count = counts[f];
      uint64_t pg = 0, ph = 0;
      for (uint32_t b = 0; b < count; ++b) {
        pg += (uint64_t)h[b * 2];
        ph += (uint64_t)h[b * 2 + 1];
      }
      uint64_t tg, th;
      if (use_parent_sums) {
        tg = (uint64_t)node_sums[node * 2];
        th = (uint64_t)node_sums[node * 2 + 1];
      } else {
        tg = pg + (uint64_t)h[stride * 2];
        th = ph + (uint64_t)h[stride * 2 + 1];
      }
      uint64_t mg = tg - pg, mh = th - ph;
      double TG = stat_value((int64_t)tg, scale[0]), TH = stat_value((int64_t)th, scale[1]);
      float w = leaf_weight(TG, TH, &p);
      orc_split best;
      memset(&best, 0, sizeof best);
      best.gain = -INFINITY;
      best.feature = -1;
      best.left_weight = w;
      best.right_weight = w;
      best.total_g = (float)TG;
      best.total_h = (float)TH;
      best.parent_weight = w;
      float parent_gain = node_gain(TG, TH, w, &p);
      const float* fc = cuts + (size_t)f * stride;
      uint64_t lg = 0, lh = 0;
      for (uint32_t b = 0; b < count; ++b) {
        lg += (uint64_t)h[b * 2];
        lh += (uint64_t)h[b * 2 + 1];
        consider(&best, (int64_t)lg, (int64_t)lh, (int64_t)(tg - lg), (int64_t)(th - lh), scale,
                 fc[b], 0, f, parent_gain, &p);
      }
      if (mg != 0 || mh != 0) {
        uint64_t rg = 0, rh = 0;
        for (int b = (int)count - 1; b >= 0; --b) {
          rg += (uint64_t)h[b * 2];
          rh += (uint64_t)h[b * 2 + 1];
          float threshold = b == 0 ? minima[f] : fc[b - 1];
          consider(&best, (int64_t)(tg - rg), (int64_t)(th - rh), (int64_t)rg, (int64_t)rh, scale,
                   threshold, 1, f, parent_gain, &p);
        }
      }
      out[(size_t)node * cols + f] = best;
    }
}

/* select_splits, kernels/boost.metal:1245-1265, with the applied parent
 * statistics of kernels/split_statistics.metal.h:17-38. */
void orc_select_splits(const orc_split* candidates, uint32_t nodes, uint32_t cols,
                       const float* scale, float reg_lambda, float reg_alpha,
                       float max_delta_step, orc_split* best) {
  for (uint32_t node = 0; node < nodes; ++node) {
    orc_split result = candidates[(size_t)node * cols];
    for (uint32_t f = 1; f < cols; ++f) {
      const orc_split* o = &candidates[(size_t)node * cols + f];
      if (o->gain > result.gain) result = *o;
    }
    if (result.feature >= 0) {
      double G = stat_value(result.left_sum_g, scale[0]) + stat_value(result.right_sum_g, scale[0]);
      double H = stat_value(result.left_sum_h, scale[1]) + stat_value(result.right_sum_h, scale[1]);
      double value = 0.0;
      if (H > 0) {
        double alpha = fabs((double)reg_alpha);
        double t = fabs(G) <= alpha ? 0.0 : (G < 0 ? G + alpha : G - alpha);
        value = -t / (H + (double)reg_lambda);
        double limit = fabs((double)max_delta_step);
        if (limit != 0 && fabs(value) > limit) value = copysign(limit, value);
      }
      result.applied_parent_weight = (float)value;
      result.applied_parent_hessian = (float)H;
    }
    best[node] = result;
  }
}

/* ------------------------------------------------------------------------ */
/* One depthwise tree.                                                       */
/* ------------------------------------------------------------------------ */

typedef struct {
  uint32_t id;
  uint32_t begin, count; /* range in the row array */
  int64_t sum_g, sum_h;
} frontier_node;

/* Level-synchronous growth with the expansion rule and node numbering of
 * tree_driver_apply (kernels/tree_driver.metal.h:54-93), then the host replay
 * of src/tree.cpp:1663-1717. Rows are partitioned by the bin form of the
 * split predicate (kernels/boost.metal:1383-1389), stably. */
int orc_grow_tree(const uint32_t* bins, uint32_t rows, uint32_t cols, const int64_t* q,
                  const float* scale, const float* cuts, uint32_t stride,
                  const uint32_t* counts, const float* minima, const orc_tree_params* tp,
                  orc_node* nodes, uint32_t capacity, float* row_leaf) {
  uint32_t max_depth = tp->max_depth;
  uint64_t node_cap = max_depth >= 31 ? 0xffffffffull : ((2ull << max_depth) - 1);
  if (node_cap > capacity) node_cap = capacity;
  orc_split* history = (orc_split*)calloc(node_cap ? node_cap : 1, sizeof(orc_split));
  uint32_t* flags = (uint32_t*)calloc(node_cap ? node_cap : 1, sizeof(uint32_t));
  uint32_t* order = (uint32_t*)malloc(((size_t)rows + 1) * sizeof(uint32_t));
  uint32_t* scratch = (uint32_t*)malloc(((size_t)rows + 1) * sizeof(uint32_t));
  for (uint32_t r = 0; r < rows; ++r) order[r] = r;
  frontier_node* frontier = (frontier_node*)malloc(sizeof(frontier_node));
  uint32_t nfront = 1, created = 1;
  frontier[0].id = 0; frontier[0].begin = 0; frontier[0].count = rows;
  frontier[0].sum_g = 0; frontier[0].sum_h = 0;
  int status = 0;
  size_t per_node = (size_t)cols * (stride + 1) * 2;
  for (uint32_t depth = 0; depth < max_depth && nfront; ++depth) {
    int64_t* hist = (int64_t*)calloc(per_node * nfront, sizeof(int64_t));
    int64_t* sums = (int64_t*)malloc(2 * nfront * sizeof(int64_t));
    orc_split* cand = (orc_split*)malloc((size_t)nfront * cols * sizeof(orc_split));
    orc_split* best = (orc_split*)malloc(nfront * sizeof(orc_split));
    for (uint32_t s = 0; s < nfront; ++s) {
      orc_histogram(bins, cols, stride, q, order + frontier[s].begin, frontier[s].count,
                    hist + per_node * s);
      sums[2 * s] = frontier[s].sum_g;
      sums[2 * s + 1] = frontier[s].sum_h;
    }
    orc_evaluate_splits(hist, nfront, cols, stride, scale, cuts, counts, minima, tp->reg_lambda,
                        tp->reg_alpha, tp->min_child_weight, tp->max_delta_step, depth != 0, sums,
                        cand);
    orc_select_splits(cand, nfront, cols, scale, tp->reg_lambda, tp->reg_alpha,
                      tp->max_delta_step, best);
    frontier_node* next = (frontier_node*)malloc(2 * nfront * sizeof(frontier_node));
    uint32_t nnext = 0;
    for (uint32_t s = 0; s < nfront; ++s) {
      uint32_t id = frontier[s].id;
      orc_split sp = best[s];
      history[id] = sp;
      flags[id] = 1;
      int expand = sp.feature >= 0 && sp.gain > 1.0e-6f && sp.gain >= tp->min_split_loss;
      if (!expand) continue;
      if (created + 2 > node_cap) {
        status = -1;
        break;
      }
      uint32_t left = created;
      created += 2;
      flags[id] |= 2;
      if (depth + 1 >= max_depth) continue;
      /* stable partition of this node's rows */
      uint32_t f = (uint32_t)sp.feature;
      int32_t k = -1;
      for (uint32_t b = 0; b < counts[f]; ++b)
        if (f32_bits(cuts[(size_t)f * stride + b]) == f32_bits(sp.threshold)) k = (int32_t)b;
      uint32_t* rows_in = order + frontier[s].begin;
      uint32_t nl = 0, nr = 0;
      for (uint32_t i = 0; i < frontier[s].count; ++i) {
        uint32_t b = bins[(size_t)rows_in[i] * cols + f];
        int go_left = b == ORC_MISSING ? (int)sp.default_left : (int32_t)b <= k;
        if (go_left) rows_in[nl++] = rows_in[i];
        else scratch[nr++] = rows_in[i];
      }
      memcpy(rows_in + nl, scratch, nr * sizeof(uint32_t));
      next[nnext].id = left;
      next[nnext].begin = frontier[s].begin;
      next[nnext].count = nl;
      next[nnext].sum_g = sp.left_sum_g;
      next[nnext].sum_h = sp.left_sum_h;
      next[nnext + 1].id = left + 1;
      next[nnext + 1].begin = frontier[s].begin + nl;
      next[nnext + 1].count = nr;
      next[nnext + 1].sum_g = sp.right_sum_g;
      next[nnext + 1].sum_h = sp.right_sum_h;
      nnext += 2;
    }
    free(hist);
    free(sums);
    free(cand);
    free(best);
    free(frontier);
    frontier = next;
    nfront = nnext;
    if (status) break;
  }
  free(frontier);
  int result = status;
  if (!status) {
    /* replay, src/tree.cpp:1663-1717 */
    uint32_t size = 1;
    memset(&nodes[0], 0, sizeof(orc_node));
    nodes[0].left = nodes[0].right = nodes[0].feature = nodes[0].parent = -1;
    for (uint32_t id = 0; id < created && !result; ++id) {
      if (id >= size) {
        result = -2;
        break;
      }
      if (!(flags[id] & 1)) continue;
      orc_split sp = history[id];
      nodes[id].cover = sp.total_h;
      if (!id) nodes[0].leaf = sp.parent_weight * tp->eta;
      if (!(flags[id] & 2)) continue;
      uint32_t left = size;
      nodes[id].left = (int32_t)left;
      nodes[id].right = (int32_t)left + 1;
      nodes[id].feature = sp.feature;
      nodes[id].threshold = sp.threshold;
      nodes[id].default_left = sp.default_left;
      nodes[id].gain = sp.gain;
      nodes[id].cover = sp.applied_parent_hessian;
      uint32_t f = (uint32_t)sp.feature;
      int32_t k = -1;
      for (uint32_t b = 0; b < counts[f]; ++b)
        if (f32_bits(cuts[(size_t)f * stride + b]) == f32_bits(sp.threshold)) k = (int32_t)b;
      nodes[id].split_bin = k;
      for (int c = 0; c < 2; ++c) {
        orc_node* n = &nodes[left + c];
        memset(n, 0, sizeof *n);
        n->left = n->right = n->feature = -1;
        n->parent = (int32_t)id;
        n->leaf = (c ? sp.right_weight : sp.left_weight) * tp->eta;
        n->cover = c ? sp.right_h : sp.left_h;
      }
      size += 2;
    }
    if (!result) {
      if (size != created) result = -3;
      else result = (int)size;
    }
  }
  if (result > 0 && row_leaf) {
    for (uint32_t r = 0; r < rows; ++r) {
      int32_t n = 0;
      while (nodes[n].left >= 0) {
        uint32_t b = bins[(size_t)r * cols + (uint32_t)nodes[n].feature];
        int go_left = b == ORC_MISSING ? (int)nodes[n].default_left : (int32_t)b <= nodes[n].split_bin;
        n = go_left ? nodes[n].left : nodes[n].right;
      }
      row_leaf[r] = nodes[n].leaf;
    }
  }
  free(history);
  free(flags);
  free(order);
  free(scratch);
  return result;
}

/* ------------------------------------------------------------------------ */
/* The host-driven tree: a queue of evaluated leaves.                        */
/* ------------------------------------------------------------------------ */

typedef struct {
  uint32_t id, depth;
  uint32_t begin, count; /* range in the row array */
  orc_split split;
} queue_leaf;

/* Queue order of src/tree.cpp:63-69: loss-guided trees pop the largest gain
 * first; ties, and every depth-wise tree, pop the smallest node id first.
 * Returns nonzero when a pops before b. */
static int leaf_before(const queue_leaf* a, const queue_leaf* b, uint32_t lossguide) {
  if (lossguide && a->split.gain != b->split.gain) return a->split.gain > b->split.gain;
  return a->id < b->id;
}

static void heap_push(queue_leaf* h, uint32_t* n, queue_leaf v, uint32_t lossguide) {
  uint32_t i = (*n)++;
  h[i] = v;
  while (i && leaf_before(&h[i], &h[(i - 1) / 2], lossguide)) {
    queue_leaf t = h[i];
    h[i] = h[(i - 1) / 2];
    h[(i - 1) / 2] = t;
    i = (i - 1) / 2;
  }
}

static queue_leaf heap_pop(queue_leaf* h, uint32_t* n, uint32_t lossguide) {
  queue_leaf top = h[0];
  h[0] = h[--(*n)];
  uint32_t i = 0;
  for (;;) {
    uint32_t l = 2 * i + 1, r = l + 1, m = i;
    if (l < *n && leaf_before(&h[l], &h[m], lossguide)) m = l;
    if (r < *n && leaf_before(&h[r], &h[m], lossguide)) m = r;
    if (m == i) break;
    queue_leaf t = h[i];
    h[i] = h[m];
    h[m] = t;
    i = m;
  }
  return top;
}

/* The best split of one node over rows [begin, begin + count) of `order`. */
static orc_split evaluate_node(const uint32_t* bins, uint32_t cols, const int64_t* q, const float* scale,
                               const float* cuts, uint32_t stride, const uint32_t* counts,
                               const float* minima, const orc_tree_params* tp, const uint32_t* order,
                               uint32_t begin, uint32_t count, int root, int64_t sum_g, int64_t sum_h) {
  size_t per_node = (size_t)cols * (stride + 1) * 2;
  int64_t* hist = (int64_t*)calloc(per_node, sizeof(int64_t));
  orc_split* cand = (orc_split*)malloc((size_t)cols * sizeof(orc_split));
  int64_t sums[2] = {sum_g, sum_h};
  orc_split best;
  orc_histogram(bins, cols, stride, q, order + begin, count, hist);
  orc_evaluate_splits(hist, 1, cols, stride, scale, cuts, counts, minima, tp->reg_lambda, tp->reg_alpha,
                      tp->min_child_weight, tp->max_delta_step, root ? 0u : 1u, sums, cand);
  orc_select_splits(cand, 1, cols, scale, tp->reg_lambda, tp->reg_alpha, tp->max_delta_step, &best);
  free(hist);
  free(cand);
  return best;
}

/* [ours, restating src/tree.cpp:291-349 and 1031-1120] Host-driven growth.
 * The root is evaluated and queued; each pass pops a batch (one leaf when
 * loss-guided, else up to 256 leaves of one depth in node-id order), keeping
 * the leaves whose split is usable (feature >= 0, gain > 1e-6, gain >=
 * min_split_loss, depth < max_depth, fewer than max_leaves leaves so far,
 * counting the root as one); the first empty batch ends the tree. Applying
 * a leaf numbers its children in pop order; while depth + 1 < max_depth and
 * the leaf count allows, the children are partitioned, evaluated and queued
 * when their gain exceeds 1e-6. max_depth 0 means unlimited. Node fields
 * follow the level-synchronous grower (cover = the evaluated total Hessian,
 * the applied parent Hessian once split). */
int orc_grow_tree_queue(const uint32_t* bins, uint32_t rows, uint32_t cols, const int64_t* q,
                        const float* scale, const float* cuts, uint32_t stride, const uint32_t* counts,
                        const float* minima, const orc_tree_params* tp, uint32_t lossguide,
                        uint32_t max_leaves, orc_node* nodes, uint32_t capacity, float* row_leaf) {
  const uint32_t max_depth = tp->max_depth;
  uint32_t* order = (uint32_t*)malloc(((size_t)rows + 1) * sizeof(uint32_t));
  uint32_t* scratch = (uint32_t*)malloc(((size_t)rows + 1) * sizeof(uint32_t));
  queue_leaf* heap = (queue_leaf*)malloc(((size_t)capacity + 1) * sizeof(queue_leaf));
  queue_leaf* batch = (queue_leaf*)malloc(256 * sizeof(queue_leaf));
  queue_leaf* kids = (queue_leaf*)malloc(512 * sizeof(queue_leaf));
  uint32_t nheap = 0, size = 1, leaves = 1;
  int result = 0;
  for (uint32_t r = 0; r < rows; ++r) order[r] = r;
  if (capacity < 1) {
    result = -1;
    goto done;
  }
  {
    queue_leaf root = {0, 0, 0, rows, evaluate_node(bins, cols, q, scale, cuts, stride, counts, minima, tp,
                                                    order, 0, rows, 1, 0, 0)};
    memset(&nodes[0], 0, sizeof(orc_node));
    nodes[0].left = nodes[0].right = nodes[0].feature = nodes[0].parent = -1;
    nodes[0].split_bin = 0;
    nodes[0].cover = root.split.total_h;
    nodes[0].leaf = root.split.parent_weight * tp->eta;
    heap_push(heap, &nheap, root, lossguide);
  }
  for (;;) {
    /* pop */
    uint32_t nb = 0;
    if (!nheap) break;
    uint32_t depth = heap[0].depth;
    do {
      queue_leaf leaf = heap_pop(heap, &nheap, lossguide);
      if (leaf.split.feature >= 0 && leaf.split.gain > 1.0e-6f && leaf.split.gain >= tp->min_split_loss &&
          (!max_depth || leaf.depth < max_depth) && (!max_leaves || leaves < max_leaves)) {
        ++leaves;
        batch[nb++] = leaf;
      }
      if (lossguide) break;
    } while (nheap && heap[0].depth == depth && nb < 256);
    if (!nb) break;
    /* apply */
    uint32_t nk = 0;
    for (uint32_t i = 0; i < nb; ++i) {
      const queue_leaf* leaf = &batch[i];
      const orc_split* sp = &leaf->split;
      if (size + 2 > capacity) {
        result = -1;
        goto done;
      }
      uint32_t left = size;
      size += 2;
      orc_node* nd = &nodes[leaf->id];
      nd->left = (int32_t)left;
      nd->right = (int32_t)left + 1;
      nd->feature = sp->feature;
      nd->threshold = sp->threshold;
      nd->default_left = sp->default_left;
      nd->gain = sp->gain;
      nd->cover = sp->applied_parent_hessian;
      uint32_t f = (uint32_t)sp->feature;
      int32_t k = -1;
      for (uint32_t b = 0; b < counts[f]; ++b)
        if (f32_bits(cuts[(size_t)f * stride + b]) == f32_bits(sp->threshold)) k = (int32_t)b;
      nd->split_bin = k;
      for (int c = 0; c < 2; ++c) {
        orc_node* n = &nodes[left + c];
        memset(n, 0, sizeof *n);
        n->left = n->right = n->feature = -1;
        n->parent = (int32_t)leaf->id;
        n->leaf = (c ? sp->right_weight : sp->left_weight) * tp->eta;
        n->cover = c ? sp->right_h : sp->left_h;
      }
      if ((!max_depth || leaf->depth + 1 < max_depth) && (!max_leaves || leaves < max_leaves)) {
        /* stable partition of this leaf's rows */
        uint32_t* rows_in = order + leaf->begin;
        uint32_t nl = 0, nr = 0;
        for (uint32_t j = 0; j < leaf->count; ++j) {
          uint32_t b = bins[(size_t)rows_in[j] * cols + f];
          int go_left = b == ORC_MISSING ? (int)sp->default_left : (int32_t)b <= k;
          if (go_left) rows_in[nl++] = rows_in[j];
          else scratch[nr++] = rows_in[j];
        }
        memcpy(rows_in + nl, scratch, nr * sizeof(uint32_t));
        /* Each child carries its parent's split until it is evaluated. */
        queue_leaf l = {left, leaf->depth + 1, leaf->begin, nl, *sp};
        queue_leaf r = {left + 1, leaf->depth + 1, leaf->begin + nl, nr, *sp};
        kids[nk] = l;
        kids[nk + 1] = r;
        nk += 2;
      }
    }
    /* evaluate the children of this batch */
    for (uint32_t i = 0; i < nk; ++i) {
      const orc_split parent = kids[i].split;
      const int right = (i & 1) != 0;
      kids[i].split = evaluate_node(bins, cols, q, scale, cuts, stride, counts, minima, tp, order,
                                    kids[i].begin, kids[i].count, 0,
                                    right ? parent.right_sum_g : parent.left_sum_g,
                                    right ? parent.right_sum_h : parent.left_sum_h);
      nodes[kids[i].id].cover = kids[i].split.total_h;
      if (kids[i].split.gain > 1.0e-6f) heap_push(heap, &nheap, kids[i], lossguide);
    }
  }
  result = (int)size;
  if (row_leaf) {
    for (uint32_t r = 0; r < rows; ++r) {
      int32_t n = 0;
      while (nodes[n].left >= 0) {
        uint32_t b = bins[(size_t)r * cols + (uint32_t)nodes[n].feature];
        int go_left = b == ORC_MISSING ? (int)nodes[n].default_left : (int32_t)b <= nodes[n].split_bin;
        n = go_left ? nodes[n].left : nodes[n].right;
      }
      row_leaf[r] = nodes[n].leaf;
    }
  }
done:
  free(order);
  free(scratch);
  free(heap);
  free(batch);
  free(kids);
  return result;
}

/* ------------------------------------------------------------------------ */
/* Base score and the boosting loop.                                         */
/* ------------------------------------------------------------------------ */

/* [ours] Deterministic binary64 sum: 1024-row chunks reduced as a pairwise
 * tree (s[i] += s[i + h] for h = 512..1), chunk sums added in chunk order.
 * The reference sums in extended precision (kernels/boost.metal:356-402). */
#define ORC_BASE_CHUNK 1024
static double fixed_order_sum(const double* v, uint32_t n) {
  double total = 0, s[ORC_BASE_CHUNK];
  for (uint32_t begin = 0; begin < n; begin += ORC_BASE_CHUNK) {
    for (uint32_t i = 0; i < ORC_BASE_CHUNK; ++i) s[i] = begin + i < n ? v[begin + i] : 0.0;
    for (uint32_t h = ORC_BASE_CHUNK / 2; h; h >>= 1)
      for (uint32_t i = 0; i < h; ++i) s[i] = s[i] + s[i + h];
    total = total + s[0];
  }
  return total;
}

/* base_partial/base_reduce/base_finalize (kernels/boost.metal:356-420) and
 * score_margins (src/objectives.cpp:17-31). */
void orc_base_score(int objective, const float* labels, const float* weights, uint32_t rows,
                    uint32_t groups, float scale_pos_weight, float* score, float* margin) {
  double* yw = (double*)malloc(((size_t)rows + 1) * sizeof(double));
  double* ww = (double*)malloc(((size_t)rows + 1) * sizeof(double));
  float* values = (float*)malloc(groups * sizeof(float));
  for (uint32_t k = 0; k < groups; ++k) {
    for (uint32_t r = 0; r < rows; ++r) {
      float y = labels[r];
      float w = weights ? weights[r] : 1.0f;
      if (objective == ORC_LOGISTIC) w = w * (y == 1.0f ? scale_pos_weight : 1.0f);
      if (objective == ORC_SOFTPROB) y = (uint32_t)y == k ? 1.0f : 0.0f;
      yw[r] = (double)y * (double)w;
      ww[r] = (double)w;
    }
    double sy = fixed_order_sum(yw, rows), sw = fixed_order_sum(ww, rows);
    values[k] = sw > 0 ? (float)(sy / sw) : (objective == ORC_SQUAREDERROR && rows == 0 ? 0.0f : 0.5f);
  }
  for (uint32_t k = 0; k < groups; ++k) {
    float s = values[k], m = s;
    if (objective == ORC_SOFTPROB) {
      float mean = 0;
      for (uint32_t j = 0; j < groups; ++j) mean += logf(fmaxf(values[j], 1.0e-6f));
      m = logf(fmaxf(s, 1.0e-6f)) - mean / (float)groups;
      s = m;
    } else if (objective == ORC_LOGISTIC) {
      float v = fminf(fmaxf(s, 1.0e-6f), 1.0f - 1.0e-6f);
      m = -logf(1.0f / v - 1.0f);
    }
    score[k] = s;
    margin[k] = m;
  }
  free(yw);
  free(ww);
  free(values);
}

int64_t orc_train(const float* X, uint32_t rows, uint32_t cols, const float* labels,
                  const float* weights, const orc_train_params* p, orc_node* nodes,
                  uint64_t node_capacity, uint32_t* tree_sizes, float* margins,
                  float* base_margin_out) {
  uint32_t groups = p->objective == ORC_SOFTPROB ? p->num_class : 1;
  uint32_t stride = orc_cut_stride(rows, p->max_bin);
  float* cuts = (float*)calloc((size_t)cols * stride, sizeof(float));
  uint32_t* counts = (uint32_t*)calloc(cols, sizeof(uint32_t));
  float* minima = (float*)calloc(cols, sizeof(float));
  uint32_t* bins = (uint32_t*)malloc(((size_t)rows * cols + 1) * sizeof(uint32_t));
  float* pairs = (float*)malloc(((size_t)rows * groups * 2 + 1) * sizeof(float));
  float* gpairs = (float*)malloc(((size_t)rows * 2 + 1) * sizeof(float));
  int64_t* q = (int64_t*)malloc(((size_t)rows * 2 + 1) * sizeof(int64_t));
  float* leaf = (float*)malloc(((size_t)rows + 1) * sizeof(float));
  float* score = (float*)malloc(groups * sizeof(float));
  float* base = (float*)malloc(groups * sizeof(float));
  orc_sketch_cuts(X, rows, cols, weights, p->max_bin, cuts, counts, minima);
  orc_quantize(X, rows, cols, cuts, stride, counts, bins);
  if (p->has_base_score) {
    for (uint32_t k = 0; k < groups; ++k) score[k] = p->base_score;
    for (uint32_t k = 0; k < groups; ++k) {
      base[k] = score[k];
      if (p->objective == ORC_LOGISTIC) {
        float v = fminf(fmaxf(score[k], 1.0e-6f), 1.0f - 1.0e-6f);
        base[k] = -logf(1.0f / v - 1.0f);
      }
    }
  } else {
    orc_base_score(p->objective, labels, weights, rows, groups, p->scale_pos_weight, score, base);
  }
  for (uint32_t k = 0; k < groups; ++k) base_margin_out[k] = base[k];
  for (uint32_t r = 0; r < rows; ++r)
    for (uint32_t k = 0; k < groups; ++k) margins[(size_t)r * groups + k] = base[k];
  uint64_t used = 0;
  int64_t result = 0;
  /* The host-driven grower for loss-guided trees, leaf budgets and depths
   * the level-synchronous driver does not take (src/tree.cpp:366-385). */
  const int queue = p->lossguide || p->max_leaves || p->tree.max_depth == 0 || p->tree.max_depth > 10;
  uint64_t tree_cap64 = 2ull * rows + 1;
  if (p->tree.max_depth && p->tree.max_depth < 31 && ((2ull << p->tree.max_depth) - 1) < tree_cap64)
    tree_cap64 = (2ull << p->tree.max_depth) - 1;
  uint32_t tree_cap = (uint32_t)tree_cap64;
  for (uint32_t round = 0; round < p->rounds && !result; ++round) {
    orc_gradients(p->objective, margins, labels, weights, rows, groups, p->scale_pos_weight, pairs);
    /* All trees of a round use the gradients of the round's start; the
     * margins advance after every tree of the round is grown. */
    float* increments = (float*)malloc(((size_t)rows * groups + 1) * sizeof(float));
    for (uint32_t k = 0; k < groups && !result; ++k) {
      for (uint32_t r = 0; r < rows; ++r) {
        gpairs[r * 2] = pairs[((size_t)r * groups + k) * 2];
        gpairs[r * 2 + 1] = pairs[((size_t)r * groups + k) * 2 + 1];
      }
      float scale[2];
      orc_gradient_scales(gpairs, rows, 1, scale);
      orc_quantize_gradients(gpairs, rows, 1, scale, q);
      if (used + tree_cap > node_capacity) {
        result = -100;
        break;
      }
      int n = queue ? orc_grow_tree_queue(bins, rows, cols, q, scale, cuts, stride, counts, minima, &p->tree,
                                          p->lossguide, p->max_leaves, nodes + used, tree_cap, leaf)
                    : orc_grow_tree(bins, rows, cols, q, scale, cuts, stride, counts, minima, &p->tree,
                                    nodes + used, tree_cap, leaf);
      if (n < 0) {
        result = n;
        break;
      }
      tree_sizes[round * groups + k] = (uint32_t)n;
      used += (uint64_t)n;
      for (uint32_t r = 0; r < rows; ++r) increments[(size_t)r * groups + k] = leaf[r];
    }
    if (!result)
      for (size_t i = 0; i < (size_t)rows * groups; ++i) margins[i] = margins[i] + increments[i];
    free(increments);
  }
  free(cuts);
  free(counts);
  free(minima);
  free(bins);
  free(pairs);
  free(gpairs);
  free(q);
  free(leaf);
  free(score);
  free(base);
  return result ? result : (int64_t)used;
}
