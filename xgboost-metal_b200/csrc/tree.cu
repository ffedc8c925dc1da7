// CUDA kernels of the histogram tree trainer (sm_100a).
//
// Reference semantics (tabulai/xgboost-metal) that each kernel reproduces:
//   quantize_kernel      kernels/boost.metal:461-499 (bin = #cuts <= x, capped)
//   gradient_kernel      kernels/boost.metal:553-601
//   mass_*/scales        kernels/gradient_quantization.metal.h:1-67
//   hist_kernel          kernels/boost.metal:700-733, histogram_missing.metal.h
//   hist2_kernel         the same sums, staged two-limb form (each row's
//                        values formed once per 32 features), and a staged
//                        three-limb form for uint8 rounds of wider values
//   eval_kernel          kernels/boost.metal:902-1005 (+ subtraction :780-794);
//                        pack_best / merge_best select across ranks
//   transpose_codes_kernel, narrow_codes_kernel: layouts of the same codes
//   control_kernel       kernels/boost.metal:1245-1265, tree_driver.metal.h:28-94,
//                        src/tree.cpp:1663-1717 (node table replay)
//   partition_kernel     kernels/boost.metal:1325-1329, 1383-1389, 1738-1765
//   base_chunk_kernel    kernels/boost.metal:356-420
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>

#include "device_math.cuh"
#include "split_select.h"
#include "tree.h"

namespace xgbb {
namespace {

constexpr int kWarp = 32;

__device__ __forceinline__ unsigned long long shfl_u64(unsigned long long v, int src) {
  return __shfl_sync(0xffffffffu, v, src);
}

// Inclusive warp scan of 64-bit integers (wrap-around).
__device__ __forceinline__ unsigned long long warp_scan_u64(unsigned long long v, int lane) {
#pragma unroll
  for (int d = 1; d < kWarp; d <<= 1) {
    unsigned long long o = __shfl_up_sync(0xffffffffu, v, d);
    if (lane >= d) v += o;
  }
  return v;
}

// Exclusive block scan for <= 1024 threads; returns the total in *total.
__device__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* total) {
  __shared__ uint32_t warp_sums[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    uint32_t o = __shfl_up_sync(0xffffffffu, x, d);
    if (lane >= d) x += o;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    uint32_t w = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      uint32_t o = __shfl_up_sync(0xffffffffu, w, d);
      if (lane >= d) w += o;
    }
    warp_sums[lane] = w;
  }
  __syncthreads();
  const uint32_t before = warp ? warp_sums[warp - 1] : 0;
  *total = warp_sums[((blockDim.x + 31) >> 5) - 1];
  __syncthreads();
  return before + x - v;
}

// ---------------------------------------------------------------------------
// Binning.
// ---------------------------------------------------------------------------
// With `staged`, every feature's cuts and counts are first copied into
// shared memory (cols * bins + cols words), so the binary searches of a
// row's features, which touch as many cut arrays as the row has features,
// read shared memory instead of thrashing L1.
template <typename CodeT>
__global__ void quantize_kernel(const float* __restrict__ X, uint32_t rows, uint32_t cols,
                                const float* __restrict__ cuts_g, const uint32_t* __restrict__ counts_g,
                                uint32_t bins, CodeT* __restrict__ codes, uint32_t stride,
                                uint32_t missing, bool staged, unsigned long long* missing_cells) {
  extern __shared__ float staged_cuts[];
  const float* cuts = cuts_g;
  const uint32_t* counts = counts_g;
  if (staged) {
    const uint32_t n = cols * bins;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) staged_cuts[i] = cuts_g[i];
    uint32_t* sc = reinterpret_cast<uint32_t*>(staged_cuts + n);
    for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) sc[i] = counts_g[i];
    __syncthreads();
    cuts = staged_cuts;
    counts = sc;
  }
  const uint64_t total = uint64_t(rows) * stride;
  uint32_t absent = 0;  // cells of this thread without a value
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < total;
       i += uint64_t(gridDim.x) * blockDim.x) {
    const uint32_t r = uint32_t(i / stride), c = uint32_t(i % stride);
    uint32_t code = missing;
    if (c < cols) {
      const float v = X[size_t(r) * cols + c];
      const uint32_t count = counts[c];
      absent += isnan(v) ? 1u : 0u;
      if (!isnan(v) && count) {
        const float* fc = cuts + size_t(c) * bins;
        uint32_t lo = 0, hi = count;
        while (lo < hi) {
          const uint32_t mid = (lo + hi) >> 1;
          if (v >= fc[mid]) lo = mid + 1;
          else hi = mid;
        }
        code = lo < count - 1 ? lo : count - 1;
      }
    }
    codes[i] = CodeT(code);
  }
  const uint32_t warp_absent = __reduce_add_sync(0xffffffffu, absent);
  if (missing_cells && (threadIdx.x & 31) == 0 && warp_absent) atomicAdd(missing_cells, warp_absent);
}

// Feature-major copy of the codes, [cols][rows], for the partition: the rows
// of a node then read their split feature from a dense column (64x64 tiles
// through shared memory, both sides coalesced).
template <typename CodeT>
__global__ void __launch_bounds__(256) transpose_codes_kernel(const CodeT* __restrict__ codes, uint32_t rows,
                                                              uint32_t cols, uint32_t stride,
                                                              CodeT* __restrict__ fm) {
  __shared__ CodeT tile[64][65];
  const uint32_t ctiles = (cols + 63) / 64;
  const uint64_t tiles = uint64_t((rows + 63) / 64) * ctiles;
  for (uint64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const uint32_t r0 = uint32_t(t / ctiles) * 64, c0 = uint32_t(t % ctiles) * 64;
    for (uint32_t i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
      const uint32_t r = i / 64, c = i % 64;
      if (r0 + r < rows && c0 + c < cols) tile[r][c] = codes[size_t(r0 + r) * stride + c0 + c];
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
      const uint32_t c = i / 64, r = i % 64;
      if (r0 + r < rows && c0 + c < cols) fm[size_t(c0 + c) * rows + r0 + r] = tile[r][c];
    }
    __syncthreads();
  }
}

// uint16 codes [rows][s16] to uint8 codes [rows][s8] (every code below 256);
// padding columns take `pad`.
__global__ void narrow_codes_kernel(const uint16_t* __restrict__ src, uint32_t rows, uint32_t cols,
                                    uint32_t s16, uint32_t s8, uint8_t pad, uint8_t* __restrict__ dst) {
  const uint64_t total = uint64_t(rows) * s8;
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < total;
       i += uint64_t(gridDim.x) * blockDim.x) {
    const uint32_t r = uint32_t(i / s8), c = uint32_t(i % s8);
    dst[i] = c < cols ? uint8_t(src[size_t(r) * s16 + c]) : pad;
  }
}

__global__ void validate_kernel(const float4* __restrict__ X4, const float* __restrict__ X,
                                uint64_t n, unsigned int* flags) {
  unsigned int nan = 0, inf = 0;
  const uint64_t n4 = X4 ? n / 4 : 0;
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n4;
       i += uint64_t(gridDim.x) * blockDim.x) {
    const float4 v = X4[i];
    nan |= isnan(v.x) | isnan(v.y) | isnan(v.z) | isnan(v.w);
    inf |= isinf(v.x) | isinf(v.y) | isinf(v.z) | isinf(v.w);
  }
  for (uint64_t i = n4 * 4 + blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n;
       i += uint64_t(gridDim.x) * blockDim.x) {
    nan |= isnan(X[i]);
    inf |= isinf(X[i]);
  }
  nan = __reduce_or_sync(0xffffffffu, nan);
  inf = __reduce_or_sync(0xffffffffu, inf);
  if ((threadIdx.x & 31) == 0) {
    if (nan) atomicOr(flags, 1u);
    if (inf) atomicOr(flags + 1, 1u);
  }
}

// ---------------------------------------------------------------------------
// Gradients and exact power-of-two scales.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 gradient_pair(int objective, const float* __restrict__ margins,
                                                float label, float weight, uint32_t row,
                                                uint32_t groups, uint32_t k, float spw) {
  const float pred = margins[size_t(row) * groups + k];
  float w = weight, g = __fsub_rn(pred, label), h = 1.0f;
  if (objective == kLogistic || objective == kLogitRaw) {
    const float prob = __fdiv_rn(1.0f, __fadd_rn(1.0f, det_expf(-pred)));
    w = __fmul_rn(w, label == 1.0f ? spw : 1.0f);
    g = __fsub_rn(prob, label);
    h = fmaxf(__fmul_rn(prob, __fsub_rn(1.0f, prob)), 1.0e-16f);
  } else if (objective == kSoftprob || objective == kSoftmax) {
    float mx = 0x1p-126f;
    for (uint32_t j = 0; j < groups; ++j) mx = fmaxf(mx, margins[size_t(row) * groups + j]);
    double denom = 0.0;
    for (uint32_t j = 0; j < groups; ++j)
      denom = __dadd_rn(denom, (double)det_expf(__fsub_rn(margins[size_t(row) * groups + j], mx)));
    const float prob = __double2float_rn(__ddiv_rn((double)det_expf(__fsub_rn(pred, mx)), denom));
    g = __fsub_rn(prob, uint32_t(label) == k ? 1.0f : 0.0f);
    return make_float2(__fmul_rn(g, w), fmaxf(__fmul_rn(fabsf(g), w), 1.0e-16f));
  }
  return make_float2(__fmul_rn(g, w), __fmul_rn(h, w));
}

// Gradient pairs [group][row]; per (group, part) the largest magnitude.
__global__ void gradient_kernel(int objective, const float* __restrict__ margins,
                                const float* __restrict__ labels, const float* __restrict__ weights,
                                uint32_t rows, uint32_t groups, float spw, float2* __restrict__ pairs,
                                MassAccum mass) {
  const uint32_t k = blockIdx.y;
  uint32_t mg = 0, mh = 0;
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const float2 p = gradient_pair(objective, margins, labels[r], weights ? weights[r] : 1.0f, r,
                                   groups, k, spw);
    pairs[size_t(k) * rows + r] = p;
    mg = max(mg, __float_as_uint(p.x) & 0x7fffffffu);
    mh = max(mh, __float_as_uint(p.y) & 0x7fffffffu);
  }
  mg = __reduce_max_sync(0xffffffffu, mg);
  mh = __reduce_max_sync(0xffffffffu, mh);
  if ((threadIdx.x & 31) == 0) {
    if (mg) atomicMax(mass.max_bits + k * 2, mg);
    if (mh) atomicMax(mass.max_bits + k * 2 + 1, mh);
  }
}

// Windowed exact sum: every magnitude is m * 2^s in units of 2^-149
// (m < 2^24); terms are accumulated as floor(m * 2^(s - L)) in 128 bits with
// L = max(s_max - 72, 0), so the sum of at most 2^32 terms cannot overflow.
__device__ __forceinline__ uint32_t window_shift(uint32_t max_bits) {
  const uint32_t e = max_bits >> 23;
  const uint32_t smax = e ? e - 1 : 0;
  return smax > 72 ? smax - 72 : 0;
}

__device__ __forceinline__ void add_term(uint32_t bits, uint32_t L, unsigned long long& lo,
                                         unsigned long long& hi) {
  const uint32_t e = (bits >> 23) & 255;
  const unsigned long long m = (bits & 0x7fffffu) | (e ? 0x800000u : 0u);
  const int s = int(e ? e - 1 : 0) - int(L);
  unsigned long long tlo, thi;
  if (s >= 64) {
    tlo = 0;
    thi = m << (s - 64);
  } else if (s >= 0) {
    tlo = m << s;
    thi = s ? (m >> (64 - s)) : 0;
  } else {
    tlo = (-s) >= 24 ? 0 : (m >> (-s));
    thi = 0;
  }
  const unsigned long long nlo = lo + tlo;
  hi += thi + (nlo < lo ? 1 : 0);
  lo = nlo;
}

__device__ __forceinline__ void atomic_add_u128(unsigned long long* lo, unsigned long long* hi,
                                                unsigned long long vlo, unsigned long long vhi) {
  const unsigned long long old = atomicAdd(lo, vlo);
  const unsigned long long carry = (old + vlo < old) ? 1ull : 0ull;
  if (vhi + carry) atomicAdd(hi, vhi + carry);
}

__global__ void mass_window_kernel(const float2* __restrict__ pairs, uint32_t rows,
                                   MassAccum mass) {
  const uint32_t k = blockIdx.y;
  const uint32_t Lg = window_shift(mass.max_bits[k * 2]);
  const uint32_t Lh = window_shift(mass.max_bits[k * 2 + 1]);
  unsigned long long glo = 0, ghi = 0, hlo = 0, hhi = 0;
  const float2* p = pairs + size_t(k) * rows;
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const float2 v = p[r];
    add_term(__float_as_uint(v.x) & 0x7fffffffu, Lg, glo, ghi);
    add_term(__float_as_uint(v.y) & 0x7fffffffu, Lh, hlo, hhi);
  }
  // Warp reduction of the 128-bit sums.
#pragma unroll
  for (int d = 16; d; d >>= 1) {
    unsigned long long a = __shfl_down_sync(0xffffffffu, glo, d),
                       b = __shfl_down_sync(0xffffffffu, ghi, d);
    unsigned long long n = glo + a;
    ghi += b + (n < glo);
    glo = n;
    a = __shfl_down_sync(0xffffffffu, hlo, d);
    b = __shfl_down_sync(0xffffffffu, hhi, d);
    n = hlo + a;
    hhi += b + (n < hlo);
    hlo = n;
  }
  if ((threadIdx.x & 31) == 0) {
    if (glo | ghi) atomic_add_u128(mass.window + k * 4, mass.window + k * 4 + 1, glo, ghi);
    if (hlo | hhi) atomic_add_u128(mass.window + k * 4 + 2, mass.window + k * 4 + 3, hlo, hhi);
  }
}

__device__ __forceinline__ int bitlen128(unsigned long long lo, unsigned long long hi) {
  return hi ? 128 - __clzll(hi) : (lo ? 64 - __clzll(lo) : 0);
}

__device__ __forceinline__ float scale_for(int bitlen_mass) {
  const int e = bitlen_mass - 149 > 0 ? bitlen_mass - 149 : 0;
  return __uint_as_float(uint32_t(62 - e + 127) << 23);
}

// One thread per (group, part). The windowed sum A satisfies
// A * 2^L <= M < (A + n) * 2^L, so bitlen(M) = bitlen(A) + L whenever
// A + n <= 2^bitlen(A); otherwise the exact fallback decides.
__global__ void scales_kernel(MassAccum mass, float2* scales, uint32_t groups,
                              unsigned long long rows_total) {
  const uint32_t i = threadIdx.x;
  if (i >= groups * 2) return;
  const unsigned long long A_lo = mass.window[2 * i], A_hi = mass.window[2 * i + 1];
  const uint32_t L = window_shift(mass.max_bits[i]);
  const int bl = bitlen128(A_lo, A_hi);
  bool decided = true;
  if (L && bl) {
    // A + n <= 2^bl ?
    const unsigned long long lo = A_lo + rows_total, hi = A_hi + (A_lo + rows_total < A_lo ? 1 : 0);
    const int bl2 = bitlen128(lo, hi);
    const bool power_of_two = __popcll(lo) + __popcll(hi) == 1;
    decided = bl2 == bl || (bl2 == bl + 1 && power_of_two);
  }
  mass.fallback[i] = decided ? 0u : 1u;
  if (decided) {
    const float s = scale_for(bl ? bl + int(L) : 0);
    reinterpret_cast<float*>(scales)[i] = s;
  }
}

// Exact fallback: 32-bit limb sums of m * 2^s (each addend < 2^32, so 64-bit
// limb sums cannot overflow for fewer than 2^32 rows), carried afterwards.
__global__ void mass_exact_kernel(const float2* __restrict__ pairs, uint32_t rows,
                                  MassAccum mass) {
  const uint32_t k = blockIdx.y;
  const bool need_g = mass.fallback[k * 2], need_h = mass.fallback[k * 2 + 1];
  if (!need_g && !need_h) return;
  __shared__ unsigned long long limbs[2][11];
  if (threadIdx.x < 22) (&limbs[0][0])[threadIdx.x] = 0;
  __syncthreads();
  const float2* p = pairs + size_t(k) * rows;
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const float2 v = p[r];
    for (int part = 0; part < 2; ++part) {
      if (!(part ? need_h : need_g)) continue;
      const uint32_t bits = __float_as_uint(part ? v.y : v.x) & 0x7fffffffu;
      const uint32_t e = bits >> 23;
      const unsigned long long m = (bits & 0x7fffffu) | (e ? 0x800000u : 0u);
      const uint32_t s = e ? e - 1 : 0, w = s / 32, b = s % 32;
      const unsigned long long t = m << b;
      if (t & 0xffffffffull) atomicAdd(&limbs[part][w], t & 0xffffffffull);
      if (t >> 32) atomicAdd(&limbs[part][w + 1], t >> 32);
    }
  }
  __syncthreads();
  if (threadIdx.x < 20) {
    const int part = threadIdx.x / 10, w = threadIdx.x % 10;
    if (limbs[part][w]) atomicAdd(mass.exact + (k * 2 + part) * 10 + w, limbs[part][w]);
  }
}

__global__ void scales_exact_kernel(MassAccum mass, float2* scales, uint32_t groups) {
  const uint32_t i = threadIdx.x;
  if (i >= groups * 2 || !mass.fallback[i]) return;
  uint32_t limb[10];
  unsigned long long carry = 0;
  for (int w = 0; w < 10; ++w) {
    const unsigned long long s = mass.exact[i * 10 + w] + carry;
    limb[w] = uint32_t(s);
    carry = s >> 32;
  }
  int bl = 0;
  for (int w = 9; w >= 0; --w)
    if (limb[w]) {
      bl = w * 32 + 32 - __clz(limb[w]);
      break;
    }
  reinterpret_cast<float*>(scales)[i] = scale_for(bl);
}

// ---------------------------------------------------------------------------
// Base score: fixed-order binary64 sums of y*w and w over 1024-row chunks.
// ---------------------------------------------------------------------------
constexpr uint32_t kBaseChunk = 1024;

__global__ void base_chunk_kernel(int objective, const float* __restrict__ labels,
                                  const float* __restrict__ weights, uint32_t rows, uint32_t k,
                                  float spw, double* __restrict__ chunk_sums) {
  __shared__ double sy[kBaseChunk], sw[kBaseChunk];
  const uint32_t base = blockIdx.x * kBaseChunk;
  for (uint32_t i = threadIdx.x; i < kBaseChunk; i += blockDim.x) {
    const uint32_t r = base + i;
    double yw = 0.0, ww = 0.0;
    if (r < rows) {
      float y = labels[r], w = weights ? weights[r] : 1.0f;
      if (objective == kLogistic || objective == kLogitRaw) w = __fmul_rn(w, y == 1.0f ? spw : 1.0f);
      if (objective == kSoftprob || objective == kSoftmax) y = uint32_t(y) == k ? 1.0f : 0.0f;
      yw = __dmul_rn((double)y, (double)w);
      ww = (double)w;
    }
    sy[i] = yw;
    sw[i] = ww;
  }
  __syncthreads();
  for (uint32_t h = kBaseChunk / 2; h; h >>= 1) {
    for (uint32_t i = threadIdx.x; i < h; i += blockDim.x) {
      sy[i] = __dadd_rn(sy[i], sy[i + h]);
      sw[i] = __dadd_rn(sw[i], sw[i + h]);
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    chunk_sums[blockIdx.x * 2] = sy[0];
    chunk_sums[blockIdx.x * 2 + 1] = sw[0];
  }
}

__global__ void fill_margins_kernel(float* margins, const float* base, uint32_t rows,
                                    uint32_t groups) {
  const uint64_t total = uint64_t(rows) * groups;
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < total;
       i += uint64_t(gridDim.x) * blockDim.x)
    margins[i] = base[i % groups];
}

// ---------------------------------------------------------------------------
// Tree driver kernels.
// ---------------------------------------------------------------------------
struct HistArgs {
  Ellpack e;
  const float2* pairs;   // gradient pairs in the order of the level's row list
  const float2* scale;
  const unsigned int* max_bits;  // largest |g| and |h| bits of this group (float bits)
  const uint32_t* rows;
  const DriverState* state;
  const uint32_t* tile_offset;
  const uint32_t* built_left;
  const uint32_t* seg_begin;
  const uint32_t* seg_count;
  longlong2* built;      // [cols_pad][pair_stride][bins + 1]
  uint32_t pair_stride;  // pairs of this level in the built layout
  bool staged;         // the staged two-limb kernel may take this level (bins + 1 <= 257)
  bool staged3;        // the staged three-limb kernel takes the levels the two-limb one leaves
  uint32_t ngroups;
  uint32_t min_limbs;  // 3 forces three-limb accumulation (tuning; results unchanged)
};

constexpr int kHistWarps = 32;          // 1024 threads, one CTA per SM
constexpr uint32_t kHistLanes = 32;     // features per CTA: lane = feature

// The (feature group, tile) items of one CTA. When the SMs split evenly
// over the feature groups, the CTAs of all groups get the same tile ranges:
// they run in step over the same rows, so the two 64-byte halves of a row's
// 128-byte line are requested together and DRAM serves each line once
// (DRAM reads 128-byte lines even for 64-byte requests). Otherwise the items
// are split into equal contiguous runs.
__device__ __forceinline__ void hist_item_range(uint32_t total_tiles, uint32_t ngroups, uint64_t& it,
                                                uint64_t& end) {
  const uint32_t grid = gridDim.x, b = blockIdx.x;
  const uint32_t per_group = grid / ngroups;
  if (per_group >= 1 && uint64_t(per_group) * ngroups * 8 >= uint64_t(grid) * 7) {
    if (b >= per_group * ngroups) {
      it = end = 0;
      return;
    }
    const uint32_t g = b / per_group, k = b % per_group;
    it = uint64_t(g) * total_tiles + uint64_t(k) * total_tiles / per_group;
    end = uint64_t(g) * total_tiles + uint64_t(k + 1) * total_tiles / per_group;
    return;
  }
  const uint64_t items = uint64_t(total_tiles) * ngroups;
  const uint64_t per = (items + grid - 1) / grid;
  it = b * per;
  end = min(items, it + per);
}

// Limbs of one value type: three signed 32-bit limbs of L bits hold the
// CTA's exact int64 per-bin sums. L >= 17 keeps the top limb (bits >= 2L of a
// sum below 2^63) inside int32. When every |q| of the round has at most 2L
// bits (L <= 21), the top limb only receives carries and values touch two
// limbs; otherwise L >= bitlen/3 and values touch three.
struct LimbPlan {
  uint32_t L, n;
  uint32_t bits;  // bit length of the largest |q| of the round
};
__device__ __forceinline__ LimbPlan limb_plan(unsigned int max_bits, float scale) {
  const float mv = __uint_as_float(max_bits & 0x7fffffffu);
  const long long qm = __float2ll_rn(__fmul_rn(mv, scale));
  const unsigned long long a = (unsigned long long)(qm < 0 ? -qm : qm);
  const uint32_t bl = a ? 64u - __clzll(a) : 0u;
  if (bl <= 42) {
    const uint32_t L = (bl + 1) / 2;
    return {L < 17 ? 17u : L, 2u, bl};
  }
  const uint32_t L = (bl + 2) / 3;
  return {L > 21 ? 21u : L, 3u, bl};
}

__device__ __forceinline__ long long combine_limbs(const int* base, uint32_t plane, uint32_t L) {
  const unsigned long long v = (unsigned long long)(long long)base[0] +
                               ((unsigned long long)(long long)base[plane] << L) +
                               ((unsigned long long)(long long)base[2 * plane] << (2 * L));
  return (long long)v;
}

// Histograms of the built child of every node pair (or of the root).
//
// One CTA per SM walks a contiguous run of (feature group, pair, row tile)
// work items. Lane f of every warp owns feature f0 + f, so the 32 lanes of an
// atomic touch 32 consecutive words ([bin][32] layout): no bank conflicts.
// Exact int64 sums live in three signed 32-bit limbs per value (shared-memory
// atomics are 32-bit), carried between limbs every 2^(31-L) rows, and are
// recombined and flushed with 64-bit global atomics when the (group, pair)
// changes.
template <typename CodeT, bool kUnitH, bool kRoot, int NG, int NH>
__device__ __forceinline__ void hist_body(const HistArgs& a, int* smem, const DriverState& st,
                                          uint32_t Lg, uint32_t Lh) {
  const uint32_t B = a.e.bins, B1 = B + 1, C = a.e.cols;
  const uint32_t plane = B1 * kHistLanes;  // ints per limb array
  int* lg = smem;                           // g limbs: 3 planes
  int* lh = smem + 3 * plane;               // h limbs: 3 planes, or counts (unit hessian)
  const uint32_t nplanes = kUnitH ? 4 : 6;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // Per-warp staging of the 32 rows of a batch: (g0, g1, g2, h0 | count) and (h1, h2).
  int4* stage4 = reinterpret_cast<int4*>(smem + nplanes * plane) + warp * 32;
  int2* stage2 = reinterpret_cast<int2*>(reinterpret_cast<int4*>(smem + nplanes * plane) + kHistWarps * 32) +
                 warp * 32;
  const uint32_t npairs = kRoot ? 1u : st.pairs;
  const uint32_t total_tiles = st.total_tiles;
  uint64_t it, end;
  hist_item_range(total_tiles, a.ngroups, it, end);
  if (it >= end) return;
  const float2 s = *a.scale;
  const uint32_t Lmax = Lg > Lh ? Lg : Lh;
  // Rows allowed between carries: a word below 2^L plus n values below 2^L, and
  // the carry that normalise() adds to limb 1, stay inside int32.
  const uint32_t norm_rows = (1u << (31 - Lmax)) - 2;
  // Every warp takes one batch of `batch` rows per sub-chunk; 21-bit limbs
  // carry every 1023 rows, so their sub-chunks are half as long.
  const uint32_t batch = Lmax >= 21 ? 16u : 32u;
  const uint32_t sub_rows = batch * kHistWarps;
  const long long qh_unit = __float2ll_rn(s.y);
  const CodeT* __restrict__ codes = static_cast<const CodeT*>(a.e.codes);
  const uint32_t stride = a.e.stride;
  // The missing code is also its shared-memory slot; it is flushed to bin B.
  const uint32_t miss_slot = a.e.missing;

  for (uint32_t i = threadIdx.x; i < nplanes * plane; i += blockDim.x) smem[i] = 0;
  __syncthreads();

  auto normalise = [&]() {
    for (uint32_t i = threadIdx.x; i < plane; i += blockDim.x) {
#pragma unroll
      for (int v = 0; v < (kUnitH ? 1 : 2); ++v) {
        int* b = (v ? lh : lg) + i;
        const uint32_t L = v ? Lh : Lg;
        int x0 = b[0];
        const int c0 = x0 >> L;  // arithmetic shift: floor division by 2^L
        x0 -= c0 * (1 << L);
        int x1 = b[plane] + c0;
        const int c1 = x1 >> L;
        x1 -= c1 * (1 << L);
        b[0] = x0;
        b[plane] = x1;
        b[2 * plane] += c1;
      }
    }
  };
  auto flush = [&](uint32_t group, uint32_t pair) {
    const uint32_t f0 = group * kHistLanes;
    for (uint32_t i = threadIdx.x; i < plane; i += blockDim.x) {
      const uint32_t slot = i / kHistLanes, f = f0 + (i % kHistLanes);
      const uint32_t bin = slot == miss_slot ? B : slot;
      const long long g = combine_limbs(lg + i, plane, Lg);
      long long h;
      if (kUnitH) h = (long long)((unsigned long long)(unsigned)lh[i] * (unsigned long long)qh_unit);
      else h = combine_limbs(lh + i, plane, Lh);
      const bool any = kUnitH ? (g != 0 || lh[i] != 0) : (g != 0 || h != 0);
      if (any && f < C) {
        longlong2* dst = a.built + (size_t(f) * a.pair_stride + pair) * B1 + bin;
        atomicAdd(reinterpret_cast<unsigned long long*>(&dst->x), (unsigned long long)g);
        atomicAdd(reinterpret_cast<unsigned long long*>(&dst->y), (unsigned long long)h);
      }
      lg[i] = 0;
      lg[i + plane] = 0;
      lg[i + 2 * plane] = 0;
      lh[i] = 0;
      if (!kUnitH) {
        lh[i + plane] = 0;
        lh[i + 2 * plane] = 0;
      }
    }
  };
  auto split = [](long long q, uint32_t L, int& c0, int& c1, int& c2) {
    const bool neg = q < 0;
    const unsigned long long m = (unsigned long long)(neg ? -q : q), mask = (1ull << L) - 1;
    c0 = int(m & mask);
    c1 = int((m >> L) & mask);
    c2 = int(m >> (2 * L));
    if (neg) {
      c0 = -c0;
      c1 = -c1;
      c2 = -c2;
    }
  };

  int64_t cur_group = -1, cur_pair = -1;
  uint32_t since = 0;  // rows added since the last carry
  for (; it < end; ++it) {
    const uint32_t group = uint32_t(it / total_tiles), t = uint32_t(it % total_tiles);
    uint32_t pair = 0;
    if (!kRoot) {
      uint32_t lo = 0, hi = npairs;
      while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (a.tile_offset[mid] <= t) lo = mid;
        else hi = mid;
      }
      pair = lo;
    }
    if (int64_t(group) != cur_group || int64_t(pair) != cur_pair) {
      if (cur_group >= 0) {
        __syncthreads();
        flush(uint32_t(cur_group), uint32_t(cur_pair));
        __syncthreads();
        since = 0;
      }
      cur_group = group;
      cur_pair = pair;
    }
    const uint32_t slot = kRoot ? 0u : 2u * pair + (a.built_left[pair] ? 0u : 1u);
    const uint32_t seg0 = a.seg_begin[slot], segn = a.seg_count[slot];
    const uint32_t begin = seg0 + (t - (kRoot ? 0u : a.tile_offset[pair])) * kTileRows;
    const uint32_t cnt = min(kTileRows, seg0 + segn - begin);
    const uint32_t f = group * kHistLanes + lane;
    // Lanes past the last feature run the same instructions on code 0: they
    // only touch their own column, which is never flushed.
    const bool active = f < C;
    for (uint32_t sub = 0; sub < cnt; sub += sub_rows) {
      const uint32_t nsub = min(sub_rows, cnt - sub);
      const uint32_t base = warp * batch;
      const uint32_t nrows = base < nsub ? min(batch, nsub - base) : 0u;
      if (nrows) {
        // Lane i: row i of the batch, its gradient pair split into limbs once.
        const bool mine = lane < nrows;
        const uint32_t my_row =
            mine ? (kRoot ? begin + sub + base + lane : __ldg(a.rows + begin + sub + base + lane)) : 0u;
        int g0 = 0, g1 = 0, g2 = 0, h0 = 0, h1 = 0, h2 = 0;
        if (mine) {
          const float2 gp = __ldg(a.pairs + begin + sub + base + lane);
          split(__float2ll_rn(__fmul_rn(gp.x, s.x)), Lg, g0, g1, g2);
          if (kUnitH) h0 = 1;
          else split(__float2ll_rn(__fmul_rn(gp.y, s.y)), Lh, h0, h1, h2);
        }
        stage4[lane] = make_int4(g0, g1, g2, h0);
        if (!kUnitH) stage2[lane] = make_int2(h1, h2);
        __syncwarp();
        // Rows past nrows carry zero limbs and code 0: their adds are no-ops.
        for (uint32_t j0 = 0; j0 < nrows; j0 += 8) {
          uint32_t code[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const uint32_t r = __shfl_sync(0xffffffffu, my_row, j0 + u);
            code[u] = (active && j0 + u < nrows) ? uint32_t(__ldg(codes + size_t(r) * stride + f)) : 0u;
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const uint32_t idx = code[u] * kHistLanes + lane;
            const int4 q4 = stage4[j0 + u];
            atomicAdd(lg + idx, q4.x);
            atomicAdd(lg + idx + plane, q4.y);
            if (NG == 3) atomicAdd(lg + idx + 2 * plane, q4.z);
            atomicAdd(lh + idx, q4.w);
            if (!kUnitH) {
              const int2 q2 = stage2[j0 + u];
              atomicAdd(lh + idx + plane, q2.x);
              if (NH == 3) atomicAdd(lh + idx + 2 * plane, q2.y);
            }
          }
        }
        __syncwarp();
      }
      since += nsub;
      if (since + sub_rows > norm_rows) {
        __syncthreads();
        normalise();
        __syncthreads();
        since = 0;
      }
    }
  }
  __syncthreads();
  flush(uint32_t(cur_group), uint32_t(cur_pair));
}

// ---------------------------------------------------------------------------
// Staged histogram: two limbs (every |q| of the round has at most 2L bits),
// or three limbs for uint8 codes with real hessians (wider values).
//
// One CTA per SM over tile-ordered (feature group, pair, tile) items, as
// hist_body, with 16 warps (12 for three limbs, whose six limb planes leave
// room for fewer stage buffers). Each warp copies the 32-feature code slices and
// the precomputed limbs of its next 32 rows into one of two shared-memory
// stage buffers with cp.async, one step ahead of the step it accumulates, and
// loads the row ids one step ahead of the copies.
//
// Accumulation: lane r owns row r of the step. It keeps the row's limbs in
// registers and reads the row's codes with 16-byte loads, so each shared
// load feeds 8 (uint16) or 16 (uint8) features. At step f (0..31) lane r
// adds to feature f ^ r: the 32 atomics of one instruction then touch 32
// different features, which the [slot][32 features] plane layout puts in
// 32 different banks. The stage stores row r's 16-byte chunk c at position
// c ^ swz(r) (swz = (r >> 1) & 3 for uint16, (r >> 2) & 1 for uint8), so the
// 8 lanes of each quarter-warp load phase read 8 different bank groups, and
// each lane permutes its loaded codes in registers (position e holds element
// e ^ r) so that the code of feature f ^ r sits at a fixed position for
// step f. Per row and 32 features this costs 4 (3 with unit hessians)
// shared atomics plus 0.5 (uint16) or 0.25 (uint8) shared loads; the carries
// out of limb 1 stay in registers (each thread owns fixed words of the
// planes), so normalisation and flush touch only shared memory and
// registers.
constexpr uint32_t kSlots = 257;                       // bins 0..255 + missing slot (<= 256)
constexpr uint32_t kPlaneWords = kSlots * kHistLanes;  // ints per plane
constexpr uint32_t kH2Warps = 16;
constexpr uint32_t kH2Threads = kH2Warps * 32;
// The three-limb form keeps six planes (197 KB), so its CTA has 12 warps and
// takes uint8 codes only: their stage buffers then fit beside the planes.
constexpr uint32_t kH3Warps = 12;
constexpr uint32_t kStageRows = 32;                    // rows per warp per step
constexpr uint32_t kStepRows = kStageRows * kH2Warps;  // rows per CTA per step
constexpr uint32_t kStageBufs = 2;                     // one step of copies in flight
// A normalisation carries only words above this magnitude; the rows between
// two normalisations are limited so that a word left below it cannot
// overflow (see hist2_kernel).
constexpr int kCarryAbove = 1 << 26;
static_assert(kPlaneWords % 2 == 0, "planes hold whole word pairs");

template <typename CodeT>
struct __align__(16) HistStage {
  CodeT codes[kStageRows][kHistLanes];
  float2 pairs[kStageRows];
};

// Limb planes of the staged kernel: g0 g1 h0 h1 (g0 g1 count with unit
// hessians) for two limbs, g0 g1 g2 h0 h1 h2 for three.
template <bool kUnitH, uint32_t kLimbs>
constexpr uint32_t staged_planes() {
  return kLimbs == 3 ? 6u : (kUnitH ? 3u : 4u);
}

template <typename CodeT, bool kUnitH, uint32_t kLimbs = 2, uint32_t kWarps = kH2Warps>
constexpr size_t hist2_smem() {
  return size_t(staged_planes<kUnitH, kLimbs>()) * kPlaneWords * sizeof(int) +
         size_t(kWarps) * kStageBufs * sizeof(HistStage<CodeT>);
}
static_assert(hist2_smem<uint16_t, false>() <= 227 * 1024 && hist2_smem<uint8_t, false, 3, kH3Warps>() <= 227 * 1024,
              "staged histogram shared memory");

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
// Shared-memory add without a compiler memory barrier: the accumulation
// loop's loads read the stage buffers, which these adds never touch, so the
// compiler may hoist the next rows' loads above them. Every other access to
// the planes is separated from the adds by a CTA barrier.
__device__ __forceinline__ void red_shared(uint32_t addr, int v) {
  asm volatile("red.shared.add.s32 [%0], %1;\n" ::"r"(addr), "r"(v));
}
// The same at a constant offset from addr (an immediate of the instruction).
template <uint32_t kOff>
__device__ __forceinline__ void red_shared_at(uint32_t addr, int v) {
  asm volatile("red.shared.add.s32 [%0+%2], %1;\n" ::"r"(addr), "r"(v), "n"(kOff));
}

// Stage position of chunk c (16 bytes) of staged row r; see hist2_kernel.
template <typename CodeT>
__device__ __forceinline__ uint32_t stage_chunk(uint32_t r, uint32_t c) {
  return sizeof(CodeT) == 2 ? (c ^ ((r >> 1) & 3u)) : (c ^ ((r >> 2) & 1u));
}
__device__ __forceinline__ uint32_t pick(uint32_t a, uint32_t b, bool p) { return p ? b : a; }
// Reorders 16 bytes of codes in registers so that position e holds element
// e ^ x: uint16 codes (8 per quad, x < 8) or uint8 codes (16 per quad, x < 16).
template <typename CodeT>
__device__ __forceinline__ void xor_permute(uint32_t (&a)[4], uint32_t x) {
  uint32_t s, p1, p2;
  if (sizeof(CodeT) == 2) {
    s = (x & 1u) ? 0x1032u : 0x3210u;  // swap the halves of each word
    p1 = x & 2u;
    p2 = x & 4u;
  } else {
    s = (x & 2u) ? ((x & 1u) ? 0x0123u : 0x1032u) : ((x & 1u) ? 0x2301u : 0x3210u);
    p1 = x & 4u;
    p2 = x & 8u;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) a[i] = __byte_perm(a[i], 0, s);
  const uint32_t t0 = pick(a[0], a[1], p1), t1 = pick(a[1], a[0], p1);
  const uint32_t t2 = pick(a[2], a[3], p1), t3 = pick(a[3], a[2], p1);
  a[0] = pick(t0, t2, p2);
  a[2] = pick(t2, t0, p2);
  a[1] = pick(t1, t3, p2);
  a[3] = pick(t3, t1, p2);
}

// Limb plans of a round; the staged kernel takes the rounds whose values all
// fit two limbs, the three-limb kernel the others. The histogram, limb and
// partition kernels make the same choice from the same inputs.
__device__ __forceinline__ bool plan_round(const float2* scale, const unsigned int* max_bits,
                                           uint32_t min_limbs, bool staged, bool unit_h, LimbPlan& pg,
                                           LimbPlan& ph) {
  const float2 s = *scale;
  pg = limb_plan(max_bits[0], s.x);
  ph = unit_h ? LimbPlan{17u, 2u, 1u} : limb_plan(max_bits[1], s.y);
  if (min_limbs >= 3) {
    // Three limbs of L = max(17, bitlen / 3) bits hold any value of the round.
    if (pg.n == 2) pg = LimbPlan{(pg.L * 2 + 2) / 3 < 17 ? 17u : (pg.L * 2 + 2) / 3, 3u, pg.bits};
    if (!unit_h && ph.n == 2) ph = LimbPlan{(ph.L * 2 + 2) / 3 < 17 ? 17u : (ph.L * 2 + 2) / 3, 3u, ph.bits};
  }
  return staged && pg.n == 2 && ph.n == 2;
}
__device__ __forceinline__ bool plan_round(const HistArgs& a, bool unit_h, LimbPlan& pg, LimbPlan& ph) {
  return plan_round(a.scale, a.max_bits, a.min_limbs, a.staged, unit_h, pg, ph);
}

// A two-limb split of q = rint(v * s) in float arithmetic on the FMA pipe,
// which the histogram kernel leaves mostly idle: l1 = rint(q * 2^-L) and
// l0 = q - l1 * 2^L. Every step is exact: q is an integer-valued float (s is
// a power of two), scaling by 2^-L and rounding to an integer are exact, and
// |l0| <= 2^(L-1) makes the fused multiply-add exact. So l0 + l1 * 2^L = q,
// with |l0| <= 2^(L-1) and |l1| <= 2^(bits - L): the bounds the staged
// kernel's normalisation interval assumes. (Ties give l0 = +2^(L-1), which
// the balanced integer split avoids; only the sum reaches the histogram.)
struct LimbSplit {
  float two_l, inv_two_l;  // 2^L, 2^-L
  __device__ __forceinline__ void operator()(float v, float s, int& l0, int& l1) const {
    const float q = rintf(__fmul_rn(v, s));
    const float hi = rintf(__fmul_rn(q, inv_two_l));
    l1 = __float2int_rn(hi);
    l0 = __float2int_rn(__fmaf_rn(-hi, two_l, q));
  }
};

__device__ __forceinline__ LimbSplit limb_split(uint32_t L) {
  return LimbSplit{__int_as_float(int(127 + L) << 23), __int_as_float(int(127 - L) << 23)};
}

// (g0, g1, h0, h1) of one row, or (g0, g1, 1, 0) with unit hessians.
__device__ __forceinline__ int4 row_limbs(float2 gp, float2 sc, const LimbSplit& sg, const LimbSplit& sh,
                                          bool unit_h) {
  int4 v;
  sg(gp.x, sc.x, v.x, v.y);
  if (unit_h) {
    v.z = 1;
    v.w = 0;
  } else {
    sh(gp.y, sc.y, v.z, v.w);
  }
  return v;
}

// The three-limb split of q = rint(v * s), in the same float arithmetic:
// l2 = rint(q * 2^-2L), r = q - l2 * 2^2L, l1 = rint(r * 2^-L),
// l0 = r - l1 * 2^L. Each step is exact. If |q| <= 2^(2L-1), l2 = 0 and r = q.
// Otherwise ulp(q) >= 2^(2L-24) divides both q and l2 * 2^2L, and
// |r| <= 2^(2L-1), so r has at most 24 significant bits; the same holds one
// level down for l0. So l0 + l1 * 2^L + l2 * 2^2L = q, with |l0|, |l1| <=
// 2^(L-1) and |l2| <= 2^(bits - 2L).
struct LimbSplit3 {
  float two_l, inv_two_l, two_2l, inv_two_2l;  // 2^L, 2^-L, 2^2L, 2^-2L
  __device__ __forceinline__ void operator()(float v, float s, int& l0, int& l1, int& l2) const {
    const float q = rintf(__fmul_rn(v, s));
    const float top = rintf(__fmul_rn(q, inv_two_2l));
    const float r = __fmaf_rn(-top, two_2l, q);
    const float mid = rintf(__fmul_rn(r, inv_two_l));
    l2 = __float2int_rn(top);
    l1 = __float2int_rn(mid);
    l0 = __float2int_rn(__fmaf_rn(-mid, two_l, r));
  }
};

__device__ __forceinline__ LimbSplit3 limb_split3(uint32_t L) {
  return LimbSplit3{__int_as_float(int(127 + L) << 23), __int_as_float(int(127 - L) << 23),
                    __int_as_float(int(127 + 2 * L) << 23), __int_as_float(int(127 - 2 * L) << 23)};
}

// Limb width of the staged three-limb kernel for values of `bits` bits:
// L = ceil((bits + 1) / 3), so that |l2| <= 2^(L-1) as well, and at least 12
// (the register limb above l2 then holds any sum below 2^63 in int32), at
// most 21.
__device__ __forceinline__ uint32_t limb3_width(uint32_t bits) {
  const uint32_t L = (bits + 3) / 3;
  return L < 12 ? 12u : (L > 21 ? 21u : L);
}


// One step of one warp: up to kStageRows rows of one item, packed into three
// registers (group < 2^22, pair < 2^10, rows of the CTA <= kStepRows).
struct HistStep {
  uint32_t gp;    // group << 10 | pair
  uint32_t row0;  // root: first row id; else index of the first row in the row list
  uint32_t meta;  // valid << 31 | cta_rows << 8 | n
  __device__ __forceinline__ bool valid() const { return meta >> 31; }
  __device__ __forceinline__ uint32_t n() const { return meta & 0xffu; }
  __device__ __forceinline__ uint32_t cta_rows() const { return (meta >> 8) & 0xffffu; }
  __device__ __forceinline__ uint32_t group() const { return gp >> 10; }
  __device__ __forceinline__ uint32_t pair() const { return gp & 0x3ffu; }
};
static_assert(kMaxFrontier / 2 <= 0x400u && kStepRows <= 0xffffu && kStageRows <= 0xffu, "HistStep packing");

template <bool kRoot, uint32_t kStep = kStepRows>
struct HistCursor {
  uint64_t it, end;
  uint32_t k;        // step within the item
  uint32_t group, pair, begin, cnt;
  uint32_t tile;     // tile of `it` within its feature group
  uint32_t total_tiles;
  uint32_t t_lo, t_hi;   // tiles of `pair`: [t_lo, t_hi)
  uint32_t seg0, segn;   // rows of the built child of `pair`

  __device__ __forceinline__ void load_pair(const HistArgs& a) {
    if (kRoot) {
      t_lo = 0;
      t_hi = total_tiles;
      seg0 = __ldg(a.seg_begin);
      segn = __ldg(a.seg_count);
      return;
    }
    t_lo = __ldg(a.tile_offset + pair);
    t_hi = __ldg(a.tile_offset + pair + 1);
    const uint32_t slot = 2u * pair + (__ldg(a.built_left + pair) ? 0u : 1u);
    seg0 = __ldg(a.seg_begin + slot);
    segn = __ldg(a.seg_count + slot);
  }
  // Full lookup (binary search over the pairs' tile offsets).
  __device__ __forceinline__ void resolve(const HistArgs& a, uint32_t npairs) {
    group = uint32_t(it / total_tiles);
    const uint32_t t = uint32_t(it % total_tiles);
    tile = t;
    pair = 0;
    if (!kRoot) {
      uint32_t lo = 0, hi = npairs;
      while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (__ldg(a.tile_offset + mid) <= t) lo = mid;
        else hi = mid;
      }
      pair = lo;
    }
    load_pair(a);
    locate(t);
  }
  __device__ __forceinline__ void locate(uint32_t t) {
    begin = seg0 + (t - t_lo) * kTileRows;
    cnt = min(kTileRows, seg0 + segn - begin);
  }
  __device__ __forceinline__ HistStep step(uint32_t warp) const {
    HistStep s;
    const bool valid = it < end;
    s.gp = group << 10 | pair;
    const uint32_t off = k * kStep;
    const uint32_t cta_rows = valid ? min(kStep, cnt - off) : 0u;
    const uint32_t w0 = off + warp * kStageRows;
    const uint32_t n = (valid && w0 < cnt) ? min(kStageRows, cnt - w0) : 0u;
    s.meta = uint32_t(valid) << 31 | cta_rows << 8 | n;
    s.row0 = begin + w0;
    return s;
  }
  // Next step; the pair advances incrementally (items of a CTA are in tile
  // order), so only a change of feature group needs the full lookup.
  __device__ __forceinline__ void advance(const HistArgs& a, uint32_t npairs) {
    if (it >= end) return;
    if ((k + 1) * kStep < cnt) {
      ++k;
      return;
    }
    k = 0;
    if (++it >= end) return;
    const uint32_t t = ++tile;
    if (t == total_tiles) {  // next feature group
      resolve(a, npairs);
      return;
    }
    if (!kRoot && t >= t_hi) {
      do {
        ++pair;
        t_lo = t_hi;
        t_hi = __ldg(a.tile_offset + pair + 1);
      } while (t >= t_hi);
      const uint32_t slot = 2u * pair + (__ldg(a.built_left + pair) ? 0u : 1u);
      seg0 = __ldg(a.seg_begin + slot);
      segn = __ldg(a.seg_count + slot);
    }
    locate(t);
  }
};

template <typename CodeT, bool kUnitH, bool kRoot, uint32_t kLimbs = 2, uint32_t kWarps = kH2Warps>
__global__ void __launch_bounds__(kWarps * 32, 1) hist2_kernel(HistArgs a) {
  static_assert(kLimbs == 2 || (kLimbs == 3 && !kUnitH && sizeof(CodeT) == 1), "staged limb forms");
  constexpr uint32_t kThreads = kWarps * 32;
  constexpr uint32_t kStep = kStageRows * kWarps;                          // rows per CTA per step
  constexpr uint32_t kOwn4 = (kPlaneWords / 4 + kThreads - 1) / kThreads;  // word quads per thread
  extern __shared__ __align__(128) int smem[];
  const DriverState st = *a.state;
  if (!st.frontier || !st.total_tiles) return;
  LimbPlan pg, ph;
  // Two limbs when every value of the round fits them; otherwise the
  // three-limb form, staged here or the unstaged three-limb kernel.
  const bool two = plan_round(a, kUnitH, pg, ph);
  if (kLimbs == 2 ? !two : (two || !a.staged3)) return;
  if (static_cast<uint32_t>(__cvta_generic_to_shared(smem)) & 127u) {
    if (threadIdx.x == 0) atomicOr(&const_cast<DriverState*>(a.state)->error, kErrLayout);
    return;
  }
  const uint32_t Lg = kLimbs == 3 ? limb3_width(pg.bits) : pg.L;
  const uint32_t Lh = kLimbs == 3 ? limb3_width(ph.bits) : ph.L;
  const LimbSplit split_g = limb_split(Lg), split_h = limb_split(Lh);
  const LimbSplit3 split3_g = limb_split3(Lg), split3_h = limb_split3(Lh);
  constexpr uint32_t kPlanes = staged_planes<kUnitH, kLimbs>();
  constexpr uint32_t kPlaneBytes = kPlaneWords * sizeof(int);
  constexpr uint32_t kSlice = kHistLanes * sizeof(CodeT);  // bytes of a row's group slice
  const uint32_t B = a.e.bins, B1 = B + 1, C = a.e.cols;
  const uint32_t words = B1 * kHistLanes;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t npairs = kRoot ? 1u : st.pairs;
  HistCursor<kRoot, kStep> cur;
  hist_item_range(st.total_tiles, a.ngroups, cur.it, cur.end);
  cur.k = 0;
  cur.total_tiles = st.total_tiles;
  if (cur.it >= cur.end) return;
  cur.resolve(a, npairs);

  HistStage<CodeT>* stage = reinterpret_cast<HistStage<CodeT>*>(smem + kPlanes * kPlaneWords) + warp * kStageBufs;
  const float2 sc = *a.scale;
  const long long qh_unit = __float2ll_rn(sc.y);
  // Limbs (LimbSplit): |l0| <= 2^(L-1), and |l1| <= 2^(L-1) as well when
  // |q| < 2^(2L-1): a row adds at most 2^per_row_bits to a word. Three limbs
  // (LimbSplit3): |l0|, |l1| <= 2^(L-1) and |l2| <= 2^(bits-2L).
  const uint32_t Lmax = kUnitH ? Lg : (Lg > Lh ? Lg : Lh);
  uint32_t per_row_bits;
  if (kLimbs == 3) {
    const uint32_t tg_bits = pg.bits > 2 * Lg ? pg.bits - 2 * Lg : 0u;
    const uint32_t th_bits = ph.bits > 2 * Lh ? ph.bits - 2 * Lh : 0u;
    const uint32_t top_bits = tg_bits > th_bits ? tg_bits : th_bits;
    per_row_bits = top_bits > Lmax - 1 ? top_bits : Lmax - 1;
  } else {
    per_row_bits = (pg.bits + 1 <= 2 * Lg && (kUnitH || ph.bits + 1 <= 2 * Lh)) ? Lmax - 1 : Lmax;
  }
  // A normalisation leaves every word at most kCarryAbove in magnitude (a
  // carried word restarts in [0, 2^L)), so `norm_rows` more rows keep it
  // inside int32.
  const uint32_t norm_rows = uint32_t((0x7fffffffull - uint64_t(kCarryAbove)) >> per_row_bits);
  const unsigned char* codes = static_cast<const unsigned char*>(a.e.codes);
  const size_t row_bytes = size_t(a.e.stride) * sizeof(CodeT);
  const uint32_t miss_slot = a.e.missing;

  for (uint32_t i = threadIdx.x; i < kPlanes * kPlaneWords; i += blockDim.x) smem[i] = 0;
  {
    int* sz = reinterpret_cast<int*>(stage - warp * kStageBufs);
    const uint32_t n = kWarps * kStageBufs * sizeof(HistStage<CodeT>) / sizeof(int);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) sz[i] = 0;
  }
  __syncthreads();

  // Carries out of the top shared limb (limb 1, or limb 2 with three limbs)
  // of the word quads tid + k * kThreads.
  int4 tg[kOwn4], th[kOwn4];
#pragma unroll
  for (uint32_t k = 0; k < kOwn4; ++k) tg[k] = th[k] = make_int4(0, 0, 0, 0);

  // Copies of one step's code slices and gradient pairs into stage buffer
  // `buf`; `id` holds the row id of lane j's row (non-root).
  // Per lane: which 16-byte part of a row's slice it copies, and where each
  // pass's piece lands in a stage buffer (fixed for the kernel).
  constexpr uint32_t kParts = kSlice / 16;  // 4 (u16) or 2 (u8)
  constexpr uint32_t kRowsPerPass = 32 / kParts;
  constexpr uint32_t kPasses = kStageRows / kRowsPerPass;
  const uint32_t part = lane % kParts;
  const uint32_t stage0 = static_cast<uint32_t>(__cvta_generic_to_shared(stage));
  uint32_t piece_at[kPasses];
#pragma unroll
  for (uint32_t pass = 0; pass < kPasses; ++pass) {
    const uint32_t r = pass * kRowsPerPass + lane / kParts;
    piece_at[pass] = r * kSlice + stage_chunk<CodeT>(r, part) * 16;
  }
  const uint32_t pair_at = static_cast<uint32_t>(offsetof(HistStage<CodeT>, pairs)) + lane * 8;
  const unsigned char* const codes_part = codes + part * 16;
  auto issue = [&](const HistStep& s, uint32_t id, uint32_t buf) {
    if (!s.n()) return;
    const uint32_t dst = stage0 + buf * uint32_t(sizeof(HistStage<CodeT>));
    const uint32_t fvalid = min(kHistLanes, C - s.group() * kHistLanes);
    const uint32_t chunks = (fvalid * sizeof(CodeT) + 15) / 16;  // 16-byte pieces of the slice
    const unsigned char* const src = codes_part + size_t(s.group()) * kSlice;
#pragma unroll
    for (uint32_t pass = 0; pass < kPasses; ++pass) {
      const uint32_t r = pass * kRowsPerPass + lane / kParts;
      const uint32_t rid = kRoot ? s.row0 + r : __shfl_sync(0xffffffffu, id, r);
      if (r < s.n() && part < chunks) cp_async16(dst + piece_at[pass], src + size_t(rid) * row_bytes);
    }
    // Lanes past n add zeros (their pairs are not read), so the stale codes
    // of their stage rows add nothing; every stale code is a valid slot.
    if (lane < s.n()) cp_async8(dst + pair_at, a.pairs + s.row0 + lane);
  };
  auto load_ids = [&](const HistStep& s) -> uint32_t {
    if (kRoot) return 0u;
    return lane < s.n() ? __ldg(a.rows + s.row0 + lane) : 0u;
  };
  // Carries of the limbs of one word whose magnitude passed kCarryAbove: a
  // floor carry from limb 0 into limb 1, from limb 1 into limb 2 (three
  // limbs), and from the top shared limb into the register limb `top`. Each
  // limb is checked after its carry in. Returns whether a word changed.
  auto carry_up = [](int& x, int& next, uint32_t L) -> bool {
    if (abs(x) <= kCarryAbove) return false;
    const int c = x >> L;  // arithmetic shift: floor division by 2^L
    x -= c * (1 << L);
    next += c;
    return true;
  };
  auto carry1 = [](int& x0, int& x1, int& top, uint32_t L) -> bool {
    bool changed = false;
    if (abs(x0) > kCarryAbove) {
      const int c0 = x0 >> L;
      x0 -= c0 * (1 << L);
      x1 += c0;
      changed = true;
    }
    if (abs(x1) > kCarryAbove) {
      const int c1 = x1 >> L;
      x1 -= c1 * (1 << L);
      top += c1;
      changed = true;
    }
    return changed;
  };
  auto carry = [&](int* p0, int* p1, int4& top, uint32_t L) {
    int4 x0 = *reinterpret_cast<int4*>(p0), x1 = *reinterpret_cast<int4*>(p1);
    bool changed = carry1(x0.x, x1.x, top.x, L);
    changed |= carry1(x0.y, x1.y, top.y, L);
    changed |= carry1(x0.z, x1.z, top.z, L);
    changed |= carry1(x0.w, x1.w, top.w, L);
    if (changed) {
      *reinterpret_cast<int4*>(p0) = x0;
      *reinterpret_cast<int4*>(p1) = x1;
    }
  };
  auto carry3 = [&](int* p0, int* p1, int* p2, int4& top, uint32_t L) {
    int4 x0 = *reinterpret_cast<int4*>(p0), x1 = *reinterpret_cast<int4*>(p1),
         x2 = *reinterpret_cast<int4*>(p2);
    bool changed = carry_up(x0.x, x1.x, L) | carry_up(x0.y, x1.y, L) | carry_up(x0.z, x1.z, L) |
                   carry_up(x0.w, x1.w, L);
    changed |= carry1(x1.x, x2.x, top.x, L);
    changed |= carry1(x1.y, x2.y, top.y, L);
    changed |= carry1(x1.z, x2.z, top.z, L);
    changed |= carry1(x1.w, x2.w, top.w, L);
    if (changed) {
      *reinterpret_cast<int4*>(p0) = x0;
      *reinterpret_cast<int4*>(p1) = x1;
      *reinterpret_cast<int4*>(p2) = x2;
    }
  };
  auto normalise = [&]() {
    __syncthreads();
#pragma unroll
    for (uint32_t k = 0; k < kOwn4; ++k) {
      const uint32_t i = 4 * (threadIdx.x + k * kThreads);
      if (i < words) {
        if (kLimbs == 3) {
          carry3(smem + i, smem + kPlaneWords + i, smem + 2 * kPlaneWords + i, tg[k], Lg);
          carry3(smem + 3 * kPlaneWords + i, smem + 4 * kPlaneWords + i, smem + 5 * kPlaneWords + i, th[k], Lh);
        } else {
          carry(smem + i, smem + kPlaneWords + i, tg[k], Lg);
          if (!kUnitH) carry(smem + 2 * kPlaneWords + i, smem + 3 * kPlaneWords + i, th[k], Lh);
        }
      }
    }
    __syncthreads();
  };
  // Three limbs: l0 + l1 * 2^L + l2 * 2^2L + top * 2^3L, modulo 2^64.
  auto combine = [](const int* p, int top, uint32_t L) -> long long {
    return (long long)((unsigned long long)(long long)p[0] +
                       ((unsigned long long)(long long)p[kPlaneWords] << L) +
                       ((unsigned long long)(long long)p[2 * kPlaneWords] << (2 * L)) +
                       ((unsigned long long)(long long)top << (3 * L)));
  };
  auto flush = [&](uint32_t group, uint32_t pair) {
    __syncthreads();
    const uint32_t f0 = group * kHistLanes;
    int* const ph0 = smem + (kLimbs == 3 ? 3 : 2) * kPlaneWords;  // h0, or the counts
#pragma unroll
    for (uint32_t k = 0; k < kOwn4; ++k) {
      const uint32_t i0 = 4 * (threadIdx.x + k * kThreads);
      if (i0 < words) {
        const int tgs[4] = {tg[k].x, tg[k].y, tg[k].z, tg[k].w};
        const int ths[4] = {th[k].x, th[k].y, th[k].z, th[k].w};
#pragma unroll
        for (uint32_t e = 0; e < 4; ++e) {
          const uint32_t i = i0 + e;
          const uint32_t slot = i / kHistLanes, f = f0 + (i % kHistLanes);
          const uint32_t bin = slot == miss_slot ? B : slot;
          long long g, h;
          bool any;
          if constexpr (kLimbs == 3) {
            g = combine(smem + i, tgs[e], Lg);
            h = combine(ph0 + i, ths[e], Lh);
            any = g != 0 || h != 0;
          } else {
            const int topg = tgs[e], toph = ths[e];
            g = (long long)((unsigned long long)(long long)smem[i] +
                            ((unsigned long long)(long long)smem[kPlaneWords + i] << Lg) +
                            ((unsigned long long)(long long)topg << (2 * Lg)));
            if (kUnitH) {
              h = (long long)((unsigned long long)(unsigned)ph0[i] * (unsigned long long)qh_unit);
              any = g != 0 || ph0[i] != 0;
            } else {
              h = (long long)((unsigned long long)(long long)ph0[i] +
                              ((unsigned long long)(long long)ph0[kPlaneWords + i] << Lh) +
                              ((unsigned long long)(long long)toph << (2 * Lh)));
              any = g != 0 || h != 0;
            }
          }
          if (any && f < C) {
            longlong2* dst = a.built + (size_t(f) * a.pair_stride + pair) * B1 + bin;
            atomicAdd(reinterpret_cast<unsigned long long*>(&dst->x), (unsigned long long)g);
            atomicAdd(reinterpret_cast<unsigned long long*>(&dst->y), (unsigned long long)h);
          }
        }
        *reinterpret_cast<int4*>(smem + i0) = make_int4(0, 0, 0, 0);
        *reinterpret_cast<int4*>(smem + kPlaneWords + i0) = make_int4(0, 0, 0, 0);
        *reinterpret_cast<int4*>(smem + 2 * kPlaneWords + i0) = make_int4(0, 0, 0, 0);
        if (kPlanes > 3) *reinterpret_cast<int4*>(smem + 3 * kPlaneWords + i0) = make_int4(0, 0, 0, 0);
        if (kPlanes > 4) {
          *reinterpret_cast<int4*>(smem + 4 * kPlaneWords + i0) = make_int4(0, 0, 0, 0);
          *reinterpret_cast<int4*>(smem + 5 * kPlaneWords + i0) = make_int4(0, 0, 0, 0);
        }
      }
      tg[k] = make_int4(0, 0, 0, 0);
      th[k] = make_int4(0, 0, 0, 0);
    }
    __syncthreads();
  };

  // Pipeline: s0 accumulates, the copies of s1 are in flight, the row ids of
  // s2 are being loaded.
  HistStep s0 = cur.step(warp);
  cur.advance(a, npairs);
  HistStep s1 = cur.step(warp);
  cur.advance(a, npairs);
  HistStep s2 = cur.step(warp);
  uint32_t id = load_ids(s0);
  issue(s0, id, 0);
  cp_async_commit();
  id = load_ids(s1);
  uint32_t buf = 0;
  int64_t cur_group = -1, cur_pair = -1;
  uint32_t since = 0;
  const uint32_t pbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  // With the planes on a 128-byte boundary, code * 128 + pbase has zero low
  // seven bits, so the lane term is or-ed in once and the feature term is a
  // constant XOR: word code * 32 + (lane ^ f) of the plane.
  const uint32_t tbase = pbase + (lane << 2);

  while (s0.valid()) {
    cp_async_wait<0>();  // this step's copies
    __syncwarp();
    // The next step's copies go out before any flush or normalisation, so
    // that memory stays busy while every warp of the CTA carries or flushes.
    issue(s1, id, buf ^ 1);
    cp_async_commit();
    id = load_ids(s2);
    if (int64_t(s0.group()) != cur_group || int64_t(s0.pair()) != cur_pair) {
      if (cur_group >= 0) {
        flush(uint32_t(cur_group), uint32_t(cur_pair));
        since = 0;
      }
      cur_group = s0.group();
      cur_pair = s0.pair();
    }
    if (since + s0.cta_rows() > norm_rows) {
      normalise();
      since = 0;
    }
    if (s0.n()) {
      HistStage<CodeT>& st0 = stage[buf];
      // Lane = row: its limbs, formed once for 32 features; lanes past n add
      // zeros. Three limbs: (g0, g1, h0, h1) in q and (g2, h2) in q3.
      int2 q3 = make_int2(0, 0);
      int4 q;
      if constexpr (kLimbs == 3) {
        q = make_int4(0, 0, 0, 0);
        if (lane < s0.n()) {
          const float2 gp = st0.pairs[lane];
          split3_g(gp.x, sc.x, q.x, q.y, q3.x);
          split3_h(gp.y, sc.y, q.z, q.w, q3.y);
        }
      } else {
        q = lane < s0.n() ? row_limbs(st0.pairs[lane], sc, split_g, split_h, kUnitH) : make_int4(0, 0, 0, 0);
      }
      constexpr uint32_t kQuads = kSlice / 16;
      constexpr uint32_t kPerQuad = 16 / sizeof(CodeT);
      uint32_t quad[kQuads][4];
      const unsigned char* row = reinterpret_cast<const unsigned char*>(&st0.codes[lane][0]);
#pragma unroll
      for (uint32_t k = 0; k < kQuads; ++k) {
        // Quad k holds features kPerQuad * (k ^ hi) + e ^ lo after the
        // permutation, hi/lo the chunk and in-chunk bits of the lane.
        const uint32_t c = k ^ (lane / kPerQuad);
        const uint4 v = *reinterpret_cast<const uint4*>(row + stage_chunk<CodeT>(lane, c) * 16);
        quad[k][0] = v.x;
        quad[k][1] = v.y;
        quad[k][2] = v.z;
        quad[k][3] = v.w;
        xor_permute<CodeT>(quad[k], lane % kPerQuad);
      }
#pragma unroll
      for (uint32_t f = 0; f < kHistLanes; ++f) {
        const uint32_t w = quad[f / kPerQuad][(f % kPerQuad) * sizeof(CodeT) / 4];
        const uint32_t code = sizeof(CodeT) == 2 ? (w >> (16 * (f & 1))) & 0xffffu : (w >> (8 * (f & 3))) & 0xffu;
        const uint32_t addr = (code * (kHistLanes * 4) + tbase) ^ (4 * f);
        if (kLimbs == 3) {
          red_shared(addr, q.x);
          red_shared_at<kPlaneBytes>(addr, q.y);
          red_shared_at<2 * kPlaneBytes>(addr, q3.x);
          red_shared_at<3 * kPlaneBytes>(addr, q.z);
          red_shared_at<4 * kPlaneBytes>(addr, q.w);
          red_shared_at<5 * kPlaneBytes>(addr, q3.y);
        } else {
          red_shared(addr, q.x);
          red_shared_at<kPlaneBytes>(addr, q.y);
          red_shared_at<2 * kPlaneBytes>(addr, q.z);
          if (!kUnitH) red_shared_at<3 * kPlaneBytes>(addr, q.w);
        }
      }
    }
    __syncwarp();
    since += s0.cta_rows();
    s0 = s1;
    s1 = s2;
    cur.advance(a, npairs);
    s2 = cur.step(warp);
    buf ^= 1;
  }
  cp_async_wait<0>();
  flush(uint32_t(cur_group), uint32_t(cur_pair));
}

template <typename CodeT, bool kUnitH, bool kRoot>
__global__ void __launch_bounds__(1024, 1) hist_kernel(HistArgs a) {
  extern __shared__ __align__(128) int smem[];
  const DriverState st = *a.state;
  if (!st.frontier || !st.total_tiles) return;
  LimbPlan pg, ph;
  // The staged kernels build this level: the two-limb one when the round's
  // values fit two limbs, else the three-limb one where it applies.
  if (plan_round(a, kUnitH, pg, ph) || a.staged3) return;
  if (pg.n == 2 && ph.n == 2) hist_body<CodeT, kUnitH, kRoot, 2, 2>(a, smem, st, pg.L, ph.L);
  else if (pg.n == 2) hist_body<CodeT, kUnitH, kRoot, 2, 3>(a, smem, st, pg.L, ph.L);
  else if (ph.n == 2) hist_body<CodeT, kUnitH, kRoot, 3, 2>(a, smem, st, pg.L, ph.L);
  else hist_body<CodeT, kUnitH, kRoot, 3, 3>(a, smem, st, pg.L, ph.L);
}

struct EvalArgs {
  Ellpack e;
  SplitMath m;
  const float2* scale;
  const DriverState* state;
  uint32_t depth;
  const longlong2* built;    // [cols_pad][pair_stride][bins + 1]
  uint32_t pair_stride;
  uint32_t f_lo, f_hi;       // features this rank evaluates
  const longlong2* prev_bank;
  longlong2* bank;
  const uint32_t* parent_slot;
  const uint32_t* built_left;
  const long long* sums;
  DevSplit* cand;
  unsigned long long* keys;
  bool write_bank;
  // Host-driven trees: `built` holds every node's own histogram,
  // [cols][pair_stride = slots][bins + 1], with no sibling subtraction.
  bool direct;
};

struct Candidate {
  float gain, lw, rw, threshold;
  uint32_t order;
  int32_t split_bin;
  uint32_t default_left;
  double LH, RH;
  long long lg, lh, rg, rh;
};

// One warp per (node, feature): the node's histogram (the built child, or the
// parent minus the built sibling), a warp-shuffle prefix scan over the bins,
// forward candidates (missing right) and, when the node has missing rows,
// backward candidates (missing left), each scored in binary64 with the
// reference's rounding points; the best candidate by (gain, scan order).
__global__ void __launch_bounds__(256, 2) eval_kernel(EvalArgs a) {
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t nslots = a.state->frontier;
  const uint32_t C = a.e.cols, B = a.e.bins, B1 = B + 1;
  const uint32_t nf = a.f_hi > a.f_lo ? a.f_hi - a.f_lo : 0u;
  const uint64_t total = uint64_t(nslots) * nf;
  const uint64_t nwarps = uint64_t(gridDim.x) * (blockDim.x >> 5);
  const float2 sc = *a.scale;
  int eg, eh;
  frexpf(sc.x, &eg);
  frexpf(sc.y, &eh);
  const double inv_g = ldexp(1.0, -(eg - 1)), inv_h = ldexp(1.0, -(eh - 1));
  for (uint64_t w = blockIdx.x * uint64_t(blockDim.x >> 5) + (threadIdx.x >> 5); w < total; w += nwarps) {
    const uint32_t slot = uint32_t(w / nf), f = a.f_lo + uint32_t(w % nf);
    const longlong2* bptr;
    const longlong2* pptr = nullptr;
    if (a.depth == 0) {
      bptr = a.built + size_t(f) * B1;
    } else if (a.direct) {
      bptr = a.built + (size_t(f) * a.pair_stride + slot) * B1;
    } else {
      const uint32_t p = slot >> 1;
      const uint32_t built_side = a.built_left[p] ? 0u : 1u;
      bptr = a.built + (size_t(f) * a.pair_stride + p) * B1;
      if ((slot & 1u) != built_side) pptr = a.prev_bank + (size_t(a.parent_slot[p]) * C + f) * B1;
    }
    // Lane `lane` holds bins [8 lane, 8 lane + 8).
    long long vg[8], vh[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t b = lane * 8 + j;
      long long g = 0, h = 0;
      if (b < B) {
        const longlong2 x = bptr[b];
        g = x.x;
        h = x.y;
        if (pptr) {
          const longlong2 y = pptr[b];
          g = (long long)((unsigned long long)y.x - (unsigned long long)g);
          h = (long long)((unsigned long long)y.y - (unsigned long long)h);
        }
      }
      vg[j] = g;
      vh[j] = h;
    }
    long long missg, missh;
    {
      const longlong2 x = bptr[B];
      missg = x.x;
      missh = x.y;
      if (pptr) {
        const longlong2 y = pptr[B];
        missg = (long long)((unsigned long long)y.x - (unsigned long long)missg);
        missh = (long long)((unsigned long long)y.y - (unsigned long long)missh);
      }
    }
    if (a.write_bank) {
      longlong2* dst = a.bank + (size_t(slot) * C + f) * B1;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t b = lane * 8 + j;
        if (b < B) dst[b] = make_longlong2(vg[j], vh[j]);
      }
      if (lane == 0) dst[B] = make_longlong2(missg, missh);
    }
    // Lane-local inclusive prefix, then the warp scan of lane totals.
    unsigned long long pg[8], ph[8];
    unsigned long long accg = 0, acch = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      accg += (unsigned long long)vg[j];
      acch += (unsigned long long)vh[j];
      pg[j] = accg;
      ph[j] = acch;
    }
    const unsigned long long incg = warp_scan_u64(accg, lane), inch = warp_scan_u64(acch, lane);
    const unsigned long long exg = incg - accg, exh = inch - acch;
    const unsigned long long Pg = shfl_u64(incg, 31), Ph = shfl_u64(inch, 31);
    unsigned long long Tg, Th;
    if (a.depth == 0) {
      Tg = Pg + (unsigned long long)missg;
      Th = Ph + (unsigned long long)missh;
    } else {
      Tg = (unsigned long long)a.sums[slot * 2];
      Th = (unsigned long long)a.sums[slot * 2 + 1];
    }
    const unsigned long long Mg = Tg - Pg, Mh = Th - Ph;
    const double TG = stat_value((long long)Tg, inv_g), TH = stat_value((long long)Th, inv_h);
    const float wparent = leaf_weight(TG, TH, a.m);
    const float parent_gain = node_gain(TG, TH, wparent, a.m);
    const uint32_t count = a.e.counts[f];
    const float* fc = a.e.cuts + size_t(f) * B;

    Candidate best;
    best.gain = -CUDART_INF_F;
    best.order = 0xffffffffu;
    auto consider = [&](unsigned long long lg, unsigned long long lh, unsigned long long rg,
                        unsigned long long rh, uint32_t order, float threshold, int32_t sbin,
                        uint32_t dl) {
      const double LG = stat_value((long long)lg, inv_g), LH = stat_value((long long)lh, inv_h);
      const double RG = stat_value((long long)rg, inv_g), RH = stat_value((long long)rh, inv_h);
      if (!valid_hessian(LH, a.m) || !valid_hessian(RH, a.m)) return;
      const float lw = leaf_weight(LG, LH, a.m), rw = leaf_weight(RG, RH, a.m);
      const float gain =
          __fsub_rn(__fadd_rn(node_gain(LG, LH, lw, a.m), node_gain(RG, RH, rw, a.m)), parent_gain);
      if (!(gain > -CUDART_INF_F)) return;
      if (gain > best.gain || (gain == best.gain && order < best.order)) {
        best.gain = gain;
        best.order = order;
        best.lw = lw;
        best.rw = rw;
        best.threshold = threshold;
        best.split_bin = sbin;
        best.default_left = dl;
        best.LH = LH;
        best.RH = RH;
        best.lg = (long long)lg;
        best.lh = (long long)lh;
        best.rg = (long long)rg;
        best.rh = (long long)rh;
      }
    };
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t b = lane * 8 + j;
      if (b < count) {
        const unsigned long long Lg = exg + pg[j], Lh = exh + ph[j];
        consider(Lg, Lh, Tg - Lg, Th - Lh, b, fc[b], int32_t(b), 0u);
      }
    }
    if (Mg != 0 || Mh != 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t b = lane * 8 + j;
        if (b < count) {
          const unsigned long long Rg = Pg - (exg + pg[j] - (unsigned long long)vg[j]);
          const unsigned long long Rh = Ph - (exh + ph[j] - (unsigned long long)vh[j]);
          consider(Tg - Rg, Th - Rh, Rg, Rh, count + (count - 1 - b),
                   b == 0 ? a.e.minima[f] : fc[b - 1], int32_t(b) - 1, 1u);
        }
      }
    }
    // Warp argmax by (gain, order).
    float bg = best.gain;
    uint32_t bo = best.order, bl = lane;
#pragma unroll
    for (int d = 16; d; d >>= 1) {
      const float og = __shfl_xor_sync(0xffffffffu, bg, d);
      const uint32_t oo = __shfl_xor_sync(0xffffffffu, bo, d);
      const uint32_t ol = __shfl_xor_sync(0xffffffffu, bl, d);
      const bool take = (og > bg) || (og == bg && oo < bo) || (og == bg && oo == bo && ol < bl);
      if (take) {
        bg = og;
        bo = oo;
        bl = ol;
      }
    }
    const bool any = bg > -CUDART_INF_F;
    if ((any && lane == bl) || (!any && lane == 0)) {
      DevSplit r;
      r.total_g = __double2float_rn(TG);
      r.total_h = __double2float_rn(TH);
      r.parent_weight = wparent;
      r.applied_parent_weight = 0.0f;
      r.applied_parent_hessian = 0.0f;
      r.pad = 0;
      if (any) {
        r.gain = best.gain;
        r.threshold = best.threshold;
        r.feature = int32_t(f);
        r.split_bin = best.split_bin;
        r.default_left = best.default_left;
        r.left_weight = best.lw;
        r.right_weight = best.rw;
        r.left_h = __double2float_rn(best.LH);
        r.right_h = __double2float_rn(best.RH);
        r.order = best.order;
        r.left_g = best.lg;
        r.left_hs = best.lh;
        r.right_g = best.rg;
        r.right_hs = best.rh;
      } else {
        r.gain = -CUDART_INF_F;
        r.threshold = 0.0f;
        r.feature = -1;
        r.split_bin = -1;
        r.default_left = 0;
        r.left_weight = wparent;
        r.right_weight = wparent;
        r.left_h = 0.0f;
        r.right_h = 0.0f;
        r.order = 0xffffffffu;
        r.left_g = r.left_hs = r.right_g = r.right_hs = 0;
      }
      a.cand[size_t(slot) * C + f] = r;
      atomicMax(a.keys + slot, split_key(r.gain, f));
    }
  }
}

struct ControlArgs {
  Ellpack e;
  TreeParams tp;
  SplitMath m;
  const float2* scale;
  DriverState* state;
  uint32_t depth;
  const uint32_t* ids;
  const long long* sums;
  const uint32_t* seg_begin;
  const uint32_t* seg_count;
  const DevSplit* cand;
  const unsigned long long* keys;
  unsigned long long* next_keys;
  uint32_t* next_ids;
  long long* next_sums;
  uint32_t* parent_slot;
  uint32_t* mode;
  float* slot_leaf;
  uint32_t* cursor_l;
  uint32_t* cursor_r;
  uint32_t* ptile_offset;
  DevNode* nodes;
  uint32_t node_capacity;
};

// Per-node selection (first feature with the largest gain), the reference's
// expansion rule and node numbering, the node table and the next frontier.
__global__ void __launch_bounds__(1024) control_kernel(ControlArgs a) {
  __shared__ uint32_t s_node_count, s_error;
  const uint32_t n = a.state->frontier;
  const uint32_t s = threadIdx.x;
  if (threadIdx.x == 0) {
    s_node_count = a.state->node_count;
    s_error = a.state->error;
  }
  __syncthreads();
  DevSplit best{};
  uint32_t expand = 0;
  if (s < n && !s_error) {
    const unsigned long long key = a.keys[s];
    const uint32_t f = 0xffffffffu - uint32_t(key & 0xffffffffu);
    best = a.cand[size_t(s) * a.e.cols + (f < a.e.cols ? f : 0u)];
    if (best.feature >= 0) {
      const float2 sc = *a.scale;
      int eg, eh;
      frexpf(sc.x, &eg);
      frexpf(sc.y, &eh);
      const double inv_g = ldexp(1.0, -(eg - 1)), inv_h = ldexp(1.0, -(eh - 1));
      const double G = __dadd_rn(stat_value(best.left_g, inv_g), stat_value(best.right_g, inv_g));
      const double H = __dadd_rn(stat_value(best.left_hs, inv_h), stat_value(best.right_hs, inv_h));
      double value = 0.0;
      if (H > 0.0) {
        const double t = fabs(G) <= a.m.alpha ? 0.0 : (G < 0.0 ? __dadd_rn(G, a.m.alpha) : __dsub_rn(G, a.m.alpha));
        value = __ddiv_rn(-t, __dadd_rn(H, a.m.lambda));
        const double limit = fabs((double)a.tp.max_delta_step);
        if (limit != 0.0 && fabs(value) > limit) value = copysign(limit, value);
      }
      best.applied_parent_weight = __double2float_rn(value);
      best.applied_parent_hessian = __double2float_rn(H);
    }
    expand = best.feature >= 0 && best.gain > 1.0e-6f && best.gain >= a.tp.min_split_loss;
  }
  uint32_t total_expand;
  const uint32_t sel = block_exclusive_scan(expand, &total_expand);
  const uint32_t node_count = s_node_count;
  const bool overflow = node_count + 2ull * total_expand > a.node_capacity;
  const bool terminal = a.depth + 1 >= a.tp.max_depth;
  const float eta = a.tp.eta;
  if (s < n && !s_error && !overflow) {
    const uint32_t id = a.ids[s];
    DevNode node = a.nodes[id];
    node.flags |= 1u;
    node.cover = best.total_h;
    if (id == 0) {
      node.leaf = __fmul_rn(best.parent_weight, eta);
      node.base_weight = best.parent_weight;
    }
    if (expand) {
      const uint32_t left = node_count + 2 * sel;
      node.left = int32_t(left);
      node.right = int32_t(left + 1);
      node.feature = best.feature;
      node.split_bin = best.split_bin;
      node.default_left = best.default_left;
      node.threshold = best.threshold;
      node.gain = best.gain;
      node.cover = best.applied_parent_hessian;
      node.base_weight = best.applied_parent_weight;
      node.flags |= 2u;
      const float ll = __fmul_rn(best.left_weight, eta), rl = __fmul_rn(best.right_weight, eta);
      DevNode c{};
      c.left = c.right = c.feature = -1;
      c.split_bin = -1;
      c.parent = int32_t(id);
      c.leaf = ll;
      c.cover = best.left_h;
      c.base_weight = ll;
      a.nodes[left] = c;
      c.leaf = rl;
      c.cover = best.right_h;
      c.base_weight = rl;
      a.nodes[left + 1] = c;
      a.mode[s] = terminal ? 2u : 1u;
      a.slot_leaf[2 * s] = ll;
      a.slot_leaf[2 * s + 1] = rl;
      if (!terminal) {
        a.next_ids[2 * sel] = left;
        a.next_ids[2 * sel + 1] = left + 1;
        a.next_sums[4 * sel] = best.left_g;
        a.next_sums[4 * sel + 1] = best.left_hs;
        a.next_sums[4 * sel + 2] = best.right_g;
        a.next_sums[4 * sel + 3] = best.right_hs;
        a.parent_slot[sel] = s;
        a.next_keys[2 * sel] = 0;
        a.next_keys[2 * sel + 1] = 0;
      }
    } else {
      a.mode[s] = 0u;
      a.slot_leaf[2 * s] = node.leaf;
    }
    a.nodes[id] = node;
    a.cursor_l[s] = a.seg_begin[s];
    a.cursor_r[s] = a.seg_begin[s] + a.seg_count[s];
  }
  const uint32_t tiles = (s < n) ? (a.seg_count[s] + kTileRows - 1) / kTileRows : 0u;
  uint32_t total_tiles;
  const uint32_t off = block_exclusive_scan(tiles, &total_tiles);
  if (s < n) a.ptile_offset[s] = off;
  if (threadIdx.x == 0) {
    if (s_error || overflow) {
      a.state->error = s_error ? s_error : kErrCapacity;
      a.state->pad0 = 0;
      a.state->pad1 = 0;
    } else {
      a.state->node_count = node_count + 2 * total_expand;
      a.state->pad0 = total_tiles;                        // partition tiles
      a.state->pad1 = terminal ? 0u : 2u * total_expand;  // next frontier
    }
    a.ptile_offset[n] = total_tiles;
  }
}

// Distributed split search: every rank evaluates its own feature range, then
// the best candidate of each slot (key + record) is gathered from all ranks
// and the overall best written where control_kernel reads it, so every rank
// selects the same split as one GPU evaluating every feature would.
__global__ void set_frontier_kernel(DriverState* state, uint32_t frontier) { state->frontier = frontier; }

struct BestRecord {
  unsigned long long key;
  DevSplit split;
};

__global__ void pack_best_kernel(const unsigned long long* keys, const DevSplit* cand, uint32_t cols,
                                 BestRecord* out) {
  for (uint32_t s = threadIdx.x; s < kMaxFrontier; s += blockDim.x) {
    BestRecord r;
    r.key = keys[s];
    const uint32_t f = key_feature(r.key);
    if (r.key && f < cols) r.split = cand[size_t(s) * cols + f];
    else r = BestRecord{};
    out[s] = r;
  }
}

__global__ void merge_best_kernel(const DriverState* state, const BestRecord* all, uint32_t ranks,
                                  uint32_t cols, unsigned long long* keys, DevSplit* cand) {
  const uint32_t n = state->frontier;
  for (uint32_t s = threadIdx.x; s < n; s += blockDim.x) {
    unsigned long long key;
    const uint32_t best =
        merge_rank_keys(ranks, [&](uint32_t r) { return all[size_t(r) * kMaxFrontier + s].key; }, &key);
    keys[s] = key;
    const uint32_t f = key_feature(key);
    if (key && f < cols) cand[size_t(s) * cols + f] = all[size_t(best) * kMaxFrontier + s].split;
  }
}

struct PartArgs {
  Ellpack e;
  const DriverState* state;
  const uint32_t* ids;
  const DevNode* nodes;
  const uint32_t* seg_begin;
  const uint32_t* seg_count;
  const uint32_t* ptile_offset;
  const uint32_t* mode;
  const float* slot_leaf;
  const uint32_t* rows;
  uint32_t* rows_next;
  const float2* pairs;       // gradient pairs in the order of `rows`
  float2* pairs_next;        // ... and of `rows_next`
  uint32_t* cursor_l;
  uint32_t* cursor_r;
  float* margins;
  uint32_t groups, group;
  bool root;
};

// Rows of every frontier node: nodes that stop add their leaf to the row's
// margin, nodes split at the last level add the child leaf, other split nodes
// move their rows, each with its gradient pair, to the two children (left
// block from the segment start, right block from the segment end), so that
// the next level reads both in row-list order. A warp owns 256 consecutive
// rows of a 2048-row tile, lane-strided so that reads and writes coalesce;
// ranks come from warp ballots, and one cursor reservation is made per tile.
constexpr uint32_t kPartThreads = 256;
constexpr uint32_t kPartWarps = kPartThreads / 32;
constexpr uint32_t kPartIter = kTileRows / kPartThreads;  // rows per lane

template <typename CodeT>
__global__ void __launch_bounds__(kPartThreads) partition_kernel(PartArgs a) {
  __shared__ uint32_t s_off[kPartWarps][2];
  const DriverState st = *a.state;
  if (!st.frontier || st.error) return;
  const uint32_t n = st.frontier, ptiles = st.pad0;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t lt_mask = (1u << lane) - 1u;
  const CodeT* __restrict__ codes = static_cast<const CodeT*>(a.e.codes);
  const CodeT* __restrict__ fm = static_cast<const CodeT*>(a.e.codes_fm);
  for (uint32_t t = blockIdx.x; t < ptiles; t += gridDim.x) {
    uint32_t lo = 0, hi = n;
    while (hi - lo > 1) {
      const uint32_t mid = (lo + hi) >> 1;
      if (a.ptile_offset[mid] <= t) lo = mid;
      else hi = mid;
    }
    const uint32_t s = lo;
    const uint32_t seg0 = a.seg_begin[s], segn = a.seg_count[s];
    const uint32_t begin = seg0 + (t - a.ptile_offset[s]) * kTileRows;
    const uint32_t cnt = min(kTileRows, seg0 + segn - begin);
    const uint32_t md = a.mode[s];
    const DevNode node = a.nodes[a.ids[s]];
    const float leaf_l = a.slot_leaf[2 * s], leaf_r = a.slot_leaf[2 * s + 1];
    const uint32_t w0 = warp * (kTileRows / kPartWarps);
    uint32_t rows[kPartIter];
    uint32_t left_bits = 0, valid_bits = 0;
#pragma unroll
    for (uint32_t k = 0; k < kPartIter; ++k) {
      const uint32_t i = w0 + k * 32 + lane;
      const bool valid = i < cnt;
      rows[k] = valid ? (a.root ? begin + i : a.rows[begin + i]) : 0u;
      valid_bits |= uint32_t(valid) << k;
    }
    // All of a lane's split codes are loaded before any is used, and all of
    // its margins before any is stored, so the random reads of a deep level
    // are in flight together.
    uint32_t code[kPartIter];
#pragma unroll
    for (uint32_t k = 0; k < kPartIter; ++k) {
      code[k] = 0;
      if (md != 0 && ((valid_bits >> k) & 1u))
        code[k] = fm ? fm[size_t(node.feature) * a.e.rows + rows[k]]
                     : codes[size_t(rows[k]) * a.e.stride + uint32_t(node.feature)];
    }
#pragma unroll
    for (uint32_t k = 0; k < kPartIter; ++k) {
      const bool left = code[k] == a.e.missing ? node.default_left != 0u : int32_t(code[k]) <= node.split_bin;
      left_bits |= uint32_t(left) << k;
    }
    if (md != 1) {
      // A stopping node adds its leaf to every row's margin; a split at the
      // last level adds the child's leaf.
      float* m[kPartIter];
      float v[kPartIter];
#pragma unroll
      for (uint32_t k = 0; k < kPartIter; ++k) {
        m[k] = a.margins + size_t(rows[k]) * a.groups + a.group;
        v[k] = ((valid_bits >> k) & 1u) ? *m[k] : 0.0f;
      }
#pragma unroll
      for (uint32_t k = 0; k < kPartIter; ++k)
        if ((valid_bits >> k) & 1u)
          *m[k] = __fadd_rn(v[k], md == 0 ? leaf_l : (((left_bits >> k) & 1u) ? leaf_l : leaf_r));
      continue;  // uniform across the block
    }
    // Per-warp totals, then warp offsets within the tile and the tile's
    // positions in the two child blocks.
    uint32_t nl = 0, nr = 0;
#pragma unroll
    for (uint32_t k = 0; k < kPartIter; ++k) {
      const bool valid = (valid_bits >> k) & 1u, left = (left_bits >> k) & 1u;
      nl += __popc(__ballot_sync(0xffffffffu, valid && left));
      nr += __popc(__ballot_sync(0xffffffffu, valid && !left));
    }
    if (lane == 0) {
      s_off[warp][0] = nl;
      s_off[warp][1] = nr;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t tl = 0, tr = 0;
      for (uint32_t w = 0; w < kPartWarps; ++w) {
        const uint32_t l = s_off[w][0], r = s_off[w][1];
        s_off[w][0] = tl;
        s_off[w][1] = tr;
        tl += l;
        tr += r;
      }
      const uint32_t lb = tl ? atomicAdd(a.cursor_l + s, tl) : 0u;
      const uint32_t rb = tr ? atomicSub(a.cursor_r + s, tr) - tr : 0u;
      for (uint32_t w = 0; w < kPartWarps; ++w) {
        s_off[w][0] += lb;
        s_off[w][1] += rb;
      }
    }
    __syncthreads();
    uint32_t lpos = s_off[warp][0], rpos = s_off[warp][1];
#pragma unroll
    for (uint32_t k = 0; k < kPartIter; ++k) {
      const bool valid = (valid_bits >> k) & 1u, left = (left_bits >> k) & 1u;
      const uint32_t bl = __ballot_sync(0xffffffffu, valid && left);
      const uint32_t br = __ballot_sync(0xffffffffu, valid && !left);
      if (valid) {
        const uint32_t pos = left ? lpos + __popc(bl & lt_mask) : rpos + __popc(br & lt_mask);
        a.rows_next[pos] = rows[k];
        const uint32_t src = begin + w0 + k * 32 + lane;
        a.pairs_next[pos] = __ldg(a.pairs + src);
      }
      lpos += __popc(bl);
      rpos += __popc(br);
    }
    __syncthreads();
  }
}

// Loads of streamed data that should leave L2 first (evict-first policy).
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint32_t ld_stream_u32(const uint32_t* p, uint64_t pol) {
  uint32_t v;
  asm volatile("ld.global.nc.L2::cache_hint.u32 %0, [%1], %2;\n" : "=r"(v) : "l"(p), "l"(pol));
  return v;
}
__device__ __forceinline__ uint32_t ld_stream_code(const uint16_t* p, uint64_t pol) {
  unsigned short v;
  asm volatile("ld.global.nc.L2::cache_hint.u16 %0, [%1], %2;\n" : "=h"(v) : "l"(p), "l"(pol));
  return v;
}
__device__ __forceinline__ uint32_t ld_stream_code(const uint8_t* p, uint64_t pol) {
  unsigned short v;
  asm volatile("ld.global.nc.L2::cache_hint.u8 %0, [%1], %2;\n" : "=h"(v) : "l"(p), "l"(pol));
  return v;
}

// The last level: every frontier node stops (its leaf goes to all its rows)
// or splits into two leaves, and no row moves. Only margins change, at
// random row ids, so the level runs in passes over ranges of row ids: each
// pass walks the whole row list but reads and writes only the margins of
// rows in [row_lo, row_hi), which then stay in L2 across the pass (the row
// ids and split codes stream through with an evict-first policy). The
// result is the partition kernel's: margin += leaf, one add per row.
template <typename CodeT>
__global__ void __launch_bounds__(kPartThreads) leaf_margin_kernel(PartArgs a, uint32_t row_lo, uint32_t row_hi) {
  const DriverState st = *a.state;
  if (!st.frontier || st.error) return;
  const uint32_t n = st.frontier, ptiles = st.pad0;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const CodeT* __restrict__ codes = static_cast<const CodeT*>(a.e.codes);
  const CodeT* __restrict__ fm = static_cast<const CodeT*>(a.e.codes_fm);
  const uint64_t pol = evict_first_policy();
  for (uint32_t t = blockIdx.x; t < ptiles; t += gridDim.x) {
    uint32_t lo = 0, hi = n;
    while (hi - lo > 1) {
      const uint32_t mid = (lo + hi) >> 1;
      if (a.ptile_offset[mid] <= t) lo = mid;
      else hi = mid;
    }
    const uint32_t s = lo;
    const uint32_t seg0 = a.seg_begin[s], segn = a.seg_count[s];
    const uint32_t begin = seg0 + (t - a.ptile_offset[s]) * kTileRows;
    const uint32_t cnt = min(kTileRows, seg0 + segn - begin);
    const uint32_t md = a.mode[s];
    const DevNode node = a.nodes[a.ids[s]];
    const float leaf_l = a.slot_leaf[2 * s], leaf_r = a.slot_leaf[2 * s + 1];
    const uint32_t w0 = warp * (kTileRows / kPartWarps);
    uint32_t rows[kPartIter], take = 0;
#pragma unroll
    for (uint32_t k = 0; k < kPartIter; ++k) {
      const uint32_t i = w0 + k * 32 + lane;
      rows[k] = 0;
      if (i < cnt) {
        rows[k] = a.root ? begin + i : ld_stream_u32(a.rows + begin + i, pol);
        take |= uint32_t(rows[k] >= row_lo && rows[k] < row_hi) << k;
      }
    }
    uint32_t code[kPartIter];
#pragma unroll
    for (uint32_t k = 0; k < kPartIter; ++k) {
      code[k] = 0;
      if (md != 0 && ((take >> k) & 1u))
        code[k] = fm ? ld_stream_code(fm + size_t(node.feature) * a.e.rows + rows[k], pol)
                     : ld_stream_code(codes + size_t(rows[k]) * a.e.stride + uint32_t(node.feature), pol);
    }
    float* m[kPartIter];
    float v[kPartIter];
#pragma unroll
    for (uint32_t k = 0; k < kPartIter; ++k) {
      m[k] = a.margins + size_t(rows[k]) * a.groups + a.group;
      v[k] = ((take >> k) & 1u) ? *m[k] : 0.0f;
    }
#pragma unroll
    for (uint32_t k = 0; k < kPartIter; ++k) {
      if (!((take >> k) & 1u)) continue;
      const bool left = code[k] == a.e.missing ? node.default_left != 0u : int32_t(code[k]) <= node.split_bin;
      *m[k] = __fadd_rn(v[k], md == 0 ? leaf_l : (left ? leaf_l : leaf_r));
    }
  }
}

// Local child counts of split nodes, [slot][left, right].
__global__ void counts_kernel(const DriverState* state, const uint32_t* seg_begin,
                              const uint32_t* seg_count, const uint32_t* mode,
                              const uint32_t* cursor_l, uint32_t* counts) {
  const uint32_t n = state->frontier;
  for (uint32_t s = threadIdx.x; s < kMaxFrontier; s += blockDim.x) {
    uint32_t l = 0, r = 0;
    if (s < n && mode[s] == 1u) {
      l = cursor_l[s] - seg_begin[s];
      r = seg_count[s] - l;
    }
    counts[2 * s] = l;
    counts[2 * s + 1] = r;
  }
}

struct PlanArgs {
  DriverState* state;
  unsigned long long* level_rows;
  uint32_t* level_nodes;
  uint32_t next_depth;
  const uint32_t* parent_slot;
  const uint32_t* seg_begin_cur;
  const uint32_t* counts_local;
  const uint32_t* counts_global;
  uint32_t* seg_begin;
  uint32_t* seg_count;
  uint32_t* built_left;
  uint32_t* tile_offset;
};

// Next level: child segments, the smaller child of each pair to build (by
// the counts over all ranks; ties build the left child,
// kernels/boost.metal:672) and the row tiles of the built children.
__global__ void __launch_bounds__(1024) plan_kernel(PlanArgs a) {
  const DriverState st = *a.state;
  const uint32_t next = st.error ? 0u : st.pad1;
  const uint32_t pairs = next / 2;
  const uint32_t p = threadIdx.x;
  uint32_t tiles = 0;
  if (p < pairs) {
    const uint32_t s = a.parent_slot[p];
    const uint32_t begin = a.seg_begin_cur[s];
    const uint32_t nl = a.counts_local[2 * s], nr = a.counts_local[2 * s + 1];
    const uint32_t gl = a.counts_global[2 * s], gr = a.counts_global[2 * s + 1];
    a.seg_begin[2 * p] = begin;
    a.seg_count[2 * p] = nl;
    a.seg_begin[2 * p + 1] = begin + nl;
    a.seg_count[2 * p + 1] = nr;
    const bool bl = gl <= gr;
    a.built_left[p] = bl ? 1u : 0u;
    tiles = ((bl ? nl : nr) + kTileRows - 1) / kTileRows;
    if (a.next_depth < kMaxDepth) atomicAdd(a.level_rows + a.next_depth, (unsigned long long)(bl ? nl : nr));
  }
  uint32_t total;
  const uint32_t off = block_exclusive_scan(tiles, &total);
  if (p < pairs) a.tile_offset[p] = off;
  __syncthreads();
  if (threadIdx.x == 0) {
    if (a.next_depth < kMaxDepth) a.level_nodes[a.next_depth] = pairs;
    a.tile_offset[pairs] = total;
    a.state->frontier = next;
    a.state->depth = a.next_depth;
    a.state->pairs = pairs;
    a.state->total_tiles = total;
  }
}

__global__ void init_tree_kernel(DriverState* state, uint32_t rows, uint32_t* ids,
                                 long long* sums, uint32_t* seg_begin, uint32_t* seg_count,
                                 uint32_t* tile_offset, uint32_t* built_left,
                                 unsigned long long* keys, DevNode* nodes,
                                 unsigned long long* level_rows, uint32_t* level_nodes) {
  for (uint32_t d = 0; d < kMaxDepth; ++d) {
    level_rows[d] = 0;
    level_nodes[d] = 0;
  }
  level_rows[0] = rows;
  level_nodes[0] = 1;
  const uint32_t tiles = (rows + kTileRows - 1) / kTileRows;
  DriverState s{};
  s.node_count = 1;
  s.frontier = 1;
  s.pairs = 1;
  s.total_tiles = tiles;
  *state = s;
  ids[0] = 0;
  sums[0] = 0;
  sums[1] = 0;
  seg_begin[0] = 0;
  seg_count[0] = rows;
  tile_offset[0] = 0;
  tile_offset[1] = tiles;
  built_left[0] = 1;
  keys[0] = 0;
  DevNode root{};
  root.left = root.right = root.parent = root.feature = -1;
  root.split_bin = -1;
  nodes[0] = root;
}

// ---------------------------------------------------------------------------
// Prediction from raw features (x < threshold goes left, NaN takes the
// default direction; kernels/boost.metal:1325-1329, 1738-1765).
// ---------------------------------------------------------------------------
__global__ void predict_kernel(const float* __restrict__ X, uint32_t rows, uint32_t cols,
                               const DevNode* __restrict__ nodes, const uint32_t* tree_begin,
                               const uint32_t* tree_group, uint32_t trees, const float* base,
                               uint32_t groups, float* out) {
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const float* x = X + size_t(r) * cols;
    for (uint32_t k = 0; k < groups; ++k) {
      float sum = base[k];
      for (uint32_t t = 0; t < trees; ++t) {
        if (tree_group[t] != k) continue;
        const DevNode* tn = nodes + tree_begin[t];
        int32_t n = 0;
        while (tn[n].left >= 0) {
          const float v = x[tn[n].feature];
          const bool left = isnan(v) ? tn[n].default_left != 0u : v < tn[n].threshold;
          n = left ? tn[n].left : tn[n].right;
        }
        sum = __fadd_rn(sum, tn[n].leaf);
      }
      out[size_t(r) * groups + k] = sum;
    }
  }
}

// The leaf each row reaches in each tree, as the node id in float32:
// out[row][tree] (pred_leaf; the reference's predict_leaf kernel).
__global__ void leaf_index_kernel(const float* __restrict__ X, uint32_t rows, uint32_t cols,
                                  const DevNode* __restrict__ nodes, const uint32_t* tree_begin,
                                  uint32_t trees, float* out) {
  for (uint32_t t = blockIdx.y; t < trees; t += gridDim.y) {
    const DevNode* tn = nodes + tree_begin[t];
    for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
      const float* x = X + size_t(r) * cols;
      int32_t n = 0;
      while (tn[n].left >= 0) {
        const float v = x[tn[n].feature];
        const bool left = isnan(v) ? tn[n].default_left != 0u : v < tn[n].threshold;
        n = left ? tn[n].left : tn[n].right;
      }
      out[size_t(r) * trees + t] = float(n);
    }
  }
}

// Output transforms (kernels/boost.metal:1855-1885) with det_expf.
__global__ void transform_kernel(int objective, float* v, uint32_t rows, uint32_t groups) {
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    float* x = v + size_t(r) * groups;
    if (objective == kSoftprob) {
      float mx = -CUDART_INF_F, denom = 0.0f;
      for (uint32_t k = 0; k < groups; ++k) mx = fmaxf(mx, x[k]);
      for (uint32_t k = 0; k < groups; ++k) denom = __fadd_rn(denom, det_expf(__fsub_rn(x[k], mx)));
      for (uint32_t k = 0; k < groups; ++k) x[k] = __fdiv_rn(det_expf(__fsub_rn(x[k], mx)), denom);
    } else if (objective == kSoftmax) {
      uint32_t best = 0;
      for (uint32_t k = 1; k < groups; ++k)
        if (x[k] > x[best]) best = k;
      x[0] = float(best);
    } else if (objective == kLogistic) {
      for (uint32_t k = 0; k < groups; ++k)
        x[k] = __fdiv_rn(1.0f, __fadd_rn(1.0f, det_expf(-x[k])));
    }
  }
}

__global__ void window_to_limbs_kernel(MassAccum m, uint32_t n) {
  const uint32_t i = threadIdx.x;
  if (i >= n) return;
  const unsigned long long lo = m.window[2 * i], hi = m.window[2 * i + 1];
  m.limbs[4 * i] = lo & 0xffffffffull;
  m.limbs[4 * i + 1] = lo >> 32;
  m.limbs[4 * i + 2] = hi & 0xffffffffull;
  m.limbs[4 * i + 3] = hi >> 32;
}

__global__ void limbs_to_window_kernel(MassAccum m, uint32_t n) {
  const uint32_t i = threadIdx.x;
  if (i >= n) return;
  unsigned long long carry = 0, w[4];
  for (int k = 0; k < 4; ++k) {
    const unsigned long long s = m.limbs[4 * i + k] + carry;
    w[k] = s & 0xffffffffull;
    carry = s >> 32;
  }
  m.window[2 * i] = w[0] | (w[1] << 32);
  m.window[2 * i + 1] = w[2] | (w[3] << 32);
}

// Blocks for `work` items at `threads` per block, at most `per_sm` blocks per
// streaming multiprocessor of the device.
int grid_for(uint64_t work, int threads, int per_sm = 16) {
  const uint64_t blocks = (work + threads - 1) / threads;
  return int(std::max<uint64_t>(1, std::min<uint64_t>(blocks, uint64_t(device_sms()) * per_sm)));
}

}  // namespace

int device_sms() {
  constexpr int kDevices = 64;
  static int cache[kDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kDevices) return 148;
  if (!cache[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// ---------------------------------------------------------------------------
// Launchers.
// ---------------------------------------------------------------------------
MassAccum mass_view(void* base, uint32_t groups) {
  char* p = static_cast<char*>(base);
  const size_t n = size_t(groups) * 2;
  MassAccum m;
  m.window = reinterpret_cast<unsigned long long*>(p);
  m.limbs = m.window + 2 * n;
  m.exact = m.limbs + 4 * n;
  m.max_bits = reinterpret_cast<unsigned int*>(m.exact + 10 * n);
  m.fallback = m.max_bits + n;
  return m;
}

void launch_window_to_limbs(MassAccum m, uint32_t groups, cudaStream_t stream) {
  window_to_limbs_kernel<<<1, 64 * ((2 * groups + 63) / 64), 0, stream>>>(m, 2 * groups);
  XGBB_CUDA(cudaGetLastError());
}

void launch_limbs_to_window(MassAccum m, uint32_t groups, cudaStream_t stream) {
  limbs_to_window_kernel<<<1, 64 * ((2 * groups + 63) / 64), 0, stream>>>(m, 2 * groups);
  XGBB_CUDA(cudaGetLastError());
}

void launch_transpose_codes(const void* codes, uint32_t rows, uint32_t cols, uint32_t stride,
                            uint32_t bytes_per_code, void* fm, cudaStream_t stream) {
  const uint64_t tiles = uint64_t((rows + 63) / 64) * ((cols + 63) / 64);
  if (!tiles) return;
  const int blocks = grid_for(tiles, 1, 16);
  if (bytes_per_code == 1)
    transpose_codes_kernel<uint8_t><<<blocks, 256, 0, stream>>>(
        static_cast<const uint8_t*>(codes), rows, cols, stride, static_cast<uint8_t*>(fm));
  else
    transpose_codes_kernel<uint16_t><<<blocks, 256, 0, stream>>>(
        static_cast<const uint16_t*>(codes), rows, cols, stride, static_cast<uint16_t*>(fm));
  XGBB_CUDA(cudaGetLastError());
}

void launch_quantize(const float* X, uint32_t rows, uint32_t cols, const float* cuts,
                     const uint32_t* counts, uint32_t bins, void* codes, uint32_t stride,
                     uint32_t bytes_per_code, uint32_t missing, unsigned long long* missing_cells,
                     cudaStream_t stream) {
  const uint64_t total = uint64_t(rows) * stride;
  if (!total) return;
  constexpr size_t kStagedMax = 160 * 1024;
  const size_t smem = (size_t(cols) * bins + cols) * 4;
  const bool staged = smem <= kStagedMax;
  static bool configured = false;
  if (!configured) {
    XGBB_CUDA(cudaFuncSetAttribute(quantize_kernel<uint8_t>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   int(kStagedMax)));
    XGBB_CUDA(cudaFuncSetAttribute(quantize_kernel<uint16_t>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   int(kStagedMax)));
    configured = true;
  }
  // Staged: one 1024-thread block per SM walks the values; otherwise many
  // small blocks.
  const int threads = staged ? 1024 : 256;
  const int blocks = staged ? int(std::min<uint64_t>(device_sms(), (total + threads - 1) / threads))
                            : grid_for(total, threads, 32);
  if (bytes_per_code == 1)
    quantize_kernel<uint8_t><<<blocks, threads, staged ? smem : 0, stream>>>(
        X, rows, cols, cuts, counts, bins, static_cast<uint8_t*>(codes), stride, missing, staged, missing_cells);
  else
    quantize_kernel<uint16_t><<<blocks, threads, staged ? smem : 0, stream>>>(
        X, rows, cols, cuts, counts, bins, static_cast<uint16_t*>(codes), stride, missing, staged, missing_cells);
  XGBB_CUDA(cudaGetLastError());
}

void launch_narrow_codes(const void* src, uint32_t rows, uint32_t cols, uint32_t s16, uint32_t s8,
                         uint32_t pad, void* dst, cudaStream_t stream) {
  const uint64_t total = uint64_t(rows) * s8;
  if (!total) return;
  narrow_codes_kernel<<<grid_for(total, 256, 16), 256, 0, stream>>>(
      static_cast<const uint16_t*>(src), rows, cols, s16, s8, uint8_t(pad), static_cast<uint8_t*>(dst));
  XGBB_CUDA(cudaGetLastError());
}

void launch_validate(const float* X, uint64_t n, unsigned int* flags, cudaStream_t stream) {
  if (!n) return;
  const bool aligned = (reinterpret_cast<uintptr_t>(X) & 15) == 0;
  validate_kernel<<<grid_for(n / 4 + 1, 256, 8), 256, 0, stream>>>(
      aligned ? reinterpret_cast<const float4*>(X) : nullptr, X, n, flags);
  XGBB_CUDA(cudaGetLastError());
}

void launch_gradients(int objective, const float* margins, const float* labels,
                      const float* weights, uint32_t rows, uint32_t groups, float spw,
                      float2* pairs, MassAccum mass, cudaStream_t stream) {
  if (!rows) return;
  const int threads = 256;
  dim3 grid(grid_for(rows, threads, 4), groups);
  gradient_kernel<<<grid, threads, 0, stream>>>(objective, margins, labels, weights, rows, groups,
                                                spw, pairs, mass);
  XGBB_CUDA(cudaGetLastError());
}

void launch_mass_window(const float2* pairs, uint32_t rows, uint32_t groups, MassAccum mass,
                        cudaStream_t stream) {
  if (!rows) return;
  const int threads = 256;
  dim3 grid(grid_for(rows, threads, 4), groups);
  mass_window_kernel<<<grid, threads, 0, stream>>>(pairs, rows, mass);
  XGBB_CUDA(cudaGetLastError());
}

void launch_scales(const float2*, uint32_t, uint32_t groups, MassAccum mass, float2* scales,
                   unsigned long long rows_total, bool, cudaStream_t stream) {
  scales_kernel<<<1, 64 * ((2 * groups + 63) / 64), 0, stream>>>(mass, scales, groups, rows_total);
  XGBB_CUDA(cudaGetLastError());
}

void launch_mass_exact(const float2* pairs, uint32_t rows, uint32_t groups, MassAccum mass,
                       cudaStream_t stream) {
  if (!rows) return;
  const int threads = 256;
  dim3 grid(grid_for(rows, threads, 4), groups);
  mass_exact_kernel<<<grid, threads, 0, stream>>>(pairs, rows, mass);
  XGBB_CUDA(cudaGetLastError());
}

void launch_scales_exact(uint32_t groups, MassAccum mass, float2* scales, cudaStream_t stream) {
  scales_exact_kernel<<<1, 64 * ((2 * groups + 63) / 64), 0, stream>>>(mass, scales, groups);
  XGBB_CUDA(cudaGetLastError());
}

void launch_base_chunks(int objective, const float* labels, const float* weights, uint32_t rows,
                        uint32_t group, float spw, double* chunk_sums, cudaStream_t stream) {
  const uint32_t chunks = (rows + kBaseChunk - 1) / kBaseChunk;
  if (!chunks) return;
  base_chunk_kernel<<<chunks, 512, 0, stream>>>(objective, labels, weights, rows, group, spw,
                                                chunk_sums);
  XGBB_CUDA(cudaGetLastError());
}

void launch_fill_margins(float* margins, const float* base, uint32_t rows, uint32_t groups,
                         cudaStream_t stream) {
  const uint64_t total = uint64_t(rows) * groups;
  if (!total) return;
  fill_margins_kernel<<<grid_for(total, 256), 256, 0, stream>>>(margins, base, rows, groups);
  XGBB_CUDA(cudaGetLastError());
}

HistConfig hist_config(const Ellpack& e, bool unit_hessian) {
  HistConfig c;
  c.feature_group = kHistLanes;
  c.smem = size_t(unit_hessian ? 4 : 6) * (e.bins + 1) * kHistLanes * sizeof(int) +
           size_t(kHistWarps) * 32 * (sizeof(int4) + (unit_hessian ? 0 : sizeof(int2)));
  c.threads = kHistWarps * 32;
  return c;
}

namespace {
template <typename CodeT, bool kUnit, bool kRoot>
void launch_hist_t(const HistArgs& args, int blocks, int threads, size_t smem, cudaStream_t stream) {
  auto kernel = hist_kernel<CodeT, kUnit, kRoot>;
  static bool configured = false;
  if (!configured) {
    XGBB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    configured = true;
  }
  kernel<<<blocks, threads, smem, stream>>>(args);
  if (args.staged) {
    // The staged kernel exits at once when the round needs three limbs (and
    // the three-limb kernel exits when it does not); the choice is made on the
    // device from the round's gradient magnitudes.
    auto staged = hist2_kernel<CodeT, kUnit, kRoot>;
    constexpr size_t smem2 = hist2_smem<CodeT, kUnit>();
    static bool configured2 = false;
    if (!configured2) {
      XGBB_CUDA(cudaFuncSetAttribute(staged, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem2)));
      configured2 = true;
    }
    staged<<<blocks, kH2Threads, smem2, stream>>>(args);
  }
  if constexpr (sizeof(CodeT) == 1 && !kUnit) {
    if (args.staged3) {
      // The staged three-limb kernel takes the rounds the two-limb one leaves
      // (the unstaged three-limb kernel above then exits at once).
      auto staged3 = hist2_kernel<CodeT, false, kRoot, 3, kH3Warps>;
      constexpr size_t smem3 = hist2_smem<CodeT, false, 3, kH3Warps>();
      static bool configured3 = false;
      if (!configured3) {
        XGBB_CUDA(cudaFuncSetAttribute(staged3, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem3)));
        configured3 = true;
      }
      staged3<<<blocks, kH3Warps * 32, smem3, stream>>>(args);
    }
  }
}
}  // namespace

void tree_init(const TreeWorkspace& ws, const TreeLaunch& tl, cudaStream_t stream) {
  init_tree_kernel<<<1, 1, 0, stream>>>(ws.state, tl.ell.rows, ws.ids[0], ws.sums[0],
                                        ws.seg_begin[0], ws.seg_count[0], ws.tile_offset,
                                        ws.built_left, ws.keys[0], ws.nodes, ws.level_rows,
                                        ws.level_nodes);
  XGBB_CUDA(cudaGetLastError());
}

namespace {
// Histograms of the built children from each row's present codes, for a
// sparse matrix (the reference's histogram_csr_accumulate,
// kernels/histogram_csr.metal.h:22-114): blocks take tiles of built rows;
// every present (feature, code) of a row adds the row's exact (g, h) with
// 64-bit global atomics, and each tile adds its rows' (g, h) sums to its
// node's totals. csr_missing_kernel then sets each built node's missing bin
// to the node total minus its present bins, mod 2^64
// (histogram_csr_finalize_missing, :117-152). Both are linear in the rows,
// so on several GPUs each rank's local histograms still sum to the global
// ones in the reduce-scatter.
struct CsrLevelArgs {
  const unsigned long long* row_ptr;  // [rows + 1]
  const uint32_t* entries;            // feature << 16 | code, present codes only
  const float2* pairs;                // this group's gradient pairs in row order
  const float2* scale;
  const uint32_t* rows;
  const DriverState* state;
  const uint32_t* tile_offset;
  const uint32_t* built_left;
  const uint32_t* seg_begin;
  const uint32_t* seg_count;
  longlong2* built;                   // [cols_pad][pair_stride][bins + 1]
  unsigned long long* totals;         // [pairs][2]
  uint32_t pair_stride, bins, cols;
  bool root;
};
constexpr int kCsrThreads = 256;

__global__ void __launch_bounds__(kCsrThreads) csr_level_hist_kernel(CsrLevelArgs a) {
  __shared__ unsigned long long tot[2];
  const DriverState st = *a.state;
  if (!st.frontier || !st.total_tiles) return;
  const uint32_t npairs = a.root ? 1u : st.pairs;
  const float2 sc = *a.scale;
  const uint32_t B1 = a.bins + 1;
  for (uint32_t t = blockIdx.x; t < st.total_tiles; t += gridDim.x) {
    uint32_t pair = 0;
    if (!a.root) {
      uint32_t lo = 0, hi = npairs;
      while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (a.tile_offset[mid] <= t) lo = mid;
        else hi = mid;
      }
      pair = lo;
    }
    const uint32_t slot = a.root ? 0u : 2u * pair + (a.built_left[pair] ? 0u : 1u);
    const uint32_t seg0 = a.seg_begin[slot], segn = a.seg_count[slot];
    const uint32_t begin = seg0 + (t - a.tile_offset[pair]) * kTileRows;
    const uint32_t cnt = min(kTileRows, seg0 + segn - begin);
    if (threadIdx.x < 2) tot[threadIdx.x] = 0;
    __syncthreads();
    unsigned long long sg = 0, sh = 0;
    for (uint32_t i = threadIdx.x; i < cnt; i += blockDim.x) {
      const uint32_t row = a.root ? begin + i : a.rows[begin + i];
      const float2 p = a.pairs[row];
      const unsigned long long qg = (unsigned long long)__float2ll_rn(__fmul_rn(p.x, sc.x));
      const unsigned long long qh = (unsigned long long)__float2ll_rn(__fmul_rn(p.y, sc.y));
      sg += qg;
      sh += qh;
      for (unsigned long long k = a.row_ptr[row], e = a.row_ptr[row + 1]; k < e; ++k) {
        const uint32_t x = a.entries[k], f = x >> 16, code = x & 0xffffu;
        if (f >= a.cols || code >= a.bins) continue;
        longlong2* dst = a.built + (size_t(f) * a.pair_stride + pair) * B1 + code;
        atomicAdd(reinterpret_cast<unsigned long long*>(&dst->x), qg);
        atomicAdd(reinterpret_cast<unsigned long long*>(&dst->y), qh);
      }
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
      sg += __shfl_down_sync(0xffffffffu, sg, d);
      sh += __shfl_down_sync(0xffffffffu, sh, d);
    }
    if ((threadIdx.x & 31) == 0) {
      atomicAdd(&tot[0], sg);
      atomicAdd(&tot[1], sh);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      atomicAdd(&a.totals[2 * pair], tot[0]);
      atomicAdd(&a.totals[2 * pair + 1], tot[1]);
    }
    __syncthreads();
  }
}

__global__ void csr_missing_kernel(const DriverState* state, bool root, longlong2* built,
                                   const unsigned long long* totals, uint32_t pair_stride, uint32_t bins,
                                   uint32_t cols) {
  const DriverState st = *state;
  if (!st.frontier || !st.total_tiles) return;
  const uint32_t npairs = root ? 1u : st.pairs;
  const uint64_t n = uint64_t(cols) * npairs;
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n; i += uint64_t(gridDim.x) * blockDim.x) {
    const uint32_t f = uint32_t(i / npairs), p = uint32_t(i % npairs);
    longlong2* h = built + (size_t(f) * pair_stride + p) * (bins + 1);
    unsigned long long g = totals[2 * p], hh = totals[2 * p + 1];
    for (uint32_t b = 0; b < bins; ++b) {
      g -= (unsigned long long)h[b].x;
      hh -= (unsigned long long)h[b].y;
    }
    h[bins].x = (long long)g;
    h[bins].y = (long long)hh;
  }
}
}  // namespace

void tree_level_hist(const TreeWorkspace& ws, const TreeLaunch& tl, uint32_t depth,
                     cudaStream_t stream) {
  const size_t bytes = size_t(max_pairs_at(depth)) * hist_node_bytes(tl.ell, tl.cols_pad);
  XGBB_CUDA(cudaMemsetAsync(ws.built, 0, bytes, stream));
  if (tl.csr_ptr) {
    XGBB_CUDA(cudaMemsetAsync(tl.csr_totals, 0, size_t(max_pairs_at(depth)) * 16, stream));
    CsrLevelArgs c;
    c.row_ptr = tl.csr_ptr;
    c.entries = tl.csr_entries;
    c.pairs = tl.pairs;
    c.scale = tl.scale;
    c.rows = ws.rows[depth & 1];
    c.state = ws.state;
    c.tile_offset = ws.tile_offset;
    c.built_left = ws.built_left;
    c.seg_begin = ws.seg_begin[depth & 1];
    c.seg_count = ws.seg_count[depth & 1];
    c.built = ws.built;
    c.totals = tl.csr_totals;
    c.pair_stride = max_pairs_at(depth);
    c.bins = tl.ell.bins;
    c.cols = tl.ell.cols;
    c.root = depth == 0;
    csr_level_hist_kernel<<<device_sms() * 8, kCsrThreads, 0, stream>>>(c);
    XGBB_CUDA(cudaGetLastError());
    csr_missing_kernel<<<grid_for(uint64_t(tl.ell.cols) * c.pair_stride, 256), 256, 0, stream>>>(
        ws.state, c.root, ws.built, tl.csr_totals, c.pair_stride, tl.ell.bins, tl.ell.cols);
    XGBB_CUDA(cudaGetLastError());
    return;
  }
  HistArgs a;
  a.e = tl.ell;
  a.pairs = depth == 0 ? tl.pairs : ws.ord[depth & 1];
  a.scale = tl.scale;
  a.rows = ws.rows[depth & 1];
  a.state = ws.state;
  a.tile_offset = ws.tile_offset;
  a.built_left = ws.built_left;
  a.seg_begin = ws.seg_begin[depth & 1];
  a.seg_count = ws.seg_count[depth & 1];
  a.built = ws.built;
  a.pair_stride = max_pairs_at(depth);
  a.staged = tl.ell.bins + 1 <= kSlots;
  a.staged3 = a.staged && tl.staged3 && tl.ell.bytes_per_code == 1 && !tl.unit_hessian;
  a.max_bits = tl.max_bits;
  a.min_limbs = tl.min_limbs;
  a.ngroups = (tl.ell.cols + kHistLanes - 1) / kHistLanes;
  const bool root = depth == 0;
  const bool u8 = tl.ell.bytes_per_code == 1;
  const int b = tl.hist_blocks, t = tl.hist_threads;
  const size_t sm = tl.hist_smem;
#define XGBB_HIST(C, U, R) launch_hist_t<C, U, R>(a, b, t, sm, stream)
  if (u8) {
    if (tl.unit_hessian) { if (root) XGBB_HIST(uint8_t, true, true); else XGBB_HIST(uint8_t, true, false); }
    else { if (root) XGBB_HIST(uint8_t, false, true); else XGBB_HIST(uint8_t, false, false); }
  } else {
    if (tl.unit_hessian) { if (root) XGBB_HIST(uint16_t, true, true); else XGBB_HIST(uint16_t, true, false); }
    else { if (root) XGBB_HIST(uint16_t, false, true); else XGBB_HIST(uint16_t, false, false); }
  }
#undef XGBB_HIST
  XGBB_CUDA(cudaGetLastError());
}

static SplitMath split_math(const TreeParams& p) {
  SplitMath m;
  m.lambda = (double)p.reg_lambda;
  m.alpha = fabs((double)p.reg_alpha);
  m.alpha2 = (double)p.reg_alpha + (double)p.reg_alpha;
  m.min_child = (double)fabsf(p.min_child_weight);
  m.max_delta = fabsf(p.max_delta_step);
  return m;
}

void tree_level_eval(const TreeWorkspace& ws, const TreeLaunch& tl, uint32_t depth,
                     cudaStream_t stream) {
  EvalArgs a;
  a.e = tl.ell;
  a.m = split_math(tl.params);
  a.scale = tl.scale;
  a.state = ws.state;
  a.depth = depth;
  a.built = ws.built;
  a.pair_stride = max_pairs_at(depth);
  a.f_lo = tl.f_lo;
  a.f_hi = tl.f_hi;
  a.prev_bank = ws.bank[(depth + 1) & 1];
  a.bank = ws.bank[depth & 1];
  a.parent_slot = ws.parent_slot;
  a.built_left = ws.built_left;
  a.sums = ws.sums[depth & 1];
  a.cand = ws.cand;
  a.keys = ws.keys[depth & 1];
  a.write_bank = depth + 1 < tl.params.max_depth;
  a.direct = false;
  eval_kernel<<<tl.eval_blocks, 256, 0, stream>>>(a);
  XGBB_CUDA(cudaGetLastError());
}

void tree_level_pack_best(const TreeWorkspace& ws, const TreeLaunch& tl, uint32_t depth, void* out,
                          cudaStream_t stream) {
  pack_best_kernel<<<1, 512, 0, stream>>>(ws.keys[depth & 1], ws.cand, tl.ell.cols,
                                          static_cast<BestRecord*>(out));
  XGBB_CUDA(cudaGetLastError());
}

void tree_level_merge_best(const TreeWorkspace& ws, const TreeLaunch& tl, uint32_t depth,
                           const void* all, uint32_t ranks, cudaStream_t stream) {
  merge_best_kernel<<<1, 512, 0, stream>>>(ws.state, static_cast<const BestRecord*>(all), ranks,
                                           tl.ell.cols, ws.keys[depth & 1], ws.cand);
  XGBB_CUDA(cudaGetLastError());
}

size_t best_record_bytes() { return sizeof(BestRecord); }
static_assert(sizeof(BestRecord) == sizeof(NodeBest) && alignof(BestRecord) == alignof(NodeBest),
              "NodeBest mirrors BestRecord");

void queue_evaluate(const Ellpack& e, const TreeParams& tp, const float2* scale, DriverState* state,
                    uint32_t slots, bool root, const longlong2* built, const long long* sums, DevSplit* cand,
                    unsigned long long* keys, NodeBest* best, int blocks, cudaStream_t stream) {
  // The node count eval_kernel reads (set by a kernel: a host copy would wait
  // for the stream's earlier collectives).
  set_frontier_kernel<<<1, 1, 0, stream>>>(state, slots);
  XGBB_CUDA(cudaGetLastError());
  XGBB_CUDA(cudaMemsetAsync(keys, 0, kMaxFrontier * sizeof(unsigned long long), stream));
  EvalArgs a{};
  a.e = e;
  a.m = split_math(tp);
  a.scale = scale;
  a.state = state;
  a.depth = root ? 0u : 1u;
  a.built = built;
  a.pair_stride = slots;
  a.f_lo = 0;
  a.f_hi = e.cols;
  a.sums = sums;
  a.cand = cand;
  a.keys = keys;
  a.write_bank = false;
  a.direct = true;
  eval_kernel<<<blocks, 256, 0, stream>>>(a);
  XGBB_CUDA(cudaGetLastError());
  pack_best_kernel<<<1, 512, 0, stream>>>(keys, cand, e.cols, reinterpret_cast<BestRecord*>(best));
  XGBB_CUDA(cudaGetLastError());
}

void tree_level_control(const TreeWorkspace& ws, const TreeLaunch& tl, uint32_t depth,
                        cudaStream_t stream) {
  ControlArgs a;
  a.e = tl.ell;
  a.tp = tl.params;
  a.m = split_math(tl.params);
  a.scale = tl.scale;
  a.state = ws.state;
  a.depth = depth;
  a.ids = ws.ids[depth & 1];
  a.sums = ws.sums[depth & 1];
  a.seg_begin = ws.seg_begin[depth & 1];
  a.seg_count = ws.seg_count[depth & 1];
  a.cand = ws.cand;
  a.keys = ws.keys[depth & 1];
  a.next_keys = ws.keys[(depth + 1) & 1];
  a.next_ids = ws.ids[(depth + 1) & 1];
  a.next_sums = ws.sums[(depth + 1) & 1];
  a.parent_slot = ws.parent_slot;
  a.mode = ws.mode;
  a.slot_leaf = ws.slot_leaf;
  a.cursor_l = ws.cursor_l;
  a.cursor_r = ws.cursor_r;
  a.ptile_offset = ws.ptile_offset;
  a.nodes = ws.nodes;
  a.node_capacity = ws.node_capacity;
  control_kernel<<<1, 1024, 0, stream>>>(a);
  XGBB_CUDA(cudaGetLastError());
}

void tree_level_partition(const TreeWorkspace& ws, const TreeLaunch& tl, uint32_t depth,
                          cudaStream_t stream) {
  PartArgs a;
  a.e = tl.ell;
  a.state = ws.state;
  a.ids = ws.ids[depth & 1];
  a.nodes = ws.nodes;
  a.seg_begin = ws.seg_begin[depth & 1];
  a.seg_count = ws.seg_count[depth & 1];
  a.ptile_offset = ws.ptile_offset;
  a.mode = ws.mode;
  a.slot_leaf = ws.slot_leaf;
  a.rows = ws.rows[depth & 1];
  a.rows_next = ws.rows[(depth + 1) & 1];
  a.pairs = depth == 0 ? tl.pairs : ws.ord[depth & 1];
  a.pairs_next = ws.ord[(depth + 1) & 1];
  a.cursor_l = ws.cursor_l;
  a.cursor_r = ws.cursor_r;
  a.margins = tl.margins;
  a.groups = tl.groups;
  a.group = tl.group;
  a.root = depth == 0;
  if (depth + 1 >= tl.params.max_depth) {
    // Last level: margins only, in passes whose margins fit well inside L2.
    constexpr uint64_t kPassBytes = 96ull << 20;
    const uint64_t bytes = uint64_t(tl.ell.rows) * 4 * std::min<uint32_t>(tl.groups, 8);
    const uint32_t passes = uint32_t(std::max<uint64_t>(1, (bytes + kPassBytes - 1) / kPassBytes));
    const uint32_t span = uint32_t((uint64_t(tl.ell.rows) + passes - 1) / passes);
    for (uint32_t p = 0; p < passes; ++p) {
      const uint32_t lo = uint32_t(std::min<uint64_t>(uint64_t(p) * span, tl.ell.rows));
      const uint32_t hi = p + 1 == passes ? 0xffffffffu : uint32_t(std::min<uint64_t>(uint64_t(p + 1) * span, tl.ell.rows));
      if (tl.ell.bytes_per_code == 1)
        leaf_margin_kernel<uint8_t><<<tl.part_blocks, kPartThreads, 0, stream>>>(a, lo, hi);
      else
        leaf_margin_kernel<uint16_t><<<tl.part_blocks, kPartThreads, 0, stream>>>(a, lo, hi);
      XGBB_CUDA(cudaGetLastError());
    }
    return;
  }
  if (tl.ell.bytes_per_code == 1)
    partition_kernel<uint8_t><<<tl.part_blocks, kPartThreads, 0, stream>>>(a);
  else
    partition_kernel<uint16_t><<<tl.part_blocks, kPartThreads, 0, stream>>>(a);
  XGBB_CUDA(cudaGetLastError());
}

void tree_level_counts(const TreeWorkspace& ws, uint32_t depth, cudaStream_t stream) {
  counts_kernel<<<1, 512, 0, stream>>>(ws.state, ws.seg_begin[depth & 1], ws.seg_count[depth & 1],
                                       ws.mode, ws.cursor_l, ws.counts_local);
  XGBB_CUDA(cudaGetLastError());
}

void tree_level_plan(const TreeWorkspace& ws, const TreeLaunch&, uint32_t next_depth,
                     cudaStream_t stream) {
  PlanArgs a;
  a.state = ws.state;
  a.level_rows = ws.level_rows;
  a.level_nodes = ws.level_nodes;
  a.next_depth = next_depth;
  a.parent_slot = ws.parent_slot;
  a.seg_begin_cur = ws.seg_begin[(next_depth + 1) & 1];
  a.counts_local = ws.counts_local;
  a.counts_global = ws.counts_global;
  a.seg_begin = ws.seg_begin[next_depth & 1];
  a.seg_count = ws.seg_count[next_depth & 1];
  a.built_left = ws.built_left;
  a.tile_offset = ws.tile_offset;
  plan_kernel<<<1, 1024, 0, stream>>>(a);
  XGBB_CUDA(cudaGetLastError());
}

void launch_predict(const float* X, uint32_t rows, uint32_t cols, const DevNode* nodes,
                    const uint32_t* tree_begin, const uint32_t* tree_group, uint32_t trees,
                    const float* base, uint32_t groups, float* out, cudaStream_t stream) {
  if (!rows) return;
  predict_kernel<<<grid_for(rows, 128), 128, 0, stream>>>(X, rows, cols, nodes, tree_begin,
                                                         tree_group, trees, base, groups, out);
  XGBB_CUDA(cudaGetLastError());
}

void launch_leaf_index(const float* X, uint32_t rows, uint32_t cols, const DevNode* nodes,
                       const uint32_t* tree_begin, uint32_t trees, float* out, cudaStream_t stream) {
  if (!rows || !trees) return;
  dim3 grid(grid_for(rows, 128), std::min<uint32_t>(trees, 65535u));
  leaf_index_kernel<<<grid, 128, 0, stream>>>(X, rows, cols, nodes, tree_begin, trees, out);
  XGBB_CUDA(cudaGetLastError());
}

void launch_transform(int objective, float* v, uint32_t rows, uint32_t groups,
                      cudaStream_t stream) {
  if (!rows) return;
  transform_kernel<<<grid_for(rows, 128), 128, 0, stream>>>(objective, v, rows, groups);
  XGBB_CUDA(cudaGetLastError());
}

}  // namespace xgbb
