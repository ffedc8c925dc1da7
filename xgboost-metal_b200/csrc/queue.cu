// Device work of host-driven trees (grower.cpp): node histograms built from
// row segments, row partitions of a batch of leaves, and the margin update of
// a finished tree. The host pops leaves from its queue and launches these per
// batch; split evaluation reuses eval_kernel (tree.cu) on the histograms.
//
// Reference semantics: histograms are the exact int64 sums of the quantised
// gradients per (node, feature, bin) (kernels/boost.metal:700-733, the
// missing bin as in kernels/histogram_missing.metal.h:13-60); the partition
// predicate is the bin form of split_left (kernels/boost.metal:1325-1329,
// 1497-1499); leaves add weight * eta to the margins (src/tree.cpp:1663-1717).
#include <cuda_runtime.h>

#include "tree.h"

namespace xgbb {
namespace {

constexpr int kQueueThreads = 256;
constexpr uint32_t kQueueFeatures = 8;  // features per histogram work item
constexpr uint32_t kQueueBins = kMaxBins + 1;

__global__ void queue_iota_kernel(uint32_t* rows, uint32_t n) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) rows[i] = i;
}

// The node (slot) whose tiles contain tile t: the last s with tiles[s] <= t.
__device__ __forceinline__ uint32_t owner_of(const uint32_t* tiles, uint32_t n, uint32_t t) {
  uint32_t lo = 0, hi = n;  // tiles[lo] <= t < tiles[hi]
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) / 2;
    if (tiles[mid] <= t) lo = mid;
    else hi = mid;
  }
  return lo;
}

// One work item = (tile of kQueueTileRows rows of one node, group of
// kQueueFeatures features), tile-major so that the CTAs of one tile read the
// same rows. The item's sums live in shared memory as 64-bit integers
// (wrap-around adds are exact mod 2^64) and are added to the node's global
// histogram once per item.
template <typename CodeT>
__global__ void __launch_bounds__(kQueueThreads) queue_hist_kernel(Ellpack e, const uint32_t* __restrict__ order,
                                                                   const float2* __restrict__ pairs,
                                                                   const float2* scale, const uint32_t* seg,
                                                                   const uint32_t* tiles, uint32_t slots,
                                                                   uint32_t total_tiles, longlong2* built) {
  __shared__ unsigned long long sg[kQueueFeatures * kQueueBins], sh[kQueueFeatures * kQueueBins];
  const uint32_t C = e.cols, B = e.bins, B1 = B + 1;
  const uint32_t groups = (C + kQueueFeatures - 1) / kQueueFeatures;
  const uint64_t items = uint64_t(total_tiles) * groups;
  const float2 sc = *scale;
  const CodeT* __restrict__ codes = static_cast<const CodeT*>(e.codes);
  const uint32_t fl = threadIdx.x % kQueueFeatures, r0 = threadIdx.x / kQueueFeatures;
  constexpr uint32_t kRowsPerPass = kQueueThreads / kQueueFeatures;
  for (uint64_t item = blockIdx.x; item < items; item += gridDim.x) {
    const uint32_t t = uint32_t(item / groups), fg = uint32_t(item % groups);
    const uint32_t s = owner_of(tiles, slots, t);
    const uint32_t begin = seg[2 * s] + (t - tiles[s]) * kQueueTileRows;
    const uint32_t end = min(seg[2 * s] + seg[2 * s + 1], begin + kQueueTileRows);
    for (uint32_t i = threadIdx.x; i < kQueueFeatures * B1; i += blockDim.x) {
      sg[i] = 0;
      sh[i] = 0;
    }
    __syncthreads();
    const uint32_t f = fg * kQueueFeatures + fl;
    if (f < C) {
      for (uint32_t i = begin + r0; i < end; i += kRowsPerPass) {
        const uint32_t row = order[i];
        const uint32_t code = codes[size_t(row) * e.stride + f];
        const uint32_t bin = code == e.missing ? B : code;
        if (bin > B) continue;  // not a code of this matrix
        const float2 p = pairs[row];
        const long long qg = __float2ll_rn(__fmul_rn(p.x, sc.x));
        const long long qh = __float2ll_rn(__fmul_rn(p.y, sc.y));
        atomicAdd(&sg[fl * B1 + bin], (unsigned long long)qg);
        atomicAdd(&sh[fl * B1 + bin], (unsigned long long)qh);
      }
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < kQueueFeatures * B1; i += blockDim.x) {
      const uint32_t ff = fg * kQueueFeatures + i / B1, b = i % B1;
      const unsigned long long g = sg[i], h = sh[i];
      if (ff < C && (g | h)) {
        longlong2* dst = built + (size_t(ff) * slots + s) * B1 + b;
        atomicAdd(reinterpret_cast<unsigned long long*>(&dst->x), g);
        atomicAdd(reinterpret_cast<unsigned long long*>(&dst->y), h);
      }
    }
    __syncthreads();
  }
}

// Exclusive scan over the CTA's threads (kQueueThreads).
__device__ __forceinline__ uint32_t cta_exclusive_scan(uint32_t v, uint32_t* total) {
  __shared__ uint32_t warp_sums[kQueueThreads / 32];
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t o = __shfl_up_sync(0xffffffffu, x, d);
    if (lane >= uint32_t(d)) x += o;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  uint32_t before = 0, sum = 0;
  for (uint32_t w = 0; w < kQueueThreads / 32; ++w) {
    if (w < warp) before += warp_sums[w];
    sum += warp_sums[w];
  }
  __syncthreads();
  *total = sum;
  return before + x - v;
}

// One CTA per tile of kQueuePartRows rows of one item: each thread takes four
// consecutive rows, the CTA claims room at the left end (rows going left) and
// the right end (rows going right) of the item's segment in `scratch` with
// one atomic each, and writes its rows there.
template <typename CodeT>
__global__ void __launch_bounds__(kQueueThreads) queue_partition_kernel(Ellpack e, const uint32_t* __restrict__ order,
                                                                        uint32_t* scratch, const uint32_t* items,
                                                                        const uint32_t* tiles, uint32_t nitems,
                                                                        uint32_t total_tiles, uint32_t* cursor) {
  __shared__ uint32_t s_base[2];
  const CodeT* __restrict__ codes = static_cast<const CodeT*>(e.codes);
  constexpr uint32_t kPer = kQueuePartRows / kQueueThreads;
  for (uint32_t t = blockIdx.x; t < total_tiles; t += gridDim.x) {
    const uint32_t it = owner_of(tiles, nitems, t);
    const uint32_t* d = items + 5 * size_t(it);
    const uint32_t seg_end = d[0] + d[1];
    const uint32_t f = d[2];
    const int32_t split_bin = int32_t(d[3]);
    const bool default_left = d[4] != 0;
    const uint32_t tile_begin = d[0] + (t - tiles[it]) * kQueuePartRows;
    const uint32_t tile_rows = min(kQueuePartRows, seg_end - tile_begin);
    const uint32_t first = threadIdx.x * kPer;
    uint32_t ids[kPer];
    uint32_t left_mask = 0, nl = 0, nv = 0;
#pragma unroll
    for (uint32_t k = 0; k < kPer; ++k) {
      ids[k] = 0;
      if (first + k < tile_rows) {
        const uint32_t row = order[tile_begin + first + k];
        const uint32_t code = f < e.cols ? uint32_t(codes[size_t(row) * e.stride + f]) : e.missing;
        const bool left = code == e.missing ? default_left : int32_t(code) <= split_bin;
        ids[k] = row;
        left_mask |= uint32_t(left) << k;
        nl += left;
        ++nv;
      }
    }
    uint32_t total_left;
    const uint32_t before_left = cta_exclusive_scan(nl, &total_left);
    const uint32_t before_all = min(first, tile_rows);
    if (threadIdx.x == 0) {
      const uint32_t total_right = tile_rows - total_left;
      s_base[0] = atomicAdd(cursor + 2 * it, total_left);
      s_base[1] = atomicSub(cursor + 2 * it + 1, total_right) - total_right;
    }
    __syncthreads();
    uint32_t l = s_base[0] + before_left, r = s_base[1] + (before_all - before_left);
#pragma unroll
    for (uint32_t k = 0; k < kPer; ++k) {
      if (k < nv) {
        if ((left_mask >> k) & 1u) scratch[l++] = ids[k];
        else scratch[r++] = ids[k];
      }
    }
    __syncthreads();
  }
}

// The partitioned segments back into the row order.
__global__ void queue_copy_back_kernel(uint32_t* order, const uint32_t* scratch, const uint32_t* items,
                                       const uint32_t* tiles, uint32_t nitems, uint32_t total_tiles) {
  for (uint32_t t = blockIdx.x; t < total_tiles; t += gridDim.x) {
    const uint32_t it = owner_of(tiles, nitems, t);
    const uint32_t seg_end = items[5 * size_t(it)] + items[5 * size_t(it) + 1];
    const uint32_t tile_begin = items[5 * size_t(it)] + (t - tiles[it]) * kQueuePartRows;
    for (uint32_t i = tile_begin + threadIdx.x; i < min(seg_end, tile_begin + kQueuePartRows); i += blockDim.x)
      order[i] = scratch[i];
  }
}

template <typename CodeT>
__global__ void queue_margin_kernel(Ellpack e, const DevNode* __restrict__ nodes, uint32_t node_count,
                                    float* margins, uint32_t groups, uint32_t group) {
  const CodeT* __restrict__ codes = static_cast<const CodeT*>(e.codes);
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < e.rows; r += gridDim.x * blockDim.x) {
    uint32_t n = 0;
    for (uint32_t step = 0; step < node_count; ++step) {
      const DevNode nd = nodes[n];
      if (nd.left < 0 || uint32_t(nd.feature) >= e.cols) break;
      const uint32_t code = codes[size_t(r) * e.stride + uint32_t(nd.feature)];
      const bool left = code == e.missing ? nd.default_left != 0u : int32_t(code) <= nd.split_bin;
      const int32_t next = left ? nd.left : nd.right;
      if (next < 0 || uint32_t(next) >= node_count) break;
      n = uint32_t(next);
    }
    float* m = margins + size_t(r) * groups + group;
    *m = __fadd_rn(*m, nodes[n].leaf);
  }
}

int grid_for(uint64_t work, int threads) {
  const uint64_t g = (work + threads - 1) / threads;
  return int(g < 1 ? 1 : (g > 148 * 16 ? 148 * 16 : g));
}

}  // namespace

void launch_queue_iota(uint32_t* rows, uint32_t n, cudaStream_t stream) {
  if (!n) return;
  queue_iota_kernel<<<grid_for(n, 256), 256, 0, stream>>>(rows, n);
  XGBB_CUDA(cudaGetLastError());
}

void launch_queue_hist(const Ellpack& e, const uint32_t* order, const float2* pairs, const float2* scale,
                       const uint32_t* seg, const uint32_t* tiles, uint32_t slots, uint32_t total_tiles,
                       longlong2* built, int blocks, cudaStream_t stream) {
  require(e.bins + 1 <= kQueueBins, "host-driven trees support at most 256 bins per feature");
  require(slots >= 1 && slots <= kMaxFrontier, "host-driven tree batch out of range");
  XGBB_CUDA(cudaMemsetAsync(built, 0, size_t(e.cols) * slots * (e.bins + 1) * sizeof(longlong2), stream));
  if (!total_tiles) return;
  const uint64_t items = uint64_t(total_tiles) * ((e.cols + kQueueFeatures - 1) / kQueueFeatures);
  const int grid = int(items < uint64_t(blocks) ? items : uint64_t(blocks));
  if (e.bytes_per_code == 1)
    queue_hist_kernel<uint8_t><<<grid, kQueueThreads, 0, stream>>>(e, order, pairs, scale, seg, tiles, slots,
                                                                   total_tiles, built);
  else
    queue_hist_kernel<uint16_t><<<grid, kQueueThreads, 0, stream>>>(e, order, pairs, scale, seg, tiles, slots,
                                                                    total_tiles, built);
  XGBB_CUDA(cudaGetLastError());
}

void launch_queue_partition(const Ellpack& e, uint32_t* order, uint32_t* scratch, const uint32_t* items,
                            const uint32_t* tiles, uint32_t nitems, uint32_t total_tiles, uint32_t* cursor,
                            int blocks, cudaStream_t stream) {
  if (!total_tiles || !nitems) return;
  const int grid = int(total_tiles < uint32_t(blocks) ? total_tiles : uint32_t(blocks));
  if (e.bytes_per_code == 1)
    queue_partition_kernel<uint8_t><<<grid, kQueueThreads, 0, stream>>>(e, order, scratch, items, tiles, nitems,
                                                                        total_tiles, cursor);
  else
    queue_partition_kernel<uint16_t><<<grid, kQueueThreads, 0, stream>>>(e, order, scratch, items, tiles, nitems,
                                                                         total_tiles, cursor);
  XGBB_CUDA(cudaGetLastError());
  queue_copy_back_kernel<<<grid, kQueueThreads, 0, stream>>>(order, scratch, items, tiles, nitems, total_tiles);
  XGBB_CUDA(cudaGetLastError());
}

void launch_queue_margins(const Ellpack& e, const DevNode* nodes, uint32_t node_count, float* margins,
                          uint32_t groups, uint32_t group, cudaStream_t stream) {
  if (!e.rows || !node_count) return;
  if (e.bytes_per_code == 1)
    queue_margin_kernel<uint8_t><<<grid_for(e.rows, 256), 256, 0, stream>>>(e, nodes, node_count, margins, groups,
                                                                             group);
  else
    queue_margin_kernel<uint16_t><<<grid_for(e.rows, 256), 256, 0, stream>>>(e, nodes, node_count, margins, groups,
                                                                              group);
  XGBB_CUDA(cudaGetLastError());
}

}  // namespace xgbb
