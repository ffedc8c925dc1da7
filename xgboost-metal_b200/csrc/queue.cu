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

#include "exec.h"
#include "queue_par.h"
#include "tree.h"

namespace xgbb {
namespace {

constexpr int kQueueThreads = 256;

__global__ void queue_iota_kernel(uint32_t* rows, uint32_t n) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) rows[i] = i;
}

// Work items (queue_hist_item) strided over the grid; each item's sums
// collect in shared memory.
template <typename CodeT>
__global__ void __launch_bounds__(kQueueThreads) queue_hist_kernel(Ellpack e, const uint32_t* __restrict__ order,
                                                                   const float2* __restrict__ pairs,
                                                                   const float2* scale, const uint32_t* seg,
                                                                   const uint32_t* tiles, uint32_t slots,
                                                                   uint32_t total_tiles, longlong2* built) {
  __shared__ unsigned long long sg[kQueueFeatures * kQueueBins], sh[kQueueFeatures * kQueueBins];
  const uint64_t items = uint64_t(total_tiles) * ((e.cols + kQueueFeatures - 1) / kQueueFeatures);
  const float2 sc = *scale;
  DeviceExec ex;
  for (uint64_t item = blockIdx.x; item < items; item += gridDim.x)
    queue_hist_item<CodeT>(ex, e, order, pairs, sc, seg, tiles, slots, item, sg, sh, built);
}

// Partition tiles (queue_partition_tile) strided over the grid.
template <typename CodeT>
__global__ void __launch_bounds__(kQueueThreads) queue_partition_kernel(Ellpack e, const uint32_t* __restrict__ order,
                                                                        uint32_t* scratch, const uint32_t* items,
                                                                        const uint32_t* tiles, uint32_t nitems,
                                                                        uint32_t total_tiles, uint32_t* cursor) {
  __shared__ uint32_t flags[kQueuePartRows], rank[kQueuePartRows], base[2];
  DeviceExec ex;
  for (uint32_t t = blockIdx.x; t < total_tiles; t += gridDim.x)
    queue_partition_tile<CodeT>(ex, e, order, scratch, items, tiles, nitems, t, cursor, flags, rank, base);
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
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < e.rows; r += gridDim.x * blockDim.x)
    queue_margin_row<CodeT>(e, nodes, node_count, margins, groups, group, r);
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
