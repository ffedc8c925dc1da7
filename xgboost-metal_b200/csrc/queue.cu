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

// Sparse rows from the ELLPACK codes: per tile of kCsrTileRows rows the
// rows' present-code counts as an exclusive scan within the tile (into
// row_ptr) and the tile's total; then the tile totals scanned; then the tile
// offsets added.
constexpr uint32_t kCsrTileRows = 4096;

template <typename CodeT>
__global__ void __launch_bounds__(kQueueThreads) csr_count_kernel(Ellpack e, unsigned long long* row_ptr,
                                                                  unsigned long long* tile_sums) {
  __shared__ uint32_t counts[kCsrTileRows];
  DeviceExec ex;
  const uint32_t r0 = blockIdx.x * kCsrTileRows;
  const uint32_t n = min(kCsrTileRows, e.rows - r0);
  ex.for_each(n, [&](uint32_t i) { counts[i] = csr_row_count<CodeT>(e, r0 + i); });
  const uint32_t total = ex.scan_exclusive(counts, n, Add32{});
  ex.for_each(n, [&](uint32_t i) { row_ptr[r0 + i] = counts[i]; });
  if (threadIdx.x == 0) tile_sums[blockIdx.x] = total;
}

__global__ void __launch_bounds__(1024) csr_scan_tiles_kernel(unsigned long long* tile_sums, uint32_t tiles,
                                                              unsigned long long* row_ptr, uint32_t rows) {
  DeviceExec ex;
  const unsigned long long total = ex.scan_exclusive(tile_sums, tiles, Add64{});
  if (threadIdx.x == 0) row_ptr[rows] = total;
}

__global__ void csr_offsets_kernel(unsigned long long* row_ptr, const unsigned long long* tile_sums, uint32_t rows) {
  const uint32_t r0 = blockIdx.x * kCsrTileRows;
  const uint32_t end = min(rows, r0 + kCsrTileRows);
  const unsigned long long off = tile_sums[blockIdx.x];
  for (uint32_t r = r0 + threadIdx.x; r < end; r += blockDim.x) row_ptr[r] += off;
}

template <typename CodeT>
__global__ void csr_fill_kernel(Ellpack e, const unsigned long long* row_ptr, uint32_t* entries) {
  for (uint32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < e.rows; r += gridDim.x * blockDim.x)
    csr_row_fill<CodeT>(e, r, row_ptr[r], entries);
}

// Sparse node histograms (queue_hist_csr_tile) strided over the grid, then
// each (feature, node) missing bin from the node totals.
__global__ void __launch_bounds__(kQueueThreads) queue_hist_csr_kernel(
    uint32_t bins, uint32_t cols, const unsigned long long* __restrict__ row_ptr, const uint32_t* __restrict__ entries,
    const uint32_t* __restrict__ order, const float2* __restrict__ pairs, const float2* scale, const uint32_t* seg,
    const uint32_t* tiles, uint32_t slots, uint32_t total_tiles, unsigned long long* node_totals, longlong2* built) {
  __shared__ unsigned long long tot[2];
  const float2 sc = *scale;
  DeviceExec ex;
  for (uint32_t t = blockIdx.x; t < total_tiles; t += gridDim.x)
    queue_hist_csr_tile(ex, bins, cols, row_ptr, entries, order, pairs, sc, seg, tiles, slots, t, tot, node_totals,
                        built);
}

__global__ void queue_fill_missing_kernel(uint32_t bins, uint32_t cols, uint32_t slots,
                                          const unsigned long long* node_totals, longlong2* built) {
  const uint64_t n = uint64_t(cols) * slots;
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n; i += uint64_t(gridDim.x) * blockDim.x)
    queue_fill_missing(bins, slots, node_totals, built, uint32_t(i / slots), uint32_t(i % slots));
}

int grid_for(uint64_t work, int threads) {
  const uint64_t g = (work + threads - 1) / threads, cap = uint64_t(device_sms()) * 16;
  return int(g < 1 ? 1 : (g > cap ? cap : g));
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

uint64_t queue_csr_row_ptr(const Ellpack& e, unsigned long long* row_ptr, unsigned long long* tile_sums,
                           cudaStream_t stream) {
  require(e.cols <= 0x10000u, "sparse rows need at most 65536 features");
  const uint32_t tiles = (e.rows + kCsrTileRows - 1) / kCsrTileRows;
  if (tiles) {
    if (e.bytes_per_code == 1) csr_count_kernel<uint8_t><<<tiles, kQueueThreads, 0, stream>>>(e, row_ptr, tile_sums);
    else csr_count_kernel<uint16_t><<<tiles, kQueueThreads, 0, stream>>>(e, row_ptr, tile_sums);
    XGBB_CUDA(cudaGetLastError());
  }
  csr_scan_tiles_kernel<<<1, 1024, 0, stream>>>(tile_sums, tiles, row_ptr, e.rows);
  XGBB_CUDA(cudaGetLastError());
  if (tiles) {
    csr_offsets_kernel<<<tiles, 256, 0, stream>>>(row_ptr, tile_sums, e.rows);
    XGBB_CUDA(cudaGetLastError());
  }
  unsigned long long nnz = 0;
  XGBB_CUDA(cudaMemcpyAsync(&nnz, row_ptr + e.rows, 8, cudaMemcpyDeviceToHost, stream));
  XGBB_CUDA(cudaStreamSynchronize(stream));
  return nnz;
}

void queue_csr_fill(const Ellpack& e, const unsigned long long* row_ptr, uint32_t* entries, cudaStream_t stream) {
  if (!e.rows) return;
  if (e.bytes_per_code == 1)
    csr_fill_kernel<uint8_t><<<grid_for(e.rows, 256), 256, 0, stream>>>(e, row_ptr, entries);
  else
    csr_fill_kernel<uint16_t><<<grid_for(e.rows, 256), 256, 0, stream>>>(e, row_ptr, entries);
  XGBB_CUDA(cudaGetLastError());
}

void launch_queue_hist_csr(const Ellpack& e, const unsigned long long* row_ptr, const uint32_t* entries,
                           const uint32_t* order, const float2* pairs, const float2* scale, const uint32_t* seg,
                           const uint32_t* tiles, uint32_t slots, uint32_t total_tiles,
                           unsigned long long* node_totals, longlong2* built, int blocks, cudaStream_t stream) {
  require(e.bins + 1 <= kQueueBins, "host-driven trees support at most 256 bins per feature");
  require(slots >= 1 && slots <= kMaxFrontier, "host-driven tree batch out of range");
  XGBB_CUDA(cudaMemsetAsync(built, 0, size_t(e.cols) * slots * (e.bins + 1) * sizeof(longlong2), stream));
  XGBB_CUDA(cudaMemsetAsync(node_totals, 0, size_t(slots) * 16, stream));
  if (total_tiles) {
    const int grid = int(total_tiles < uint32_t(blocks) ? total_tiles : uint32_t(blocks));
    queue_hist_csr_kernel<<<grid, kQueueThreads, 0, stream>>>(e.bins, e.cols, row_ptr, entries, order, pairs, scale,
                                                              seg, tiles, slots, total_tiles, node_totals, built);
    XGBB_CUDA(cudaGetLastError());
  }
  queue_fill_missing_kernel<<<grid_for(uint64_t(e.cols) * slots, 256), 256, 0, stream>>>(e.bins, e.cols, slots,
                                                                                          node_totals, built);
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
