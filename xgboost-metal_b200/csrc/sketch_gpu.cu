// Quantile cuts on the GPU: the data-parallel sketch of sketch_par.h run with
// one thread block per task.
//
//   sketch_runs_kernel    one block per feature: the feature's runs in row
//                         order, a chunk of rows at a time
//                         (kernels/quantile.metal.h:19-140)
//   sketch_batch_kernel   one block per batch of 2 * limit runs: sorted,
//                         summarised and pruned (:216-240, :192-214)
//   sketch_reduce_kernel  one block per feature: the batch summaries
//                         combined and pruned level by level, then the cuts
//                         (:266-400)
//
// Features are processed in groups sized to the free device memory; each
// group's runs and summaries take about 16 bytes per row and feature.
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "common.h"
#include "exec.h"
#include "sketch.h"
#include "sketch_par.h"
#include "tree.h"

namespace xgbb {
namespace {

using namespace sketch;

constexpr int kSketchThreads = 1024;
constexpr uint32_t kChunkRows = 4096;

// Runs of feature f0 + blockIdx.x into runs[blockIdx.x * rows ...];
// stats[blockIdx.x] = (runs, elements, nonmissing).
__global__ void __launch_bounds__(kSketchThreads) sketch_runs_kernel(const float* __restrict__ X, uint32_t rows,
                                                                     uint32_t cols, const float* __restrict__ weights,
                                                                     uint32_t f0, Run* runs, uint32_t* stats) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ RunCarry carry;
  __shared__ float last_w;
  float* sv = reinterpret_cast<float*>(smem);
  ChunkWork c{sv,
              sv + kChunkRows,
              reinterpret_cast<uint32_t*>(sv + 2 * kChunkRows),
              reinterpret_cast<uint32_t*>(sv + 3 * kChunkRows),
              reinterpret_cast<uint32_t*>(sv + 4 * kChunkRows),
              reinterpret_cast<uint32_t*>(sv + 5 * kChunkRows),
              reinterpret_cast<uint32_t*>(sv + 6 * kChunkRows),
              &last_w};
  const uint32_t f = f0 + blockIdx.x;
  Run* out = runs + size_t(blockIdx.x) * rows;
  if (threadIdx.x == 0) carry = RunCarry{0, 0, 0, 0, 0.0f, 0.0f};
  __syncthreads();
  DeviceExec ex;
  for (uint32_t r0 = 0; r0 < rows; r0 += kChunkRows) {
    const uint32_t n = min(kChunkRows, rows - r0);
    runs_chunk(
        ex,
        [&](uint32_t i, float& v, float& w) {
          v = X[size_t(r0 + i) * cols + f];
          w = weights ? weights[r0 + i] : 1.0f;
        },
        n, weights == nullptr, carry, out, c);
  }
  if (threadIdx.x == 0) {
    stats[3 * blockIdx.x] = carry.runs;
    stats[3 * blockIdx.x + 1] = carry.elements;
    stats[3 * blockIdx.x + 2] = carry.nonmissing;
  }
}

__global__ void __launch_bounds__(kSketchThreads) sketch_batch_kernel(const Run* runs, const BatchTask* tasks,
                                                                      uint32_t ntasks, Entry* summaries,
                                                                      uint32_t* sizes, unsigned char* scratch,
                                                                      size_t scratch_stride, uint32_t cap) {
  const BatchWork bw = batch_work_at(scratch + size_t(blockIdx.x) * scratch_stride, cap);
  DeviceExec ex;
  for (uint32_t t = blockIdx.x; t < ntasks; t += gridDim.x) {
    const BatchTask task = tasks[t];
    const uint32_t n = summarize_par(ex, runs + task.run_begin, task.size, task.limit, bw.keys, bw.sorted, bw.entries,
                                     summaries + task.summary_at, bw.w);
    if (threadIdx.x == 0) sizes[task.size_slot] = n;
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kSketchThreads) sketch_reduce_kernel(const Entry* summaries, const uint32_t* sizes,
                                                                       const ReduceTask* tasks, unsigned char* work,
                                                                       uint32_t max_bin, uint32_t stride, float* cuts,
                                                                       uint32_t* counts) {
  const ReduceTask t = tasks[blockIdx.x];
  const ReduceWork r = reduce_work_at(work + t.work_at, t.limit, t.budget, t.levels);
  DeviceExec ex;
  const uint32_t n = reduce_feature(ex, summaries + t.summary_at, sizes + t.first_size, t.nbatch, t.limit, t.budget,
                                    t.levels, max_bin, r, cuts + size_t(t.feature) * stride);
  if (threadIdx.x == 0) counts[t.feature] = n;
}

struct Device {
  void* p = nullptr;
  size_t n = 0;
  void need(size_t bytes) {
    if (bytes <= n) return;
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
    XGBB_CUDA(cudaMalloc(&p, std::max<size_t>(bytes, 256)));
    n = std::max<size_t>(bytes, 256);
  }
  ~Device() {
    if (p) cudaFree(p);
  }
  template <class T>
  T* as() const {
    return static_cast<T*>(p);
  }
};

}  // namespace

void sketch_cuts_device(const float* X, uint32_t rows, uint32_t cols, const float* weights, uint32_t max_bin,
                        float* cuts, uint32_t* counts, float* minima, cudaStream_t stream) {
  const uint32_t stride = cut_stride(rows, max_bin);
  std::fill(cuts, cuts + size_t(cols) * stride, 0.0f);
  std::fill(counts, counts + cols, 0u);
  std::fill(minima, minima + cols, -INFINITY);
  if (!cols) return;
  const size_t runs_smem = 7 * size_t(kChunkRows) * 4;
  XGBB_CUDA(cudaFuncSetAttribute(sketch_runs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(runs_smem)));
  const int sms = device_sms();
  // Features per group: runs and batch summaries take about 16 bytes per row
  // and feature; keep them within a quarter of the free memory.
  size_t free_b = 0, total_b = 0;
  XGBB_CUDA(cudaMemGetInfo(&free_b, &total_b));
  const size_t per_feature = std::max<size_t>(size_t(rows) * 16, 1);
  const uint32_t group = uint32_t(std::max<size_t>(1, std::min<size_t>(cols, free_b / 4 / per_feature)));
  Device d_cuts, d_counts, d_runs, d_stats, d_summaries, d_sizes, d_tasks, d_scratch, d_rtasks, d_work;
  d_cuts.need(size_t(cols) * stride * 4);
  d_counts.need(size_t(cols) * 4);
  XGBB_CUDA(cudaMemsetAsync(d_cuts.p, 0, size_t(cols) * stride * 4, stream));
  std::vector<uint32_t> stats;
  for (uint32_t f0 = 0; f0 < cols; f0 += group) {
    const uint32_t nf = std::min(group, cols - f0);
    d_runs.need(size_t(nf) * std::max(rows, 1u) * sizeof(Run));
    d_stats.need(size_t(nf) * 3 * 4);
    sketch_runs_kernel<<<nf, kSketchThreads, runs_smem, stream>>>(X, rows, cols, weights, f0, d_runs.as<Run>(),
                                                                   d_stats.as<uint32_t>());
    XGBB_CUDA(cudaGetLastError());
    stats.assign(size_t(nf) * 3, 0);
    XGBB_CUDA(cudaMemcpyAsync(stats.data(), d_stats.p, stats.size() * 4, cudaMemcpyDeviceToHost, stream));
    XGBB_CUDA(cudaStreamSynchronize(stream));
    const GroupPlan plan = plan_group(stats.data(), nf, f0, rows, max_bin);
    const std::vector<BatchTask>& tasks = plan.tasks;
    const std::vector<ReduceTask>& rtasks = plan.reduce;
    const uint64_t summary_at = plan.summary_entries, work_at = plan.work_bytes;
    const uint32_t cap = plan.cap, sizes_n = plan.sizes;
    d_summaries.need(size_t(summary_at) * sizeof(Entry));
    d_sizes.need(size_t(sizes_n) * 4);
    d_work.need(size_t(work_at));
    if (!tasks.empty()) {
      const size_t scratch_stride = batch_scratch_bytes(cap);
      const uint32_t grid = uint32_t(std::min<size_t>(tasks.size(), size_t(sms) * 2));
      d_scratch.need(scratch_stride * grid);
      d_tasks.need(tasks.size() * sizeof(BatchTask));
      XGBB_CUDA(cudaMemcpyAsync(d_tasks.p, tasks.data(), tasks.size() * sizeof(BatchTask), cudaMemcpyHostToDevice,
                                stream));
      sketch_batch_kernel<<<grid, kSketchThreads, 0, stream>>>(d_runs.as<Run>(), d_tasks.as<BatchTask>(),
                                                              uint32_t(tasks.size()), d_summaries.as<Entry>(),
                                                              d_sizes.as<uint32_t>(), d_scratch.as<unsigned char>(),
                                                              scratch_stride, cap);
      XGBB_CUDA(cudaGetLastError());
    }
    d_rtasks.need(rtasks.size() * sizeof(ReduceTask));
    XGBB_CUDA(cudaMemcpyAsync(d_rtasks.p, rtasks.data(), rtasks.size() * sizeof(ReduceTask), cudaMemcpyHostToDevice,
                              stream));
    sketch_reduce_kernel<<<nf, kSketchThreads, 0, stream>>>(d_summaries.as<Entry>(), d_sizes.as<uint32_t>(),
                                                            d_rtasks.as<ReduceTask>(), d_work.as<unsigned char>(),
                                                            max_bin, stride, d_cuts.as<float>(),
                                                            d_counts.as<uint32_t>());
    XGBB_CUDA(cudaGetLastError());
    // The next group reuses the buffers.
    XGBB_CUDA(cudaStreamSynchronize(stream));
  }
  XGBB_CUDA(cudaMemcpyAsync(cuts, d_cuts.p, size_t(cols) * stride * 4, cudaMemcpyDeviceToHost, stream));
  XGBB_CUDA(cudaMemcpyAsync(counts, d_counts.p, size_t(cols) * 4, cudaMemcpyDeviceToHost, stream));
  XGBB_CUDA(cudaStreamSynchronize(stream));
}

}  // namespace xgbb
