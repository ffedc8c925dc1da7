// Quantile cuts on the GPU: the data-parallel sketch of sketch_par.h run with
// one thread block per task.
//
//   sketch_runs_kernel    the runs of each feature in row order
//                         (kernels/quantile.metal.h:19-140), rows split into
//                         segments: a counting pass, a serial link of the
//                         segments per feature (sketch_link_kernel), a
//                         writing pass, then the weights of runs that span
//                         segments (sketch_links_kernel)
//   sketch_batch_kernel   one block per batch of 2 * limit runs: sorted (keys
//                         in shared memory), summarised and pruned
//                         (:216-240, :192-214)
//   sketch_merge_kernel   one level of the merge tree over the batch
//                         summaries, every merge of the level at once
//   sketch_finish_kernel  per feature whose merges all overflowed: the
//                         tree's left-over nodes merged and the cuts (:266-400)
//   sketch_reduce_kernel  per other feature: the level-by-level reduction
//
// Features are processed in groups sized to the free device memory; each
// group's runs and summaries take about 24 bytes per row and feature.
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
// Shared memory for the batch sort keys and for the searched keys of merges
// (a larger need falls back to the global scratch).
constexpr size_t kSketchSmem = 220 * 1024;

// Runs of every feature of the group, rows split into gridDim.y segments of
// seg_rows rows processed at the same time. Pass 1 (pass2 false): each
// segment from an empty carry, counting only. Pass 2: each segment from the
// carry sketch_link_kernel gave it, writing feature f0 + blockIdx.x's runs
// into runs[blockIdx.x * rows ...].
constexpr int kRunsThreads = 512;
constexpr uint32_t kRunsChunk = 2048;
constexpr size_t kRunsSmem = 7 * size_t(kRunsChunk) * sizeof(float);
__global__ void __launch_bounds__(kRunsThreads) sketch_runs_kernel(const float* __restrict__ X, uint32_t rows,
                                                                   uint32_t cols, const float* __restrict__ weights,
                                                                   uint32_t f0, uint32_t seg_rows, bool pass2,
                                                                   RunCarry* pass1, SegmentLink* link, Run* runs) {
  extern __shared__ __align__(16) float sv[];  // 7 * kRunsChunk words
  __shared__ RunCarry carry;
  __shared__ float last_w;
  ChunkWork c{sv,
              sv + kRunsChunk,
              reinterpret_cast<uint32_t*>(sv + 2 * kRunsChunk),
              reinterpret_cast<uint32_t*>(sv + 3 * kRunsChunk),
              reinterpret_cast<uint32_t*>(sv + 4 * kRunsChunk),
              reinterpret_cast<uint32_t*>(sv + 5 * kRunsChunk),
              reinterpret_cast<uint32_t*>(sv + 6 * kRunsChunk),
              &last_w};
  const uint32_t f = f0 + blockIdx.x, seg = blockIdx.x * gridDim.y + blockIdx.y;
  const uint32_t lo = min(rows, blockIdx.y * seg_rows), hi = min(rows, lo + seg_rows);
  if (threadIdx.x == 0) carry = pass2 ? link[seg].in : RunCarry{0, 0, 0, 0, 0.0f, 0.0f, 0.0f};
  __syncthreads();
  const RunOut out{runs + size_t(blockIdx.x) * rows, pass2, pass2 ? link[seg].in.runs : 0u,
                   pass2 ? &link[seg].cont_w : nullptr};
  DeviceExec ex;
  for (uint32_t r0 = lo; r0 < hi; r0 += kRunsChunk) {
    const uint32_t n = min(kRunsChunk, hi - r0);
    runs_chunk(
        ex,
        [&](uint32_t i, float& v, float& w) {
          v = X[size_t(r0 + i) * cols + f];
          w = weights ? weights[r0 + i] : 1.0f;
        },
        n, weights == nullptr, carry, out, c);
  }
  if (!pass2 && threadIdx.x == 0) pass1[seg] = carry;
}

// One thread per feature: the segments' carries in order (link_segments),
// and the feature's (runs, elements, nonmissing).
__global__ void sketch_link_kernel(const float* __restrict__ X, uint32_t rows, uint32_t cols,
                                   const float* __restrict__ weights, uint32_t f0, uint32_t nf, uint32_t nseg,
                                   uint32_t seg_rows, const RunCarry* pass1, SegmentLink* link, uint32_t* stats) {
  const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= nf) return;
  const uint32_t f = f0 + j;
  link_segments(
      pass1 + size_t(j) * nseg, nseg, weights == nullptr, link + size_t(j) * nseg,
      [&](uint32_t s, uint32_t k, float& v, float& w) {
        const size_t r = size_t(s) * seg_rows + k;
        v = X[r * cols + f];
        w = weights ? weights[r] : 1.0f;
      },
      [&](uint32_t s) { return min(rows, (s + 1) * seg_rows) - min(rows, s * seg_rows); }, stats + 3 * j);
}

// One thread per feature: runs that span segments take their final weights.
__global__ void sketch_links_kernel(uint32_t rows, uint32_t nf, uint32_t nseg, const SegmentLink* link, Run* runs) {
  const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j < nf) finish_links(link + size_t(j) * nseg, nseg, runs + size_t(j) * rows);
}

// With `in_shared`, the sort keys live in shared memory (pow2_ceil(cap)
// words) and, once sorted, the same space holds the rank sums the prune
// searches. With `radix` as well, the sort is the block radix sort, whose
// scratch takes the same space.
__global__ void __launch_bounds__(kSketchThreads) sketch_batch_kernel(const Run* runs, const BatchTask* tasks,
                                                                      uint32_t ntasks, Entry* summaries,
                                                                      uint32_t* sizes, unsigned char* scratch,
                                                                      size_t scratch_stride, uint32_t cap,
                                                                      bool in_shared, bool radix, bool work_shared) {
  extern __shared__ __align__(16) unsigned char fast[];
  BatchWork bw = batch_work_at(scratch + size_t(blockIdx.x) * scratch_stride, cap);
  if (in_shared) {
    bw.keys = reinterpret_cast<unsigned long long*>(fast);
    bw.w.fa = reinterpret_cast<float*>(fast);
  }
  if (work_shared) {
    // The summary's per-index words (head flags, group weights, rank sums,
    // the prune's choices) in shared memory too: they are first written
    // after the radix sort, whose scratch they then overwrite.
    uint32_t* wb = reinterpret_cast<uint32_t*>(fast);
    bw.w.u = wb;
    bw.w.v = wb + cap + 2;
    bw.w.f = reinterpret_cast<float*>(bw.w.v + cap + 2);
    bw.w.fa = bw.w.f + cap + 2;
  }
  DeviceExec ex;
  for (uint32_t t = blockIdx.x; t < ntasks; t += gridDim.x) {
    const BatchTask task = tasks[t];
    const uint32_t n = summarize_par(ex, runs + task.run_begin, task.size, task.limit, bw.keys, bw.sorted, bw.entries,
                                     summaries + task.summary_at, bw.w, radix ? fast : nullptr);
    if (threadIdx.x == 0) sizes[task.size_slot] = n;
    __syncthreads();
  }
}

// One level of the merge tree; the searched keys (2 * big floats) in shared
// memory when `in_shared`.
__global__ void __launch_bounds__(kSketchThreads) sketch_merge_kernel(const MergeTask* tasks, uint32_t ntasks,
                                                                      Entry* entries, uint32_t* sizes,
                                                                      uint32_t* irregular, unsigned char* scratch,
                                                                      size_t scratch_stride, uint32_t big,
                                                                      bool in_shared) {
  extern __shared__ __align__(16) unsigned char fast[];
  MergeWork m = merge_work_at(scratch + size_t(blockIdx.x) * scratch_stride, big);
  if (in_shared) {
    m.w.fa = reinterpret_cast<float*>(fast);
    m.w.fb = m.w.fa + big;
  }
  DeviceExec ex;
  for (uint32_t t = blockIdx.x; t < ntasks; t += gridDim.x) merge_node(ex, tasks[t], entries, sizes, irregular, m);
}

// A feature whose merges all overflowed: its cuts from the tree's left-over
// nodes. Other features return at once (sketch_reduce_kernel takes them).
__global__ void __launch_bounds__(kSketchThreads) sketch_finish_kernel(const FinishTask* tasks, const FinishRes* res,
                                                                       const Entry* entries, const uint32_t* sizes,
                                                                       const uint32_t* irregular, unsigned char* work,
                                                                       uint32_t max_bin, uint32_t stride, float* cuts,
                                                                       uint32_t* counts, bool in_shared) {
  extern __shared__ __align__(16) unsigned char fast[];
  const FinishTask t = tasks[blockIdx.x];
  if (irregular[t.local]) return;
  ReduceWork r = reduce_work_at(work + t.work_at, t.limit, t.budget, t.levels);
  if (in_shared) {
    r.w.fa = reinterpret_cast<float*>(fast);
    r.w.fb = r.w.fa + reduce_big(t.limit, t.budget);
  }
  DeviceExec ex;
  const uint32_t n = finish_tree(ex, t, res, entries, sizes, max_bin, r, cuts + size_t(t.feature) * stride);
  if (threadIdx.x == 0) counts[t.feature] = n;
}

// The level-by-level reduction of the features the tree could not take.
__global__ void __launch_bounds__(kSketchThreads) sketch_reduce_kernel(const Entry* summaries, const uint32_t* sizes,
                                                                       const ReduceTask* tasks,
                                                                       const uint32_t* irregular, unsigned char* work,
                                                                       uint32_t max_bin, uint32_t stride, float* cuts,
                                                                       uint32_t* counts, bool in_shared) {
  extern __shared__ __align__(16) unsigned char fast[];
  if (!irregular[blockIdx.x]) return;
  const ReduceTask t = tasks[blockIdx.x];
  ReduceWork r = reduce_work_at(work + t.work_at, t.limit, t.budget, t.levels);
  if (in_shared) {
    r.w.fa = reinterpret_cast<float*>(fast);
    r.w.fb = r.w.fa + reduce_big(t.limit, t.budget);
  }
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
  XGBB_CUDA(cudaFuncSetAttribute(sketch_runs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kRunsSmem)));
  for (const void* k : {reinterpret_cast<const void*>(sketch_batch_kernel), reinterpret_cast<const void*>(sketch_merge_kernel),
                        reinterpret_cast<const void*>(sketch_finish_kernel),
                        reinterpret_cast<const void*>(sketch_reduce_kernel)})
    XGBB_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSketchSmem)));
  const int sms = device_sms();
  // Features per group: runs (8 bytes per row), batch summaries and the
  // tree's nodes (up to 16 bytes per row) within half of the free memory.
  size_t free_b = 0, total_b = 0;
  XGBB_CUDA(cudaMemGetInfo(&free_b, &total_b));
  const size_t per_feature = std::max<size_t>(size_t(rows) * 24, 1);
  const uint32_t groups = uint32_t((cols + std::max<size_t>(1, std::min<size_t>(cols, free_b / 2 / per_feature)) - 1) /
                                   std::max<size_t>(1, std::min<size_t>(cols, free_b / 2 / per_feature)));
  const uint32_t group = (cols + groups - 1) / groups;  // balanced groups
  Device d_cuts, d_counts, d_runs, d_stats, d_summaries, d_sizes, d_tasks, d_scratch, d_rtasks, d_work, d_pass1,
      d_link, d_mtasks, d_ftasks, d_res, d_irregular;
  d_cuts.need(size_t(cols) * stride * 4);
  d_counts.need(size_t(cols) * 4);
  XGBB_CUDA(cudaMemsetAsync(d_cuts.p, 0, size_t(cols) * stride * 4, stream));
  std::vector<uint32_t> stats;
  Trace trace("sketch");
  for (uint32_t f0 = 0; f0 < cols; f0 += group) {
    const uint32_t nf = std::min(group, cols - f0);
    d_runs.need(size_t(nf) * std::max(rows, 1u) * sizeof(Run));
    trace.mark("group scratch", stream);
    d_stats.need(size_t(nf) * 3 * 4);
    // Segments of whole chunks, about 4 blocks per SM in all.
    const uint32_t chunks = std::max(1u, (rows + kRunsChunk - 1) / kRunsChunk);
    const uint32_t nseg = std::max(1u, std::min(chunks, (4u * uint32_t(sms) + nf - 1) / nf));
    const uint32_t seg_rows = (chunks + nseg - 1) / nseg * kRunsChunk;
    d_pass1.need(size_t(nf) * nseg * sizeof(RunCarry));
    d_link.need(size_t(nf) * nseg * sizeof(SegmentLink));
    const dim3 rgrid(nf, nseg);
    sketch_runs_kernel<<<rgrid, kRunsThreads, kRunsSmem, stream>>>(X, rows, cols, weights, f0, seg_rows, false,
                                                                    d_pass1.as<RunCarry>(), d_link.as<SegmentLink>(),
                                                                    d_runs.as<Run>());
    XGBB_CUDA(cudaGetLastError());
    sketch_link_kernel<<<(nf + 127) / 128, 128, 0, stream>>>(X, rows, cols, weights, f0, nf, nseg, seg_rows,
                                                              d_pass1.as<RunCarry>(), d_link.as<SegmentLink>(),
                                                              d_stats.as<uint32_t>());
    XGBB_CUDA(cudaGetLastError());
    sketch_runs_kernel<<<rgrid, kRunsThreads, kRunsSmem, stream>>>(X, rows, cols, weights, f0, seg_rows, true,
                                                                    d_pass1.as<RunCarry>(), d_link.as<SegmentLink>(),
                                                                    d_runs.as<Run>());
    XGBB_CUDA(cudaGetLastError());
    sketch_links_kernel<<<(nf + 127) / 128, 128, 0, stream>>>(rows, nf, nseg, d_link.as<SegmentLink>(),
                                                               d_runs.as<Run>());
    XGBB_CUDA(cudaGetLastError());
    stats.assign(size_t(nf) * 3, 0);
    XGBB_CUDA(cudaMemcpyAsync(stats.data(), d_stats.p, stats.size() * 4, cudaMemcpyDeviceToHost, stream));
    XGBB_CUDA(cudaStreamSynchronize(stream));
    trace.mark("runs", stream);
    const GroupPlan plan = plan_group(stats.data(), nf, f0, rows, max_bin);
    const TreePlan tree = plan_tree(plan);
    trace.mark("plan", stream);
    const std::vector<BatchTask>& tasks = plan.tasks;
    const std::vector<ReduceTask>& rtasks = plan.reduce;
    const uint32_t cap = plan.cap;
    d_summaries.need(size_t(tree.entries) * sizeof(Entry));
    d_sizes.need(size_t(tree.sizes) * 4);
    d_work.need(size_t(plan.work_bytes));
    d_irregular.need(size_t(nf) * 4);
    XGBB_CUDA(cudaMemsetAsync(d_irregular.p, 0, size_t(nf) * 4, stream));
    if (!tasks.empty()) {
      const size_t scratch_stride = batch_scratch_bytes(cap);
      const size_t keys_bytes = size_t(pow2_ceil(cap)) * 8;
      const bool in_shared = keys_bytes <= kSketchSmem;
      const size_t radix_bytes = radix_sort_bytes(cap, kSketchThreads / 32);
      const bool radix = in_shared && radix_bytes <= kSketchSmem && cap < 65536;
      const size_t work_bytes = size_t(4) * (cap + 2) * 4;
      const bool work_shared = radix && work_bytes <= kSketchSmem;
      const size_t batch_smem = radix ? std::max({keys_bytes, radix_bytes, work_shared ? work_bytes : size_t(0)})
                                      : in_shared ? keys_bytes : 0;
      const uint32_t grid = uint32_t(std::min<size_t>(tasks.size(), size_t(sms) * (in_shared ? 1 : 2)));
      d_scratch.need(scratch_stride * grid);
      d_tasks.need(tasks.size() * sizeof(BatchTask));
      XGBB_CUDA(cudaMemcpyAsync(d_tasks.p, tasks.data(), tasks.size() * sizeof(BatchTask), cudaMemcpyHostToDevice,
                                stream));
      sketch_batch_kernel<<<grid, kSketchThreads, batch_smem, stream>>>(
          d_runs.as<Run>(), d_tasks.as<BatchTask>(), uint32_t(tasks.size()), d_summaries.as<Entry>(),
          d_sizes.as<uint32_t>(), d_scratch.as<unsigned char>(), scratch_stride, cap, in_shared, radix,
          work_shared);
      XGBB_CUDA(cudaGetLastError());
    }
    trace.mark("batch summaries", stream);
    uint32_t big = 2;
    for (const ReduceTask& rt : rtasks) big = std::max(big, reduce_big(rt.limit, rt.budget));
    const size_t fast_bytes = size_t(2) * big * sizeof(float);
    const bool fast_shared = fast_bytes <= kSketchSmem;
    const size_t fast_smem = fast_shared ? fast_bytes : 0;
    // The merge tree, one launch per level (the tasks of all levels uploaded
    // once, back to back).
    std::vector<MergeTask> all;
    std::vector<size_t> level_at;
    for (const auto& level : tree.levels) {
      level_at.push_back(all.size());
      all.insert(all.end(), level.begin(), level.end());
    }
    if (!all.empty()) {
      const size_t mstride = merge_scratch_bytes(big);
      size_t widest = 0;
      for (const auto& level : tree.levels) widest = std::max(widest, level.size());
      const uint32_t mgrid = uint32_t(std::min<size_t>(widest, size_t(sms) * (fast_shared ? 2 : 4)));
      d_scratch.need(std::max(d_scratch.n, mstride * mgrid));
      d_mtasks.need(all.size() * sizeof(MergeTask));
      XGBB_CUDA(cudaMemcpyAsync(d_mtasks.p, all.data(), all.size() * sizeof(MergeTask), cudaMemcpyHostToDevice,
                                stream));
      for (size_t l = 0; l < tree.levels.size(); ++l) {
        const uint32_t n = uint32_t(tree.levels[l].size());
        if (!n) continue;
        sketch_merge_kernel<<<std::min(n, mgrid), kSketchThreads, fast_smem, stream>>>(
            d_mtasks.as<MergeTask>() + level_at[l], n, d_summaries.as<Entry>(), d_sizes.as<uint32_t>(),
            d_irregular.as<uint32_t>(), d_scratch.as<unsigned char>(), mstride, big, fast_shared);
        XGBB_CUDA(cudaGetLastError());
      }
    }
    trace.mark("merge tree", stream);
    d_ftasks.need(tree.finish.size() * sizeof(FinishTask));
    d_res.need(std::max<size_t>(tree.res.size(), 1) * sizeof(FinishRes));
    XGBB_CUDA(cudaMemcpyAsync(d_ftasks.p, tree.finish.data(), tree.finish.size() * sizeof(FinishTask),
                              cudaMemcpyHostToDevice, stream));
    if (!tree.res.empty())
      XGBB_CUDA(cudaMemcpyAsync(d_res.p, tree.res.data(), tree.res.size() * sizeof(FinishRes), cudaMemcpyHostToDevice,
                                stream));
    sketch_finish_kernel<<<nf, kSketchThreads, fast_smem, stream>>>(
        d_ftasks.as<FinishTask>(), d_res.as<FinishRes>(), d_summaries.as<Entry>(), d_sizes.as<uint32_t>(),
        d_irregular.as<uint32_t>(), d_work.as<unsigned char>(), max_bin, stride, d_cuts.as<float>(),
        d_counts.as<uint32_t>(), fast_shared);
    XGBB_CUDA(cudaGetLastError());
    d_rtasks.need(rtasks.size() * sizeof(ReduceTask));
    XGBB_CUDA(cudaMemcpyAsync(d_rtasks.p, rtasks.data(), rtasks.size() * sizeof(ReduceTask), cudaMemcpyHostToDevice,
                              stream));
    sketch_reduce_kernel<<<nf, kSketchThreads, fast_smem, stream>>>(
        d_summaries.as<Entry>(), d_sizes.as<uint32_t>(), d_rtasks.as<ReduceTask>(), d_irregular.as<uint32_t>(),
        d_work.as<unsigned char>(), max_bin, stride, d_cuts.as<float>(), d_counts.as<uint32_t>(), fast_shared);
    XGBB_CUDA(cudaGetLastError());
    // The next group reuses the buffers.
    XGBB_CUDA(cudaStreamSynchronize(stream));
    trace.mark("finish and reduce", stream);
  }
  XGBB_CUDA(cudaMemcpyAsync(cuts, d_cuts.p, size_t(cols) * stride * 4, cudaMemcpyDeviceToHost, stream));
  XGBB_CUDA(cudaMemcpyAsync(counts, d_counts.p, size_t(cols) * 4, cudaMemcpyDeviceToHost, stream));
  XGBB_CUDA(cudaStreamSynchronize(stream));
  trace.mark("cuts to the host", stream);
}

}  // namespace xgbb
