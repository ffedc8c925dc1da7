#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace xgbb {
// Cut stride of a matrix: max(1, min(max_bin, rows)) (src/data.cpp:1232).
uint32_t cut_stride(uint32_t rows, uint32_t max_bin);
// cuts[f * stride + i] for i < counts[f]; minima[f] = -inf.
void sketch_cuts(const float* X, uint32_t rows, uint32_t cols, const float* weights,
                 uint32_t max_bin, float* cuts, uint32_t* counts, float* minima, int threads);
// The same cuts computed on the GPU (sketch_gpu.cu) from a device matrix X
// [rows][cols] and optional device weights; results land in host arrays.
void sketch_cuts_device(const float* X, uint32_t rows, uint32_t cols, const float* weights, uint32_t max_bin,
                        float* cuts, uint32_t* counts, float* minima, cudaStream_t stream);
}  // namespace xgbb
