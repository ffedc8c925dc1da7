#pragma once
#include <cstdint>

namespace xgbb {
// Cut stride of a matrix: max(1, min(max_bin, rows)) (src/data.cpp:1232).
uint32_t cut_stride(uint32_t rows, uint32_t max_bin);
// cuts[f * stride + i] for i < counts[f]; minima[f] = -inf.
void sketch_cuts(const float* X, uint32_t rows, uint32_t cols, const float* weights,
                 uint32_t max_bin, float* cuts, uint32_t* counts, float* minima, int threads);
}  // namespace xgbb
