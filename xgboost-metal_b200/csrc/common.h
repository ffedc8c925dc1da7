// Shared host/device declarations of the B200 histogram tree trainer.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

namespace xgbb {

// Thrown by every failed check; the C ABI turns it into a -1 return and a
// thread-local message (the reference's convention, src/c_api.cpp:33-40).
struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};

inline void require(bool ok, const std::string& message) {
  if (!ok) throw Error(message);
}

inline void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Error(std::string(what) + ": " + cudaGetErrorString(e));
}
#define XGBB_CUDA(call) ::xgbb::cuda_check((call), #call)

constexpr uint32_t kMaxDepth = 10;         // device driver limit (src/tree.cpp:376-384)
constexpr uint32_t kMaxBins = 256;         // bins per feature, missing bin excluded
constexpr uint32_t kMaxFrontier = 1u << (kMaxDepth - 1);
constexpr uint32_t kMassBuckets = 8;       // 8 x 32-bit windows cover float magnitudes
constexpr uint32_t kTileRows = 2048;       // rows per histogram work item

enum Objective : int { kSquaredError = 0, kLogistic = 1, kLogitRaw = 2, kSoftprob = 3, kSoftmax = 4 };

// A split candidate / chosen split (one per node and feature, then per node).
// Integer child sums are exact; float fields follow the reference's Split
// record (include/metalgb/shared.h:124-134).
struct DevSplit {
  float gain, threshold;
  int32_t feature, split_bin;  // present row goes left iff bin <= split_bin
  uint32_t default_left;
  float left_weight, right_weight, parent_weight;
  float left_h, right_h, total_g, total_h;
  float applied_parent_weight, applied_parent_hessian;
  uint32_t order, pad;
  long long left_g, left_hs, right_g, right_hs;
};
static_assert(sizeof(DevSplit) == 96, "DevSplit layout");

// Model node (device node table, node id = index). Mirrors the replayed
// host node of src/tree.cpp:1663-1717 plus the bin form of the split.
struct DevNode {
  int32_t left, right, parent, feature;
  int32_t split_bin;
  uint32_t default_left;
  float threshold, leaf, cover, gain, base_weight;
  uint32_t flags;  // 1 = evaluated, 2 = expanded
};
static_assert(sizeof(DevNode) == 48, "DevNode layout");

struct TreeParams {
  uint32_t max_depth;
  float eta, reg_lambda, reg_alpha, min_child_weight, max_delta_step, min_split_loss;
};

// Tree driver state (device). Kernels read live counts from here so that one
// fixed launch sequence (captured once as a CUDA graph) serves every tree.
struct DriverState {
  uint32_t node_count, frontier, depth, error;
  uint32_t pairs, total_tiles, pad0, pad1;
};
enum : uint32_t { kErrCapacity = 1, kErrNode = 2, kErrLayout = 4 };

}  // namespace xgbb
