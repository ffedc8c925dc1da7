// Shared host/device declarations of the B200 histogram tree trainer.
#pragma once
#include <cuda_runtime.h>

#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
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
// The same for a literal message, which then costs nothing until a check
// fails (checks run once per element of large arrays).
inline void require(bool ok, const char* message) {
  if (!ok) throw Error(message);
}

inline void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Error(std::string(what) + ": " + cudaGetErrorString(e));
}
#define XGBB_CUDA(call) ::xgbb::cuda_check((call), #call)

// Phase timing of host-driven work for diagnosis: with XGBB_TRACE=1 each
// mark waits for `stream` and prints the wall time since the previous mark
// to stderr; otherwise marks cost nothing.
class Trace {
 public:
  explicit Trace(const char* scope) : scope_(scope), on_(enabled()) {
    if (on_) t_ = now();
  }
  void mark(const char* what, cudaStream_t stream) {
    if (!on_) return;
    cudaStreamSynchronize(stream);
    const double t = now();
    std::fprintf(stderr, "[xgbb trace] %s: %s %.1f ms\n", scope_, what, (t - t_) * 1e3);
    t_ = t;
  }

 private:
  static bool enabled() {
    static const bool on = [] {
      const char* v = std::getenv("XGBB_TRACE");
      return v && v[0] == '1';
    }();
    return on;
  }
  static double now() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
  }
  const char* scope_;
  bool on_;
  double t_ = 0;
};

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
