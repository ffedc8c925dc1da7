// Gradient pairs and their exact power-of-two scales computed into buffers the
// caller owns, without any device allocation: the scale accumulators live in
// one fixed array of this library instead of a per-call buffer.
//
// Limit: at most kNoAllocMaxGroups output groups (the scratch is
// kNoAllocMaxGroups * mass_bytes(1) = 17,408 bytes). Larger requests are
// rejected before anything is enqueued.
//
// What must start at zero: every accumulator of the scratch (max_bits,
// fallback, window, limbs, exact) is summed or max-reduced into by the
// gradient and magnitude kernels, so each call clears the part it uses with
// cudaMemsetAsync on the caller's stream before its first kernel. Nothing
// else is read before it is written.
//
// Overlapping calls race: the scratch is one array per device, so two calls
// that can run at the same time on one device (different streams, or
// different host threads without ordering) corrupt each other's scales. Calls
// on one stream are ordered and safe.
//
// Set-up: the first call on each device looks the scratch address up with
// cudaGetSymbolAddress (which may load this library's device code); make that
// first call before any stream capture on that device. The address is kept
// with the id of the device context it was found in; after a device reset
// the next call finds the new context and looks the address up again, so
// that call too belongs outside any capture.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "common.h"
#include "tree.h"

namespace {
constexpr uint32_t kNoAllocMaxGroups = 64;
constexpr size_t kScratchBytes = kNoAllocMaxGroups * 2 * (4 + 4 + 16 + 32 + 80);
constexpr int kMaxDevices = 64;
}  // namespace

static __device__ __align__(256) unsigned char g_gradient_scratch[kScratchBytes];

namespace xgbb {
namespace {
static_assert(kScratchBytes == kNoAllocMaxGroups * 2 * (4 + 4 + 16 + 32 + 80), "scratch size");

// Id of the calling thread's current context (cuCtxGetId: unique for the
// life of the process), or 0 when there is none or it cannot be read. The
// driver calls are reached through the runtime's entry-point lookup, so the
// library links no driver library.
unsigned long long current_context_id() {
  using GetCurrent = int (*)(void**);
  using GetId = int (*)(void*, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(f);
    f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(f);
    cudaGetLastError();
  });
  void* ctx = nullptr;
  unsigned long long id = 0;
  if (get_current && get_id && get_current(&ctx) == 0 && ctx && get_id(ctx, &id) == 0) return id;
  return 0;
}

// The array's device address in the current context. It is looked up once
// per device and kept with the id of the context it belongs to; a device
// reset (cudaDeviceReset) ends that context, and the next one maps the array
// afresh, so a different (or unreadable) context id means a new lookup.
void* scratch_address() {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  static unsigned long long ctx[kMaxDevices] = {};
  int dev = 0;
  XGBB_CUDA(cudaGetDevice(&dev));
  require(dev >= 0 && dev < kMaxDevices, "device ordinal out of range for the gradient scratch");
  std::lock_guard<std::mutex> lock(mu);
  const unsigned long long id = current_context_id();
  if (!addr[dev] || id == 0 || id != ctx[dev]) {
    XGBB_CUDA(cudaGetSymbolAddress(&addr[dev], g_gradient_scratch));
    ctx[dev] = current_context_id();  // the lookup made the device's context current
  }
  return addr[dev];
}
}  // namespace

void gradients_no_alloc(int objective, const float* margins, const float* labels,
                        const float* weights, uint64_t rows, uint32_t groups,
                        float scale_pos_weight, float2* pairs, float2* scales, cudaStream_t stream) {
  require(objective >= kSquaredError && objective <= kSoftmax, "unknown objective code");
  require(groups >= 1, "groups must be at least 1");
  require(groups <= kNoAllocMaxGroups,
          "groups = " + std::to_string(groups) + " exceeds the " + std::to_string(kNoAllocMaxGroups) +
              " output groups the fixed gradient scratch holds (" + std::to_string(kScratchBytes) +
              " bytes); use XGBBGradientsHost or training, which size their buffers per call");
  require(rows >= 1 && rows <= 0xffffffffull, "rows must be between 1 and 4294967295");
  require(margins && labels && pairs && scales, "margins, labels, pairs and scales must be device pointers");
  void* base = scratch_address();
  const size_t used = mass_bytes(groups);
  XGBB_CUDA(cudaMemsetAsync(base, 0, used, stream));
  const MassAccum m = mass_view(base, groups);
  const uint32_t n = uint32_t(rows);
  launch_gradients(objective, margins, labels, weights, n, groups, scale_pos_weight, pairs, m, stream);
  launch_mass_window(pairs, n, groups, m, stream);
  launch_scales(pairs, n, groups, m, scales, rows, true, stream);
  launch_mass_exact(pairs, n, groups, m, stream);
  launch_scales_exact(groups, m, scales, stream);
}

}  // namespace xgbb
