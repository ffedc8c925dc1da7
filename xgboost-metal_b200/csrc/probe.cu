// Throughput probes of the shared-memory pipe, for sizing the histogram
// kernels' limb scheme. Each block fills one SM (its shared memory rules out
// a second block) and runs `iters` passes of 32 feature steps per warp, with
// the histogram kernels' addressing: lane j adds to word code * 32 + (j ^ f)
// of a plane, so the 32 lanes of every instruction hit 32 different banks,
// and the codes are pseudo-random bins in [0, 256].
//
//   variant 0  red.shared.add.s32, 4 per code (the staged kernel's g0 g1 h0 h1)
//   variant 1  red.shared.add.s32, 1 per code
//   variant 2  st.shared.b32, 4 per code (the same traffic without atomics)
//   variant 3  atom.shared.add.u64, 2 per code (one 64-bit word each for g, h)
//
// The result is SM cycles per warp-level shared instruction: the block's
// clock64 span over (warps x iters x 32 x instructions per code).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <vector>

#include "common.h"

namespace xgbb {
namespace {

constexpr uint32_t kProbeBins = 257, kProbeLanes = 32;
constexpr uint32_t kProbePlaneWords = kProbeBins * kProbeLanes;

template <int V>
__global__ void __launch_bounds__(1024, 1) probe_kernel(uint32_t iters, unsigned long long* cycles, int* sink) {
  extern __shared__ __align__(16) int sm[];
  constexpr uint32_t words = 4 * kProbePlaneWords;  // four int planes or two u64 planes
  for (uint32_t i = threadIdx.x; i < words; i += blockDim.x) sm[i] = 0;
  __syncthreads();
  const uint32_t lane = threadIdx.x & 31, lane4 = lane * 4;
  const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(sm));
  constexpr uint32_t kPlaneBytes = kProbePlaneWords * 4;
  uint32_t x = 0x9e3779b9u * (threadIdx.x + 1) + 0x85ebca6bu * blockIdx.x;
  const long long t0 = clock64();
  for (uint32_t it = 0; it < iters; ++it) {
    uint32_t codes[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      x = x * 1664525u + 1013904223u;
      codes[j] = x;
    }
#pragma unroll
    for (uint32_t f = 0; f < 32; ++f) {
      const uint32_t code = (codes[f / 4] >> (8 * (f & 3))) & 0xffu;
      const int v = int(x >> 13) - (1 << 18);
      if (V == 3) {
        const uint32_t addr = base + code * 256 + (((lane ^ f) & 31) * 8);
        asm volatile("{ .reg .u64 t; atom.shared.add.u64 t, [%0], %1; }\n" ::"r"(addr), "l"((long long)v));
        asm volatile("{ .reg .u64 t; atom.shared.add.u64 t, [%0], %1; }\n" ::"r"(addr + 2 * kPlaneBytes),
                     "l"((long long)v));
      } else {
        const uint32_t addr = base + code * 128 + (lane4 ^ (4 * f));
        if (V == 2) {
          asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(addr), "r"(v));
          asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(addr + kPlaneBytes), "r"(v));
          asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(addr + 2 * kPlaneBytes), "r"(v));
          asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(addr + 3 * kPlaneBytes), "r"(v));
        } else {
          asm volatile("red.shared.add.s32 [%0], %1;\n" ::"r"(addr), "r"(v));
          if (V == 0) {
            asm volatile("red.shared.add.s32 [%0], %1;\n" ::"r"(addr + kPlaneBytes), "r"(v));
            asm volatile("red.shared.add.s32 [%0], %1;\n" ::"r"(addr + 2 * kPlaneBytes), "r"(v));
            asm volatile("red.shared.add.s32 [%0], %1;\n" ::"r"(addr + 3 * kPlaneBytes), "r"(v));
          }
        }
      }
    }
  }
  __syncthreads();
  const long long t1 = clock64();
  if (threadIdx.x == 0) cycles[blockIdx.x] = static_cast<unsigned long long>(t1 - t0);
  // Keep the planes observable.
  if (threadIdx.x == 0) atomicAdd(sink, sm[blockIdx.x % words]);
}

}  // namespace

double probe_shared_pipe(int variant, uint32_t warps, uint32_t iters) {
  if (variant < 0 || variant > 3) throw Error("Unknown probe variant.");
  if (warps < 1 || warps > 32 || iters < 1) throw Error("Probe needs 1-32 warps and at least one pass.");
  int dev = 0, sms = 0;
  XGBB_CUDA(cudaGetDevice(&dev));
  XGBB_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const size_t smem = size_t(4) * kProbePlaneWords * 4;
  unsigned long long* d_cycles = nullptr;
  int* d_sink = nullptr;
  XGBB_CUDA(cudaMalloc(&d_cycles, size_t(sms) * 8));
  XGBB_CUDA(cudaMalloc(&d_sink, 4));
  auto launch = [&](auto kernel) {
    XGBB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    kernel<<<sms, warps * 32, smem>>>(iters, d_cycles, d_sink);
  };
  for (int rep = 0; rep < 2; ++rep) {  // the first launch warms up
    switch (variant) {
      case 0: launch(probe_kernel<0>); break;
      case 1: launch(probe_kernel<1>); break;
      case 2: launch(probe_kernel<2>); break;
      default: launch(probe_kernel<3>); break;
    }
  }
  XGBB_CUDA(cudaGetLastError());
  std::vector<unsigned long long> cyc(sms);
  const cudaError_t e = cudaMemcpy(cyc.data(), d_cycles, size_t(sms) * 8, cudaMemcpyDeviceToHost);
  cudaFree(d_cycles);
  cudaFree(d_sink);
  XGBB_CUDA(e);
  std::sort(cyc.begin(), cyc.end());
  const double per_code = variant == 0 || variant == 2 ? 4.0 : variant == 3 ? 2.0 : 1.0;
  return double(cyc[cyc.size() / 2]) / (double(warps) * iters * 32.0 * per_code);
}

}  // namespace xgbb
