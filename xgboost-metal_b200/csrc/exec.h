// Executors for block-structured algorithms: the same algorithm code runs as
// a CUDA thread block (DeviceExec: each loop strided over the block's threads
// with a barrier after it, block-wide scans, device atomics) and serially on
// the host (HostExec), which is how the tests check the kernels' index and
// scan logic on the CPU against the oracle.
//
// Contract for algorithm code: every executor call is reached by all threads
// of the block (control flow depends only on values every thread reads after
// a barrier), and a loop body touches no location another index of the same
// loop writes, except through the atomic helpers.
#pragma once
#include <cmath>
#include <cstdint>
#include <vector>

#if defined(__CUDACC__)
#define XGBB_HD __host__ __device__
#else
#define XGBB_HD
#endif

namespace xgbb {

// Associative combining operations with their identities.
struct Add32 {
  XGBB_HD uint32_t operator()(uint32_t a, uint32_t b) const { return a + b; }
  XGBB_HD static uint32_t identity() { return 0u; }
};
struct Add64 {
  XGBB_HD unsigned long long operator()(unsigned long long a, unsigned long long b) const { return a + b; }
  XGBB_HD static unsigned long long identity() { return 0ull; }
};
struct MaxU32 {
  XGBB_HD uint32_t operator()(uint32_t a, uint32_t b) const { return a > b ? a : b; }
  XGBB_HD static uint32_t identity() { return 0u; }
};
// Addition saturating above 2^24 (associative on non-negative integers).
struct SatAdd24 {
  XGBB_HD uint32_t operator()(uint32_t a, uint32_t b) const {
    const uint32_t s = a + b;
    return (s > (1u << 24) + 1 || s < a) ? (1u << 24) + 1 : s;
  }
  XGBB_HD static uint32_t identity() { return 0u; }
};
// Right-biased maximum: b unless b < a. Associative, and a left fold of it
// from `init` is the serial clamp `if (x < prev) x = prev; prev = x`.
struct KeepMax {
  XGBB_HD float operator()(float a, float b) const { return b < a ? a : b; }
  XGBB_HD static float identity() { return -INFINITY; }
};

// Serial executor. `notes` counts algorithm-specific events (hand-overs to
// serial forms) for the tests.
struct HostExec {
  uint64_t notes[8] = {};
  void note(uint32_t kind) { ++notes[kind & 7]; }
  template <class F>
  void for_each(uint32_t n, F&& f) {
    for (uint32_t i = 0; i < n; ++i) f(i);
  }
  template <class T, class Op>
  T scan_exclusive(T* a, uint32_t n, Op op) {
    T acc = Op::identity();
    for (uint32_t i = 0; i < n; ++i) {
      const T x = a[i];
      a[i] = acc;
      acc = op(acc, x);
    }
    return acc;
  }
  template <class T, class Op>
  void scan_inclusive(T* a, uint32_t n, T init, Op op) {
    T acc = init;
    for (uint32_t i = 0; i < n; ++i) a[i] = acc = op(acc, a[i]);
  }
  // order[i] = index of the i-th smallest of key[0, n), ties in index order
  // (the device's radix sort gives the same order). The other pointers are
  // the device form's scratch and go unused here.
  void stable_order(uint32_t* key, uint16_t* order, uint32_t n, uint32_t*, uint16_t*, uint32_t*) {
    std::vector<uint32_t> idx(n), tmp(n);
    for (uint32_t i = 0; i < n; ++i) idx[i] = i;
    for (uint32_t shift = 0; shift < 32; shift += 8) {  // LSD counting sort, stable
      uint32_t count[257] = {};
      for (uint32_t i = 0; i < n; ++i) ++count[((key[idx[i]] >> shift) & 255u) + 1];
      for (uint32_t d = 0; d < 256; ++d) count[d + 1] += count[d];
      for (uint32_t i = 0; i < n; ++i) tmp[count[(key[idx[i]] >> shift) & 255u]++] = idx[i];
      idx.swap(tmp);
    }
    for (uint32_t i = 0; i < n; ++i) order[i] = uint16_t(idx[i]);
  }
  void add_u64(unsigned long long* p, unsigned long long v) { *p += v; }
  uint32_t add_u32(uint32_t* p, uint32_t v) {
    const uint32_t old = *p;
    *p = old + v;
    return old;
  }
  uint32_t sub_u32(uint32_t* p, uint32_t v) {
    const uint32_t old = *p;
    *p = old - v;
    return old;
  }
};

#if defined(__CUDACC__)
// Block executor: loop bodies strided over the block's threads with a
// barrier after each loop; scans over arrays by contiguous per-thread chunks
// and a warp-shuffle scan of the chunk totals, each operation applied left to
// right.
struct DeviceExec {
  __device__ void note(uint32_t) {}

  template <class F>
  __device__ void for_each(uint32_t n, F&& f) {
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) f(i);
    __syncthreads();
  }

  // Exclusive block scan of one value per thread; *total gets the fold of all.
  template <class T, class Op>
  __device__ T block_scan(T x, Op op, T* total) {
    __shared__ unsigned long long warp_buf[32];
    T* warp_tot = reinterpret_cast<T*>(warp_buf);
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
    T v = x;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const T o = __shfl_up_sync(0xffffffffu, v, d);
      if (lane >= uint32_t(d)) v = op(o, v);
    }
    if (lane == 31) warp_tot[warp] = v;
    __syncthreads();
    if (warp == 0) {
      T w = lane < nwarps ? warp_tot[lane] : Op::identity();
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const T o = __shfl_up_sync(0xffffffffu, w, d);
        if (lane >= uint32_t(d)) w = op(o, w);
      }
      warp_tot[lane] = w;
    }
    __syncthreads();
    const T before_warp = warp ? warp_tot[warp - 1] : Op::identity();
    const T prev_lane = __shfl_up_sync(0xffffffffu, v, 1);
    const T excl = lane ? op(before_warp, prev_lane) : before_warp;
    *total = warp_tot[nwarps - 1];
    __syncthreads();
    return excl;
  }

  // Stable radix sort (8-bit digits, four passes) of n < 65536 32-bit keys:
  // order[i] = index of the i-th smallest, ties in index order. key, order
  // and key2, order2 (n entries each) are shared scratch, cnt holds
  // 256 * (warps + 1) counters. Warp w ranks the elements of its contiguous
  // segment row by row, lanes with equal digits found by __match_any_sync,
  // and the offsets are scanned digit-major then warp, so equal keys keep
  // their input order. key is left permuted.
  __device__ void stable_order(uint32_t* key, uint16_t* order, uint32_t n, uint32_t* key2, uint16_t* order2,
                               uint32_t* cnt) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const uint32_t stride = nw + 1;  // counter of (digit d, warp w): cnt[d * stride + w]
    const uint32_t seg = (n + nw - 1) / nw;
    const uint32_t lo = min(n, warp * seg), hi = min(n, lo + seg);
    const uint32_t lt = (1u << lane) - 1u;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) order[i] = uint16_t(i);
    uint32_t *ka = key, *kb = key2;
    uint16_t *oa = order, *ob = order2;
    for (uint32_t shift = 0; shift < 32; shift += 8) {
      for (uint32_t i = threadIdx.x; i < 256 * stride; i += blockDim.x) cnt[i] = 0;
      __syncthreads();
      for (uint32_t base = lo; base < hi; base += 32) {
        const uint32_t e = base + lane;
        const bool valid = e < hi;
        const uint32_t d = valid ? (ka[e] >> shift) & 255u : 256u + lane;
        const uint32_t m = __match_any_sync(0xffffffffu, d);
        if (valid && (m & lt) == 0) cnt[d * stride + warp] += __popc(m);
        __syncwarp();
      }
      __syncthreads();
      scan_exclusive(cnt, 256 * stride, Add32{});
      for (uint32_t base = lo; base < hi; base += 32) {
        const uint32_t e = base + lane;
        const bool valid = e < hi;
        const uint32_t d = valid ? (ka[e] >> shift) & 255u : 256u + lane;
        const uint32_t m = __match_any_sync(0xffffffffu, d);
        if (valid) {
          const uint32_t pos = cnt[d * stride + warp] + __popc(m & lt);
          kb[pos] = ka[e];
          ob[pos] = oa[e];
        }
        __syncwarp();
        if (valid && (m & lt) == 0) cnt[d * stride + warp] += __popc(m);
        __syncwarp();
      }
      __syncthreads();
      uint32_t* tk = ka;
      ka = kb;
      kb = tk;
      uint16_t* to = oa;
      oa = ob;
      ob = to;
    }
  }

  template <class T, class Op>
  __device__ T scan_exclusive(T* a, uint32_t n, Op op) {
    const uint32_t chunk = (n + blockDim.x - 1) / blockDim.x;
    const uint32_t lo = min(n, threadIdx.x * chunk), hi = min(n, lo + chunk);
    T acc = Op::identity();
    for (uint32_t i = lo; i < hi; ++i) acc = op(acc, a[i]);
    T total;
    T run = block_scan(acc, op, &total);
    for (uint32_t i = lo; i < hi; ++i) {
      const T x = a[i];
      a[i] = run;
      run = op(run, x);
    }
    __syncthreads();
    return total;
  }

  template <class T, class Op>
  __device__ void scan_inclusive(T* a, uint32_t n, T init, Op op) {
    const uint32_t chunk = (n + blockDim.x - 1) / blockDim.x;
    const uint32_t lo = min(n, threadIdx.x * chunk), hi = min(n, lo + chunk);
    T acc = Op::identity();
    for (uint32_t i = lo; i < hi; ++i) acc = op(acc, a[i]);
    T total;
    T run = op(init, block_scan(acc, op, &total));
    for (uint32_t i = lo; i < hi; ++i) a[i] = run = op(run, a[i]);
    __syncthreads();
  }

  __device__ void add_u64(unsigned long long* p, unsigned long long v) { atomicAdd(p, v); }
  __device__ uint32_t add_u32(uint32_t* p, uint32_t v) { return atomicAdd(p, v); }
  __device__ uint32_t sub_u32(uint32_t* p, uint32_t v) { return atomicSub(p, v); }
};
#endif

}  // namespace xgbb
