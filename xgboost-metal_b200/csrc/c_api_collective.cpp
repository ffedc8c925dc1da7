// Host-side collective entry points of the upstream ABI over the NCCL
// communicator of row-sharded training: broadcast and all-reduce of host
// buffers (staged through device memory, waits bounded by the communicator's
// time limit), rank metadata, messages and error signalling. Upstream's
// tracker (a TCP rendezvous service) has no counterpart: ranks bootstrap NCCL
// from a unique id shared out of band (XGBBNcclUniqueId).
#include <cuda_runtime.h>
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <type_traits>
#include <vector>

#include "c_api_common.h"
#include "comm.h"
#include "xgboost/c_api.h"

using namespace xgbb::capi;
using xgbb::Error;
using xgbb::require;

namespace {

// Runs `collective(device_send, device_recv, stream)` on device copies of a
// host buffer and returns the received bytes.
template <class F>
std::vector<char> staged(const void* send, size_t send_bytes, size_t recv_bytes, const char* what, F collective) {
  xgbb::DeviceBuffer dsend(std::max<size_t>(send_bytes, 1)), drecv(std::max<size_t>(recv_bytes, 1));
  cudaStream_t s = nullptr;
  cudaEvent_t ev = nullptr;
  XGBB_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  std::vector<char> out(recv_bytes);
  try {
    XGBB_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    if (send_bytes) XGBB_CUDA(cudaMemcpyAsync(dsend.get(), send, send_bytes, cudaMemcpyHostToDevice, s));
    collective(dsend.get(), drecv.get(), s);
    if (recv_bytes) XGBB_CUDA(cudaMemcpyAsync(out.data(), drecv.get(), recv_bytes, cudaMemcpyDeviceToHost, s));
    XGBB_CUDA(cudaEventRecord(ev, s));
    xgbb::Comm::get().wait(ev, what);
  } catch (...) {
    if (ev) cudaEventDestroy(ev);
    if (!xgbb::Comm::get().failed()) cudaStreamDestroy(s);
    throw;
  }
  cudaEventDestroy(ev);
  cudaStreamDestroy(s);
  return out;
}

// IEEE binary16 <-> binary32, round to nearest even.
float half_to_float(uint16_t h) {
  const uint32_t sign = uint32_t(h & 0x8000u) << 16, e = (h >> 10) & 31, m = h & 0x3ffu;
  uint32_t out;
  if (e == 31) out = sign | 0x7f800000u | (m << 13);
  else if (e) out = sign | ((e + 112) << 23) | (m << 13);
  else if (!m) out = sign;
  else {
    int sh = __builtin_clz(m) - 21;
    out = sign | (uint32_t(113 - sh) << 23) | (((m << sh) & 0x3ffu) << 13);
  }
  float f;
  std::memcpy(&f, &out, 4);
  return f;
}

uint16_t float_to_half(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint16_t sign = uint16_t((x >> 16) & 0x8000u);
  const uint32_t abs = x & 0x7fffffffu;
  if (abs >= 0x7f800000u) return uint16_t(sign | 0x7c00u | (abs > 0x7f800000u ? 0x200u : 0u));
  if (abs >= 0x477ff000u) return uint16_t(sign | 0x7c00u);  // rounds past the largest half
  const int e = int(abs >> 23) - 127;
  if (e >= -14) {
    // Normal half: keep 10 mantissa bits, round the 13 dropped bits to even.
    uint32_t m = abs & 0x7fffffu;
    uint32_t h = uint32_t(e + 15) << 10 | (m >> 13);
    const uint32_t rest = m & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) ++h;
    return uint16_t(sign | h);
  }
  if (e < -25) return sign;
  // Subnormal half: the value in units of 2^-24, rounded to even; the
  // 24-bit significand loses its lowest -e - 1 bits.
  const uint32_t m = (abs & 0x7fffffu) | 0x800000u;
  const int shift = -e - 1;
  uint32_t h = m >> shift;
  const uint32_t rest = m & ((1u << shift) - 1), halfway = 1u << (shift - 1);
  if (rest > halfway || (rest == halfway && (h & 1u))) ++h;
  return uint16_t(sign | h);
}

template <class T>
T combine(T a, T b, int op) {
  switch (op) {
    case 0: return a > b ? a : b;
    case 1: return a < b ? a : b;
    case 2: return T(a + b);
  }
  if constexpr (std::is_integral_v<T>) {
    if (op == 3) return T(a & b);
    if (op == 4) return T(a | b);
    if (op == 5) return T(a ^ b);
  }
  throw Error("Bitwise all-reduce needs an integer data type.");
}

template <class T>
void reduce_into(char* buf, const std::vector<char>& all, size_t count, int world, int op) {
  T* out = reinterpret_cast<T*>(buf);
  for (size_t i = 0; i < count; ++i) {
    T acc;
    std::memcpy(&acc, all.data() + i * sizeof(T), sizeof(T));
    for (int r = 1; r < world; ++r) {
      T v;
      std::memcpy(&v, all.data() + (size_t(r) * count + i) * sizeof(T), sizeof(T));
      acc = combine(acc, v, op);
    }
    out[i] = acc;
  }
}

}  // namespace

// include/xgboost/c_api.h:1798
XGB_DLL int XGCommunicatorIsDistributed(void) { return xgbb::Comm::get().world() > 1 ? 1 : 0; }

// include/xgboost/c_api.h:1809: through the log callback, else stderr.
XGB_DLL int XGCommunicatorPrint(char const* message) {
  return guarded([&] {
    require(message != nullptr, "Null message.");
    log_message(message);
  });
}

// include/xgboost/c_api.h:1817
XGB_DLL int XGCommunicatorGetProcessorName(const char** name_str) {
  return guarded([&] {
    char host[256] = {};
    require(gethostname(host, sizeof host - 1) == 0, "Cannot read the host name.");
    results.str = host;
    *name_str = results.str.c_str();
  });
}

// include/xgboost/c_api.h:1835: `size` bytes from `root` to every rank.
XGB_DLL int XGCommunicatorBroadcast(void* send_receive_buffer, size_t size, int root) {
  return guarded([&] {
    xgbb::Comm& c = xgbb::Comm::get();
    require(root >= 0 && root < c.world(), "Broadcast root is out of range.");
    if (!c.active() || size == 0) return;
    require(send_receive_buffer != nullptr, "Null broadcast buffer.");
    const auto got = staged(send_receive_buffer, size, size, "a host broadcast",
                            [&](void* dsend, void* drecv, cudaStream_t s) {
                              XGBB_CUDA(cudaMemcpyAsync(drecv, dsend, size, cudaMemcpyDeviceToDevice, s));
                              c.broadcast(drecv, size, root, s);
                            });
    std::memcpy(send_receive_buffer, got.data(), size);
  });
}

// include/xgboost/c_api.h:1858: data_type 0 f16, 1 f32, 2 f64, 3 long double,
// 4-7 i8/i16/i32/i64, 8-11 u8/u16/u32/u64; op 0 max, 1 min, 2 sum, 3 and,
// 4 or, 5 xor (python-package/xgboost/collective.py:246-282). The buffers of
// all ranks are gathered and reduced in rank order on the host.
XGB_DLL int XGCommunicatorAllreduce(void* send_receive_buffer, size_t count, int data_type, int op) {
  return guarded([&] {
    static const size_t sizes[] = {2, 4, 8, sizeof(long double), 1, 2, 4, 8, 1, 2, 4, 8};
    require(data_type >= 0 && data_type <= 11, "Unknown all-reduce data type.");
    require(op >= 0 && op <= 5, "Unknown all-reduce operation.");
    xgbb::Comm& c = xgbb::Comm::get();
    if (!c.active() || count == 0) return;
    require(send_receive_buffer != nullptr, "Null all-reduce buffer.");
    const size_t bytes = count * sizes[data_type];
    const int world = c.world();
    const auto all = staged(send_receive_buffer, bytes, bytes * world, "a host all-reduce",
                            [&](void* dsend, void* drecv, cudaStream_t s) { c.all_gather(dsend, drecv, bytes, s); });
    char* buf = static_cast<char*>(send_receive_buffer);
    switch (data_type) {
      case 0: {
        std::vector<char> widened(count * world * 4);
        for (size_t i = 0; i < count * world; ++i) {
          uint16_t h;
          std::memcpy(&h, all.data() + i * 2, 2);
          const float f = half_to_float(h);
          std::memcpy(widened.data() + i * 4, &f, 4);
        }
        std::vector<float> acc(count);
        reduce_into<float>(reinterpret_cast<char*>(acc.data()), widened, count, world, op);
        for (size_t i = 0; i < count; ++i) {
          const uint16_t h = float_to_half(acc[i]);
          std::memcpy(buf + i * 2, &h, 2);
        }
        break;
      }
      case 1: reduce_into<float>(buf, all, count, world, op); break;
      case 2: reduce_into<double>(buf, all, count, world, op); break;
      case 3: reduce_into<long double>(buf, all, count, world, op); break;
      case 4: reduce_into<int8_t>(buf, all, count, world, op); break;
      case 5: reduce_into<int16_t>(buf, all, count, world, op); break;
      case 6: reduce_into<int32_t>(buf, all, count, world, op); break;
      case 7: reduce_into<int64_t>(buf, all, count, world, op); break;
      case 8: reduce_into<uint8_t>(buf, all, count, world, op); break;
      case 9: reduce_into<uint16_t>(buf, all, count, world, op); break;
      case 10: reduce_into<uint32_t>(buf, all, count, world, op); break;
      case 11: reduce_into<uint64_t>(buf, all, count, world, op); break;
    }
  });
}

// Aborts this rank's communicator; the others see their collectives fail.
XGB_DLL int XGCommunicatorSignalError(void) {
  return guarded([&] { xgbb::Comm::get().signal_error(); });
}

namespace {
[[noreturn]] void no_tracker() {
  throw Error("Trackers are not used by the CUDA backend: ranks bootstrap NCCL from a unique id shared out "
              "of band (XGBBNcclUniqueId; xgboost.collective.init(nccl_unique_id=...)).");
}
}  // namespace

// include/xgboost/c_api.h:1697-1742
XGB_DLL int XGTrackerCreate(char const* config, TrackerHandle* handle) {
  (void)config, (void)handle;
  return guarded([] { no_tracker(); });
}
XGB_DLL int XGTrackerWorkerArgs(TrackerHandle handle, char const** args) {
  (void)handle, (void)args;
  return guarded([] { no_tracker(); });
}
XGB_DLL int XGTrackerRun(TrackerHandle handle, char const* config) {
  (void)handle, (void)config;
  return guarded([] { no_tracker(); });
}
XGB_DLL int XGTrackerWaitFor(TrackerHandle handle, char const* config) {
  (void)handle, (void)config;
  return guarded([] { no_tracker(); });
}
XGB_DLL int XGTrackerFree(TrackerHandle handle) {
  return guarded([&] { require(handle == nullptr, "Unknown tracker handle."); });
}
