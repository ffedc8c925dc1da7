#include "comm.h"

#include <dlfcn.h>
#include <nccl.h>

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>

#include "common.h"

namespace xgbb {
namespace {

// NCCL is resolved at run time, when a communicator is first needed, and an
// NCCL already loaded into the process (for example by a framework that
// shares it) is reused. Linking it at load time would pin whichever
// libnccl.so.2 the loader finds first into every process that merely imports
// the library, and a later framework needing a newer NCCL would then fail to
// resolve its symbols.
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*abort)(ncclComm_t) = nullptr;
  ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*reduce_scatter)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                 cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  static std::string failure;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      failure = std::string("NCCL is required for multi-GPU training and could not be loaded: ") + dlerror();
      return;
    }
    auto sym = [&](const char* name) {
      void* p = dlsym(h, name);
      if (!p && failure.empty()) failure = std::string("NCCL symbol not found: ") + name;
      return p;
    };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.init_rank_config = reinterpret_cast<decltype(api.init_rank_config)>(sym("ncclCommInitRankConfig"));
    api.destroy = reinterpret_cast<decltype(api.destroy)>(sym("ncclCommDestroy"));
    api.abort = reinterpret_cast<decltype(api.abort)>(sym("ncclCommAbort"));
    api.async_error = reinterpret_cast<decltype(api.async_error)>(sym("ncclCommGetAsyncError"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
    api.broadcast = reinterpret_cast<decltype(api.broadcast)>(sym("ncclBroadcast"));
    api.reduce_scatter = reinterpret_cast<decltype(api.reduce_scatter)>(sym("ncclReduceScatter"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
  });
  require(failure.empty(), failure);
  return api;
}

void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) throw Error(std::string(what) + ": " + nccl().error_string(r));
}
#define XGBB_NCCL(call) nccl_check((call), #call)
using Clock = std::chrono::steady_clock;
double seconds_since(Clock::time_point t) { return std::chrono::duration<double>(Clock::now() - t).count(); }
ncclComm_t as_comm(void* p) { return static_cast<ncclComm_t>(p); }

// XGBB_TRACE=1 logs every collective this rank issues (stderr).
bool tracing() {
  static const bool on = [] {
    const char* v = std::getenv("XGBB_TRACE");
    return v && *v && *v != '0';
  }();
  return on;
}
void trace(int rank, const char* op, size_t count) {
  if (tracing()) {
    std::fprintf(stderr, "[xgbb rank %d] %s %zu\n", rank, op, count);
    std::fflush(stderr);
  }
}
}  // namespace

Comm& Comm::get() {
  static Comm instance;
  return instance;
}

std::string nccl_unique_id_hex() {
  ncclUniqueId id;
  XGBB_NCCL(nccl().get_unique_id(&id));
  std::string out;
  char buf[3];
  for (size_t i = 0; i < sizeof(id.internal); ++i) {
    std::snprintf(buf, sizeof buf, "%02x", static_cast<unsigned char>(id.internal[i]));
    out += buf;
  }
  return out;
}

void Comm::init(int rank, int world, const std::string& id_hex, int device) {
  require(world >= 1 && rank >= 0 && rank < world, "invalid rank / world size");
  finalize();
  rank_ = rank;
  world_ = world;
  if (world == 1) return;
  ncclUniqueId id;
  require(id_hex.size() == 2 * sizeof(id.internal), "nccl_unique_id must be a hex string of the NCCL id");
  for (size_t i = 0; i < sizeof(id.internal); ++i)
    id.internal[i] = char(std::stoi(id_hex.substr(2 * i, 2), nullptr, 16));
  XGBB_CUDA(cudaSetDevice(device));
  ncclComm_t c = nullptr;
  trace(rank, "init", size_t(world));
  // A non-blocking communicator: joining, and any call NCCL cannot finish at
  // once, return ncclInProgress and are waited for here within the time
  // limit, so a rank that never joins ends in an error instead of a hang.
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  const ncclResult_t r = nccl().init_rank_config(&c, world, id, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) nccl_check(r, "ncclCommInitRankConfig");
  comm_ = c;
  failed_ = false;
  settle("communicator initialisation (a rank did not join)");
  trace(rank, "init done", size_t(world));
}

void Comm::set_timeout(double seconds) {
  require(seconds > 0, "communicator timeout must be positive");
  timeout_s_ = seconds;
}

// Aborting ends the communicator's kernels, but may wait on a proxy thread
// that talks to the failed rank: it runs on a thread of its own, the error is
// raised at once, and the process is expected to exit after it.
void Comm::abort_detached() {
  trace(rank_, "abort", 0);
  void* c = comm_;
  if (c && !failed_) std::thread([c] { nccl().abort(as_comm(c)); }).detach();
  failed_ = true;
}

void Comm::fail(const std::string& what) {
  abort_detached();
  throw Error(what);
}

// Waits until NCCL has finished a call that returned ncclInProgress.
void Comm::settle(const char* what) {
  const auto start = Clock::now();
  for (;;) {
    ncclResult_t e = ncclSuccess;
    nccl_check(nccl().async_error(as_comm(comm_), &e), "ncclCommGetAsyncError");
    if (e == ncclSuccess) return;
    if (e != ncclInProgress) fail(std::string("NCCL error during ") + what + ": " + nccl().error_string(e));
    if (seconds_since(start) > timeout_s_)
      fail(std::string("NCCL ") + what + " did not complete within " + std::to_string(timeout_s_) + " s");
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

void Comm::call(ncclResult_t r, const char* what) {
  if (r == ncclInProgress) settle(what);
  else if (r != ncclSuccess) fail(std::string(what) + ": " + nccl().error_string(r));
}

// Host wait for stream work that contains collectives (`ev` recorded after
// it): polls the event and NCCL's asynchronous error; past the time limit (a
// rank failed or left) the communicator is aborted and an Error raised.
void Comm::wait(cudaEvent_t ev, const char* what) {
  if (!active()) {
    XGBB_CUDA(cudaEventSynchronize(ev));
    return;
  }
  require(!failed_, "the communicator was aborted after an earlier failure; the process should exit");
  trace(rank_, what, 0);
  const auto start = Clock::now();
  for (;;) {
    const cudaError_t q = cudaEventQuery(ev);
    if (q == cudaSuccess) return;
    if (q != cudaErrorNotReady) XGBB_CUDA(q);
    ncclResult_t e = ncclSuccess;
    nccl_check(nccl().async_error(as_comm(comm_), &e), "ncclCommGetAsyncError");
    if (e != ncclSuccess && e != ncclInProgress)
      fail(std::string("NCCL error while waiting for ") + what + ": " + nccl().error_string(e));
    if (seconds_since(start) > timeout_s_)
      fail(std::string(what) + " did not complete within " + std::to_string(timeout_s_) +
           " s; a rank may have failed or left (communicator aborted)");
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

// Device-wide synchronisation under the same limit: the synchronising call
// runs on a helper thread while this one watches NCCL and the clock.
void Comm::wait_device(const char* what) {
  if (!active()) {
    XGBB_CUDA(cudaDeviceSynchronize());
    return;
  }
  require(!failed_, "the communicator was aborted after an earlier failure; the process should exit");
  int dev = 0;
  XGBB_CUDA(cudaGetDevice(&dev));
  auto done = std::make_shared<std::atomic<bool>>(false);
  auto err = std::make_shared<cudaError_t>(cudaSuccess);
  std::thread t([dev, done, err] {
    cudaSetDevice(dev);
    *err = cudaDeviceSynchronize();
    *done = true;
  });
  const auto start = Clock::now();
  std::string failure;
  while (!*done) {
    ncclResult_t e = ncclSuccess;
    if (nccl().async_error(as_comm(comm_), &e) == ncclSuccess && e != ncclSuccess && e != ncclInProgress) {
      failure = std::string("NCCL error while waiting for ") + what + ": " + nccl().error_string(e);
      break;
    }
    if (seconds_since(start) > timeout_s_) {
      failure = std::string(what) + " did not complete within " + std::to_string(timeout_s_) +
                " s; a rank may have failed or left (communicator aborted)";
      break;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
  if (!failure.empty()) {
    t.detach();  // stays blocked behind the aborted communicator's kernels
    fail(failure);
  }
  t.join();
  XGBB_CUDA(*err);
}

void Comm::add_release_hook(const void* owner, std::function<void()> fn) { hooks_[owner] = std::move(fn); }
void Comm::remove_release_hook(const void* owner) { hooks_.erase(owner); }

void Comm::finalize() {
  auto hooks = std::move(hooks_);
  hooks_.clear();
  for (auto& kv : hooks) kv.second();
  if (comm_) {
    if (!failed_) nccl().destroy(as_comm(comm_));
    comm_ = nullptr;
  }
  failed_ = false;
  rank_ = 0;
  world_ = 1;
}

void Comm::sum_u64(void* buf, size_t count, cudaStream_t s) {
  if (!active() || !count) return;
  trace(rank_, "sum_u64", count);
  require(!failed_, "the communicator was aborted after an earlier failure; the process should exit");
  call(nccl().all_reduce(buf, buf, count, ncclUint64, ncclSum, as_comm(comm_), s), "ncclAllReduce");
}
void Comm::sum_u32(void* buf, size_t count, cudaStream_t s) {
  if (!active() || !count) return;
  trace(rank_, "sum_u32", count);
  require(!failed_, "the communicator was aborted after an earlier failure; the process should exit");
  call(nccl().all_reduce(buf, buf, count, ncclUint32, ncclSum, as_comm(comm_), s), "ncclAllReduce");
}
void Comm::max_u32(void* buf, size_t count, cudaStream_t s) {
  if (!active() || !count) return;
  trace(rank_, "max_u32", count);
  require(!failed_, "the communicator was aborted after an earlier failure; the process should exit");
  call(nccl().all_reduce(buf, buf, count, ncclUint32, ncclMax, as_comm(comm_), s), "ncclAllReduce");
}
void Comm::sum_f64(void* buf, size_t count, cudaStream_t s) {
  if (!active() || !count) return;
  trace(rank_, "sum_f64", count);
  require(!failed_, "the communicator was aborted after an earlier failure; the process should exit");
  call(nccl().all_reduce(buf, buf, count, ncclFloat64, ncclSum, as_comm(comm_), s), "ncclAllReduce");
}
void Comm::broadcast(void* buf, size_t bytes, int root, cudaStream_t s) {
  if (!active() || !bytes) return;
  trace(rank_, "broadcast", bytes);
  require(!failed_, "the communicator was aborted after an earlier failure; the process should exit");
  call(nccl().broadcast(buf, buf, bytes, ncclUint8, root, as_comm(comm_), s), "ncclBroadcast");
}
void Comm::reduce_scatter_u64(void* buf, size_t count, cudaStream_t s) {
  if (!active() || !count) return;
  trace(rank_, "reduce_scatter_u64", count);
  require(!failed_, "the communicator was aborted after an earlier failure; the process should exit");
  auto* b = static_cast<unsigned long long*>(buf);
  call(nccl().reduce_scatter(b, b + size_t(rank_) * count, count, ncclUint64, ncclSum, as_comm(comm_), s),
       "ncclReduceScatter");
}
void Comm::all_gather(const void* send, void* recv, size_t bytes, cudaStream_t s) {
  if (!active() || !bytes) return;
  trace(rank_, "all_gather", bytes);
  require(!failed_, "the communicator was aborted after an earlier failure; the process should exit");
  call(nccl().all_gather(send, recv, bytes, ncclUint8, as_comm(comm_), s), "ncclAllGather");
}
void Comm::barrier(cudaStream_t s) {
  if (!active()) return;
  static thread_local void* scratch = nullptr;
  if (!scratch) XGBB_CUDA(cudaMalloc(&scratch, 8));
  sum_u64(scratch, 1, s);
  cudaEvent_t ev;
  XGBB_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  XGBB_CUDA(cudaEventRecord(ev, s));
  try {
    wait(ev, "barrier");
  } catch (...) {
    cudaEventDestroy(ev);
    throw;
  }
  cudaEventDestroy(ev);
}

}  // namespace xgbb
