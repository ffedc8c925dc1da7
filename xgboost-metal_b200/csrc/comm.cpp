#include "comm.h"

#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

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
  ncclResult_t (*init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
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
    api.init_rank = reinterpret_cast<decltype(api.init_rank)>(sym("ncclCommInitRank"));
    api.destroy = reinterpret_cast<decltype(api.destroy)>(sym("ncclCommDestroy"));
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
  ncclComm_t c;
  trace(rank, "init", size_t(world));
  XGBB_NCCL(nccl().init_rank(&c, world, id, rank));
  trace(rank, "init done", size_t(world));
  comm_ = c;
}

void Comm::add_release_hook(const void* owner, std::function<void()> fn) { hooks_[owner] = std::move(fn); }
void Comm::remove_release_hook(const void* owner) { hooks_.erase(owner); }

void Comm::finalize() {
  auto hooks = std::move(hooks_);
  hooks_.clear();
  for (auto& kv : hooks) kv.second();
  if (comm_) {
    nccl().destroy(as_comm(comm_));
    comm_ = nullptr;
  }
  rank_ = 0;
  world_ = 1;
}

void Comm::sum_u64(void* buf, size_t count, cudaStream_t s) {
  if (!active() || !count) return;
  trace(rank_, "sum_u64", count);
  XGBB_NCCL(nccl().all_reduce(buf, buf, count, ncclUint64, ncclSum, as_comm(comm_), s));
}
void Comm::sum_u32(void* buf, size_t count, cudaStream_t s) {
  if (!active() || !count) return;
  trace(rank_, "sum_u32", count);
  XGBB_NCCL(nccl().all_reduce(buf, buf, count, ncclUint32, ncclSum, as_comm(comm_), s));
}
void Comm::max_u32(void* buf, size_t count, cudaStream_t s) {
  if (!active() || !count) return;
  trace(rank_, "max_u32", count);
  XGBB_NCCL(nccl().all_reduce(buf, buf, count, ncclUint32, ncclMax, as_comm(comm_), s));
}
void Comm::sum_f64(void* buf, size_t count, cudaStream_t s) {
  if (!active() || !count) return;
  trace(rank_, "sum_f64", count);
  XGBB_NCCL(nccl().all_reduce(buf, buf, count, ncclFloat64, ncclSum, as_comm(comm_), s));
}
void Comm::broadcast(void* buf, size_t bytes, int root, cudaStream_t s) {
  if (!active() || !bytes) return;
  trace(rank_, "broadcast", bytes);
  XGBB_NCCL(nccl().broadcast(buf, buf, bytes, ncclUint8, root, as_comm(comm_), s));
}
void Comm::reduce_scatter_u64(void* buf, size_t count, cudaStream_t s) {
  if (!active() || !count) return;
  trace(rank_, "reduce_scatter_u64", count);
  auto* b = static_cast<unsigned long long*>(buf);
  XGBB_NCCL(nccl().reduce_scatter(b, b + size_t(rank_) * count, count, ncclUint64, ncclSum, as_comm(comm_), s));
}
void Comm::all_gather(const void* send, void* recv, size_t bytes, cudaStream_t s) {
  if (!active() || !bytes) return;
  trace(rank_, "all_gather", bytes);
  XGBB_NCCL(nccl().all_gather(send, recv, bytes, ncclUint8, as_comm(comm_), s));
}
void Comm::barrier(cudaStream_t s) {
  if (!active()) return;
  static thread_local void* scratch = nullptr;
  if (!scratch) XGBB_CUDA(cudaMalloc(&scratch, 8));
  sum_u64(scratch, 1, s);
  XGBB_CUDA(cudaStreamSynchronize(s));
}

}  // namespace xgbb
