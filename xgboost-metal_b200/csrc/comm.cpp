#include "comm.h"

#include <nccl.h>

#include <cstdio>
#include <cstring>

#include "common.h"

namespace xgbb {
namespace {
void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) throw Error(std::string(what) + ": " + ncclGetErrorString(r));
}
#define XGBB_NCCL(call) nccl_check((call), #call)
ncclComm_t as_comm(void* p) { return static_cast<ncclComm_t>(p); }
}  // namespace

Comm& Comm::get() {
  static Comm instance;
  return instance;
}

std::string nccl_unique_id_hex() {
  ncclUniqueId id;
  XGBB_NCCL(ncclGetUniqueId(&id));
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
  XGBB_NCCL(ncclCommInitRank(&c, world, id, rank));
  comm_ = c;
}

void Comm::finalize() {
  if (comm_) {
    ncclCommDestroy(as_comm(comm_));
    comm_ = nullptr;
  }
  rank_ = 0;
  world_ = 1;
}

void Comm::sum_u64(void* buf, size_t count, cudaStream_t s) {
  if (!active() || !count) return;
  XGBB_NCCL(ncclAllReduce(buf, buf, count, ncclUint64, ncclSum, as_comm(comm_), s));
}
void Comm::sum_u32(void* buf, size_t count, cudaStream_t s) {
  if (!active() || !count) return;
  XGBB_NCCL(ncclAllReduce(buf, buf, count, ncclUint32, ncclSum, as_comm(comm_), s));
}
void Comm::max_u32(void* buf, size_t count, cudaStream_t s) {
  if (!active() || !count) return;
  XGBB_NCCL(ncclAllReduce(buf, buf, count, ncclUint32, ncclMax, as_comm(comm_), s));
}
void Comm::sum_f64(void* buf, size_t count, cudaStream_t s) {
  if (!active() || !count) return;
  XGBB_NCCL(ncclAllReduce(buf, buf, count, ncclFloat64, ncclSum, as_comm(comm_), s));
}
void Comm::broadcast(void* buf, size_t bytes, int root, cudaStream_t s) {
  if (!active() || !bytes) return;
  XGBB_NCCL(ncclBroadcast(buf, buf, bytes, ncclUint8, root, as_comm(comm_), s));
}
void Comm::barrier(cudaStream_t s) {
  if (!active()) return;
  static thread_local void* scratch = nullptr;
  if (!scratch) XGBB_CUDA(cudaMalloc(&scratch, 8));
  sum_u64(scratch, 1, s);
  XGBB_CUDA(cudaStreamSynchronize(s));
}

}  // namespace xgbb
