// Row-sharded training across GPUs: one process per GPU, one NCCL
// communicator per process. Every rank holds a contiguous shard of the rows;
// integer histograms, child row counts and the exact gradient masses are
// summed over ranks, so each rank takes the same decisions as one GPU would.
#pragma once
#include <cuda_runtime.h>
#include <nccl.h>

#include <cstddef>
#include <cstdint>
#include <functional>
#include <map>
#include <string>

namespace xgbb {

class Comm {
 public:
  static Comm& get();
  // `id_hex` is an NCCL unique id produced by nccl_unique_id_hex() on one rank
  // and shared with the others out of band.
  void init(int rank, int world, const std::string& id_hex, int device);
  void finalize();
  bool active() const { return world_ > 1; }
  int rank() const { return rank_; }
  int world() const { return world_; }
  void sum_u64(void* buf, size_t count, cudaStream_t s);
  void sum_u32(void* buf, size_t count, cudaStream_t s);
  void max_u32(void* buf, size_t count, cudaStream_t s);
  void sum_f64(void* buf, size_t count, cudaStream_t s);
  void broadcast(void* buf, size_t bytes, int root, cudaStream_t s);
  // In-place reduce-scatter of uint64 sums: `buf` holds world() chunks of
  // `count` words; this rank's chunk (at rank() * count) receives the sums.
  void reduce_scatter_u64(void* buf, size_t count, cudaStream_t s);
  // `bytes` from every rank, concatenated in rank order into `recv`.
  void all_gather(const void* send, void* recv, size_t bytes, cudaStream_t s);
  void barrier(cudaStream_t s);
  // Work that must be released before the communicator is destroyed: CUDA
  // graphs holding NCCL calls would otherwise keep ncclCommDestroy waiting.
  void add_release_hook(const void* owner, std::function<void()> fn);
  void remove_release_hook(const void* owner);
  // Host waits for stream work that contains collectives (the event recorded
  // after it) and for the whole device, bounded by the timeout: on an NCCL
  // error or the timeout the communicator is aborted and an Error raised.
  void wait(cudaEvent_t ev, const char* what);
  void wait_device(const char* what);
  void set_timeout(double seconds);
  bool failed() const { return failed_; }
  // Aborts the communicator on this rank (XGCommunicatorSignalError): the
  // other ranks' pending and next collectives fail within their time limit.
  void signal_error() { abort_detached(); }

 private:
  void settle(const char* what);
  void call(ncclResult_t r, const char* what);
  void abort_detached();
  [[noreturn]] void fail(const std::string& what);
  int rank_ = 0, world_ = 1;
  void* comm_ = nullptr;
  bool failed_ = false;
  double timeout_s_ = 600.0;
  std::map<const void*, std::function<void()>> hooks_;
};

std::string nccl_unique_id_hex();

}  // namespace xgbb
