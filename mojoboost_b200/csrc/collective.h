// Cross-device reductions for data-parallel training (one process per GPU).
//
// Replaces the reference's CPU data-parallel exchange (distributed.mojo:505-533:
// allreduce of each node's Float64 gradient/hessian sums and Int counts) with
// NCCL collectives over NVLink on integer histogram cells, following the
// device contract the reference recorded but never built
// (distributed_gpu.mojo:34-78: one global fixed-point scale, then an exact
// integer sum in any order).  NCCL is loaded at run time (libnccl.so.2, the
// copy PyTorch ships or the system one), so a single-GPU fit never needs it.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace mtb {

class Collective {
 public:
  // Loads NCCL; false (with the reason) when it cannot be loaded.
  static bool load(std::string* why);
  // Writes a fresh 128-byte NCCL unique id (call on one rank, broadcast it).
  static void unique_id(uint8_t out[128]);

  // Joins the communicator.  `timeout_s` bounds every host wait of this
  // communicator: joining (a rank that never joins), the completion of work
  // queued behind a collective (a rank that stopped participating) and NCCL's
  // own asynchronous set-up.  Past it the communicator is aborted (its queued
  // kernels end) and the wait throws, so no rank blocks forever on another.
  Collective(const uint8_t id[128], int rank, int world, double timeout_s);
  ~Collective();
  Collective(const Collective&) = delete;
  Collective& operator=(const Collective&) = delete;

  int rank() const { return rank_; }
  int world() const { return world_; }

  void allreduce_sum_i32(int* buf, size_t n, cudaStream_t st);
  void allreduce_sum_i64(long long* buf, size_t n, cudaStream_t st);
  void allreduce_max_u64(unsigned long long* buf, size_t n, cudaStream_t st);
  void allreduce_sum_f64(double* buf, size_t n, cudaStream_t st);
  void allgather_f64(const double* send, double* recv, size_t n_per_rank, cudaStream_t st);
  void allgather_bytes(const void* send, void* recv, size_t bytes_per_rank, cudaStream_t st);
  // In place, for each of n_slots slots of slot_len int32 (slots back to
  // back from `base`): the sum over ranks of this rank's chunk
  // [rank * chunk, (rank + 1) * chunk) of every slot, slot_len = world * chunk.
  // One NCCL group.
  void reduce_scatter_slots_i32(int* base, size_t n_slots, size_t slot_len, size_t chunk, cudaStream_t st);
  // The same for int64 elements (slot_len and chunk in int64 elements).
  void reduce_scatter_slots_i64(long long* base, size_t n_slots, size_t slot_len, size_t chunk, cudaStream_t st);
  // Throws if the communicator reported an asynchronous error (and aborts it).
  void check();
  // Host waits bounded by the timeout (see the constructor): until the
  // stream's queued work (or the event) completes.
  void sync(cudaStream_t st);
  void wait(cudaEvent_t ev);
  // Aborts the communicator (idempotent): NCCL kernels still waiting for a
  // peer end, and the communicator is unusable afterwards.
  void abort();
  bool aborted() const { return comm_ == nullptr; }
  double timeout_s() const { return timeout_s_; }

 private:
  // Polls until NCCL's asynchronous state leaves "in progress" (non-blocking
  // communicator), within the timeout.
  void settle(const char* what);
  void reduce_scatter_slots(void* base, size_t elem, int dtype, size_t n_slots, size_t slot_len, size_t chunk,
                            cudaStream_t st);
  void* comm_ = nullptr;
  double timeout_s_ = 300.0;
  cudaEvent_t ev_ = nullptr;
  int rank_ = 0;
  int world_ = 1;
};

}  // namespace mtb
