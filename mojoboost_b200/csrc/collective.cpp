// NCCL loaded with dlopen; see collective.h.
#include "collective.h"

#include <dlfcn.h>
#include <stdlib.h>
#include <string.h>

#include <chrono>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>

namespace mtb {

namespace {

// The few NCCL types and entry points used here (nccl.h, NCCL 2.x ABI).
typedef int nccl_result_t;
typedef struct {
  char internal[128];
} nccl_unique_id_t;
typedef void* nccl_comm_t;
enum { kNcclSuccess = 0, kNcclInProgress = 7, kNcclInt8 = 0, kNcclInt32 = 2, kNcclInt64 = 4, kNcclUint64 = 5, kNcclFloat64 = 8 };
// The leading fields of ncclConfig_t as NCCL 2.14 laid them out; newer
// libraries read `size` and treat the fields past it as unset.
struct nccl_config_t {
  size_t size;
  unsigned int magic;
  unsigned int version;
  int blocking;
  int cga_cluster_size;
  int min_ctas;
  int max_ctas;
  const char* net_name;
};
constexpr int kNcclConfigUndefInt = -2147483647 - 1;
enum { kNcclSum = 0, kNcclMax = 2 };

struct Api {
  nccl_result_t (*get_unique_id)(nccl_unique_id_t*);
  nccl_result_t (*comm_init_rank)(nccl_comm_t*, int, nccl_unique_id_t, int);
  nccl_result_t (*comm_init_rank_config)(nccl_comm_t*, int, nccl_unique_id_t, int, nccl_config_t*);
  nccl_result_t (*comm_destroy)(nccl_comm_t);
  nccl_result_t (*comm_abort)(nccl_comm_t);
  nccl_result_t (*all_reduce)(const void*, void*, size_t, int, int, nccl_comm_t, cudaStream_t);
  nccl_result_t (*all_gather)(const void*, void*, size_t, int, nccl_comm_t, cudaStream_t);
  nccl_result_t (*reduce_scatter)(const void*, void*, size_t, int, int, nccl_comm_t, cudaStream_t);
  nccl_result_t (*group_start)();
  nccl_result_t (*group_end)();
  nccl_result_t (*get_async_error)(nccl_comm_t, nccl_result_t*);
  const char* (*error_string)(nccl_result_t);
};

Api g_api;
bool g_loaded = false;
std::string g_why;
std::once_flag g_once;

void do_load() {
  const char* env = getenv("MOJOTREES_NCCL_LIB");
  const char* names[] = {env, "libnccl.so.2", "libnccl.so"};
  void* h = nullptr;
  for (const char* n : names) {
    if (!n || !*n) continue;
    h = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
    if (h) break;
  }
  if (!h) {
    g_why = "libnccl.so.2 could not be loaded (set MOJOTREES_NCCL_LIB or import torch first)";
    return;
  }
  auto sym = [&](const char* s) {
    void* p = dlsym(h, s);
    if (!p && g_why.empty()) g_why = std::string("NCCL symbol missing: ") + s;
    return p;
  };
  g_api.get_unique_id = (decltype(g_api.get_unique_id))sym("ncclGetUniqueId");
  g_api.comm_init_rank = (decltype(g_api.comm_init_rank))sym("ncclCommInitRank");
  // optional: without it joining is not bounded by the timeout
  g_api.comm_init_rank_config = (decltype(g_api.comm_init_rank_config))dlsym(h, "ncclCommInitRankConfig");
  g_api.comm_destroy = (decltype(g_api.comm_destroy))sym("ncclCommDestroy");
  g_api.comm_abort = (decltype(g_api.comm_abort))sym("ncclCommAbort");
  g_api.all_reduce = (decltype(g_api.all_reduce))sym("ncclAllReduce");
  g_api.all_gather = (decltype(g_api.all_gather))sym("ncclAllGather");
  g_api.reduce_scatter = (decltype(g_api.reduce_scatter))sym("ncclReduceScatter");
  g_api.group_start = (decltype(g_api.group_start))sym("ncclGroupStart");
  g_api.group_end = (decltype(g_api.group_end))sym("ncclGroupEnd");
  g_api.get_async_error = (decltype(g_api.get_async_error))sym("ncclCommGetAsyncError");
  g_api.error_string = (decltype(g_api.error_string))sym("ncclGetErrorString");
  g_loaded = g_why.empty();
}

void ck(nccl_result_t r, const char* what) {
  if (r != kNcclSuccess)
    throw std::runtime_error(std::string("NCCL ") + what + " failed: " +
                             (g_api.error_string ? g_api.error_string(r) : "unknown error"));
}

}  // namespace

bool Collective::load(std::string* why) {
  std::call_once(g_once, do_load);
  if (!g_loaded && why) *why = g_why;
  return g_loaded;
}

void Collective::unique_id(uint8_t out[128]) {
  std::string why;
  if (!load(&why)) throw std::runtime_error(why);
  nccl_unique_id_t id;
  ck(g_api.get_unique_id(&id), "ncclGetUniqueId");
  memcpy(out, id.internal, 128);
}

Collective::Collective(const uint8_t id[128], int rank, int world, double timeout_s)
    : rank_(rank), world_(world), timeout_s_(timeout_s > 0 ? timeout_s : 300.0) {
  std::string why;
  if (!load(&why)) throw std::runtime_error(why);
  if (world < 1 || rank < 0 || rank >= world) throw std::runtime_error("invalid rank / world size");
  nccl_unique_id_t uid;
  memcpy(uid.internal, id, 128);
  nccl_comm_t c = nullptr;
  if (g_api.comm_init_rank_config) {
    // non-blocking: the join returns at once and is polled, so a rank that
    // never joins costs the timeout, not the process
    nccl_config_t cfg = {sizeof(nccl_config_t), 0xcafebeefu, 21400u, 0, kNcclConfigUndefInt,
                         kNcclConfigUndefInt, kNcclConfigUndefInt, nullptr};
    const nccl_result_t r = g_api.comm_init_rank_config(&c, world, uid, rank, &cfg);
    if (r != kNcclSuccess && r != kNcclInProgress) {
      if (c) g_api.comm_abort(c);
      ck(r, "ncclCommInitRankConfig");
    }
    comm_ = c;
    settle("joining the communicator");
  } else {
    ck(g_api.comm_init_rank(&c, world, uid, rank), "ncclCommInitRank");
    comm_ = c;
  }
  if (cudaEventCreateWithFlags(&ev_, cudaEventDisableTiming) != cudaSuccess) {
    abort();
    throw std::runtime_error("cudaEventCreate failed");
  }
}

Collective::~Collective() {
  if (ev_) cudaEventDestroy(ev_);
  if (comm_) g_api.comm_destroy((nccl_comm_t)comm_);
}

void Collective::abort() {
  if (!comm_) return;
  g_api.comm_abort((nccl_comm_t)comm_);
  comm_ = nullptr;
}

void Collective::settle(const char* what) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    if (!comm_) throw std::runtime_error(std::string("NCCL communicator was aborted before ") + what);
    nccl_result_t st = kNcclSuccess;
    const nccl_result_t r = g_api.get_async_error((nccl_comm_t)comm_, &st);
    if (r != kNcclSuccess || (st != kNcclSuccess && st != kNcclInProgress)) {
      abort();
      ck(r != kNcclSuccess ? r : st, what);
    }
    if (st == kNcclSuccess) return;
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s_) {
      abort();
      throw std::runtime_error(std::string("NCCL timed out after ") + std::to_string(timeout_s_) + " s " + what +
                               " (a rank did not join or stopped participating); the communicator was aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

void Collective::wait(cudaEvent_t ev) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t q = cudaEventQuery(ev);
    if (q == cudaSuccess) return;
    if (q != cudaErrorNotReady)
      throw std::runtime_error(std::string("CUDA error while waiting: ") + cudaGetErrorString(q));
    if (comm_) {
      nccl_result_t st = kNcclSuccess;
      g_api.get_async_error((nccl_comm_t)comm_, &st);
      if (st != kNcclSuccess && st != kNcclInProgress) {
        abort();
        ck(st, "asynchronous operation");
      }
    }
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s_) {
      // the queued NCCL kernels wait for a peer that is gone: aborting ends
      // them, and the work queued behind them then drains
      abort();
      cudaEventSynchronize(ev);
      throw std::runtime_error("data-parallel fit timed out after " + std::to_string(timeout_s_) +
                               " s waiting for the other ranks (a rank stopped participating); the NCCL "
                               "communicator was aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

void Collective::sync(cudaStream_t st) {
  if (cudaEventRecord(ev_, st) != cudaSuccess) throw std::runtime_error("cudaEventRecord failed");
  wait(ev_);
}

#define MTB_NCCL_CALL(call, what)                                         \
  do {                                                                    \
    if (!comm_) throw std::runtime_error("NCCL communicator was aborted"); \
    const nccl_result_t r_ = (call);                                      \
    if (r_ == kNcclInProgress)                                            \
      settle(what);                                                       \
    else                                                                  \
      ck(r_, what);                                                       \
  } while (0)

void Collective::allreduce_sum_i32(int* buf, size_t n, cudaStream_t st) {
  MTB_NCCL_CALL(g_api.all_reduce(buf, buf, n, kNcclInt32, kNcclSum, (nccl_comm_t)comm_, st), "ncclAllReduce");
}

void Collective::allreduce_sum_i64(long long* buf, size_t n, cudaStream_t st) {
  MTB_NCCL_CALL(g_api.all_reduce(buf, buf, n, kNcclInt64, kNcclSum, (nccl_comm_t)comm_, st), "ncclAllReduce");
}

void Collective::allreduce_max_u64(unsigned long long* buf, size_t n, cudaStream_t st) {
  MTB_NCCL_CALL(g_api.all_reduce(buf, buf, n, kNcclUint64, kNcclMax, (nccl_comm_t)comm_, st), "ncclAllReduce");
}

void Collective::allreduce_sum_f64(double* buf, size_t n, cudaStream_t st) {
  MTB_NCCL_CALL(g_api.all_reduce(buf, buf, n, kNcclFloat64, kNcclSum, (nccl_comm_t)comm_, st), "ncclAllReduce");
}

void Collective::allgather_f64(const double* send, double* recv, size_t n_per_rank, cudaStream_t st) {
  MTB_NCCL_CALL(g_api.all_gather(send, recv, n_per_rank, kNcclFloat64, (nccl_comm_t)comm_, st), "ncclAllGather");
}

void Collective::check() {
  if (!comm_) throw std::runtime_error("NCCL communicator was aborted");
  nccl_result_t e = kNcclSuccess;
  ck(g_api.get_async_error((nccl_comm_t)comm_, &e), "ncclCommGetAsyncError");
  if (e != kNcclSuccess) {
    g_api.comm_abort((nccl_comm_t)comm_);
    comm_ = nullptr;
    ck(e, "asynchronous operation");
  }
}

void Collective::allgather_bytes(const void* send, void* recv, size_t bytes_per_rank, cudaStream_t st) {
  MTB_NCCL_CALL(g_api.all_gather(send, recv, bytes_per_rank, kNcclInt8, (nccl_comm_t)comm_, st), "ncclAllGather");
}

void Collective::reduce_scatter_slots_i32(int* base, size_t n_slots, size_t slot_len, size_t chunk, cudaStream_t st) {
  reduce_scatter_slots(base, sizeof(int), kNcclInt32, n_slots, slot_len, chunk, st);
}

void Collective::reduce_scatter_slots_i64(long long* base, size_t n_slots, size_t slot_len, size_t chunk,
                                          cudaStream_t st) {
  reduce_scatter_slots(base, sizeof(long long), kNcclInt64, n_slots, slot_len, chunk, st);
}

void Collective::reduce_scatter_slots(void* base, size_t elem, int dtype, size_t n_slots, size_t slot_len,
                                      size_t chunk, cudaStream_t st) {
  if (chunk * (size_t)world_ != slot_len) throw std::runtime_error("reduce-scatter: slot length is not world x chunk");
  if (!comm_) throw std::runtime_error("NCCL communicator was aborted");
  ck(g_api.group_start(), "ncclGroupStart");
  nccl_result_t r = kNcclSuccess;
  for (size_t i = 0; i < n_slots && (r == kNcclSuccess || r == kNcclInProgress); ++i) {
    char* slot = static_cast<char*>(base) + i * slot_len * elem;
    // in place: rank r's result lands on its own chunk of the slot
    r = g_api.reduce_scatter(slot, slot + (size_t)rank_ * chunk * elem, chunk, dtype, kNcclSum,
                             (nccl_comm_t)comm_, st);
  }
  const nccl_result_t e = g_api.group_end();
  if (r != kNcclInProgress) ck(r, "ncclReduceScatter");
  if (e == kNcclInProgress || r == kNcclInProgress)
    settle("ncclGroupEnd");
  else
    ck(e, "ncclGroupEnd");
}

}  // namespace mtb
