// Host orchestration of the B200 GBDT training path.
//
// Per fit: bins uploaded once (feature-major) and transposed on the device to
// the row-major copy the histogram kernel streams.  Per round: derivatives,
// the scale reduction and the quantizer run as three short kernels; then one
// tree is grown as a fixed launch sequence (see gbdt_device.cuh) with no host
// synchronisation until the round ends, where the tree's node table is read
// back and the early-stop rule of boosting.mojo:2898-2907 is applied.
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>

#include <algorithm>
#include <chrono>
#include <map>
#include <mutex>
#include <thread>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "gbdt_device.cuh"
#include "gbdt_kernels.cuh"
#include "hist_launch.cuh"
#include "sparse_hist.cuh"
#include "collective.h"
#include "device_binning.h"
#include "trainer.h"

namespace mtb {

#define MTB_CUDA(call)                                                                       \
  do {                                                                                       \
    cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess)                                                                   \
      throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(e_) + " at " \
                               + #call);                                                     \
  } while (0)

int cuda_device_count() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

namespace {

// Initial raw scores: every row's K scores set to the per-class base.
__global__ void k_fill_raw(double* __restrict__ raw, const double* __restrict__ base, long long n, int K) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    raw[i] = base[i % K];
}

// Device memory of the fits comes from a per-process cache: a fit's buffers
// go back to it when the fit ends, and the next fit on the same device takes
// blocks of the sizes it needs from it instead of calling cudaMalloc (whose
// cost for the ~4 GB a configs[1] fit allocates varies between tens and
// hundreds of milliseconds).  Sizes are rounded up to 2 MB, a cached block
// is reused for a request at most 1/8 smaller, the cache holds at most a
// quarter of the device's memory, and a failed cudaMalloc empties it and
// retries (MOJOTREES_NO_MEMORY_CACHE=1: no cache).  Returning a block
// synchronises the device, as cudaFree does.
class DeviceCache {
 public:
  static DeviceCache& get() {
    static DeviceCache c;
    return c;
  }
  void* take(size_t bytes) {
    int dev = 0;
    MTB_CUDA(cudaGetDevice(&dev));
    {
      std::lock_guard<std::mutex> lock(mu_);
      auto& m = free_[dev];
      for (auto it = m.lower_bound(bytes); it != m.end() && it->first <= bytes + bytes / 8;) {
        void* p = it->second;
        const size_t sz = it->first;
        it = m.erase(it);
        held_[dev] -= sz;
        cudaPointerAttributes a;
        if (cudaPointerGetAttributes(&a, p) == cudaSuccess && a.type == cudaMemoryTypeDevice && a.device == dev)
          return p;
        cudaGetLastError();  // a block from a context that no longer exists: dropped
      }
    }
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaErrorMemoryAllocation) {
      cudaGetLastError();
      release(dev);
      e = cudaMalloc(&p, bytes);
    }
    if (e != cudaSuccess) throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(e) + " (cudaMalloc)");
    return p;
  }
  void give(void* p, size_t bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
      cudaGetLastError();
      cudaFree(p);
      return;
    }
    std::lock_guard<std::mutex> lock(mu_);
    if (!limit_.count(dev)) {
      size_t fr = 0, total = 0;
      cudaMemGetInfo(&fr, &total);
      limit_[dev] = getenv("MOJOTREES_NO_MEMORY_CACHE") ? 0 : total / 4;
    }
    if (held_[dev] + bytes > limit_[dev]) {
      cudaFree(p);
      return;
    }
    free_[dev].emplace(bytes, p);
    held_[dev] += bytes;
  }
  void release(int dev) {
    std::lock_guard<std::mutex> lock(mu_);
    for (auto& kv : free_[dev]) cudaFree(kv.second);
    free_[dev].clear();
    held_[dev] = 0;
  }

 private:
  std::mutex mu_;
  std::map<int, std::multimap<size_t, void*>> free_;
  std::map<int, size_t> held_, limit_;
};

template <typename T>
struct DevBuf {
  T* p = nullptr;
  size_t n = 0;
  size_t bytes = 0;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  void alloc(size_t count) {
    free();
    n = count;
    if (count) {
      bytes = (sizeof(T) * count + (2u << 20) - 1) & ~(size_t)((2u << 20) - 1);
      p = static_cast<T*>(DeviceCache::get().take(bytes));
    }
  }
  void free() {
    if (p) DeviceCache::get().give(p, bytes);
    p = nullptr;
    n = 0;
    bytes = 0;
  }
  ~DevBuf() { free(); }
};

// CUDA events around launches (profile_phases): a pool of events reused
// across trees, so timing adds two event records per launch and nothing else.
struct EventTimer {
  bool on;
  cudaStream_t s;
  std::vector<cudaEvent_t> pool;
  std::vector<double*> accs;
  size_t used = 0;
  EventTimer(bool enabled, cudaStream_t st) : on(enabled), s(st) {}
  ~EventTimer() {
    for (auto e : pool) cudaEventDestroy(e);
  }
  void begin(double* target) {
    if (!on) return;
    while (pool.size() < used + 2) {
      cudaEvent_t e;
      cudaEventCreate(&e);
      pool.push_back(e);
    }
    cudaEventRecord(pool[used], s);
    accs.push_back(target);
  }
  void end() {
    if (!on) return;
    cudaEventRecord(pool[used + 1], s);
    used += 2;
  }
  void collect() {
    for (size_t i = 0; i < accs.size(); ++i) {
      float ms = 0.f;
      cudaEventSynchronize(pool[2 * i + 1]);
      cudaEventElapsedTime(&ms, pool[2 * i], pool[2 * i + 1]);
      *accs[i] += ms;
    }
    accs.clear();
    used = 0;
  }
};

}  // namespace

void train_gpu(const BinnedInput& in, const TrainConfig& cfg, Model& model) {
  const long long N = in.n_rows;
  const int F = in.n_features;
  const int B = in.n_bins;
  if (N < 1 || F < 1) throw std::runtime_error("empty training matrix");
  if (N >= (1ll << 31)) throw Unsupported("more than 2^31-1 rows on one device");
  if (B < 2 || B > 256) throw std::runtime_error("n_bins must be in [2, 256]");
  if (cfg.num_leaves < 2 || cfg.num_leaves > kMaxLeaves)
    throw Unsupported("num_leaves must be in [2, " + std::to_string(kMaxLeaves) + "] on the device path");
  if (cfg.feature_fraction <= 0.0 || cfg.feature_fraction > 1.0)
    throw std::runtime_error("feature_fraction must be in (0, 1]");
  const int K = cfg.objective == OBJECTIVE_MULTICLASS ? cfg.num_class : 1;
  if (cfg.objective == OBJECTIVE_MULTICLASS && (K < 2 || K > 64))
    throw Unsupported("num_class must be in [2, 64] on the device path");
  const int mode = cfg.use_quantized_grad ? MODE_QUANT : MODE_FIXED;
  // fixed point with the 2^52 bound and Int64 cells (gpu_histogram_precision=int64)
  const bool wide = mode == MODE_FIXED && cfg.hist_int64;
  if (mode == MODE_QUANT && (cfg.num_grad_quant_bins < 2 || cfg.num_grad_quant_bins > 254 ||
                             cfg.num_grad_quant_bins % 2 != 0))
    throw Unsupported("num_grad_quant_bins must be even and in [2, 254] on the device path");
  const bool const_h = cfg.objective == OBJECTIVE_L2;
  for (int f = 0; f < F; ++f)
    if (in.n_cats[f] >= B) throw std::runtime_error("categorical feature has more categories than bins");

  int dev = cfg.gpu_device_id;
  if (cuda_device_count() < 1) throw Unsupported("no CUDA device is available");
  if (dev >= 0) MTB_CUDA(cudaSetDevice(dev));
  MTB_CUDA(cudaGetDevice(&dev));
  cudaDeviceProp prop;
  MTB_CUDA(cudaGetDeviceProperties(&prop, dev));
  const int n_sm = prop.multiProcessorCount;

  cudaStream_t st;
  MTB_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  struct StreamGuard {
    cudaStream_t s;
    ~StreamGuard() { cudaStreamDestroy(s); }
  } sg{st};

  TrainStats stats;
  auto t0 = std::chrono::steady_clock::now();
  // MOJOTREES_TRACE_UPLOAD=1 prints the set-up phases to stderr
  const bool trace_up = getenv("MOJOTREES_TRACE_UPLOAD") != nullptr;
  auto mark = [&](const char* what) {
    if (!trace_up) return;
    cudaStreamSynchronize(st);
    fprintf(stderr, "setup: %-28s %8.1f ms\n", what,
            std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() * 1e3);
  };
  const int Fp = (F + 15) / 16 * 16;
  DevBuf<uint8_t> d_bins_cm, d_bins_rm;
  d_bins_cm.alloc((size_t)F * N);
  d_bins_rm.alloc((size_t)Fp * N);
  mark("bin buffers allocated");
  if (in.dense_fm) {
    if (!in.mapper) throw std::runtime_error("dense input without a bin mapper");
    transform_on_device(*in.mapper, in.dense_fm, N, d_bins_cm.p, st);
  } else {
    upload_host(in.bins_fm, (int64_t)F * N, d_bins_cm.p, st);
  }
  mark("bins on the device");
  {
    dim3 grid((unsigned)((N + 255) / 256), Fp / 16);
    k_transpose_bins<<<grid, 256, 0, st>>>(d_bins_cm.p, d_bins_rm.p, N, F, Fp);
    stats.kernel_launches++;
  }
  DevBuf<double> d_y, d_raw, d_prob;
  mark("bins uploaded, transposed");
  d_y.alloc(N);
  upload_host(in.labels, (int64_t)sizeof(double) * N, d_y.p, st);
  d_raw.alloc((size_t)N * K);
  if (K > 1) d_prob.alloc((size_t)N * K);

  // Initial scores (boosting.mojo:521-577; multiclass :4207-4225).  Across
  // devices the label sum is each shard's sequential sum combined in rank
  // order (exact for binary and class labels, whose sums are integers).
  Collective* coll = in.coll;
  const int world = coll ? coll->world() : 1;
  // Host waits: with other ranks, bounded by the communicator's timeout
  // (past it the communicator is aborted and the wait throws).
  const char* stall_env = getenv("MOJOTREES_DP_TEST_STALL_RANK");
  const int test_stall_rank = stall_env ? atoi(stall_env) : -1;
  const int test_stall_after =
      getenv("MOJOTREES_DP_TEST_STALL_AFTER_ROUNDS") ? atoi(getenv("MOJOTREES_DP_TEST_STALL_AFTER_ROUNDS")) : 1;
  const double test_stall_s = getenv("MOJOTREES_DP_TEST_STALL_S") ? atof(getenv("MOJOTREES_DP_TEST_STALL_S")) : 0.0;
  auto host_sync = [&]() {
    if (coll)
      coll->sync(st);
    else
      MTB_CUDA(cudaStreamSynchronize(st));
  };
  const long long N_global = coll ? in.n_rows_global : N;
  mark("labels, raw allocated");
  DevBuf<double> d_red;
  d_red.alloc(2 * (size_t)std::max(world, K) + 8);
  // every rank learns whether any rank's input is invalid before any throws
  auto agree = [&](const std::string& local_error) {
    if (!coll) {
      if (!local_error.empty()) throw std::runtime_error(local_error);
      return;
    }
    unsigned long long flag = local_error.empty() ? 0ull : 1ull;
    MTB_CUDA(cudaMemcpyAsync(d_red.p, &flag, 8, cudaMemcpyHostToDevice, st));
    coll->allreduce_max_u64(reinterpret_cast<unsigned long long*>(d_red.p), 1, st);
    MTB_CUDA(cudaMemcpyAsync(&flag, d_red.p, 8, cudaMemcpyDeviceToHost, st));
    host_sync();
    if (flag) throw std::runtime_error(local_error.empty() ? "invalid input on another rank" : local_error);
  };
  // FIXED mode sums |g| over 1024-row blocks of global rows, so its shards
  // must align to them; QUANT mode only needs global row ids (max is exact)
  agree(coll && mode == MODE_FIXED && coll->rank() < world - 1 && N % 1024 != 0
            ? "fixed-point data-parallel shards other than the last must hold a multiple of 1024 rows"
            : "");
  std::vector<double> base(K);
  if (K == 1) {
    double mean = 0.0;
    std::string err;
    if (cfg.objective == OBJECTIVE_BINARY) {
      // 0/1 labels: the sequential sum is the count of ones, exact in any
      // order, so it is counted in parallel together with the label check
      long long ones = 0, bad = 0;
#pragma omp parallel for reduction(+ : ones, bad) schedule(static)
      for (long long r = 0; r < N; ++r) {
        const double v = in.labels[r];
        ones += v == 1.0 ? 1 : 0;
        bad += (v == 0.0 || v == 1.0) ? 0 : 1;
      }
      if (bad) err = "binary labels must be 0 or 1";
      mean = (double)ones;
    } else {
      for (long long r = 0; r < N; ++r) mean += 1.0 * in.labels[r];
    }
    agree(err);
    if (coll) {
      MTB_CUDA(cudaMemcpyAsync(d_red.p + world, &mean, 8, cudaMemcpyHostToDevice, st));
      coll->allgather_f64(d_red.p + world, d_red.p, 1, st);
      std::vector<double> parts(world);
      MTB_CUDA(cudaMemcpyAsync(parts.data(), d_red.p, 8 * world, cudaMemcpyDeviceToHost, st));
      host_sync();
      mean = parts[0];
      for (int q = 1; q < world; ++q) mean += parts[q];
    }
    mean /= (double)N_global;
    if (cfg.objective == OBJECTIVE_BINARY) {
      double p = mean < 1e-15 ? 1e-15 : (mean > 1.0 - 1e-15 ? 1.0 - 1e-15 : mean);
      base[0] = std::log(p / (1.0 - p));
    } else {
      base[0] = mean;
    }
  } else {
    std::vector<double> cw(K, 0.0);
    std::string err;
    for (long long r = 0; r < N; ++r) {
      double y = in.labels[r];
      int k = (int)y;
      if (!(y >= 0.0) || (double)k != y || k >= K) {
        err = "class labels must be in 0..num_class-1";
        break;
      }
      cw[k] += 1.0;
    }
    agree(err);
    if (coll) {
      MTB_CUDA(cudaMemcpyAsync(d_red.p, cw.data(), 8 * K, cudaMemcpyHostToDevice, st));
      coll->allreduce_sum_f64(d_red.p, K, st);
      MTB_CUDA(cudaMemcpyAsync(cw.data(), d_red.p, 8 * K, cudaMemcpyDeviceToHost, st));
      host_sync();
    }
    double tw = (double)N_global;
    for (int k = 0; k < K; ++k) {
      double q = cw[k] / tw;
      q = q < 1e-15 ? 1e-15 : (q > 1.0 - 1e-15 ? 1.0 - 1e-15 : q);
      base[k] = std::log(q);
    }
  }
  {
    // raw[r * K + k] = base[k], filled on the device
    MTB_CUDA(cudaMemcpyAsync(d_red.p, base.data(), sizeof(double) * K, cudaMemcpyHostToDevice, st));
    const long long n_raw = N * (long long)K;
    const unsigned blocks = (unsigned)std::min<long long>((n_raw + 255) / 256, 148ll * 16);
    if (n_raw > 0) {
      k_fill_raw<<<blocks, 256, 0, st>>>(d_raw.p, d_red.p, n_raw, K);
      MTB_CUDA(cudaGetLastError());
      stats.kernel_launches++;
    }
    host_sync();
  }

  mark("initial scores");
  DevBuf<int> d_missing, d_ncats, d_feats;
  d_missing.alloc(F);
  d_ncats.alloc(F);
  d_feats.alloc(F);
  MTB_CUDA(cudaMemcpyAsync(d_missing.p, in.missing_bin, sizeof(int) * F, cudaMemcpyHostToDevice, st));
  MTB_CUDA(cudaMemcpyAsync(d_ncats.p, in.n_cats, sizeof(int) * F, cudaMemcpyHostToDevice, st));

  const size_t pair_bytes = mode == MODE_QUANT ? 2 : wide ? 16 : 8;
  DevBuf<int> d_rows0, d_rows1;
  DevBuf<unsigned char> d_pairs0, d_pairs1;
  d_rows0.alloc(N);
  d_rows1.alloc(N);
  d_pairs0.alloc((size_t)N * pair_bytes);
  d_pairs1.alloc((size_t)N * pair_bytes);
  DevBuf<float> d_g, d_h;
  d_g.alloc(N);
  d_h.alloc(N);
  // FIXED-mode |g|, |h| partials: one per 1024 global rows.  Across devices
  // every rank gathers all ranks' partials (P per rank, the last rank's tail
  // zero-padded) so all reduce the same global pairwise tree.
  long long n_part = (N + 1023) / 1024;
  long long P_rank = n_part;
  if (coll) {
    unsigned long long mx = (unsigned long long)n_part;
    MTB_CUDA(cudaMemcpyAsync(d_red.p, &mx, 8, cudaMemcpyHostToDevice, st));
    coll->allreduce_max_u64(reinterpret_cast<unsigned long long*>(d_red.p), 1, st);
    MTB_CUDA(cudaMemcpyAsync(&mx, d_red.p, 8, cudaMemcpyDeviceToHost, st));
    host_sync();
    P_rank = (long long)mx;
    n_part = P_rank * world;
    // The gathered partials are block r * P_rank + j of rank r, so the global
    // tree equals the single-device one only when every shard but the last
    // holds exactly P_rank blocks and starts at global row r * P_rank * 1024
    // (the last shard's missing blocks are the zero padding at the end).
    std::string err;
    if (mode == MODE_FIXED && coll->rank() < world - 1 && (N != P_rank * 1024))
      err = "fixed-point data-parallel shards other than the last must all hold the same number of rows";
    else if (mode == MODE_FIXED && in.row_offset != (long long)coll->rank() * P_rank * 1024)
      err = "row_offset of a fixed-point data-parallel shard must be its rank times the common shard size";
    agree(err);
  }
  DevBuf<double> d_pg, d_ph, d_tg, d_th, d_pg_all, d_ph_all;
  d_pg.alloc(P_rank);
  d_ph.alloc(P_rank);
  if (coll) {
    d_pg_all.alloc(n_part);
    d_ph_all.alloc(n_part);
  }
  d_tg.alloc(n_part / 1000 + 16);
  d_th.alloc(n_part / 1000 + 16);
  DevBuf<RoundScales> d_sc;
  d_sc.alloc(1);
  DevBuf<TreeState> d_ts;
  d_ts.alloc(1);
  // Data-parallel histogram exchange.  Default: all-reduce of the batch's
  // work slots, every rank scanning every feature.  MOJOTREES_DP_EXCHANGE=
  // feature: each rank owns a block of Fb feature ids; the work slots are
  // reduce-scattered by those blocks, each rank scans its own active
  // features, and the per-child bests are all-gathered and merged.
  const char* dpx = getenv("MOJOTREES_DP_EXCHANGE");
  const bool dp_feature = coll && world > 1 && dpx && std::string(dpx) == "feature";
  const int Fb = dp_feature ? (F + world - 1) / world : F;  // feature ids a rank owns
  // cells of one histogram slot, in int32 words (an Int64 cell takes two)
  const long long cell_words = wide ? 2 : 1;
  const long long slot_cells = (long long)(dp_feature ? Fb * world : F) * 3 * B * cell_words;
  // Leaves expanded per iteration (speculative leaf batching); 1 grows one
  // split per iteration as the reference does.  MOJOTREES_BATCH overrides.
  int batch_cap = kMaxBatch;
  // MOJOTREES_SCAN=compact selects the split scan whose candidate evaluation
  // is one out-of-line routine (same arithmetic, smaller code)
  const char* scan_env = getenv("MOJOTREES_SCAN");
  const bool scan_compact = scan_env && std::string(scan_env) == "compact";
  if (const char* e = getenv("MOJOTREES_BATCH")) batch_cap = atoi(e);
  batch_cap = std::max(1, std::min(std::min(batch_cap, kMaxBatch), cfg.num_leaves - 1));
  // Histogram slots: the root, one per expansion (at most num_leaves - 1
  // committed splits, plus speculative ones the commit kernel keeps within
  // the remaining budget), then batch_cap work slots the builds land in.
  const int hist_slots = 2 * cfg.num_leaves + batch_cap;
  const int work_base = hist_slots;
  DevBuf<int> d_hist;
  d_hist.alloc((size_t)slot_cells * (hist_slots + batch_cap));
  DevBuf<FeatBest> d_fb;
  d_fb.alloc((size_t)2 * batch_cap * F);
  DevBuf<long long> d_begins;
  DevBuf<int> d_bufs;
  DevBuf<double> d_values;
  d_begins.alloc(kMaxPool);
  d_bufs.alloc(kMaxPool);
  // leaf-table entries the raw update stages in shared memory (12 B each in
  // the slot scatter, 8 B in the score pass;
  // larger tables are searched in global memory), and its grid: a few
  // resident blocks per SM, each staging the table once
  const int table_stage = std::min(4 * cfg.num_leaves + 2 * kMaxBatch + 2, 2400);
  const unsigned update_grid = (unsigned)std::max(1ll, std::min<long long>((N + 255) / 256, (long long)n_sm * 8));
  d_values.alloc(kMaxPool);
  static_assert(kMaxPool <= 65536, "leaf-table slots are 16-bit");
  DevBuf<unsigned short> d_slot;  // each row's leaf-table entry, rewritten every tree
  d_slot.alloc(N);
  host_sync();
  mark("work buffers");
  stats.upload_seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();

  // Histogram launch geometry: as many features per CTA as one SM's shared
  // memory holds, row chunks sized to fill every SM, CTAs of a feature group
  // in clusters of up to 8 that merge through DSMEM.
  HistLaunch hl = choose_hist_launch(mode, const_h, mode == MODE_QUANT ? cfg.num_grad_quant_bins : 0, B, Fp, n_sm, N,
                                     wide);
  // MOJOTREES_PDL=1 launches the iteration kernels as programmatic
  // dependents of one another (each may be scheduled while its predecessor
  // finishes).  Off by default: measured within 1% at configs[1] and 10%
  // slower at configs[2], whose waiting CTAs hold SMs the running kernel's
  // clusters need.
  const bool pdl = getenv("MOJOTREES_PDL") != nullptr;
  hl.pdl = pdl;

  // Sparse histograms (fixed-point modes): used when every feature's cells
  // fit one CTA and a row lists under 40% of its bins outside the features'
  // default bins.  MOJOTREES_HIST_SPARSE=0 never uses them, =1 whenever
  // the cells fit.
  int sparse_planes = 0, sparse_bp = 1;
  DevBuf<int> d_default_bin;
  DevBuf<long long> d_row_ptr;
  DevBuf<uint32_t> d_entries;
  {
    const char* sp_env = getenv("MOJOTREES_HIST_SPARSE");
    const int want = sp_env ? atoi(sp_env) : -1;
    while (sparse_bp < B) sparse_bp <<= 1;
    const int planes = const_h ? 2 : 3;
    if (want != 0 && mode == MODE_FIXED && !wide && B <= 256 &&
        sparse_hist_smem(planes, F, sparse_bp) <= 227 * 1024) {
      d_default_bin.alloc(F);
      k_sparse_default_bins<<<F, 256, 0, st>>>(d_bins_cm.p, N, d_default_bin.p);
      DevBuf<long long> d_counts, d_block_sums;
      d_counts.alloc(N);
      d_row_ptr.alloc(N + 1);
      const long long nb = (N + kScanChunk - 1) / kScanChunk;
      d_block_sums.alloc(nb);
      const unsigned rgrid = (unsigned)std::min<long long>((N + 255) / 256, (long long)n_sm * 16);
      k_sparse_rows<<<rgrid, 256, Fp, st>>>(d_bins_rm.p, N, F, Fp, d_default_bin.p, d_counts.p, nullptr, nullptr);
      k_prefix_blocks<<<(unsigned)nb, kScanChunk, 0, st>>>(d_counts.p, N, d_row_ptr.p, d_block_sums.p);
      k_prefix_sums<<<1, 1024, 0, st>>>(d_block_sums.p, nb);
      k_prefix_add<<<(unsigned)nb, kScanChunk, 0, st>>>(N, d_row_ptr.p, d_block_sums.p);
      stats.kernel_launches += 5;
      long long nnz = 0;
      MTB_CUDA(cudaMemcpyAsync(&nnz, d_row_ptr.p + N, sizeof(long long), cudaMemcpyDeviceToHost, st));
      MTB_CUDA(cudaStreamSynchronize(st));
      if (want == 1 || (double)nnz < 0.4 * (double)F * (double)N) {
        d_entries.alloc((size_t)std::max(1ll, nnz));
        k_sparse_rows<<<rgrid, 256, Fp, st>>>(d_bins_rm.p, N, F, Fp, d_default_bin.p, nullptr, d_row_ptr.p,
                                              d_entries.p);
        stats.kernel_launches++;
        sparse_planes = planes;
        stats.hist_sparse_entries = (double)nnz;
        MTB_CUDA(cudaFuncSetAttribute(planes == 2 ? k_hist_sparse<2> : k_hist_sparse<3>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)sparse_hist_smem(planes, F, sparse_bp)));
      } else {
        d_row_ptr.free();
        d_default_bin.free();
      }
    }
  }
  // partition geometry (MOJOTREES_PART_ITEMS / MOJOTREES_PART_BLOCKS_PER_SM
  // override the rows per thread of a tile and the resident blocks per SM)
  int part_bps = 4;
  if (const char* e = getenv("MOJOTREES_PART_BLOCKS_PER_SM")) part_bps = std::max(1, atoi(e));
  const int part_grid = n_sm * part_bps;
  const int part_threads = 256;
  int part_items = 4;  // rows per thread per partition tile
  if (const char* e = getenv("MOJOTREES_PART_ITEMS")) part_items = atoi(e);
  part_items = part_items <= 1 ? 1 : part_items == 2 ? 2 : part_items <= 4 ? 4 : 8;
  auto launch_partition = [&]() {
#define MTB_PART(IT)                                                                                      \
  if (mode == MODE_QUANT)                                                                                 \
    launch_chained(pdl, k_partition<uint16_t, IT>, part_grid, part_threads, 0, st, d_ts.p,                \
                   (const uint8_t*)d_bins_cm.p, N, d_rows0.p, d_rows1.p,                                  \
                   reinterpret_cast<uint16_t*>(d_pairs0.p), reinterpret_cast<uint16_t*>(d_pairs1.p),      \
                   d_hist.p, slot_cells, work_base);                                                      \
  else if (wide)                                                                                          \
    launch_chained(pdl, k_partition<longlong2, IT>, part_grid, part_threads, 0, st, d_ts.p,               \
                   (const uint8_t*)d_bins_cm.p, N, d_rows0.p, d_rows1.p,                                  \
                   reinterpret_cast<longlong2*>(d_pairs0.p), reinterpret_cast<longlong2*>(d_pairs1.p),    \
                   d_hist.p, slot_cells, work_base);                                                      \
  else                                                                                                    \
    launch_chained(pdl, k_partition<int2, IT>, part_grid, part_threads, 0, st, d_ts.p,                    \
                   (const uint8_t*)d_bins_cm.p, N, d_rows0.p, d_rows1.p,                                  \
                   reinterpret_cast<int2*>(d_pairs0.p), reinterpret_cast<int2*>(d_pairs1.p), d_hist.p,   \
                   slot_cells, work_base);
    if (part_items == 1) { MTB_PART(1) }
    else if (part_items == 2) { MTB_PART(2) }
    else if (part_items == 4) { MTB_PART(4) }
    else { MTB_PART(8) }
#undef MTB_PART
  };
  // MOJOTREES_TRACE=1 prints every tree iteration to stderr (with
  // CUDA_LAUNCH_BLOCKING=1 the last line names the iteration that stalled)
  const bool trace = getenv("MOJOTREES_TRACE") != nullptr;
  CommitParams cp;
  cp.num_leaves = cfg.num_leaves;
  cp.batch_cap = batch_cap;
  cp.hist_slots = hist_slots;
  cp.tile_rows = 256 * part_items;
  {
    // each speculative batch is picked from bottleneck keys in one
    // block-parallel pass; MOJOTREES_COMMIT_SELECT=replay replays the pick
    // loop serially instead (same batches up to ties, more pick steps)
    const char* sel = getenv("MOJOTREES_COMMIT_SELECT");
    cp.ranked_select = (sel && std::string(sel) == "replay") ? 0 : 1;
  }
  const size_t commit_smem = commit_smem_bytes(cfg.num_leaves);
  const int commit_cap = commit_info_cap(cfg.num_leaves);
  MTB_CUDA(cudaFuncSetAttribute(k_commit, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)commit_smem));

  // The host learns that a tree is done through mapped host memory written by
  // the commit kernel; it stays at most kLookahead iterations ahead of the
  // device, so at most that many no-op iterations run after the last one.
  constexpr int kRing = 64, kLookahead = 2;
  int* h_done = nullptr;
  int* d_done = nullptr;
  MTB_CUDA(cudaHostAlloc(&h_done, sizeof(int) * kRing, cudaHostAllocMapped));
  struct HostGuard {
    int* p;
    ~HostGuard() { cudaFreeHost(p); }
  } hg{h_done};
  MTB_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&d_done), h_done, 0));
  std::vector<cudaEvent_t> iter_ev(kRing, nullptr);
  struct IterEventGuard {
    std::vector<cudaEvent_t>& e;
    ~IterEventGuard() {
      for (auto x : e)
        if (x) cudaEventDestroy(x);
    }
  } ieg{iter_ev};
  for (auto& e : iter_ev) MTB_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));

  model.objective = cfg.objective;
  model.num_class = K;
  model.n_features = F;
  model.learning_rate = cfg.learning_rate;
  model.base_scores = base;
  model.trees.clear();

  const int M = 2 * cfg.num_leaves - 1;
  std::vector<HostNode> nodes_host((size_t)M);
  TreeHeader hdr;
  EventTimer timer(cfg.profile_phases, st);
  EventTimer hist_timer(cfg.profile_phases || cfg.profile_histogram, st);

  ScanParams sp;
  sp.B = B;
  sp.mode = mode;
  sp.const_hess = const_h ? 1 : 0;
  sp.min_data_in_leaf = cfg.min_data_in_leaf;
  sp.lambda_l2 = cfg.lambda_l2;
  sp.lambda_l1 = cfg.lambda_l1;
  sp.min_child_hess = cfg.min_sum_hessian_in_leaf;
  sp.max_cat_to_onehot = cfg.max_cat_to_onehot;
  sp.max_cat_threshold = cfg.max_cat_threshold;
  sp.cat_smooth = cfg.cat_smooth;
  sp.cat_l2 = cfg.cat_l2;
  sp.min_data_per_group = cfg.min_data_per_group;

  auto t_fit = std::chrono::steady_clock::now();
  int launches = 0;
  // MOJOTREES_TRACE_HIST=1 prints every histogram launch (device time, items,
  // built rows) to stderr; it synchronises after each launch (diagnostic only)
  const bool trace_hist = getenv("MOJOTREES_TRACE_HIST") != nullptr;
  cudaEvent_t th0 = nullptr, th1 = nullptr;
  struct TraceEvents {
    cudaEvent_t &a, &b;
    ~TraceEvents() {
      if (a) cudaEventDestroy(a);
      if (b) cudaEventDestroy(b);
    }
  } trace_events{th0, th1};
  if (trace_hist) {
    MTB_CUDA(cudaEventCreate(&th0));
    MTB_CUDA(cudaEventCreate(&th1));
  }
  auto hist = [&]() {
    hist_timer.begin(&stats.hist_ms);
    if (trace_hist) MTB_CUDA(cudaEventRecord(th0, st));
    if (sparse_planes)
      launch_chained(pdl, sparse_planes == 2 ? k_hist_sparse<2> : k_hist_sparse<3>, n_sm, kSparseThreads,
                     sparse_hist_smem(sparse_planes, F, sparse_bp), st, batch_of(d_ts.p),
                     (const uint32_t*)d_entries.p, (const long long*)d_row_ptr.p, (const int*)d_default_bin.p, F, B,
                     sparse_bp, (const int*)d_rows0.p, (const int*)d_rows1.p,
                     reinterpret_cast<const int2*>(d_pairs0.p), reinterpret_cast<const int2*>(d_pairs1.p), d_hist.p,
                     slot_cells, work_base, hl.min_rows_per_cta, hl.owned ? 1 : 0);
    else
      launch_hist(hl, st, batch_of(d_ts.p), d_bins_rm.p, Fp, F, B, d_rows0.p, d_rows1.p, d_pairs0.p, d_pairs1.p,
                  d_hist.p, slot_cells, work_base);
    hist_timer.end();
    if (trace_hist) {
      MTB_CUDA(cudaEventRecord(th1, st));
      Batch hb;
      MTB_CUDA(cudaMemcpyAsync(&hb, batch_of(d_ts.p), sizeof(Batch), cudaMemcpyDeviceToHost, st));
      MTB_CUDA(cudaStreamSynchronize(st));
      float ms = 0.f;
      MTB_CUDA(cudaEventElapsedTime(&ms, th0, th1));
      long long rows = 0;
      std::string sizes;
      for (int i = 0; i < hb.n_items; ++i) {
        const BatchItem& P = hb.items[i];
        const long long nl = (long long)P.cursor_left;
        const long long c = P.built_is_left ? nl : P.count - nl;
        rows += c;
        sizes += " " + std::to_string(c);
      }
      fprintf(stderr, "mojotrees hist: us %.1f items %d rows %lld sizes%s\n", ms * 1000.0, hb.n_items, rows,
              sizes.c_str());
    }
  };
  // the built children's cells summed over every device's rows (exact int32)
  // Only the first `slots` work slots can be in use: iteration i of a tree
  // expands at most 2^i leaves (the virtual tree has one more unexpanded node
  // than it has expanded ones, and every expanded node came from an earlier
  // iteration), and items take work slots 0, 1, ... in batch order.
  auto reduce_work = [&](int iteration) {
    const size_t slots = (size_t)std::min(batch_cap, 1 << std::min(iteration, 5));
    if (dp_feature && wide)
      coll->reduce_scatter_slots_i64(reinterpret_cast<long long*>(d_hist.p + (size_t)work_base * slot_cells), slots,
                                     (size_t)slot_cells / 2, (size_t)Fb * 3 * B, st);
    else if (dp_feature)
      coll->reduce_scatter_slots_i32(d_hist.p + (size_t)work_base * slot_cells, slots, (size_t)slot_cells,
                                     (size_t)Fb * 3 * B, st);
    else if (coll && wide)
      coll->allreduce_sum_i64(reinterpret_cast<long long*>(d_hist.p + (size_t)work_base * slot_cells),
                              (size_t)slot_cells / 2 * slots, st);
    else if (coll)
      coll->allreduce_sum_i32(d_hist.p + (size_t)work_base * slot_cells, (size_t)slot_cells * slots, st);
  };
  DevBuf<ChildRec> d_rec, d_rec_all;
  if (dp_feature) {
    d_rec.alloc(2 * (size_t)kMaxBatch);
    d_rec_all.alloc(2 * (size_t)kMaxBatch * world);
  }

  const long long grid1024 = (N + 1023) / 1024;
  const unsigned grid256 = (unsigned)((N + 255) / 256);
  std::vector<cudaEvent_t> round_ev;
  struct EventGuard {
    std::vector<cudaEvent_t>& e;
    ~EventGuard() {
      for (auto x : e) cudaEventDestroy(x);
    }
  } eg{round_ev};
  auto mark_round = [&]() {
    cudaEvent_t e;
    MTB_CUDA(cudaEventCreate(&e));
    round_ev.push_back(e);
    MTB_CUDA(cudaEventRecord(e, st));
  };
  mark_round();
  std::vector<size_t> round_trees;  // trees after each round
  for (int it = 0; it < cfg.num_iterations; ++it) {
    if (K > 1) {
      k_softmax<<<grid256, 256, 0, st>>>(d_raw.p, d_prob.p, N, K);
      launches++;
    }
    bool progress = false;
    size_t first_tree = model.trees.size();
    for (int k = 0; k < K; ++k) {
      // ---- derivatives, scales, quantized pairs
      timer.begin(&stats.grad_ms);
      MTB_CUDA(cudaMemsetAsync(d_sc.p, 0, sizeof(RoundScales), st));
      if (coll && mode == MODE_FIXED) {
        MTB_CUDA(cudaMemsetAsync(d_pg.p, 0, sizeof(double) * P_rank, st));
        MTB_CUDA(cudaMemsetAsync(d_ph.p, 0, sizeof(double) * P_rank, st));
      }
      if (K == 1)
        k_grad<<<(unsigned)std::min<long long>(grid1024, 2ll * n_sm), 1024, 0, st>>>(
            d_raw.p, d_y.p, d_g.p, d_h.p, N, cfg.objective, mode, d_pg.p, d_ph.p, d_sc.p);
      else
        k_grad_softmax<<<(unsigned)grid1024, 1024, 0, st>>>(d_prob.p, d_y.p, d_g.p, d_h.p, N, K, k, mode, d_pg.p,
                                                            d_ph.p, d_sc.p);
      launches++;
      const double* tot_g = d_pg.p;
      const double* tot_h = d_ph.p;
      if (mode == MODE_QUANT && coll)
        coll->allreduce_max_u64(reinterpret_cast<unsigned long long*>(&d_sc.p->g_total), 2, st);
      if (mode == MODE_FIXED) {
        // pairwise levels: 1024 partials -> 1, outputs packed one after another
        long long n = n_part, off = 0;
        const double* ig = d_pg.p;
        const double* ih = d_ph.p;
        if (coll) {
          coll->allgather_f64(d_pg.p, d_pg_all.p, P_rank, st);
          coll->allgather_f64(d_ph.p, d_ph_all.p, P_rank, st);
          ig = d_pg_all.p;
          ih = d_ph_all.p;
        }
        while (n > 1) {
          long long nb = (n + 1023) / 1024;
          double* og = d_tg.p + off;
          double* oh = d_th.p + off;
          k_pairwise_level<<<(unsigned)nb, 1024, 0, st>>>(ig, ih, n, og, oh);
          launches++;
          ig = og;
          ih = oh;
          off += nb;
          n = nb;
        }
        tot_g = ig;
        tot_h = ih;
      }
      // With other ranks, wait for the tree's first exchange before queueing
      // work that depends on it: a rank that stopped participating between
      // trees is detected here (the bounded wait aborts the communicator),
      // with none of this rank's work queued behind the aborted collective.
      if (coll) coll->sync(st);
      k_scales<<<1, 32, 0, st>>>(d_sc.p, tot_g, tot_h, mode, const_h ? 1 : 0, cfg.num_grad_quant_bins, wide ? 1 : 0);
      uint64_t gs = mt_quant_stream(cfg.quant_seed, it, k, 0);
      uint64_t hs = mt_quant_stream(cfg.quant_seed, it, k, 1);
      if (mode == MODE_QUANT)
        k_quantize<MODE_QUANT><<<grid256, 256, 0, st>>>(d_g.p, d_h.p, N, in.row_offset, d_sc.p, const_h, gs, hs,
                                                         d_rows0.p, d_pairs0.p);
      else if (wide)
        k_quantize<MODE_FIXED, true><<<grid256, 256, 0, st>>>(d_g.p, d_h.p, N, in.row_offset, d_sc.p, const_h, gs, hs,
                                                               d_rows0.p, d_pairs0.p);
      else
        k_quantize<MODE_FIXED><<<grid256, 256, 0, st>>>(d_g.p, d_h.p, N, in.row_offset, d_sc.p, const_h, gs, hs,
                                                         d_rows0.p, d_pairs0.p);
      launches += 2;
      timer.end();

      // ---- active features of this tree (sampling.mojo:424-463)
      std::vector<int> feats;
      {
        int tree_index = K > 1 ? it * K + k : it;
        if (cfg.feature_fraction >= 1.0) {
          for (int f = 0; f < F; ++f) feats.push_back(f);
        } else {
          const uint64_t mask = 0x7FFFFFFFFFFFFFFFull;
          uint64_t h = mt_splitmix64((uint64_t)(int64_t)cfg.feature_fraction_seed & mask);
          h = mt_splitmix64(h ^ ((uint64_t)(int64_t)tree_index & mask));
          uint64_t stream = mt_splitmix64(h ^ 0ull);
          int count = (int)((double)F * cfg.feature_fraction + 0.5);
          int floor_count = F >= 2 ? 2 : F;
          count = std::max(count, floor_count);
          count = std::min(count, F);
          if (count >= F) {
            for (int f = 0; f < F; ++f) feats.push_back(f);
          } else {
            int chosen = 0;
            for (int i = 0; i < F && chosen < count; ++i) {
              double prob = (double)(count - chosen) / (double)(F - i);
              if (mt_uniform(stream + (uint64_t)i) < prob) {
                feats.push_back(i);
                ++chosen;
              }
            }
          }
        }
      }
      if (dp_feature) {  // this rank scans the active features of its own block
        std::vector<int> own;
        for (int f : feats)
          if (f / Fb == coll->rank()) own.push_back(f);
        feats.swap(own);
      }
      const int n_active = (int)feats.size();
      if (n_active > 0)
        MTB_CUDA(cudaMemcpyAsync(d_feats.p, feats.data(), sizeof(int) * n_active, cudaMemcpyHostToDevice, st));
      sp.n_active = n_active;
      const unsigned scan_grid = (unsigned)((2ll * batch_cap * n_active + kScanWarps - 1) / kScanWarps);

      // ---- grow the tree: iterations of partition -> histogram -> scan ->
      // commit, each expanding up to batch_cap leaves, until the commit
      // kernel reports the tree done
      k_tree_init<<<1, 32, 0, st>>>(d_ts.p, N);
      launches++;
      int launched = 0;
      for (int i = 0;; ++i) {
        if (i >= kLookahead) {
          const int q = (i - kLookahead) % kRing;
          if (coll)
            coll->wait(iter_ev[q]);
          else
            MTB_CUDA(cudaEventSynchronize(iter_ev[q]));
          if (reinterpret_cast<volatile int*>(h_done)[q]) break;
        }
        if (i > cfg.num_leaves) break;  // bound: every iteration after the root commits a split
        if (trace) fprintf(stderr, "mojotrees trace: tree %zu iteration %d\n", model.trees.size(), i);
        timer.begin(&stats.partition_ms);
        launch_partition();
        timer.end();
        // "iteration i - 1 committed": recorded after this partition rather
        // than after that commit, so the commit -> partition launch stays a
        // programmatic dependency (the partition starts only once the commit
        // grid has completed)
        if (i > 0) MTB_CUDA(cudaEventRecord(iter_ev[(i - 1) % kRing], st));
        hist();
        reduce_work(i);
        timer.begin(&stats.scan_ms);
        if (!dp_feature) {
          launch_chained(pdl,
                         wide ? (scan_compact ? k_scan_t<true, false, true> : k_scan_t<false, false, true>)
                              : (scan_compact ? k_scan_t<true, false> : k_scan_t<false, false>),
                         scan_grid, kScanWarps * 32, 0, st, d_ts.p, d_hist.p, slot_cells, d_feats.p, d_missing.p,
                         d_ncats.p, d_sc.p, sp, d_fb.p, work_base, (ChildRec*)nullptr);
        } else {
          // this rank's per-child bests -> every rank's -> the merged leaves
          MTB_CUDA(cudaMemsetAsync(d_rec.p, 0, sizeof(ChildRec) * 2 * (size_t)batch_cap, st));
          if (n_active > 0)
            (wide ? (scan_compact ? k_scan_t<true, true, true> : k_scan_t<false, true, true>)
                  : (scan_compact ? k_scan_t<true, true> : k_scan_t<false, true>))<<<scan_grid, kScanWarps * 32, 0, st>>>(
                d_ts.p, d_hist.p, slot_cells, d_feats.p, d_missing.p, d_ncats.p, d_sc.p, sp, d_fb.p, work_base,
                d_rec.p);
          coll->allgather_bytes(d_rec.p, d_rec_all.p, sizeof(ChildRec) * 2 * (size_t)batch_cap, st);
          k_merge_children<<<1, 2 * kMaxBatch, 0, st>>>(d_ts.p, d_rec_all.p, world, 2 * batch_cap, d_sc.p, sp);
          launches += 1;
        }
        timer.end();
        timer.begin(&stats.commit_ms);
        launch_chained(pdl, k_commit, 1, kCommitThreads, commit_smem, st, d_ts.p, d_missing.p, cp, commit_cap,
                       d_done, i % kRing);
        timer.end();
        launches += 4;
        launched++;
      }
      stats.hist_launches += launched;
      k_leaf_table<<<1, 1024, sizeof(long long) * table_stage, st>>>(d_ts.p, d_begins.p, d_bufs.p, d_values.p,
                                                                      table_stage);
      k_row_slots<<<update_grid, 256, 12 * (size_t)table_stage, st>>>(d_ts.p, d_begins.p, d_bufs.p, d_rows0.p,
                                                                     d_rows1.p, d_slot.p, N, table_stage);
      k_update_raw<<<update_grid, 256, 8 * (size_t)table_stage, st>>>(d_ts.p, d_values.p, d_slot.p, d_raw.p, N, K,
                                                                     k, cfg.learning_rate, table_stage);
      launches += 3;
      MTB_CUDA(cudaGetLastError());
      MTB_CUDA(cudaMemcpyAsync(&hdr, &d_ts.p->hdr, sizeof(TreeHeader), cudaMemcpyDeviceToHost, st));
      MTB_CUDA(cudaMemcpyAsync(nodes_host.data(), d_ts.p->nodes, sizeof(HostNode) * M, cudaMemcpyDeviceToHost, st));
      host_sync();
      timer.collect();
      hist_timer.collect();
      if (hdr.error || !hdr.done) throw std::runtime_error("device trainer reported an internal error");
      stats.iterations += hdr.iterations;
      stats.expansions += (hdr.n_pool - 1) / 2;
      stats.pick_steps += hdr.pick_steps;
      if (coll) coll->check();
      std::vector<HostNode> tree(nodes_host.begin(), nodes_host.begin() + hdr.n_nodes);
      bool trivial = hdr.n_leaves == 1 && std::fabs(tree[0].value) < 1e-12;
      if (!trivial) progress = true;
      model.trees.push_back(std::move(tree));
    }
    stats.rounds++;
    mark_round();
    if (coll && test_stall_rank == coll->rank() && stats.rounds == test_stall_after) {
      // Test hook (off unless MOJOTREES_DP_TEST_STALL_RANK names this rank):
      // after a completed round, with nothing of this rank in flight, it
      // stops participating for MOJOTREES_DP_TEST_STALL_S seconds (its
      // communicator and memory stay valid meanwhile), then fails.
      std::this_thread::sleep_for(std::chrono::duration<double>(test_stall_s));
      throw std::runtime_error("injected failure: rank " + std::to_string(coll->rank()) +
                               " stopped participating after round " + std::to_string(stats.rounds));
    }
    stats.round_hist_ms.push_back(stats.hist_ms);  // cumulative; differenced below
    stats.round_hist_launches.push_back((double)stats.hist_launches);
    stats.round_launches.push_back((double)launches);
    round_trees.push_back(model.trees.size());
    if (!progress) {
      // boosting.mojo:2898-2907 / :4153-4162: a round that grew nothing ends the fit
      model.trees.resize(first_tree);
      break;
    }
  }
  host_sync();
  for (size_t i = 0; i + 1 < round_ev.size(); ++i) {
    float ms = 0.f;
    MTB_CUDA(cudaEventElapsedTime(&ms, round_ev[i], round_ev[i + 1]));
    stats.round_ms.push_back(ms);
  }
  stats.fit_seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t_fit).count();
  stats.kernel_launches += launches;
  // rows read by histogram builds: every root plus the smaller child of every split
  for (size_t t = 0; t < model.trees.size(); ++t) {
    const auto& tr = model.trees[t];
    stats.hist_rows += (double)tr[0].count;
    for (const auto& nd : tr)
      if (nd.feature >= 0) stats.hist_rows += (double)std::min(tr[nd.left].count, tr[nd.right].count);
  }
  stats.hist_bytes = stats.hist_rows * (double)(F + (mode == MODE_QUANT ? 2 : 8));
  for (size_t r = stats.round_hist_ms.size(); r-- > 1;) {
    stats.round_hist_ms[r] -= stats.round_hist_ms[r - 1];
    stats.round_hist_launches[r] -= stats.round_hist_launches[r - 1];
    stats.round_launches[r] -= stats.round_launches[r - 1];
  }
  stats.round_hist_rows.assign(round_trees.size(), 0.0);
  for (size_t r = 0; r < round_trees.size(); ++r) {
    const size_t t0 = r ? round_trees[r - 1] : 0;
    for (size_t t = t0; t < std::min(round_trees[r], model.trees.size()); ++t) {
      const auto& tr = model.trees[t];
      stats.round_hist_rows[r] += (double)tr[0].count;
      for (const auto& nd : tr)
        if (nd.feature >= 0) stats.round_hist_rows[r] += (double)std::min(tr[nd.left].count, tr[nd.right].count);
    }
  }
  if (cfg.keep_training_scores) {
    model.train_scores.resize((size_t)N * K);
    MTB_CUDA(cudaMemcpy(model.train_scores.data(), d_raw.p, sizeof(double) * N * K, cudaMemcpyDeviceToHost));
  }
  model.stats = stats;
}

}  // namespace mtb
