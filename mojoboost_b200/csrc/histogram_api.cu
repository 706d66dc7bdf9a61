// Standalone entry point of the per-leaf histogram kernel (the hot kernel of
// the trainer) for callers and tests that want one histogram of one row set:
// the quantized-gradient build of gpu_active_rows.mojo:3903
// (_range_hist_atomic_kernel) over int8 gradient / hessian pairs.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>
#include <string.h>

#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/mojotrees.h"
#include "capi_util.h"
#include "gbdt_device.cuh"
#include "gbdt_kernels.cuh"
#include "hist_launch.cuh"
#include "trainer.h"

namespace mtb {
namespace {

struct DevMem {
  void* p = nullptr;
  explicit DevMem(size_t bytes) { MTB_CUDA(cudaMalloc(&p, bytes ? bytes : 1)); }
  ~DevMem() { cudaFree(p); }
};

// Job descriptor of one histogram build over positions [0, n_sel) of
// rows/pairs: a one-item batch whose built child is the whole selection.
Batch one_item_batch(long long n_sel) {
  Batch b;
  memset(&b, 0, sizeof b);
  b.n_items = 1;
  b.root = 1;
  BatchItem& P = b.items[0];
  P.built_is_left = 1;
  P.count = n_sel;
  P.cursor_left = (unsigned long long)n_sel;
  return b;
}

// Bytes of the descriptor the kernel reads for a one-item batch.
constexpr size_t kOneItemBatchBytes = offsetof(Batch, items) + sizeof(BatchItem);

// Launches the histogram kernel for positions [0, n_sel) of rows/pairs into
// `work` (zeroed here); `d_batch` is device memory for the job descriptor.
void launch_leaf_hist(const uint8_t* d_bins_rm, int F, int Fp, int B, const int* d_rows, const uint16_t* d_pairs,
                      long long n_sel, int quant_bins, Batch* d_batch, int* d_work, cudaStream_t st) {
  Batch b = one_item_batch(n_sel);
  MTB_CUDA(cudaMemcpyAsync(d_batch, &b, kOneItemBatchBytes, cudaMemcpyHostToDevice, st));
  const long long cells = (long long)F * 3 * B;
  MTB_CUDA(cudaMemsetAsync(d_work, 0, sizeof(int) * cells, st));
  int dev = 0, n_sm = 0;
  MTB_CUDA(cudaGetDevice(&dev));
  MTB_CUDA(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
  HistLaunch hl = choose_hist_launch(MODE_QUANT, false, quant_bins, B, Fp, n_sm);
  launch_hist(hl, st, d_batch, d_bins_rm, Fp, F, B, d_rows, d_rows, d_pairs, d_pairs, d_work, cells, 0);
  MTB_CUDA(cudaGetLastError());
}

}  // namespace
}  // namespace mtb

extern "C" int32_t mojotrees_b200_histogram_u8(const uint8_t* bins, int64_t n_rows, int64_t n_features,
                                               int32_t n_bins, const int32_t* rows, int64_t n_sel,
                                               const int8_t* grad_q, const uint8_t* hess_q,
                                               int32_t num_grad_quant_bins, int32_t* out_hist,
                                               MojoTreesError* error) {
  using namespace mtb;
  capi_clear_error(error);
  try {
    if (!bins || !grad_q || !hess_q || !out_hist) throw std::invalid_argument("null pointer argument");
    if (n_rows < 1 || n_features < 1 || n_sel < 0) throw std::invalid_argument("sizes must be positive");
    if (n_rows >= (1ll << 31)) throw std::invalid_argument("more than 2^31-1 rows");
    if (n_bins < 2 || n_bins > 256) throw std::invalid_argument("n_bins must be in [2, 256]");
    if (num_grad_quant_bins < 2 || num_grad_quant_bins > 254 || num_grad_quant_bins % 2)
      throw std::invalid_argument("num_grad_quant_bins must be even and in [2, 254]");
    if (!rows) n_sel = n_rows;
    const int F = (int)n_features, B = n_bins, Fp = (F + 15) / 16 * 16;
    const int lim = num_grad_quant_bins / 2;
    std::vector<int> rsel((size_t)n_sel);
    std::vector<uint16_t> pairs((size_t)n_sel);
    for (int64_t i = 0; i < n_sel; ++i) {
      int64_t r = rows ? rows[i] : i;
      if (r < 0 || r >= n_rows) throw std::invalid_argument("row id out of range");
      if (grad_q[r] < -lim || grad_q[r] > lim || hess_q[r] > num_grad_quant_bins)
        throw std::invalid_argument("quantized gradient outside [-bins/2, bins/2] or hessian above bins");
      rsel[i] = (int)r;
      pairs[i] = (uint16_t)((uint8_t)grad_q[r]) | (uint16_t)((uint16_t)hess_q[r] << 8);
    }
    for (int64_t k = 0; k < n_rows * n_features; ++k)
      if (bins[k] >= B) throw std::invalid_argument("bin value >= n_bins");
    if (cuda_device_count() < 1) throw Unsupported("no CUDA device is available");
    // row-major bins with a 16-byte row stride, as the trainer keeps them
    std::vector<uint8_t> rm((size_t)n_rows * Fp, 0);
    for (int64_t f = 0; f < F; ++f)
      for (int64_t r = 0; r < n_rows; ++r) rm[(size_t)r * Fp + f] = bins[f * n_rows + r];
    const size_t cells = (size_t)F * 3 * B;
    DevMem d_bins(rm.size()), d_rows(sizeof(int) * rsel.size()), d_pairs(sizeof(uint16_t) * pairs.size()),
        d_batch(kOneItemBatchBytes), d_work(sizeof(int) * cells);
    cudaStream_t st = 0;
    MTB_CUDA(cudaMemcpy(d_bins.p, rm.data(), rm.size(), cudaMemcpyHostToDevice));
    MTB_CUDA(cudaMemcpy(d_rows.p, rsel.data(), sizeof(int) * rsel.size(), cudaMemcpyHostToDevice));
    MTB_CUDA(cudaMemcpy(d_pairs.p, pairs.data(), sizeof(uint16_t) * pairs.size(), cudaMemcpyHostToDevice));
    if (n_sel > 0)
      launch_leaf_hist((const uint8_t*)d_bins.p, F, Fp, B, (const int*)d_rows.p, (const uint16_t*)d_pairs.p, n_sel,
                       num_grad_quant_bins, (Batch*)d_batch.p, (int*)d_work.p, st);
    else
      MTB_CUDA(cudaMemset(d_work.p, 0, sizeof(int) * cells));
    MTB_CUDA(cudaMemcpy(out_hist, d_work.p, sizeof(int) * cells, cudaMemcpyDeviceToHost));
    return MOJOTREES_OK;
  } catch (const std::invalid_argument& e) {
    capi_set_error(error, e.what());
    return MOJOTREES_ERROR_INVALID_ARGUMENT;
  } catch (const Unsupported& e) {
    capi_set_error(error, e.what());
    return MOJOTREES_ERROR_UNSUPPORTED;
  } catch (const std::exception& e) {
    capi_set_error(error, e.what());
    return MOJOTREES_ERROR_TRAINING;
  }
}

// ---------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot call cudaMalloc: callers that hand the GPU's memory to
// their own pool allocator and forbid others from taking any, and
// latency-critical paths that must not take the allocator's locks.  For them
// the job descriptor and the accumulation cells of the histogram live in one
// fixed device array, reserved when the library is loaded and held by every
// GPU that loads it until the process exits.  The caller passes device
// pointers for the inputs and the output; nothing is allocated per call.
// The job descriptor is written by a one-thread kernel on the call's stream,
// so the call makes no host-to-device copy.
// ---------------------------------------------------------------------------
namespace mtb {
namespace {

// Largest histogram the array holds: 128 features x 256 bins x (g, h, count).
constexpr long long kNoAllocMaxCells = 128ll * 256 * 3;
constexpr size_t kNoAllocBatchBytes = (kOneItemBatchBytes + 255) / 256 * 256;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBatchBytes + kNoAllocMaxCells * 4];

struct NoAllocDevice {
  bool ready = false;
  unsigned char* scratch = nullptr;  // device address of g_noalloc_scratch
  HistLaunch hl;
  int hl_B = -1, hl_Fp = -1, hl_qb = -1;
};
constexpr int kMaxDevices = 64;
NoAllocDevice g_noalloc_dev[kMaxDevices];
std::mutex g_noalloc_mutex;

// Writes the one-item job descriptor of one_item_batch() on the device.
__global__ void k_noalloc_descriptor(Batch* b, long long n_sel) {
  unsigned char* p = reinterpret_cast<unsigned char*>(b);
  for (size_t i = 0; i < kOneItemBatchBytes; ++i) p[i] = 0;
  b->n_items = 1;
  b->root = 1;
  b->items[0].built_is_left = 1;
  b->items[0].count = n_sel;
  b->items[0].cursor_left = (unsigned long long)n_sel;
}

}  // namespace
}  // namespace mtb

extern "C" int32_t mojotrees_b200_histogram_u8_noalloc(const uint8_t* bins_rm, int64_t n_rows, int64_t n_features,
                                                       int32_t n_bins, const int32_t* rows, int64_t n_sel,
                                                       const uint16_t* pairs, int32_t num_grad_quant_bins,
                                                       int32_t* out_hist, void* stream, MojoTreesError* error) {
  using namespace mtb;
  capi_clear_error(error);
  try {
    if (!bins_rm || !rows || !pairs || !out_hist) throw std::invalid_argument("null pointer argument");
    if (n_rows < 1 || n_features < 1 || n_sel < 1) throw std::invalid_argument("sizes must be positive");
    if (n_rows >= (1ll << 31)) throw std::invalid_argument("more than 2^31-1 rows");
    if (n_bins < 2 || n_bins > 256) throw std::invalid_argument("n_bins must be in [2, 256]");
    if (num_grad_quant_bins < 2 || num_grad_quant_bins > 254 || num_grad_quant_bins % 2)
      throw std::invalid_argument("num_grad_quant_bins must be even and in [2, 254]");
    const long long cells = n_features * 3 * (long long)n_bins;
    if (cells > kNoAllocMaxCells)
      throw std::invalid_argument("n_features * n_bins exceeds the allocation-free limit of 128 * 256 "
                                  "(use mojotrees_b200_histogram_u8)");
    int dev = 0;
    MTB_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) throw std::runtime_error("device index out of range");
    const int F = (int)n_features, B = n_bins, Fp = (F + 15) / 16 * 16;
    NoAllocDevice* d = &g_noalloc_dev[dev];
    HistLaunch hl;  // this call's launch geometry, copied while the lock is held
    unsigned char* scratch = nullptr;
    {
      std::lock_guard<std::mutex> lock(g_noalloc_mutex);
      if (!d->ready) {
        // once per device, with that device current: the array's device address
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess)
          throw std::runtime_error(std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
        d->scratch = static_cast<unsigned char*>(ptr);
        d->ready = true;
      }
      if (d->hl_B != B || d->hl_Fp != Fp || d->hl_qb != num_grad_quant_bins) {
        int n_sm = 0;
        MTB_CUDA(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
        d->hl = choose_hist_launch(MODE_QUANT, false, num_grad_quant_bins, B, Fp, n_sm);
        d->hl_B = B;
        d->hl_Fp = Fp;
        d->hl_qb = num_grad_quant_bins;
      }
      hl = d->hl;
      scratch = d->scratch;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    Batch* batch = reinterpret_cast<Batch*>(scratch);
    int* work = reinterpret_cast<int*>(scratch + kNoAllocBatchBytes);
    k_noalloc_descriptor<<<1, 1, 0, st>>>(batch, n_sel);
    MTB_CUDA(cudaGetLastError());
    MTB_CUDA(cudaMemsetAsync(work, 0, sizeof(int) * cells, st));  // the array keeps the last call's cells
    launch_hist(hl, st, batch, bins_rm, Fp, F, B, rows, rows, pairs, pairs, work, cells, 0);
    MTB_CUDA(cudaGetLastError());
    MTB_CUDA(cudaMemcpyAsync(out_hist, work, sizeof(int) * cells, cudaMemcpyDeviceToDevice, st));
    return MOJOTREES_OK;
  } catch (const std::invalid_argument& e) {
    capi_set_error(error, e.what());
    return MOJOTREES_ERROR_INVALID_ARGUMENT;
  } catch (const std::exception& e) {
    capi_set_error(error, e.what());
    return MOJOTREES_ERROR_TRAINING;
  }
}

// ---------------------------------------------------------------------------
// Shared-memory atomic throughput probe: the roofline of the histogram kernel.
//
// The histogram's inner loop is one red.shared.add.u32 per (row, feature,
// plane) into a bank-per-lane layout (no bank conflicts, no same-address
// collisions in an instruction).  This probe issues the same instruction
// pattern at the same geometry (1024 threads, the same shared memory per
// CTA, one CTA per SM) with no global traffic, and reports the rate the SMs
// sustain: lane-atomics per second over the whole GPU.
// ---------------------------------------------------------------------------
namespace mtb {
namespace {

constexpr int kProbeWords = 48 * 1024;  // 192 KB, the HL_QUANT16 histogram's shared memory

__global__ void __launch_bounds__(1024) k_smem_red_probe(int iters, unsigned int* sink) {
  extern __shared__ __align__(16) unsigned int probe_smem[];
  for (int i = threadIdx.x; i < kProbeWords; i += blockDim.x) probe_smem[i] = 0u;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const uint32_t base = (uint32_t)__cvta_generic_to_shared(probe_smem) + 4u * lane;
  uint32_t x = 2654435761u * (threadIdx.x + 1) + blockIdx.x;
  for (int it = 0; it < iters; ++it) {
    x = x * 1664525u + 1013904223u;  // pseudo-random bins, as rows bring them
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t a = base + (((x >> (8 * j)) & 0xffu) << 7);
      shared_red_add(a + j * 32768u, 1u);
      shared_red_add(a + 131072u + (j >> 1) * 32768u, 2u);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) atomicAdd(sink, probe_smem[blockIdx.x & 1023]);
}

}  // namespace
}  // namespace mtb

extern "C" int32_t mojotrees_b200_shared_atomic_peak(double* out_lane_atomics_per_s, MojoTreesError* error) {
  using namespace mtb;
  capi_clear_error(error);
  try {
    if (!out_lane_atomics_per_s) throw std::invalid_argument("null pointer argument");
    if (cuda_device_count() < 1) throw Unsupported("no CUDA device is available");
    int dev = 0, n_sm = 0;
    MTB_CUDA(cudaGetDevice(&dev));
    MTB_CUDA(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
    const size_t smem = sizeof(unsigned int) * kProbeWords;
    MTB_CUDA(cudaFuncSetAttribute(k_smem_red_probe, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    DevMem sink(sizeof(unsigned int));
    const int iters = 4096;
    cudaEvent_t a, b;
    MTB_CUDA(cudaEventCreate(&a));
    MTB_CUDA(cudaEventCreate(&b));
    float best = 1e30f;
    for (int rep = 0; rep < 4; ++rep) {  // the first launch warms up
      MTB_CUDA(cudaEventRecord(a, 0));
      k_smem_red_probe<<<n_sm, 1024, smem, 0>>>(iters, (unsigned int*)sink.p);
      MTB_CUDA(cudaEventRecord(b, 0));
      MTB_CUDA(cudaEventSynchronize(b));
      float ms = 0.f;
      MTB_CUDA(cudaEventElapsedTime(&ms, a, b));
      if (rep > 0 && ms < best) best = ms;
    }
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    MTB_CUDA(cudaGetLastError());
    const double lane_atomics = (double)n_sm * 1024.0 * iters * 8.0;
    *out_lane_atomics_per_s = lane_atomics / (best * 1e-3);
    return MOJOTREES_OK;
  } catch (const std::invalid_argument& e) {
    capi_set_error(error, e.what());
    return MOJOTREES_ERROR_INVALID_ARGUMENT;
  } catch (const Unsupported& e) {
    capi_set_error(error, e.what());
    return MOJOTREES_ERROR_UNSUPPORTED;
  } catch (const std::exception& e) {
    capi_set_error(error, e.what());
    return MOJOTREES_ERROR_TRAINING;
  }
}

// ---------------------------------------------------------------------------
// Self-check of the divide-free dequantization (quot_exact): the correctly
// rounded quotient of integer histogram sums by quantizer units, compared on
// the device with the divide it replaces.
// ---------------------------------------------------------------------------
namespace mtb {
namespace {

__global__ void k_check_quotients(long long n, unsigned long long seed, unsigned long long* mismatches) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  unsigned long long bad = 0;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const uint64_t r0 = mt_splitmix64(seed + 2 * (uint64_t)i), r1 = mt_splitmix64(seed + 2 * (uint64_t)i + 1);
    // sums: integers up to 2^40 in magnitude (a few small ones exactly);
    // units: lim / max with lim in {1..127} and max a float32 in [1e-12, 1e38]
    long long q = (long long)(r0 >> 24) - (1ll << 39);
    if ((r0 & 15) == 0) q = (long long)(r0 >> 60) - 8;
    const int lim = 1 + (int)((r1 >> 57) & 127) % 127;
    const float mx = __uint_as_float((unsigned int)(0x2B8CBCCCu + (unsigned int)((r1 & 0xffffffffu) % 0x53000000u)));
    const double units = (double)lim / (double)mx;
    const double a = (double)q;
    const double want = a / units;
    const double got = quot_exact(a, units, 1.0 / units);
    if (__double_as_longlong(want) != __double_as_longlong(got)) ++bad;
  }
  if (bad) atomicAdd(mismatches, bad);
}

}  // namespace
}  // namespace mtb

extern "C" int32_t mojotrees_b200_check_quotients(int64_t n, uint64_t seed, int64_t* out_mismatches,
                                                  MojoTreesError* error) {
  using namespace mtb;
  capi_clear_error(error);
  try {
    if (!out_mismatches || n < 0) throw std::invalid_argument("invalid argument");
    if (cuda_device_count() < 1) throw Unsupported("no CUDA device is available");
    DevMem d(sizeof(unsigned long long));
    MTB_CUDA(cudaMemset(d.p, 0, sizeof(unsigned long long)));
    k_check_quotients<<<148 * 8, 256>>>(n, seed, (unsigned long long*)d.p);
    MTB_CUDA(cudaGetLastError());
    unsigned long long bad = 0;
    MTB_CUDA(cudaMemcpy(&bad, d.p, sizeof bad, cudaMemcpyDeviceToHost));
    *out_mismatches = (int64_t)bad;
    return MOJOTREES_OK;
  } catch (const std::invalid_argument& e) {
    capi_set_error(error, e.what());
    return MOJOTREES_ERROR_INVALID_ARGUMENT;
  } catch (const Unsupported& e) {
    capi_set_error(error, e.what());
    return MOJOTREES_ERROR_UNSUPPORTED;
  } catch (const std::exception& e) {
    capi_set_error(error, e.what());
    return MOJOTREES_ERROR_TRAINING;
  }
}
