// Device transform of float64 columns into uint8 bins (see device_binning.h).
#include "device_binning.h"

#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <chrono>
#include <map>
#include <mutex>
#include <cstdio>
#include <stdexcept>
#include <string>
#include <vector>

namespace mtb {
namespace {

#define MTB_CUDA_BIN(call)                                                                   \
  do {                                                                                       \
    cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess)                                                                   \
      throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(e_) + " at " \
                               + #call);                                                     \
  } while (0)

// Per-feature description of the mapper, in device memory.
struct FeatureBins {
  int64_t edge_off;  // first edge of the feature in `edges`
  int n_edges;
  int missing_bin;   // -1 when none
  int is_cat;
  int pad;
  int64_t code_off;  // first kept code in `codes`
  int n_codes;
  int pad2;
};

constexpr int kBinThreads = 256;

// One block per (row block, feature of the chunk): the feature's edges (at
// most 255) or kept codes staged in shared memory, then every value binned
// exactly as BinMapper::bin_value does.  The chunk holds rows [r0, r0 +
// chunk_rows) of features f0.. as consecutive columns of chunk_rows values.
__global__ void __launch_bounds__(kBinThreads) k_bin_columns(const double* __restrict__ x, int64_t chunk_rows,
                                                             int64_t r0_chunk, int64_t n_rows, int f0,
                                                             const FeatureBins* __restrict__ fb,
                                                             const double* __restrict__ edges,
                                                             const int64_t* __restrict__ codes,
                                                             uint8_t* __restrict__ out, int64_t rows_per_block) {
  __shared__ double s_edge[256];
  __shared__ int64_t s_code[256];
  const int fl = blockIdx.y;
  const FeatureBins d = fb[f0 + fl];
  if (d.is_cat) {
    for (int i = threadIdx.x; i < d.n_codes; i += blockDim.x) s_code[i] = codes[d.code_off + i];
  } else {
    for (int i = threadIdx.x; i < d.n_edges; i += blockDim.x) s_edge[i] = edges[d.edge_off + i];
  }
  __syncthreads();
  const double* col = x + (int64_t)fl * chunk_rows;
  uint8_t* dst = out + (int64_t)(f0 + fl) * n_rows + r0_chunk;
  const int64_t r0 = (int64_t)blockIdx.x * rows_per_block;
  const int64_t r1 = r0 + rows_per_block < chunk_rows ? r0 + rows_per_block : chunk_rows;
  for (int64_t r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
    const double v = col[r];
    int bin;
    if (d.is_cat) {
      bin = 0;
      if (v >= 0.0 && v < 2147483648.0) {
        const int64_t code = (int64_t)v;
        int lo = 0, hi = d.n_codes;  // first kept code >= code
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (s_code[mid] < code) lo = mid + 1;
          else hi = mid;
        }
        if (lo < d.n_codes && s_code[lo] == code) bin = lo + 1;
      }
    } else if (v != v && d.missing_bin >= 0) {
      bin = d.missing_bin;
    } else {
      const double value = v != v ? 0.0 : v;
      int lo = 0, hi = d.n_edges;  // number of edges below value
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (value <= s_edge[mid]) hi = mid;
        else lo = mid + 1;
      }
      bin = lo;
    }
    dst[r] = (uint8_t)bin;
  }
}

template <typename T>
struct DeviceArray {
  T* p = nullptr;
  explicit DeviceArray(size_t n) { MTB_CUDA_BIN(cudaMalloc(&p, sizeof(T) * (n ? n : 1))); }
  ~DeviceArray() { cudaFree(p); }
};

// Three 32 MB page-registered host buffers, three device buffers and their
// events: the staging of the column uploads.  Registering and allocating
// them costs tens of milliseconds, so each device keeps one set from its
// first upload until the process exits (96 MB pinned host memory and 96 MB
// device memory); an upload that finds the set in use by another thread
// makes a set of its own for the call.
constexpr int kStages = 3;
constexpr size_t kStageBytes = 32u << 20;
struct StagingSet {
  uint8_t* h[kStages] = {};
  bool reg[kStages] = {};
  void* d[kStages] = {};
  cudaEvent_t e[kStages] = {};
  void create() {
    for (int i = 0; i < kStages; ++i) {
      h[i] = static_cast<uint8_t*>(aligned_alloc(4096, kStageBytes));
      if (!h[i]) throw std::runtime_error("host staging allocation failed");
      MTB_CUDA_BIN(cudaHostRegister(h[i], kStageBytes, cudaHostRegisterDefault));
      reg[i] = true;
      MTB_CUDA_BIN(cudaMalloc(&d[i], kStageBytes));
      MTB_CUDA_BIN(cudaEventCreateWithFlags(&e[i], cudaEventDisableTiming));
    }
  }
  void destroy() {
    for (int i = 0; i < kStages; ++i) {
      if (e[i]) {
        cudaEventSynchronize(e[i]);
        cudaEventDestroy(e[i]);
      }
      if (reg[i]) cudaHostUnregister(h[i]);
      free(h[i]);
      if (d[i]) cudaFree(d[i]);
      e[i] = nullptr;
      reg[i] = false;
      h[i] = nullptr;
      d[i] = nullptr;
    }
  }
};
std::mutex g_staging_mutex;
std::map<int, StagingSet> g_staging;
std::map<int, bool> g_staging_busy;

// The device's cached set (or a fresh one for this call when it is in use),
// released at scope exit.
struct Staging {
  StagingSet own;
  StagingSet* set = nullptr;
  int dev = -1;
  Staging() {
    MTB_CUDA_BIN(cudaGetDevice(&dev));
    {
      std::lock_guard<std::mutex> lock(g_staging_mutex);
      if (!g_staging_busy[dev]) {
        g_staging_busy[dev] = true;
        set = &g_staging[dev];
      }
    }
    if (!set) {
      set = &own;
      own.create();
      return;
    }
    if (!set->h[0]) {
      try {
        set->create();
      } catch (...) {
        set->destroy();
        std::lock_guard<std::mutex> lock(g_staging_mutex);
        g_staging_busy[dev] = false;
        throw;
      }
    }
  }
  ~Staging() {
    for (int i = 0; i < kStages; ++i)
      if (set->e[i]) cudaEventSynchronize(set->e[i]);
    if (set == &own) {
      own.destroy();
    } else {
      std::lock_guard<std::mutex> lock(g_staging_mutex);
      g_staging_busy[dev] = false;
    }
  }
};

}  // namespace

void transform_on_device(const BinMapper& m, const double* x, int64_t n_rows, uint8_t* d_bins,
                         cudaStream_t st) {
  const int F = m.n_features;
  std::vector<FeatureBins> fb((size_t)F);
  for (int f = 0; f < F; ++f) {
    FeatureBins& d = fb[f];
    memset(&d, 0, sizeof d);
    d.is_cat = (!m.is_cat.empty() && m.is_cat[f]) ? 1 : 0;
    d.missing_bin = m.missing_bin[f];
    d.edge_off = m.edge_offsets[f];
    d.n_edges = (int)(m.edge_offsets[f + 1] - m.edge_offsets[f]);
    d.code_off = m.cat_offsets.empty() ? 0 : m.cat_offsets[f];
    d.n_codes = m.n_categories(f);
    if (d.n_edges > 256 || d.n_codes > 256) throw std::runtime_error("more than 256 edges or codes in a feature");
  }
  DeviceArray<FeatureBins> d_fb(F);
  DeviceArray<double> d_edges(m.edges.size());
  DeviceArray<int64_t> d_codes(m.cat_codes.size());
  MTB_CUDA_BIN(cudaMemcpyAsync(d_fb.p, fb.data(), sizeof(FeatureBins) * F, cudaMemcpyHostToDevice, st));
  if (!m.edges.empty())
    MTB_CUDA_BIN(cudaMemcpyAsync(d_edges.p, m.edges.data(), sizeof(double) * m.edges.size(),
                                 cudaMemcpyHostToDevice, st));
  if (!m.cat_codes.empty())
    MTB_CUDA_BIN(cudaMemcpyAsync(d_codes.p, m.cat_codes.data(), sizeof(int64_t) * m.cat_codes.size(),
                                 cudaMemcpyHostToDevice, st));

  // The column-major matrix is streamed in chunks of kStageBytes: several
  // whole features when a column is short, else a row range of one feature.
  // Each chunk is copied by all host threads into one of the kStages
  // page-locked staging buffers, sent to the device and binned there; the
  // memcpy of a chunk overlaps the DMA of the previous one.  The buffers are
  // ordinary allocations registered with the driver, which pins pages several
  // times faster than cudaHostAlloc, kept per device (StagingSet).
  // MOJOTREES_TRACE_UPLOAD=1 prints the phase times of this function to stderr
  const bool trace = getenv("MOJOTREES_TRACE_UPLOAD") != nullptr;
  auto clk = [] { return std::chrono::steady_clock::now(); };
  const auto tt0 = clk();
  double t_wait = 0.0, t_copy = 0.0;
  const int64_t chunk_elems_max = (int64_t)kStageBytes / (int64_t)sizeof(double);
  int64_t chunk_rows, per_chunk;
  if (n_rows >= chunk_elems_max) {
    chunk_rows = chunk_elems_max;
    per_chunk = 1;
  } else {
    chunk_rows = std::max<int64_t>(1, n_rows);
    per_chunk = std::max<int64_t>(1, std::min<int64_t>({(int64_t)F, chunk_elems_max / chunk_rows, 65535}));
  }
  Staging stg;
  StagingSet& sg = *stg.set;
  const int64_t rows_per_block = 8192;
  const auto tt1 = clk();
  int k = 0;
  for (int f0 = 0; f0 < F; f0 += (int)per_chunk) {
    const int nf = (int)std::min<int64_t>(per_chunk, F - f0);
    for (int64_t r0 = 0; r0 < n_rows; r0 += chunk_rows) {
      const int64_t nr = std::min<int64_t>(chunk_rows, n_rows - r0);
      // the buffer's previous DMA must have finished before it is refilled
      const auto ta = clk();
      MTB_CUDA_BIN(cudaEventSynchronize(sg.e[k]));
      const auto tb = clk();
      double* dst = reinterpret_cast<double*>(sg.h[k]);
      // nf columns of nr values each, packed back to back
      const int64_t elems = (int64_t)nf * nr;
      const int64_t piece = 1 << 17;
#pragma omp parallel for schedule(static)
      for (int64_t b = 0; b < elems; b += piece) {
        int64_t o = b;
        const int64_t end = std::min<int64_t>(b + piece, elems);
        while (o < end) {
          const int64_t fl = o / nr, r = o - fl * nr;
          const int64_t n = std::min<int64_t>(end - o, nr - r);
          memcpy(dst + o, x + (int64_t)(f0 + fl) * n_rows + r0 + r, sizeof(double) * n);
          o += n;
        }
      }
      if (trace) {
        t_wait += std::chrono::duration<double>(tb - ta).count();
        t_copy += std::chrono::duration<double>(clk() - tb).count();
      }
      MTB_CUDA_BIN(cudaMemcpyAsync(sg.d[k], dst, sizeof(double) * elems, cudaMemcpyHostToDevice, st));
      MTB_CUDA_BIN(cudaEventRecord(sg.e[k], st));
      const unsigned row_blocks = (unsigned)((nr + rows_per_block - 1) / rows_per_block);
      k_bin_columns<<<dim3(row_blocks, nf), kBinThreads, 0, st>>>(static_cast<const double*>(sg.d[k]), nr, r0,
                                                                 n_rows, f0, d_fb.p,
                                                                 d_edges.p, d_codes.p, d_bins, rows_per_block);
      MTB_CUDA_BIN(cudaGetLastError());
      k = (k + 1) % kStages;
    }
  }
  MTB_CUDA_BIN(cudaStreamSynchronize(st));
  if (trace)
    fprintf(stderr, "upload: setup %.1f ms, stream %.1f ms (buffer waits %.1f, host copies %.1f), %lld x %d values\n",
            std::chrono::duration<double>(tt1 - tt0).count() * 1e3,
            std::chrono::duration<double>(clk() - tt1).count() * 1e3, t_wait * 1e3, t_copy * 1e3,
            (long long)n_rows, F);
}

// Host data (pre-binned uint8 columns, labels) to the device through the
// same page-registered staging buffers as the float64 columns: 32 MB pieces, each
// copied into a staging buffer by all host threads while the previous
// piece's DMA runs (a plain copy from pageable memory moved ~6 GB/s).
void upload_host(const void* src, int64_t bytes, void* dst_dev, cudaStream_t st) {
  const uint8_t* bins = static_cast<const uint8_t*>(src);
  uint8_t* d_bins = static_cast<uint8_t*>(dst_dev);
  constexpr int64_t kPiece = (int64_t)kStageBytes;
  // registering the staging buffers costs ~25 ms: below 1 GB a direct copy
  // from pageable memory is cheaper
  if (bytes < (1ll << 30)) {
    MTB_CUDA_BIN(cudaMemcpyAsync(d_bins, bins, (size_t)bytes, cudaMemcpyHostToDevice, st));
    MTB_CUDA_BIN(cudaStreamSynchronize(st));
    return;
  }
  Staging stg;
  StagingSet& sg = *stg.set;
  int k = 0;
  for (int64_t off = 0; off < bytes; off += kPiece) {
    const int64_t len = std::min<int64_t>(kPiece, bytes - off);
    MTB_CUDA_BIN(cudaEventSynchronize(sg.e[k]));  // the buffer's previous DMA is done
    uint8_t* dst = sg.h[k];
    const int64_t part = 1 << 20;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < len; b += part) memcpy(dst + b, bins + off + b, (size_t)std::min<int64_t>(part, len - b));
    MTB_CUDA_BIN(cudaMemcpyAsync(d_bins + off, dst, (size_t)len, cudaMemcpyHostToDevice, st));
    MTB_CUDA_BIN(cudaEventRecord(sg.e[k], st));
    k = (k + 1) % kStages;
  }
  MTB_CUDA_BIN(cudaStreamSynchronize(st));
}

}  // namespace mtb
