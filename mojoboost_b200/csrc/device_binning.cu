// Device transform of float64 columns into uint8 bins (see device_binning.h).
#include "device_binning.h"

#include <string.h>

#include <algorithm>
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

// One block per (row chunk, feature of the chunk): the feature's edges (at
// most 255) or kept codes staged in shared memory, then every value binned
// exactly as BinMapper::bin_value does.
__global__ void __launch_bounds__(kBinThreads) k_bin_columns(const double* __restrict__ x, int64_t n_rows,
                                                             int f0, const FeatureBins* __restrict__ fb,
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
  const double* col = x + (int64_t)fl * n_rows;
  uint8_t* dst = out + (int64_t)(f0 + fl) * n_rows;
  const int64_t r0 = (int64_t)blockIdx.x * rows_per_block;
  const int64_t r1 = r0 + rows_per_block < n_rows ? r0 + rows_per_block : n_rows;
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

  // chunks of whole features, about 256 MB of float64 each
  const int64_t col_bytes = n_rows * (int64_t)sizeof(double);
  const int per_chunk = (int)std::max<int64_t>(1, std::min<int64_t>(F, (256ll << 20) / col_bytes));
  const int64_t chunk_elems = (int64_t)per_chunk * n_rows;
  double* h_stage[2] = {nullptr, nullptr};
  DeviceArray<double> d_stage0(chunk_elems), d_stage1(chunk_elems);
  double* d_stage[2] = {d_stage0.p, d_stage1.p};
  cudaEvent_t done[2] = {nullptr, nullptr};
  struct Cleanup {
    double** h;
    cudaEvent_t* e;
    ~Cleanup() {
      for (int i = 0; i < 2; ++i) {
        if (h[i]) cudaFreeHost(h[i]);
        if (e[i]) cudaEventDestroy(e[i]);
      }
    }
  } cleanup{h_stage, done};
  for (int i = 0; i < 2; ++i) {
    MTB_CUDA_BIN(cudaHostAlloc(&h_stage[i], sizeof(double) * chunk_elems, cudaHostAllocDefault));
    MTB_CUDA_BIN(cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming));
  }
  const int64_t rows_per_block = 8192;
  const unsigned row_blocks = (unsigned)((n_rows + rows_per_block - 1) / rows_per_block);
  int k = 0;
  for (int f0 = 0; f0 < F; f0 += per_chunk, k ^= 1) {
    const int nf = std::min(per_chunk, F - f0);
    const int64_t elems = (int64_t)nf * n_rows;
    // the buffer's previous DMA must have finished before it is refilled
    MTB_CUDA_BIN(cudaEventSynchronize(done[k]));
    const double* src = x + (int64_t)f0 * n_rows;
    double* dst = h_stage[k];
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < elems; b += (1 << 20)) {
      const int64_t n = std::min<int64_t>(1 << 20, elems - b);
      memcpy(dst + b, src + b, sizeof(double) * n);
    }
    MTB_CUDA_BIN(cudaMemcpyAsync(d_stage[k], h_stage[k], sizeof(double) * elems, cudaMemcpyHostToDevice, st));
    MTB_CUDA_BIN(cudaEventRecord(done[k], st));
    k_bin_columns<<<dim3(row_blocks, nf), kBinThreads, 0, st>>>(d_stage[k], n_rows, f0, d_fb.p, d_edges.p,
                                                               d_codes.p, d_bins, rows_per_block);
    MTB_CUDA_BIN(cudaGetLastError());
  }
  MTB_CUDA_BIN(cudaStreamSynchronize(st));
}

}  // namespace mtb
