// Prediction on the device (mojotrees_predict_ex with MOJOTREES_DEVICE_GPU;
// the reference's gpu_predict.mojo).  Rows are binned on the device by the
// chunked column transform the dense trainer uses, then one thread per row
// walks every tree of the requested iterations, summing exactly as the host
// predictor does: s = fma(learning_rate, leaf, s) in tree order, from the
// base score (boosting.mojo:1722-1727, 3747-3757).  IEEE fma is exact on both
// sides, so device raw scores equal the host's bit for bit.
#include <cuda_runtime.h>

#include <algorithm>

#include <stdexcept>
#include <string>
#include <vector>

#include "device_binning.h"
#include "predict.h"

namespace mtb {
namespace {

#define MTB_CUDA_PRED(call)                                                                  \
  do {                                                                                       \
    cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess)                                                                   \
      throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(e_) + " at " \
                               + #call);                                                     \
  } while (0)

template <typename T>
struct Dev {
  T* p = nullptr;
  explicit Dev(size_t n) { MTB_CUDA_PRED(cudaMalloc(&p, sizeof(T) * (n ? n : 1))); }
  ~Dev() { cudaFree(p); }
  Dev(const Dev&) = delete;
  Dev& operator=(const Dev&) = delete;
};

// Tree walk of tree.mojo:483-503 on feature-major bins.
__device__ __forceinline__ double walk(const HostNode* __restrict__ t, const uint8_t* __restrict__ bins,
                                       long long r, long long n) {
  int node = 0;
  while (true) {
    const int f = __ldg(&t[node].feature);
    if (f < 0) break;
    const HostNode& nd = t[node];
    const int b = bins[(long long)f * n + r];
    bool left;
    if (__ldg(&nd.is_cat)) left = b > 0 && b < 256 && ((__ldg(&nd.bits[b >> 6]) >> (b & 63)) & 1ull);
    else if (b == __ldg(&nd.mbin)) left = __ldg(&nd.dleft) != 0;
    else left = b <= __ldg(&nd.thr);
    node = left ? __ldg(&nd.left) : __ldg(&nd.right);
  }
  return __ldg(&t[node].value);
}

// out[r * K + k] = base[k] (when the range starts at iteration 0) + the
// shrunk leaves of trees (i * K + k), i in the range, in order.  tree_off[j]
// is the first node of the j-th tree of the range.
__global__ void __launch_bounds__(256) k_predict_raw(const HostNode* __restrict__ nodes,
                                                     const long long* __restrict__ tree_off,
                                                     const uint8_t* __restrict__ bins, long long n, int K,
                                                     long long n_iter, bool with_base, double lr,
                                                     const double* __restrict__ base, double* __restrict__ out) {
  for (long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += (long long)gridDim.x * blockDim.x) {
    for (int k = 0; k < K; ++k) {
      double s = with_base ? base[k] : 0.0;
      for (long long i = 0; i < n_iter; ++i) s = fma(lr, walk(nodes + tree_off[i * K + k], bins, r, n), s);
      out[r * K + k] = s;
    }
  }
}

}  // namespace

void predict_raw_device(const Model& m, const double* data, int64_t n_rows, int64_t it0, int64_t it1,
                        double* out) {
  if (!m.has_mapper) throw std::runtime_error("model has no bin mapper");
  const int K = m.num_class;
  const int F = m.n_features;
  if (n_rows == 0) return;
  const long long n_iter = it1 - it0;
  std::vector<HostNode> nodes;
  std::vector<long long> off;
  for (long long i = it0; i < it1; ++i)
    for (int k = 0; k < K; ++k) {
      const auto& t = m.trees[(size_t)(i * K + k)];
      off.push_back((long long)nodes.size());
      nodes.insert(nodes.end(), t.begin(), t.end());
    }
  cudaStream_t st;
  MTB_CUDA_PRED(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  struct StreamGuard {
    cudaStream_t s;
    ~StreamGuard() { cudaStreamDestroy(s); }
  } sg{st};
  Dev<uint8_t> d_bins((size_t)F * n_rows);
  Dev<HostNode> d_nodes(nodes.size());
  Dev<long long> d_off(off.size());
  Dev<double> d_base(K), d_out((size_t)n_rows * K);
  transform_on_device(m.mapper, data, n_rows, d_bins.p, st);
  if (!nodes.empty())
    MTB_CUDA_PRED(cudaMemcpyAsync(d_nodes.p, nodes.data(), sizeof(HostNode) * nodes.size(), cudaMemcpyHostToDevice, st));
  if (!off.empty())
    MTB_CUDA_PRED(cudaMemcpyAsync(d_off.p, off.data(), sizeof(long long) * off.size(), cudaMemcpyHostToDevice, st));
  MTB_CUDA_PRED(cudaMemcpyAsync(d_base.p, m.base_scores.data(), sizeof(double) * K, cudaMemcpyHostToDevice, st));
  int dev = 0, n_sm = 148;
  MTB_CUDA_PRED(cudaGetDevice(&dev));
  MTB_CUDA_PRED(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
  const long long want = (n_rows + 255) / 256;
  const unsigned blocks = (unsigned)std::max<long long>(1, std::min<long long>(want, (long long)n_sm * 8));
  k_predict_raw<<<blocks, 256, 0, st>>>(d_nodes.p, d_off.p, d_bins.p, n_rows, K, n_iter, it0 == 0,
                                        m.learning_rate, d_base.p, d_out.p);
  MTB_CUDA_PRED(cudaGetLastError());
  MTB_CUDA_PRED(cudaMemcpyAsync(out, d_out.p, sizeof(double) * (size_t)n_rows * K, cudaMemcpyDeviceToHost, st));
  MTB_CUDA_PRED(cudaStreamSynchronize(st));
}

}  // namespace mtb
