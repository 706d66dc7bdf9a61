// Launch geometry and launchers of the histogram kernel, shared by the
// trainer and the standalone histogram entry points.
#pragma once
#include <cuda_runtime.h>

#include <stdlib.h>

#include <algorithm>
#include <cstddef>
#include <stdexcept>
#include <string>

#include "gbdt_device.cuh"
#include "gbdt_kernels.cuh"

namespace mtb {
namespace {

#ifndef MTB_CUDA
#define MTB_CUDA(call)                                                                       \
  do {                                                                                       \
    cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess)                                                                   \
      throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(e_) + " at " \
                               + #call);                                                     \
  } while (0)
#endif

inline const Plan* plan_of(const TreeState* ts) {
  return reinterpret_cast<const Plan*>(reinterpret_cast<const char*>(ts) + offsetof(TreeState, plan));
}

struct HistLaunch {
  int cluster = 1;  // CTAs per thread-block cluster along grid y
  int min_rows_per_cta = 512;  // a leaf uses ceil(rows / this) CTAs at most
  int vpr = 1;
  int groups = 1;
  int threads = 512;
  int row_ctas = 1;
  size_t smem = 0;
};

cudaLaunchConfig_t hist_config(const HistLaunch& hl, int cs, int row_ctas, cudaStream_t st, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(hl.groups, row_ctas);
  lc.blockDim = dim3(hl.threads);
  lc.dynamicSmemBytes = hl.smem;
  lc.stream = st;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = cs;
  attr[0].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  return lc;
}

template <int VPR, int MODE, bool CH>
cudaError_t prepare_hist_t(const HistLaunch& hl, int cs, int* n_clusters) {
  auto k = k_hist<VPR, MODE, CH>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t lc = hist_config(hl, cs, hl.row_ctas / cs * cs, 0, attr);
  return cudaOccupancyMaxActiveClusters(n_clusters, k, &lc);
}

template <int VPR, int MODE, bool CH>
void launch_hist_t(const HistLaunch& hl, cudaStream_t st, const Plan* plan, const uint8_t* bins_rm, int Fp, int F,
                   int B, const int* r0, const int* r1, const void* p0, const void* p1, int* hist,
                   long long slot_cells, long long rpf, int ws) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t lc = hist_config(hl, hl.cluster, hl.row_ctas, st, attr);
  MTB_CUDA(cudaLaunchKernelEx(&lc, k_hist<VPR, MODE, CH>, plan, bins_rm, Fp, F, B, r0, r1, p0, p1, hist, slot_cells,
                              rpf, ws, hl.min_rows_per_cta));
}

#define MTB_VPR_SWITCH(EXPR)                                                                  \
  switch (hl.vpr) {                                                                            \
    case 1: { constexpr int V = 1; EXPR; } break;                                              \
    case 2: { constexpr int V = 2; EXPR; } break;                                              \
    case 3: { constexpr int V = 3; EXPR; } break;                                              \
    case 4: { constexpr int V = 4; EXPR; } break;                                              \
    case 5: { constexpr int V = 5; EXPR; } break;                                              \
    case 6: { constexpr int V = 6; EXPR; } break;                                              \
    case 7: { constexpr int V = 7; EXPR; } break;                                              \
    case 8: { constexpr int V = 8; EXPR; } break;                                              \
    default: throw std::runtime_error("bad histogram vector count");                           \
  }

template <int MODE, bool CH>
cudaError_t prepare_hist(const HistLaunch& hl, int cs, int* n_clusters) {
  cudaError_t e = cudaErrorInvalidValue;
  MTB_VPR_SWITCH(e = (prepare_hist_t<V, MODE, CH>(hl, cs, n_clusters)))
  return e;
}

template <int MODE, bool CH>
void launch_hist(const HistLaunch& hl, cudaStream_t st, const Plan* plan, const uint8_t* bins_rm, int Fp, int F,
                 int B, const int* r0, const int* r1, const void* p0, const void* p1, int* hist, long long slot_cells,
                 long long rpf, int ws) {
  MTB_VPR_SWITCH((launch_hist_t<V, MODE, CH>(hl, st, plan, bins_rm, Fp, F, B, r0, r1, p0, p1, hist, slot_cells, rpf, ws)))
}


// As many features per CTA as one SM's shared memory holds, row chunks sized
// to fill every SM, CTAs of a feature group in clusters of up to 8 that merge
// through DSMEM.
inline HistLaunch choose_hist_launch(int mode, bool const_h, int B, int Fp, int n_sm) {
  HistLaunch hl;
  size_t cell_bytes = (mode == MODE_QUANT || const_h) ? 8 : 12;  // two or three 32-bit planes
  // MOJOTREES_HIST_SMEM_KB / MOJOTREES_HIST_CLUSTER override the shared-memory
  // budget per CTA and the largest cluster size (tuning knobs)
  size_t budget = 100 * 1024;
  if (const char* e = getenv("MOJOTREES_HIST_SMEM_KB")) budget = (size_t)atoi(e) * 1024;
  int max_cs = 8;
  if (const char* e = getenv("MOJOTREES_HIST_CLUSTER")) max_cs = atoi(e);
  int fg_max = (int)(budget / ((size_t)B * cell_bytes)) / 16 * 16;
  fg_max = std::max(16, std::min(128, fg_max));
  int vmax = fg_max / 16;
  int vecs = Fp / 16;
  hl.groups = (vecs + vmax - 1) / vmax;
  hl.vpr = (vecs + hl.groups - 1) / hl.groups;
  hl.smem = (size_t)hl.vpr * 16 * B * cell_bytes;
  int per_sm = std::max(1, (int)((228 * 1024) / (hl.smem + 1024)));
  hl.threads = per_sm >= 2 ? 512 : 1024;
  per_sm = std::min(per_sm, 2048 / hl.threads);
  hl.row_ctas = std::max(1, (n_sm * per_sm + hl.groups - 1) / hl.groups);
  hl.cluster = 1;
  for (int cs : {8, 4, 2, 1}) {
    if (hl.row_ctas < cs || cs > max_cs) continue;
    int n_clusters = 0;
    cudaError_t oe;
    if (mode == MODE_QUANT) oe = prepare_hist<MODE_QUANT, false>(hl, cs, &n_clusters);
    else if (const_h) oe = prepare_hist<MODE_FIXED, true>(hl, cs, &n_clusters);
    else oe = prepare_hist<MODE_FIXED, false>(hl, cs, &n_clusters);
    if (oe == cudaSuccess && n_clusters >= 1) {
      hl.cluster = cs;
      break;
    }
    cudaGetLastError();
  }
  hl.row_ctas = std::max(hl.cluster, hl.row_ctas / hl.cluster * hl.cluster);
  if (const char* e = getenv("MOJOTREES_HIST_MIN_ROWS")) hl.min_rows_per_cta = std::max(1, atoi(e));
  return hl;
}

}  // namespace
}  // namespace mtb
