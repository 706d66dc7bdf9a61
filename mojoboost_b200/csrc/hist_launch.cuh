// Launch geometry and launchers of the histogram kernel, shared by the
// trainer and the standalone histogram entry points.
#pragma once
#include <cuda_runtime.h>

#include <stdlib.h>

#include <algorithm>
#include <cstddef>
#include <stdexcept>
#include <string>
#include <utility>

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

// Launches k on st; with pdl, as a programmatic dependent of the kernel
// before it on the stream (the kernel must begin with pdl_enter()).
template <typename... KArgs, typename... Args>
void launch_chained(bool pdl, void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                    Args&&... args) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = pdl ? 1 : 0;
  MTB_CUDA(cudaLaunchKernelEx(&lc, k, std::forward<Args>(args)...));
}

inline const Batch* batch_of(const TreeState* ts) {
  return reinterpret_cast<const Batch*>(reinterpret_cast<const char*>(ts) + offsetof(TreeState, batch));
}

struct HistLaunch {
  int layout = HL_QUANT;       // shared-memory cell layout (HistLayout)
  int cluster = 1;             // CTAs per thread-block cluster along grid y
  int min_rows_per_cta = 512;  // a batch uses ceil(rows / this) CTAs at most
  int npl = 1;                 // features per lane (feature group = 32 * npl)
  int groups = 1;
  int threads = 512;
  int row_ctas = 1;
  size_t smem = 0;
  long long rows_per_flush = 1ll << 40;
  bool pdl = false;            // launch as a programmatic dependent (trainer iterations)
  bool owned = true;           // may give items clusters of their own (k_hist); MOJOTREES_HIST_CONTIGUOUS=1: never
  int g_lim = 0;               // HL_QUANT16: offset making g non-negative
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
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = hl.pdl ? 2 : 1;
  return lc;
}

template <int NPL, int L>
cudaError_t prepare_hist_t(const HistLaunch& hl, int cs, int* n_clusters) {
  auto k = k_hist<NPL, L>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t lc = hist_config(hl, cs, hl.row_ctas / cs * cs, 0, attr);
  return cudaOccupancyMaxActiveClusters(n_clusters, k, &lc);
}

template <int NPL, int L>
void launch_hist_t(const HistLaunch& hl, cudaStream_t st, const Batch* batch, const uint8_t* bins_rm, int Fp, int F,
                   int B, const int* r0, const int* r1, const void* p0, const void* p1, int* hist,
                   long long slot_cells, int ws) {
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t lc = hist_config(hl, hl.cluster, hl.row_ctas, st, attr);
  MTB_CUDA(cudaLaunchKernelEx(&lc, k_hist<NPL, L>, batch, bins_rm, Fp, F, B, r0, r1, p0, p1, hist, slot_cells,
                              hl.rows_per_flush, hl.g_lim, ws, hl.min_rows_per_cta, hl.owned ? 1 : 0));
}

// Every (layout, features per lane) instance the launch geometry can pick.
#define MTB_HIST_SWITCH(EXPR)                                                                         \
  switch (hl.layout * 8 + hl.npl) {                                                                    \
    case HL_QUANT * 8 + 1: { constexpr int V = 1, L = HL_QUANT; EXPR; } break;                        \
    case HL_QUANT * 8 + 2: { constexpr int V = 2, L = HL_QUANT; EXPR; } break;                        \
    case HL_QUANT * 8 + 4: { constexpr int V = 4, L = HL_QUANT; EXPR; } break;                        \
    case HL_QUANT16 * 8 + 2: { constexpr int V = 2, L = HL_QUANT16; EXPR; } break;                    \
    case HL_QUANT16 * 8 + 4: { constexpr int V = 4, L = HL_QUANT16; EXPR; } break;                    \
    case HL_QUANT16R * 8 + 2: { constexpr int V = 2, L = HL_QUANT16R; EXPR; } break;                  \
    case HL_QUANT16R * 8 + 4: { constexpr int V = 4, L = HL_QUANT16R; EXPR; } break;                  \
    case HL_FIXED_CH * 8 + 1: { constexpr int V = 1, L = HL_FIXED_CH; EXPR; } break;                  \
    case HL_FIXED_CH * 8 + 2: { constexpr int V = 2, L = HL_FIXED_CH; EXPR; } break;                  \
    case HL_FIXED_CH * 8 + 4: { constexpr int V = 4, L = HL_FIXED_CH; EXPR; } break;                  \
    case HL_FIXED * 8 + 1: { constexpr int V = 1, L = HL_FIXED; EXPR; } break;                        \
    case HL_FIXED * 8 + 2: { constexpr int V = 2, L = HL_FIXED; EXPR; } break;                        \
    case HL_FIXED * 8 + 4: { constexpr int V = 4, L = HL_FIXED; EXPR; } break;                        \
    case HL_W52 * 8 + 1: { constexpr int V = 1, L = HL_W52; EXPR; } break;                            \
    case HL_W52CH * 8 + 1: { constexpr int V = 1, L = HL_W52CH; EXPR; } break;                        \
    default: throw std::runtime_error("bad histogram layout");                                         \
  }

inline cudaError_t prepare_hist(const HistLaunch& hl, int cs, int* n_clusters) {
  cudaError_t e = cudaErrorInvalidValue;
  MTB_HIST_SWITCH(e = (prepare_hist_t<V, L>(hl, cs, n_clusters)))
  return e;
}

inline void launch_hist(const HistLaunch& hl, cudaStream_t st, const Batch* batch, const uint8_t* bins_rm, int Fp,
                        int F, int B, const int* r0, const int* r1, const void* p0, const void* p1, int* hist,
                        long long slot_cells, int ws) {
  MTB_HIST_SWITCH((launch_hist_t<V, L>(hl, st, batch, bins_rm, Fp, F, B, r0, r1, p0, p1, hist, slot_cells, ws)))
}

// Cell layout and flush span for a fit.  quant_bins: the int8 gradient range
// (|g| <= quant_bins / 2, h <= quant_bins); 0 for the fixed-point modes.
inline void choose_hist_layout(HistLaunch& hl, int mode, bool const_h, int quant_bins, bool wide = false) {
  if (wide) {
    hl.layout = const_h ? HL_W52CH : HL_W52;
    hl.rows_per_flush = 1ll << 40;  // Int64 cells: sums stay below 2^53, counts below 2^31 per CTA
    return;
  }
  if (mode == MODE_QUANT) {
    const long long gl = quant_bins / 2, hlim = quant_bins;
    const long long rpf16 = std::min<long long>(65535 / (2 * gl), 65535 / hlim);
    if (rpf16 >= 2048 && !getenv("MOJOTREES_HIST_NO_PACK")) {
      hl.layout = HL_QUANT16;
      hl.rows_per_flush = rpf16;
      hl.g_lim = (int)gl;
    } else {
      // plane 0 holds g * 2^15 + count: count < 2^15 and |sum g| < 2^16 per flush
      hl.layout = HL_QUANT;
      hl.rows_per_flush = std::min<long long>((1ll << 15) - 1, ((1ll << 16) - 1) / gl);
    }
  } else {
    hl.layout = const_h ? HL_FIXED_CH : HL_FIXED;
    hl.rows_per_flush = 1ll << 40;
  }
}

// Features per lane: the fewest feature groups (each group re-reads the
// rows) whose cells fit the shared-memory budget, then the smallest such
// group.  Row chunks are sized to fill every SM; CTAs of a feature group form
// clusters of up to 8 that merge through DSMEM.
// n_rows > 0 (row ids below it) lets 16-bit packed cells with narrow
// quantizers use HL_QUANT16R; MOJOTREES_HIST_NO_ROWPACK turns that off.
inline HistLaunch choose_hist_launch(int mode, bool const_h, int quant_bins, int B, int Fp, int n_sm,
                                     long long n_rows = 0, bool wide = false) {
  HistLaunch hl;
  choose_hist_layout(hl, mode, const_h, quant_bins, wide);
  if (hl.layout == HL_QUANT16 && n_rows > 0 && n_rows <= (1ll << 26) && quant_bins <= 7
      && !getenv("MOJOTREES_HIST_NO_ROWPACK"))
    hl.layout = HL_QUANT16R;
  // MOJOTREES_HIST_SMEM_KB / MOJOTREES_HIST_CLUSTER override the shared-memory
  // budget per CTA and the cluster size (tuning knobs)
  size_t budget = 220 * 1024;
  if (const char* e = getenv("MOJOTREES_HIST_SMEM_KB")) budget = (size_t)atoi(e) * 1024;
  int max_cs = 8, force_cs = 0;
  if (const char* e = getenv("MOJOTREES_HIST_CLUSTER")) force_cs = max_cs = atoi(e);
  auto smem_of = [&](int npl) {
    return (size_t)4 * hist_layout_words(hl.layout, 32 * npl * kHistBinsPad) + (size_t)kHistBatchSmem;
  };
  hl.npl = 0;
  hl.groups = 1 << 30;
  for (int npl : {1, 2, 4}) {
    if ((hl.layout == HL_QUANT16 || hl.layout == HL_QUANT16R) && npl == 1) continue;
    if ((hl.layout == HL_W52 || hl.layout == HL_W52CH) && npl != 1) continue;
    int groups = (Fp + 32 * npl - 1) / (32 * npl);
    if ((smem_of(npl) <= budget || hl.npl == 0) && groups < hl.groups) {
      hl.npl = npl;
      hl.groups = groups;
    }
  }
  hl.smem = smem_of(hl.npl);
  int per_sm = std::max(1, (int)((228 * 1024) / (hl.smem + 1024)));
  hl.threads = kHistThreads;
  per_sm = std::min(per_sm, 2048 / hl.threads);
  // Clusters of CS CTAs must fit inside one GPC, so fewer than
  // n_sm * per_sm / CS may be resident at once.  The grid holds exactly the
  // resident clusters (a second wave would double the launch), split evenly
  // among the feature groups; the cluster size kept is the one that leaves
  // the most CTAs resident (larger on ties: fewer partial cells to merge).
  hl.cluster = 1;
  hl.row_ctas = std::max(1, n_sm * per_sm / hl.groups);
  int best_ctas = 0;
  for (int cs : {8, 4, 2, 1}) {
    if (cs > max_cs) continue;
    int n_clusters = 0;
    HistLaunch probe = hl;
    probe.row_ctas = cs;
    cudaError_t oe = prepare_hist(probe, cs, &n_clusters);
    if (oe != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    int per_group = n_clusters / hl.groups;
    if (per_group < 1) continue;
    if (per_group * cs * hl.groups > best_ctas || cs == force_cs) {
      best_ctas = per_group * cs * hl.groups;
      hl.cluster = cs;
      hl.row_ctas = per_group * cs;
      if (cs == force_cs) break;
    }
  }
  if (const char* e = getenv("MOJOTREES_HIST_MIN_ROWS")) hl.min_rows_per_cta = std::max(1, atoi(e));
  if (getenv("MOJOTREES_HIST_CONTIGUOUS")) hl.owned = false;
  return hl;
}

}  // namespace
}  // namespace mtb
