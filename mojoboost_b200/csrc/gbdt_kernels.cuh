// sm_100a kernels of the GBDT training path.  Included by trainer.cu only.
//
// Arithmetic contract (bit-exact against the CPU oracle):
//   * derivatives are computed in Float64 and narrowed to Float32 exactly as
//     boosting.mojo:676-812 does, with mt_exp (identical on host and device);
//   * FIXED mode quantizes with Int32(rint(x_f32 * s_f32)) for a power-of-two
//     s (histogram.mojo:3618-3640); QUANT mode with seeded stochastic rounding
//     (quantized_gradient.mojo:1479-1545);
//   * histogram cells are integers, so accumulation order is irrelevant;
//   * the split scan evaluates the reference gain on exact integer prefix
//     sums, dequantized by an exact power-of-two multiply (FIXED) or by the
//     reference's division f64(q) / units (QUANT, quantized_gradient.mojo:1324).
// The translation unit is compiled with -fmad=false so no multiply-add is
// contracted behind the arithmetic spelled here.
#pragma once
#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gbdt_device.cuh"
#include "mt_math.h"

namespace mtb {
// Kernels have internal linkage: each translation unit that launches them
// (trainer.cu, histogram_api.cu) carries its own instantiation.
namespace {

// ---------------------------------------------------------------------------
// Layout kernels
// ---------------------------------------------------------------------------

// bins_cm [F][n] -> bins_rm [n][Fp]; thread per (row, 16-feature vector).
__global__ void k_transpose_bins(const uint8_t* __restrict__ cm, uint8_t* __restrict__ rm,
                                 long long n, int F, int Fp) {
  long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  int v = blockIdx.y;
  if (r >= n) return;
  uint8_t b[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    int f = v * 16 + k;
    b[k] = f < F ? cm[(long long)f * n + r] : (uint8_t)0;
  }
  uint4 out;
  memcpy(&out, b, 16);
  *reinterpret_cast<uint4*>(rm + r * Fp + v * 16) = out;
}

// ---------------------------------------------------------------------------
// Derivatives and scales
// ---------------------------------------------------------------------------

enum Objective : int { OBJ_L2 = 0, OBJ_LOGISTIC = 1, OBJ_SOFTMAX = 2 };

__device__ __forceinline__ double narrow32(double v) { return (double)(float)v; }

// Warp pairwise sum of adjacent lanes: lane 0 ends with the power-of-two tree
// over the warp's 32 consecutive values.
__device__ __forceinline__ double warp_pairwise(double v) {
#pragma unroll
  for (int k = 1; k < 32; k <<= 1) {
    double o = __shfl_down_sync(0xffffffffu, v, k);
    if ((threadIdx.x & (2 * k - 1)) == 0) v = v + o;
  }
  return v;
}

// Block of 1024 threads: pairwise tree over 1024 consecutive values.
__device__ __forceinline__ double block_pairwise_1024(double v, double* sm32) {
  v = warp_pairwise(v);
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) sm32[w] = v;
  __syncthreads();
  double r = 0.0;
  if (w == 0) {
    r = warp_pairwise(sm32[lane]);
  }
  return r;
}

__device__ __forceinline__ void atomic_max_nonneg(double* addr, double v) {
  atomicMax(reinterpret_cast<unsigned long long*>(addr), (unsigned long long)__double_as_longlong(v));
}

// Per-row derivatives for L2 / logistic, narrowed to Float32.  1024 threads,
// one row each.  FIXED mode writes per-block pairwise |g|, |h| partials;
// QUANT mode folds max |g|, max |h| into the round's scales.
__global__ void __launch_bounds__(1024) k_grad(const double* __restrict__ raw, const double* __restrict__ y,
                                               float* __restrict__ g32, float* __restrict__ h32,
                                               long long n, int objective, int mode,
                                               double* __restrict__ part_g, double* __restrict__ part_h,
                                               RoundScales* sc) {
  __shared__ double sm[32];
  long long r = (long long)blockIdx.x * 1024 + threadIdx.x;
  double g = 0.0, h = 0.0;
  if (r < n) {
    double rr = raw[r];
    double yy = y[r];
    if (objective == OBJ_LOGISTIC) {
      double p = mt_sigmoid(rr);
      g = narrow32(1.0 * (p - yy));
      double hh = p * (1.0 - p);
      if (hh < 1e-16) hh = 1e-16;
      h = narrow32(1.0 * hh);
    } else {
      g = narrow32(1.0 * (rr - yy));
      h = 1.0;
    }
    g32[r] = (float)g;
    h32[r] = (float)h;
  }
  if (mode == MODE_FIXED) {
    double sg = block_pairwise_1024(fabs(g), sm);
    if (threadIdx.x == 0) part_g[blockIdx.x] = sg;
    double sh = block_pairwise_1024(fabs(h), sm);
    if (threadIdx.x == 0) part_h[blockIdx.x] = sh;
  } else {
    double ag = fabs(g), ah = fabs(h);
    for (int k = 16; k > 0; k >>= 1) {
      ag = fmax(ag, __shfl_down_sync(0xffffffffu, ag, k));
      ah = fmax(ah, __shfl_down_sync(0xffffffffu, ah, k));
    }
    if ((threadIdx.x & 31) == 0) {
      atomic_max_nonneg(&sc->g_total, ag);
      atomic_max_nonneg(&sc->h_total, ah);
    }
  }
}

// Softmax probabilities of every row (boosting.mojo:3529-3572), K <= 64.
__global__ void k_softmax(const double* __restrict__ raw, double* __restrict__ prob, long long n, int K) {
  long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  const double* rp = raw + r * K;
  double* pp = prob + r * K;
  double m = rp[0];
  for (int k = 1; k < K; ++k)
    if (rp[k] > m) m = rp[k];
  double total = 0.0;
  for (int k = 0; k < K; ++k) {
    double e = mt_exp(rp[k] - m);
    pp[k] = e;
    total = total + e;
  }
  for (int k = 0; k < K; ++k) pp[k] = pp[k] / total;
}

// Class-k softmax derivatives (boosting.mojo:3621-3677) with the same
// partial/maximum side outputs as k_grad.
__global__ void __launch_bounds__(1024) k_grad_softmax(const double* __restrict__ prob, const double* __restrict__ y,
                                                       float* __restrict__ g32, float* __restrict__ h32,
                                                       long long n, int K, int k, int mode,
                                                       double* __restrict__ part_g, double* __restrict__ part_h,
                                                       RoundScales* sc) {
  __shared__ double sm[32];
  long long r = (long long)blockIdx.x * 1024 + threadIdx.x;
  double g = 0.0, h = 0.0;
  if (r < n) {
    double p = prob[r * K + k];
    double yy = (int)y[r] == k ? 1.0 : 0.0;
    double factor = (double)K / (double)(K - 1);
    g = narrow32(1.0 * (p - yy));
    double hh = factor * p * (1.0 - p);
    if (hh < 1e-16) hh = 1e-16;
    h = narrow32(1.0 * hh);
    g32[r] = (float)g;
    h32[r] = (float)h;
  }
  if (mode == MODE_FIXED) {
    double sg = block_pairwise_1024(fabs(g), sm);
    if (threadIdx.x == 0) part_g[blockIdx.x] = sg;
    double sh = block_pairwise_1024(fabs(h), sm);
    if (threadIdx.x == 0) part_h[blockIdx.x] = sh;
  } else {
    double ag = fabs(g), ah = fabs(h);
    for (int s = 16; s > 0; s >>= 1) {
      ag = fmax(ag, __shfl_down_sync(0xffffffffu, ag, s));
      ah = fmax(ah, __shfl_down_sync(0xffffffffu, ah, s));
    }
    if ((threadIdx.x & 31) == 0) {
      atomic_max_nonneg(&sc->g_total, ag);
      atomic_max_nonneg(&sc->h_total, ah);
    }
  }
}

// One level of the pairwise reduction of block partials (1024 -> 1).
__global__ void __launch_bounds__(1024) k_pairwise_level(const double* __restrict__ in_g, const double* __restrict__ in_h,
                                                         long long n, double* __restrict__ out_g,
                                                         double* __restrict__ out_h) {
  __shared__ double sm[32];
  long long i = (long long)blockIdx.x * 1024 + threadIdx.x;
  double g = i < n ? in_g[i] : 0.0;
  double h = i < n ? in_h[i] : 0.0;
  double sg = block_pairwise_1024(g, sm);
  if (threadIdx.x == 0) out_g[blockIdx.x] = sg;
  double sh = block_pairwise_1024(h, sm);
  if (threadIdx.x == 0) out_h[blockIdx.x] = sh;
}

// Scales of the round from the reduced totals (FIXED: quantized_gradient.mojo:908;
// QUANT: :1343-1453).  `fixed_totals` is null in QUANT mode.
__global__ void k_scales(RoundScales* sc, const double* fixed_g, const double* fixed_h, int mode, int const_hess,
                         int quant_bins) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  if (mode == MODE_FIXED) {
    sc->g_total = *fixed_g;
    sc->h_total = *fixed_h;
    sc->gsf = mt_fixed_point_scale(sc->g_total);
    sc->hsf = mt_fixed_point_scale(sc->h_total);
    sc->g_inv = 1.0 / (double)sc->gsf;
    sc->h_inv = 1.0 / (double)sc->hsf;
    sc->hq_const = __float2int_rn(__fmul_rn(1.0f, sc->hsf));
  } else {
    double gmax = sc->g_total < 1e-12 ? 1e-12 : sc->g_total;
    double hmax = sc->h_total < 1e-12 ? 1e-12 : sc->h_total;
    sc->g_lim = (double)(quant_bins / 2);
    sc->h_lim = const_hess ? 1.0 : (double)quant_bins;
    sc->g_units = sc->g_lim / gmax;
    sc->h_units = const_hess ? 1.0 / hmax : sc->h_lim / hmax;
  }
}

// Tree start: identity row list and the quantized pair of every row.
template <int MODE>
__global__ void k_quantize(const float* __restrict__ g32, const float* __restrict__ h32, long long n,
                           long long row_offset, const RoundScales* __restrict__ sc, int const_hess,
                           uint64_t g_stream, uint64_t h_stream, int* __restrict__ rows, void* __restrict__ pairs) {
  long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  rows[r] = (int)r;
  float g = g32[r], h = h32[r];
  if (MODE == MODE_FIXED) {
    int gq = __float2int_rn(__fmul_rn(g, sc->gsf));
    int hq = const_hess ? sc->hq_const : __float2int_rn(__fmul_rn(h, sc->hsf));
    reinterpret_cast<int2*>(pairs)[r] = make_int2(gq, hq);
  } else {
    long long gr = row_offset + r;
    long long qg = mt_quantize_stochastic((double)g, sc->g_units, sc->g_lim, g_stream + (uint64_t)gr);
    long long qh = mt_quantize_stochastic((double)h, sc->h_units, sc->h_lim, h_stream + (uint64_t)gr);
    uint16_t packed = (uint16_t)((uint8_t)(int8_t)qg) | (uint16_t)((uint16_t)(uint8_t)qh << 8);
    reinterpret_cast<uint16_t*>(pairs)[r] = packed;
  }
}

// ---------------------------------------------------------------------------
// Tree control
// ---------------------------------------------------------------------------

__device__ __forceinline__ void clear_node(NodeRec& nd, double value, long long count) {
  nd.feature = -1;
  nd.thr = -1;
  nd.left = -1;
  nd.right = -1;
  nd.dleft = 0;
  nd.mbin = -1;
  nd.is_cat = 0;
  nd.pad = 0;
  nd.bits[0] = nd.bits[1] = nd.bits[2] = nd.bits[3] = 0;
  nd.value = value;
  nd.gain = 0.0;
  nd.count = count;
}

// Tree start: one leaf (the root) covering this device's rows in buffer 0.
__global__ void k_tree_init(TreeState* ts, long long n_local) {
  if (threadIdx.x != 0) return;
  ts->hdr.n_leaves = 1;
  ts->hdr.n_nodes = 1;
  ts->hdr.done = 0;
  ts->hdr.error = 0;
  ts->hdr.scan_ticket = 0;
  LeafRec& L = ts->leaves[0];
  L.node = 0;
  L.buf = 0;
  L.hist_slot = 0;
  L.depth = 0;
  L.begin = 0;
  L.count = n_local;
  L.split.found = 0;
  L.split.gain = 0.0;
  clear_node(ts->nodes[0], 0.0, 0);
  Plan& P = ts->plan;
  P.active = 1;
  P.n_children = 1;
  P.child_slot[0] = 0;
  P.child_hist[0] = 0;
  P.child_node[0] = 0;
  P.built_hist = 0;
  P.sib_hist = -1;
  P.built_is_left = 1;
  P.begin = 0;
  P.count = n_local;
  P.dst_buf = 0;
  P.cursor_left = (unsigned long long)n_local;
  P.cursor_right = 0;
}

// Leaf pick (growth_policy.mojo:659-677): max gain > 0, lowest frontier slot
// on ties.  Records the split in the tree and lays out the children.
// Runs on one 256-thread block.
__device__ void block_pick(TreeState* ts, const int* __restrict__ missing_bin, int num_leaves) {
  __shared__ double s_gain[256];
  __shared__ int s_slot[256];
  int t = threadIdx.x;
  if (ts->hdr.done || ts->hdr.n_leaves >= num_leaves) {
    if (t == 0) {
      ts->hdr.done = 1;
      ts->plan.active = 0;
    }
    return;
  }
  int nl = ts->hdr.n_leaves;
  double bg = 0.0;
  int bs = -1;
  for (int i = t; i < nl; i += 256) {
    const SplitRec& s = ts->leaves[i].split;
    if (s.found && s.gain > 0.0 && s.gain > bg) {
      bg = s.gain;
      bs = i;
    }
  }
  s_gain[t] = bg;
  s_slot[t] = bs;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (t < w) {
      double og = s_gain[t + w];
      int os = s_slot[t + w];
      if (os >= 0 && (s_slot[t] < 0 || og > s_gain[t] || (og == s_gain[t] && os < s_slot[t]))) {
        s_gain[t] = og;
        s_slot[t] = os;
      }
    }
    __syncthreads();
  }
  if (t != 0) return;
  Plan& P = ts->plan;
  int best = s_slot[0];
  if (best < 0) {
    ts->hdr.done = 1;
    P.active = 0;
    return;
  }
  LeafRec L = ts->leaves[best];
  const SplitRec& s = L.split;
  long long n_parent = ts->nodes[L.node].count;
  long long n_left = s.n_left;
  long long n_right = n_parent - n_left;
  int left_node = ts->hdr.n_nodes;
  int right_node = left_node + 1;
  ts->hdr.n_nodes += 2;
  NodeRec& pn = ts->nodes[L.node];
  pn.feature = s.feature;
  pn.gain = s.gain;
  pn.left = left_node;
  pn.right = right_node;
  pn.is_cat = s.is_cat;
  if (s.is_cat) {
    pn.thr = -1;
    pn.dleft = 0;
    pn.mbin = -1;
    for (int w = 0; w < 4; ++w) pn.bits[w] = s.bits[w];
  } else {
    pn.thr = s.bin;
    pn.dleft = s.default_left;
    pn.mbin = missing_bin[s.feature];
  }
  clear_node(ts->nodes[left_node], 0.0, n_left);
  clear_node(ts->nodes[right_node], 0.0, n_right);
  int new_slot = nl;
  int built_is_left = n_left <= n_right ? 1 : 0;
  P.active = 1;
  P.parent_slot = best;
  P.built_hist = new_slot;
  P.sib_hist = L.hist_slot;
  P.built_is_left = built_is_left;
  P.feature = s.feature;
  P.threshold = s.bin;
  P.default_left = s.default_left;
  P.missing_bin = s.is_cat ? -1 : missing_bin[s.feature];
  P.is_cat = s.is_cat;
  for (int w = 0; w < 4; ++w) P.bits[w] = s.bits[w];
  P.src_buf = L.buf;
  P.dst_buf = 1 - L.buf;
  P.depth = L.depth + 1;
  P.begin = L.begin;
  P.count = L.count;
  P.cursor_left = 0;
  P.cursor_right = 0;
  P.n_children = 2;
  P.child_slot[0] = best;
  P.child_slot[1] = new_slot;
  P.child_hist[0] = built_is_left ? new_slot : L.hist_slot;
  P.child_hist[1] = built_is_left ? L.hist_slot : new_slot;
  P.child_node[0] = left_node;
  P.child_node[1] = right_node;
  // Children take their frontier slots now; ranges are completed by the
  // finish kernel once the partition has counted this device's rows.
  for (int c = 0; c < 2; ++c) {
    LeafRec& C = ts->leaves[P.child_slot[c]];
    C.node = P.child_node[c];
    C.buf = P.dst_buf;
    C.hist_slot = P.child_hist[c];
    C.depth = P.depth;
    C.split.found = 0;
    C.split.gain = 0.0;
  }
  ts->hdr.n_leaves = nl + 1;
}

__device__ __forceinline__ bool goes_left(const Plan& P, int bin) {
  if (P.is_cat) {
    if (bin <= 0 || bin >= 256) return false;
    return (P.bits[bin >> 6] >> (bin & 63)) & 1ull;
  }
  if (bin == P.missing_bin) return P.default_left != 0;
  return bin <= P.threshold;
}

// Partition of the parent range into this device's left rows (from the front,
// each tile's rows in order) and right rows (from the back).  Also zeroes the
// histogram slot the built child will accumulate into.
template <typename PairT, int ITEMS>
__global__ void __launch_bounds__(256) k_partition(TreeState* ts, const uint8_t* __restrict__ bins_cm, long long n,
                                                   int* __restrict__ rows0, int* __restrict__ rows1,
                                                   PairT* __restrict__ pairs0, PairT* __restrict__ pairs1,
                                                   int* __restrict__ hist, long long slot_cells, int work_slot) {
  const Plan& P = ts->plan;
  if (!P.active) return;
  // zero the work slot the built child accumulates into
  {
    int* hs = hist + (long long)work_slot * slot_cells;
    long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = tid; i < slot_cells; i += stride) hs[i] = 0;
  }
  const int* src_rows = P.src_buf ? rows1 : rows0;
  int* dst_rows = P.src_buf ? rows0 : rows1;
  const PairT* src_pairs = P.src_buf ? pairs1 : pairs0;
  PairT* dst_pairs = P.src_buf ? pairs0 : pairs1;
  const uint8_t* col = bins_cm + (long long)P.feature * n;
  const long long begin = P.begin, count = P.count, end = P.begin + P.count;
  constexpr int TILE = 256 * ITEMS;
  long long n_tiles = (count + TILE - 1) / TILE;
  __shared__ int s_warp_l[8];
  __shared__ unsigned long long s_base_l, s_base_r;
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (long long tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
    long long t0 = begin + tile * TILE;
    int rr[ITEMS];
    PairT pp[ITEMS];
    bool valid[ITEMS], left[ITEMS];
    int my_l = 0, my_valid = 0;
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
      long long i = t0 + (long long)j * 256 + threadIdx.x;
      valid[j] = i < end;
      if (valid[j]) {
        rr[j] = src_rows[i];
        pp[j] = src_pairs[i];
        left[j] = goes_left(P, col[rr[j]]);
      } else {
        left[j] = false;
      }
      my_l += left[j];
      my_valid += valid[j];
    }
    // tile totals
    int wl = my_l, wv = my_valid;
    for (int k = 16; k > 0; k >>= 1) {
      wl += __shfl_xor_sync(0xffffffffu, wl, k);
      wv += __shfl_xor_sync(0xffffffffu, wv, k);
    }
    __shared__ int s_wv[8];
    if (lane == 0) {
      s_warp_l[w] = wl;
      s_wv[w] = wv;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int tl = 0, tv = 0;
      for (int k = 0; k < 8; ++k) {
        tl += s_warp_l[k];
        tv += s_wv[k];
      }
      s_base_l = atomicAdd(&ts->plan.cursor_left, (unsigned long long)tl);
      unsigned long long nr = (unsigned long long)(tv - tl);
      unsigned long long o = atomicAdd(&ts->plan.cursor_right, nr);
      s_base_r = (unsigned long long)end - o - nr;  // rights fill from the back
    }
    __syncthreads();
    // ranks in element order (j major, thread minor)
    int run_l = 0, run_r = 0;
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
      unsigned bl = __ballot_sync(0xffffffffu, left[j]);
      unsigned bv = __ballot_sync(0xffffffffu, valid[j]);
      unsigned br = bv & ~bl;
      __shared__ int s_cl[8], s_cr[8];
      if (lane == 0) {
        s_cl[w] = __popc(bl);
        s_cr[w] = __popc(br);
      }
      __syncthreads();
      int pre_l = 0, pre_r = 0, tot_l = 0, tot_r = 0;
      for (int k = 0; k < 8; ++k) {
        if (k < w) {
          pre_l += s_cl[k];
          pre_r += s_cr[k];
        }
        tot_l += s_cl[k];
        tot_r += s_cr[k];
      }
      unsigned below = (1u << lane) - 1u;
      if (valid[j]) {
        if (left[j]) {
          long long dst = begin + (long long)s_base_l + run_l + pre_l + __popc(bl & below);
          dst_rows[dst] = rr[j];
          dst_pairs[dst] = pp[j];
        } else {
          long long dst = (long long)s_base_r + run_r + pre_r + __popc(br & below);
          dst_rows[dst] = rr[j];
          dst_pairs[dst] = pp[j];
        }
      }
      run_l += tot_l;
      run_r += tot_r;
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------------------
// Histogram of one leaf: privatised shared-memory integer cells per CTA,
// flushed with global integer atomics.
// ---------------------------------------------------------------------------

// Shared-memory cells (32-bit atomics only; one CTA owns FG features):
//   QUANT           plane 0: g * 2^15 + count (signed, exact while a flush
//                   covers < 32768 rows and |sum g| < 2^16), plane 1: h
//   FIXED, const h  plane 0: g, plane 1: count
//   FIXED           plane 0: g, plane 1: h, plane 2: count
// Global cells are int32 [slot][F][3][B] (g, h, count): every sum is bounded
// by 2^30 + n (FIXED, quantized_gradient.mojo:98-99) or by B * n (QUANT).
constexpr int kQuantCountBits = 15;

struct HistJob {
  long long begin, count;
  int buf;
};

__device__ __forceinline__ HistJob hist_job(const Plan& P) {
  HistJob j;
  long long nl = (long long)P.cursor_left;
  if (P.built_is_left) {
    j.begin = P.begin;
    j.count = nl;
  } else {
    j.begin = P.begin + nl;
    j.count = P.count - nl;
  }
  j.buf = P.dst_buf;
  return j;
}

// CTAs of one feature group are launched in thread-block clusters of CS along
// grid y.  Each CTA accumulates its rows into its own shared-memory cells;
// the cluster then merges the CS copies through distributed shared memory
// (each CTA sums one CS-th of the cells across its peers) and only the
// merged cells reach global memory, with one int32 atomic per plane.  Small
// leaves activate fewer clusters (>= min_rows_per_cta rows per CTA); a cluster
// that has no rows exits as a whole.  Every build lands in the work slot;
// the scan kernel moves it into the child's slot after any cross-device sum.
template <int VPR, int MODE, bool CONST_H>
__global__ void __launch_bounds__(1024) k_hist(const Plan* __restrict__ plan, const uint8_t* __restrict__ bins_rm,
                                               int Fp, int F, int B, const int* __restrict__ rows0,
                                               const int* __restrict__ rows1, const void* __restrict__ pairs0,
                                               const void* __restrict__ pairs1, int* __restrict__ hist,
                                               long long slot_cells, long long rows_per_flush, int work_slot,
                                               int min_rows_per_cta) {
  namespace cg = cooperative_groups;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int FG = VPR * 16;
  constexpr int NPLANE = (MODE == MODE_FIXED && !CONST_H) ? 3 : 2;
  if (!plan->active) return;  // uniform across the grid
  const HistJob job = hist_job(*plan);
  if (job.count <= 0) return;
  cg::cluster_group cluster = cg::this_cluster();
  const int cs = (int)cluster.num_blocks();
  const int crank = (int)cluster.block_rank();
  const long long n_clusters = gridDim.y / cs;
  const long long cid = blockIdx.y / cs;
  const long long mrc = min_rows_per_cta;
  long long want = (job.count + mrc * cs - 1) / (mrc * cs);
  long long nce = want < n_clusters ? want : n_clusters;
  if (cid >= nce) return;  // the whole cluster leaves together
  const long long cchunk = (job.count + nce - 1) / nce;
  const long long c0 = job.begin + cid * cchunk;
  long long c1 = c0 + cchunk;
  if (c1 > job.begin + job.count) c1 = job.begin + job.count;
  const long long sub = (cchunk + cs - 1) / cs;  // rows per CTA, identical across the cluster
  const long long s = c0 + crank * sub;
  long long e = s + sub;
  if (e > c1) e = c1;
  const long long n_pass = (sub + rows_per_flush - 1) / rows_per_flush;
  const int f0 = blockIdx.x * FG;
  const int cells = FG * B;
  unsigned int* p0 = reinterpret_cast<unsigned int*>(smem_raw);
  unsigned int* p1 = p0 + cells;
  unsigned int* p2 = p1 + cells;
  const int* rows = job.buf ? rows1 : rows0;
  const void* pairs = job.buf ? pairs1 : pairs0;
  const int v = threadIdx.x % VPR;
  const int rsub = threadIdx.x / VPR;
  const int rpi = blockDim.x / VPR;  // rows per iteration
  // threads beyond rpi * VPR idle (blockDim need not divide by VPR); the last
  // group may extend past the row
  const bool vec_ok = f0 + v * 16 < Fp && rsub < rpi;
  int* hs = hist + (long long)work_slot * slot_cells;
  const int slice = (cells + cs - 1) / cs;
  const int m0 = crank * slice;
  const int m1 = m0 + slice < cells ? m0 + slice : cells;
  for (long long pass = 0; pass < n_pass; ++pass) {
    long long ps = s + pass * rows_per_flush;
    long long pe = ps + rows_per_flush < e ? ps + rows_per_flush : e;
    for (int c = threadIdx.x; c < cells * NPLANE; c += blockDim.x) p0[c] = 0u;
    __syncthreads();
    // two rows in flight per thread: both gathers are issued before the
    // shared-memory atomics of either, so the atomic pipe stays fed
    for (long long i = ps + rsub; vec_ok && i < pe; i += 2 * rpi) {
      const long long i2 = i + rpi;
      const bool two = i2 < pe;
      int r0 = __ldg(rows + i);
      int r1 = two ? __ldg(rows + i2) : r0;
      unsigned int a0[2], a1[2];
      const unsigned int a2 = 1u;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        long long ii = u == 0 ? i : (two ? i2 : i);
        if (MODE == MODE_QUANT) {
          uint16_t pr = __ldg(reinterpret_cast<const uint16_t*>(pairs) + ii);
          int g = (int)(int8_t)(pr & 0xff);
          a0[u] = (unsigned int)(g * (1 << kQuantCountBits) + 1);
          a1[u] = (unsigned int)(pr >> 8);
        } else {
          int2 pr = __ldg(reinterpret_cast<const int2*>(pairs) + ii);
          a0[u] = (unsigned int)pr.x;
          a1[u] = CONST_H ? 1u : (unsigned int)pr.y;
        }
      }
      uint4 bv0 = __ldg(reinterpret_cast<const uint4*>(bins_rm + (long long)r0 * Fp + f0 + v * 16));
      uint4 bv1 = __ldg(reinterpret_cast<const uint4*>(bins_rm + (long long)r1 * Fp + f0 + v * 16));
      const int base = v * 16 * B;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (u == 1 && !two) break;
        const uint4 bv = u == 0 ? bv0 : bv1;
        const unsigned int w[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          int cell = base + k * B + (int)((w[k >> 2] >> (8 * (k & 3))) & 0xffu);
          atomicAdd(&p0[cell], a0[u]);
          atomicAdd(&p1[cell], a1[u]);
          if (NPLANE == 3) atomicAdd(&p2[cell], a2);
        }
      }
    }
    cluster.sync();
    for (int c = m0 + threadIdx.x; c < m1; c += blockDim.x) {
      int fl = c / B;
      int f = f0 + fl;
      if (f >= F) continue;
      int g = 0, h = 0, cnt = 0;
      for (int rk = 0; rk < cs; ++rk) {
        const unsigned int* q0 = cluster.map_shared_rank(p0, rk);
        const unsigned int* q1 = q0 + cells;
        if (MODE == MODE_QUANT) {
          unsigned int x = q0[c];
          cnt += (int)(x & ((1u << kQuantCountBits) - 1u));
          g += (int)x >> kQuantCountBits;
          h += (int)q1[c];
        } else if (CONST_H) {
          g += (int)q0[c];
          cnt += (int)q1[c];
        } else {
          g += (int)q0[c];
          h += (int)q1[c];
          cnt += (int)q1[c + cells];
        }
      }
      if (cnt == 0) continue;
      int bin = c - fl * B;
      int* cellp = hs + (f * 3) * B + bin;
      atomicAdd(cellp, g);
      if (!(MODE == MODE_FIXED && CONST_H)) atomicAdd(cellp + B, h);
      atomicAdd(cellp + 2 * B, cnt);
    }
    cluster.sync();  // peers finished reading before anyone re-zeroes
  }
}

// ---------------------------------------------------------------------------
// Subtract + split scan: one warp per (child, active feature).
// ---------------------------------------------------------------------------

struct ScanParams {
  int n_active;
  int B;
  int mode;
  int const_hess;
  int min_data_in_leaf;
  double lambda_l2, lambda_l1, min_child_hess;
  int max_cat_to_onehot, max_cat_threshold;
  double cat_smooth, cat_l2;
  int min_data_per_group;
};

__device__ __forceinline__ double soft_l1(double s, double l1) {
  if (l1 <= 0.0) return s;
  double mag = fabs(s) - l1;
  if (mag <= 0.0) return 0.0;
  return s > 0.0 ? mag : -mag;
}

__device__ __forceinline__ double leaf_score(double g, double h, double l1, double l2) {
  double t = soft_l1(g, l1);
  return t * t / (h + l2);
}

// Dequantize an exact integer sum.
__device__ __forceinline__ double deq(long long q, int mode, double inv, double units) {
  return mode == MODE_FIXED ? (double)q * inv : (double)q / units;
}

constexpr int kScanThreads = 256;  // one thread per bin (B <= 256)

// Block-wide inclusive sum of three int64 values per thread (bin order).
__device__ __forceinline__ void block_scan3(long long& a, long long& b, long long& c, long long* sw /*[3][8]*/) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int k = 1; k < 32; k <<= 1) {
    long long oa = __shfl_up_sync(0xffffffffu, a, k);
    long long ob = __shfl_up_sync(0xffffffffu, b, k);
    long long oc = __shfl_up_sync(0xffffffffu, c, k);
    if (lane >= k) {
      a += oa;
      b += ob;
      c += oc;
    }
  }
  if (lane == 31) {
    sw[w] = a;
    sw[8 + w] = b;
    sw[16 + w] = c;
  }
  __syncthreads();
  long long pa = 0, pb = 0, pc = 0;
  for (int q = 0; q < w; ++q) {
    pa += sw[q];
    pb += sw[8 + q];
    pc += sw[16 + q];
  }
  a += pa;
  b += pb;
  c += pc;
}

// One block per (child, active feature), one thread per bin: sibling
// subtraction, exact integer prefix sums, the reference gain per candidate
// threshold, and a block arg-max that keeps the serial scan's tie rule
// (first maximum in bin order, missing-left candidate before default-right).
__device__ void scan_body(TreeState* __restrict__ ts, int* __restrict__ hist, long long slot_cells,
                          const int* __restrict__ feats, const int* __restrict__ missing_bin,
                          const int* __restrict__ n_cats, const RoundScales* __restrict__ sc, ScanParams sp,
                          FeatBest* __restrict__ out, int root, int work_slot) {
  __shared__ int s_cells[3][256];
  __shared__ long long s_w[24];
  __shared__ double s_gain[8];
  __shared__ int s_key[8];
  __shared__ long long s_nl[8];
  const Plan& P = ts->plan;
  if (!P.active) return;  // uniform
  const int c = blockIdx.x;
  if (c >= P.n_children) return;  // uniform
  const int j = blockIdx.y;
  const int t = threadIdx.x;
  const int lane = t & 31, w = t >> 5;
  const int B = sp.B;
  const int f = feats[j];
  int* hs = hist + (long long)P.child_hist[c] * slot_cells + (long long)f * 3 * B;
  const bool built = root || P.child_hist[c] != P.sib_hist;
  const int* wk = hist + (long long)work_slot * slot_cells + (long long)f * 3 * B;
  const int mode = sp.mode;
  // built child: the (reduced) work slot; sibling: parent - built, in place
  int vg = 0, vh = 0, vc = 0;
  if (t < B) {
    int wg = __ldcg(wk + t), wh = __ldcg(wk + B + t), wc = __ldcg(wk + 2 * B + t);
    if (built) {
      vg = wg;
      vh = wh;
      vc = wc;
    } else {
      vg = __ldcg(hs + t) - wg;
      vh = __ldcg(hs + B + t) - wh;
      vc = __ldcg(hs + 2 * B + t) - wc;
    }
    hs[t] = vg;
    hs[B + t] = vh;
    hs[2 * B + t] = vc;
    if (sp.const_hess && mode == MODE_FIXED) vh = (int)((long long)sc->hq_const * vc);
  }
  s_cells[0][t] = vg;
  s_cells[1][t] = vh;
  s_cells[2][t] = vc;
  long long Lg = vg, Lh = vh, Lc = vc;  // inclusive prefix through bin t
  block_scan3(Lg, Lh, Lc, s_w);
  __shared__ long long s_tot[3];
  if (t == kScanThreads - 1) {
    s_tot[0] = Lg;
    s_tot[1] = Lh;
    s_tot[2] = Lc;
  }
  __syncthreads();
  const long long Tg = s_tot[0], Th = s_tot[1], Tc = s_tot[2];
  if (j == 0 && t == 0) {
    ts->totals[c].g = Tg;
    ts->totals[c].h = Th;
    ts->totals[c].c = Tc;
  }
  const double g_inv = sc->g_inv, h_inv = sc->h_inv, gu = sc->g_units, hu = sc->h_units;
  const double l1 = sp.lambda_l1, l2 = sp.lambda_l2, mch = sp.min_child_hess;
  const long long mdl = sp.min_data_in_leaf;
  const double tg = deq(Tg, mode, g_inv, gu), th = deq(Th, mode, h_inv, hu);
  FeatBest fb;
  fb.gain = 0.0;
  fb.bin = -1;
  fb.flags = 0;
  fb.n_left = 0;
  fb.bits[0] = fb.bits[1] = fb.bits[2] = fb.bits[3] = 0;
  if (n_cats[f] >= 0) {
    // categorical: serial search on thread 0 (categorical.mojo:478-780) over
    // the exact per-category sums
    if (t == 0) {
      int n_cat = n_cats[f];
      double parent = leaf_score(tg, th, l1, l2);
      if (n_cat >= 2 && n_cat + 1 <= sp.max_cat_to_onehot) {
        for (int q = 1; q <= n_cat && q < B; ++q) {
          long long qg = s_cells[0][q], qh = s_cells[1][q], cc = s_cells[2][q];
          double lgv = deq(qg, mode, g_inv, gu), lhv = deq(qh, mode, h_inv, hu);
          if (cc < mdl || lhv < mch) continue;
          if (Tc - cc < mdl) continue;
          double rh = mode == MODE_FIXED ? th - lhv : deq(Th - qh, mode, h_inv, hu);
          if (rh < mch) continue;
          double rg = mode == MODE_FIXED ? tg - lgv : deq(Tg - qg, mode, g_inv, gu);
          double gain = leaf_score(lgv, lhv, l1, l2) + leaf_score(rg, rh, l1, l2) - parent;
          if (gain > fb.gain) {
            fb.gain = gain;
            fb.flags = 1 | 4;
            fb.n_left = cc;
            fb.bits[0] = fb.bits[1] = fb.bits[2] = fb.bits[3] = 0;
            fb.bits[q >> 6] |= 1ull << (q & 63);
          }
        }
      } else if (n_cat >= 2) {
        int cand[256];
        double key[256];
        int used = 0;
        for (int q = 1; q <= n_cat && q < B; ++q) {
          if (!((double)s_cells[2][q] >= sp.cat_smooth)) continue;
          double gv = deq(s_cells[0][q], mode, g_inv, gu);
          double hv = deq(s_cells[1][q], mode, h_inv, hu);
          double kv = gv / (hv + sp.cat_smooth);
          int p = used;  // insertion keeps equal keys in category order (stable)
          while (p > 0 && key[p - 1] > kv) {
            key[p] = key[p - 1];
            cand[p] = cand[p - 1];
            --p;
          }
          key[p] = kv;
          cand[p] = q;
          ++used;
        }
        if (used >= 2) {
          int max_num_cat = sp.max_cat_threshold < (used + 1) / 2 ? sp.max_cat_threshold : (used + 1) / 2;
          if (max_num_cat < 0) max_num_cat = 0;
          double cl2 = l2 + sp.cat_l2;
          for (int d = 0; d < 2; ++d) {
            int dir = d == 0 ? 1 : -1;
            int start = d == 0 ? 0 : used - 1;
            int pos = start;
            long long cnt_group = 0, qg = 0, qh = 0, qc = 0;
            int steps = used < max_num_cat ? used : max_num_cat;
            for (int i = 0; i < steps; ++i) {
              int q = cand[pos];
              pos += dir;
              qg += s_cells[0][q];
              qh += s_cells[1][q];
              qc += s_cells[2][q];
              cnt_group += s_cells[2][q];
              double lgv = deq(qg, mode, g_inv, gu), lhv = deq(qh, mode, h_inv, hu);
              if (qc < mdl || lhv < mch) continue;
              long long rc = Tc - qc;
              if (rc < mdl || rc < sp.min_data_per_group) break;
              double rh = mode == MODE_FIXED ? th - lhv : deq(Th - qh, mode, h_inv, hu);
              if (rh < mch) break;
              if (cnt_group < sp.min_data_per_group) continue;
              cnt_group = 0;
              double rg = mode == MODE_FIXED ? tg - lgv : deq(Tg - qg, mode, g_inv, gu);
              double gain = leaf_score(lgv, lhv, l1, cl2) + leaf_score(rg, rh, l1, cl2) - parent;
              if (gain > fb.gain) {
                fb.gain = gain;
                fb.flags = 1 | 4;
                fb.n_left = qc;
                fb.bits[0] = fb.bits[1] = fb.bits[2] = fb.bits[3] = 0;
                int q2 = start;
                for (int k = 0; k <= i; ++k) {
                  int tt = cand[q2];
                  fb.bits[tt >> 6] |= 1ull << (tt & 63);
                  q2 += dir;
                }
              }
            }
          }
        }
      }
      out[(long long)c * sp.n_active + j] = fb;
    }
    return;
  }
  const int mb = missing_bin[f];
  const int n_scan = mb >= 0 ? mb : B;
  long long mg = 0, mh = 0, mc = 0;
  if (mb >= 0) {
    mg = s_cells[0][mb];
    mh = s_cells[1][mb];
    mc = s_cells[2][mb];
  }
  const double pg = soft_l1(tg, l1);
  const double parent = pg * pg / (th + l2);
  const double parent_q = leaf_score(tg, th, l1, l2);
  double best_gain = 0.0;
  int best_key = 0x7fffffff;  // 2*bin + order
  long long best_nl = 0;
  const int b = t;
  if (b < n_scan && !(b == n_scan - 1 && mc == 0)) {
    if (mb >= 0) {
      long long Dg = Lg + mg, Dh = Lh + mh, Dc = Lc + mc;
      double dlg = deq(Dg, mode, g_inv, gu), dlh = deq(Dh, mode, h_inv, hu);
      double drg = mode == MODE_FIXED ? tg - dlg : deq(Tg - Dg, mode, g_inv, gu);
      double drh = mode == MODE_FIXED ? th - dlh : deq(Th - Dh, mode, h_inv, hu);
      if (!(dlh < mch || drh < mch || Dc < mdl || Tc - Dc < mdl)) {
        double gain;
        if (mode == MODE_FIXED) {
          double tl = soft_l1(dlg, l1), tr = soft_l1(drg, l1);
          gain = tl * tl / (dlh + l2) + tr * tr / (drh + l2) - parent;
        } else {
          gain = leaf_score(dlg, dlh, l1, l2) + leaf_score(drg, drh, l1, l2) - parent_q;
        }
        if (gain > best_gain) {
          best_gain = gain;
          best_key = 2 * b;
          best_nl = Dc;
        }
      }
    }
    if (mb < 0 || mc > 0) {
      double lgv = deq(Lg, mode, g_inv, gu), lhv = deq(Lh, mode, h_inv, hu);
      double rg = mode == MODE_FIXED ? tg - lgv : deq(Tg - Lg, mode, g_inv, gu);
      double rh = mode == MODE_FIXED ? th - lhv : deq(Th - Lh, mode, h_inv, hu);
      if (!(lhv < mch || rh < mch || Lc < mdl || Tc - Lc < mdl)) {
        double gain;
        if (mode == MODE_FIXED) {
          double tl = soft_l1(lgv, l1), tr = soft_l1(rg, l1);
          gain = tl * tl / (lhv + l2) + tr * tr / (rh + l2) - parent;
        } else {
          gain = leaf_score(lgv, lhv, l1, l2) + leaf_score(rg, rh, l1, l2) - parent_q;
        }
        if (gain > best_gain) {
          best_gain = gain;
          best_key = 2 * b + 1;
          best_nl = Lc;
        }
      }
    }
  }
  // block arg-max: higher gain, then lower key (earlier in the serial scan)
  for (int k = 16; k > 0; k >>= 1) {
    double og = __shfl_xor_sync(0xffffffffu, best_gain, k);
    int ok = __shfl_xor_sync(0xffffffffu, best_key, k);
    long long on = __shfl_xor_sync(0xffffffffu, best_nl, k);
    if (og > best_gain || (og == best_gain && ok < best_key)) {
      best_gain = og;
      best_key = ok;
      best_nl = on;
    }
  }
  if (lane == 0) {
    s_gain[w] = best_gain;
    s_key[w] = best_key;
    s_nl[w] = best_nl;
  }
  __syncthreads();
  if (t == 0) {
    for (int q = 1; q < kScanThreads / 32; ++q) {
      if (s_gain[q] > best_gain || (s_gain[q] == best_gain && s_key[q] < best_key)) {
        best_gain = s_gain[q];
        best_key = s_key[q];
        best_nl = s_nl[q];
      }
    }
    if (best_key != 0x7fffffff && best_gain > 0.0) {
      fb.gain = best_gain;
      fb.bin = best_key >> 1;
      fb.flags = 1 | ((best_key & 1) ? 0 : 2);
      fb.n_left = best_nl;
    }
    out[(long long)c * sp.n_active + j] = fb;
  }
}

// Cross-feature fold (ascending feature, strict >), guards, leaf values and
// the children's ranges.
__device__ void block_finish(TreeState* __restrict__ ts, const FeatBest* __restrict__ fbs,
                             const int* __restrict__ feats, const RoundScales* __restrict__ sc, ScanParams sp,
                             int root) {
  __shared__ double s_gain[256];
  __shared__ int s_j[256];
  Plan& P = ts->plan;
  if (!P.active) return;
  int t = threadIdx.x;
  for (int c = 0; c < P.n_children; ++c) {
    double bg = 0.0;
    int bj = -1;
    for (int j = t; j < sp.n_active; j += 256) {
      const FeatBest& fb = fbs[(long long)c * sp.n_active + j];
      if ((fb.flags & 1) && fb.gain > bg) {
        bg = fb.gain;
        bj = j;
      }
    }
    s_gain[t] = bg;
    s_j[t] = bj;
    __syncthreads();
    for (int w = 128; w > 0; w >>= 1) {
      if (t < w) {
        double og = s_gain[t + w];
        int oj = s_j[t + w];
        if (oj >= 0 && (s_j[t] < 0 || og > s_gain[t] || (og == s_gain[t] && oj < s_j[t]))) {
          s_gain[t] = og;
          s_j[t] = oj;
        }
      }
      __syncthreads();
    }
    if (t == 0) {
      LeafRec& L = ts->leaves[P.child_slot[c]];
      const ChildTotals tot = ts->totals[c];
      long long n_rows = tot.c;
      SplitRec s;
      s.found = 0;
      s.gain = 0.0;
      s.feature = -1;
      s.bin = -1;
      s.default_left = 0;
      s.is_cat = 0;
      s.pad = 0;
      s.n_left = 0;
      s.bits[0] = s.bits[1] = s.bits[2] = s.bits[3] = 0;
      int bj = s_j[0];
      if (bj >= 0 && !(n_rows < 2 * (long long)sp.min_data_in_leaf || n_rows < 2)) {
        const FeatBest& fb = fbs[(long long)c * sp.n_active + bj];
        s.found = 1;
        s.gain = fb.gain;
        s.feature = feats[bj];
        s.bin = fb.bin;
        s.default_left = (fb.flags & 2) ? 1 : 0;
        s.is_cat = (fb.flags & 4) ? 1 : 0;
        s.n_left = fb.n_left;
        for (int q = 0; q < 4; ++q) s.bits[q] = fb.bits[q];
      }
      L.split = s;
      double gd = sp.mode == MODE_FIXED ? (double)tot.g * sc->g_inv : (double)tot.g / sc->g_units;
      double hd = sp.mode == MODE_FIXED ? (double)tot.h * sc->h_inv : (double)tot.h / sc->h_units;
      double value = -soft_l1(gd, sp.lambda_l1) / (hd + sp.lambda_l2);
      NodeRec& nd = ts->nodes[P.child_node[c]];
      nd.value = value;
      nd.count = n_rows;
      if (!root) {
        long long nl = (long long)P.cursor_left;
        if (c == 0) {
          L.begin = P.begin;
          L.count = nl;
        } else {
          L.begin = P.begin + nl;
          L.count = P.count - nl;
        }
      }
    }
    __syncthreads();
  }
}

// Subtract + scan of every (child, active feature); the last block to finish
// then folds the per-feature bests (block_finish) and picks the next leaf to
// split (block_pick), so one split costs three launches: partition,
// histogram, scan.
__global__ void __launch_bounds__(kScanThreads) k_scan(TreeState* __restrict__ ts, int* __restrict__ hist,
                                                           long long slot_cells, const int* __restrict__ feats,
                                                           const int* __restrict__ missing_bin,
                                                           const int* __restrict__ n_cats,
                                                           const RoundScales* __restrict__ sc, ScanParams sp,
                                                           FeatBest* __restrict__ out, int root, int work_slot,
                                                           int num_leaves) {
  __shared__ int s_last;
  scan_body(ts, hist, slot_cells, feats, missing_bin, n_cats, sc, sp, out, root, work_slot);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned int total = gridDim.x * gridDim.y;
    unsigned int ticket = atomicAdd(&ts->hdr.scan_ticket, 1u);
    s_last = ticket == total - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  block_finish(ts, out, feats, sc, sp, root);
  __syncthreads();
  block_pick(ts, missing_bin, num_leaves);
  __syncthreads();
  if (threadIdx.x == 0) ts->hdr.scan_ticket = 0;
}

// After the last split: leaves sorted by range start, for the raw update.
__global__ void __launch_bounds__(1024) k_leaf_table(const TreeState* __restrict__ ts, long long* __restrict__ begins,
                                                     int* __restrict__ order) {
  int nl = ts->hdr.n_leaves;
  // Sort key: range start, then empty leaves before the non-empty one that
  // shares the start, then slot.  The raw update's search for the last start
  // <= position then always lands on the leaf that owns the position.
  for (int i = threadIdx.x; i < nl; i += blockDim.x) {
    long long bi = ts->leaves[i].begin * 2 + (ts->leaves[i].count > 0 ? 1 : 0);
    int rank = 0;
    for (int k = 0; k < nl; ++k) {
      long long bk = ts->leaves[k].begin * 2 + (ts->leaves[k].count > 0 ? 1 : 0);
      if (bk < bi || (bk == bi && k < i)) ++rank;
    }
    begins[rank] = ts->leaves[i].begin;
    order[rank] = i;
  }
}

// raw[row * K + k] = fma(lr, value(leaf of row), raw[row * K + k])
// (boosting.mojo:1991-2111, explicit fused multiply-add).
__global__ void k_update_raw(const TreeState* __restrict__ ts, const long long* __restrict__ begins,
                             const int* __restrict__ order, const int* __restrict__ rows0,
                             const int* __restrict__ rows1, double* __restrict__ raw, long long n, int K, int k,
                             double lr) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int nl = ts->hdr.n_leaves;
  int lo = 0, hi = nl - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (begins[mid] <= i) lo = mid;
    else hi = mid - 1;
  }
  const LeafRec* L = &ts->leaves[order[lo]];
  const int* rows = L->buf ? rows1 : rows0;
  int r = rows[i];
  double v = ts->nodes[L->node].value;
  double* p = raw + (long long)r * K + k;
  *p = fma(lr, v, *p);
}

}  // namespace
}  // namespace mtb
