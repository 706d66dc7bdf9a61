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

#include <type_traits>

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

// Block maxima of two non-negative values folded into the round's scales: one
// atomic per block and value (same-address atomics from every warp would
// serialise in L2).  sm holds 32 doubles; every thread of the block calls it.
__device__ __forceinline__ void block_max_to(double ag, double ah, double* sm, RoundScales* sc) {
  __shared__ double smh[32];
  for (int k = 16; k > 0; k >>= 1) {
    ag = fmax(ag, __shfl_down_sync(0xffffffffu, ag, k));
    ah = fmax(ah, __shfl_down_sync(0xffffffffu, ah, k));
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) {
    sm[w] = ag;
    smh[w] = ah;
  }
  __syncthreads();
  if (w == 0) {
    ag = lane < (int)(blockDim.x >> 5) ? sm[lane] : 0.0;
    ah = lane < (int)(blockDim.x >> 5) ? smh[lane] : 0.0;
    for (int k = 16; k > 0; k >>= 1) {
      ag = fmax(ag, __shfl_down_sync(0xffffffffu, ag, k));
      ah = fmax(ah, __shfl_down_sync(0xffffffffu, ah, k));
    }
    if (lane == 0) {
      atomic_max_nonneg(&sc->g_total, ag);
      atomic_max_nonneg(&sc->h_total, ah);
    }
  }
}

// Per-row derivatives for L2 / logistic, narrowed to Float32.  1024 threads,
// one row of each 1024-row chunk each.  FIXED mode writes per-chunk pairwise
// |g|, |h| partials; QUANT mode folds max |g|, max |h| into the round's
// scales.
__global__ void __launch_bounds__(1024) k_grad(const double* __restrict__ raw, const double* __restrict__ y,
                                               float* __restrict__ g32, float* __restrict__ h32,
                                               long long n, int objective, int mode,
                                               double* __restrict__ part_g, double* __restrict__ part_h,
                                               RoundScales* sc) {
  // Each block walks 1024-row chunks c = blockIdx.x, + gridDim.x, ... with
  // the next chunk's raw scores and labels loaded while this one is
  // computed; the fixed-point partial sums stay one per 1024-row chunk (the
  // pairwise order the scale depends on), the quantized maxima are folded
  // over the block's chunks before one atomic per block.
  __shared__ double sm[32];
  const long long n_chunks = (n + 1023) / 1024;
  double mg = 0.0, mh = 0.0;
  double nr = 0.0, ny = 0.0;
  long long c = blockIdx.x;
  if (c < n_chunks) {
    const long long r = c * 1024 + threadIdx.x;
    if (r < n) {
      nr = raw[r];
      ny = y[r];
    }
  }
  for (; c < n_chunks; c += gridDim.x) {
    const double rr = nr, yy = ny;
    const long long r = c * 1024 + threadIdx.x;
    if (c + gridDim.x < n_chunks) {
      const long long rn = r + (long long)gridDim.x * 1024;
      if (rn < n) {
        nr = raw[rn];
        ny = y[rn];
      }
    }
    double g = 0.0, h = 0.0;
    if (r < n) {
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
      if (threadIdx.x == 0) part_g[c] = sg;
      double sh = block_pairwise_1024(fabs(h), sm);
      if (threadIdx.x == 0) part_h[c] = sh;
    } else {
      mg = fmax(mg, fabs(g));
      mh = fmax(mh, fabs(h));
    }
  }
  if (mode != MODE_FIXED) block_max_to(mg, mh, sm, sc);
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
    block_max_to(fabs(g), fabs(h), sm, sc);
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
                         int quant_bins, int wide) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  sc->wide = wide;
  if (mode == MODE_FIXED) {
    sc->g_total = *fixed_g;
    sc->h_total = *fixed_h;
    sc->gsf = wide ? mt_fixed_point_scale52(sc->g_total) : mt_fixed_point_scale(sc->g_total);
    sc->hsf = wide ? mt_fixed_point_scale52(sc->h_total) : mt_fixed_point_scale(sc->h_total);
    sc->g_inv = 1.0 / (double)sc->gsf;
    sc->h_inv = 1.0 / (double)sc->hsf;
    sc->hq_const = wide ? 0 : __float2int_rn(__fmul_rn(1.0f, sc->hsf));
    sc->hq_const64 = wide ? __double2ll_rn(1.0 * (double)sc->hsf) : 0;
  } else {
    double gmax = sc->g_total < 1e-12 ? 1e-12 : sc->g_total;
    double hmax = sc->h_total < 1e-12 ? 1e-12 : sc->h_total;
    sc->g_lim = (double)(quant_bins / 2);
    sc->h_lim = const_hess ? 1.0 : (double)quant_bins;
    sc->g_units = sc->g_lim / gmax;
    sc->h_units = const_hess ? 1.0 / hmax : sc->h_lim / hmax;
    // reciprocals for the divide-free dequantization (deq)
    sc->g_inv = 1.0 / sc->g_units;
    sc->h_inv = 1.0 / sc->h_units;
  }
}

// Tree start: identity row list and the quantized pair of every row.
// WIDE (fixed point with the 2^52 bound): Int64(rint(f64(g) * s)), exact
// product, ties to even; pairs are longlong2.
template <int MODE, bool WIDE = false>
__global__ void k_quantize(const float* __restrict__ g32, const float* __restrict__ h32, long long n,
                           long long row_offset, const RoundScales* __restrict__ sc, int const_hess,
                           uint64_t g_stream, uint64_t h_stream, int* __restrict__ rows, void* __restrict__ pairs) {
  long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  rows[r] = (int)r;
  float g = g32[r], h = h32[r];
  if (MODE == MODE_FIXED && WIDE) {
    const long long gq = __double2ll_rn(__dmul_rn((double)g, (double)sc->gsf));
    const long long hq = const_hess ? sc->hq_const64 : __double2ll_rn(__dmul_rn((double)h, (double)sc->hsf));
    reinterpret_cast<longlong2*>(pairs)[r] = make_longlong2(gq, hq);
  } else if (MODE == MODE_FIXED) {
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
// Tree control: speculative leaf batching
//
// The reference grows a tree one split at a time (growth_policy.mojo:659-677,
// tree.mojo:3767-4256): pick the frontier leaf with the largest gain, split
// it, compute both children's best splits, repeat.  A leaf's children and
// their best splits depend only on that leaf's rows, so they can be computed
// before the leaf is picked.  Each iteration here therefore expands up to K
// frontier leaves at once (the K largest gains, never more than the remaining
// leaf budget): one partition launch, one histogram launch and one scan
// launch for all of them.  The scan's last block then replays the reference's
// sequential pick loop over the known gains and commits every split whose
// children are already computed, in exactly the reference's order (node ids,
// frontier slots and tie rules unchanged), stopping at the first pick that
// still needs an expansion.  The committed tree is identical to the
// sequential one; a leaf expanded but never committed (the leaf budget ran
// out first) stays a leaf.
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

__device__ __forceinline__ void clear_split(SplitRec& s) {
  s.found = 0;
  s.gain = 0.0;
  s.feature = -1;
  s.bin = -1;
  s.default_left = 0;
  s.is_cat = 0;
  s.pad = 0;
  s.n_left = 0;
  s.bits[0] = s.bits[1] = s.bits[2] = s.bits[3] = 0;
}

// Tree start: the root is leaf 0 / node 0 / frontier slot 0 / histogram slot
// 0, covering this device's rows in buffer 0; the first batch builds it.
__global__ void k_tree_init(TreeState* ts, long long n_local) {
  if (threadIdx.x != 0) return;
  TreeHeader& H = ts->hdr;
  H.n_leaves = 1;
  H.n_nodes = 1;
  H.done = 0;
  H.error = 0;
  H.scan_ticket = 0;
  H.n_pool = 1;
  H.n_hist = 1;
  H.iterations = 0;
  H.pick_steps = 0;
  LeafRec& L = ts->pool[0];
  L.node = 0;
  L.parent = -1;
  L.buf = 0;
  L.hist_slot = 0;
  L.state = 0;
  L.child[0] = L.child[1] = -1;
  L.exp_buf = 0;
  L.begin = 0;
  L.count = n_local;
  L.gcount = 0;
  L.value = 0.0;
  clear_split(L.split);
  ts->slot_leaf[0] = 0;
  LeafInfo& I0 = ts->info[0];
  I0.gain = -1.0;
  I0.child[0] = I0.child[1] = -1;
  I0.expanded = 0;
  I0.pad = 0;
  for (int c = 0; c < 2 * kMaxBatch; ++c) ts->child_done[c] = 0;
  clear_node(ts->nodes[0], 0.0, 0);
  Batch& Bt = ts->batch;
  Bt.n_items = 1;
  Bt.root = 1;
  Bt.n_tiles = 0;
  BatchItem& P = Bt.items[0];
  P.leaf = 0;
  P.child[0] = 0;
  P.child[1] = -1;
  P.built_is_left = 1;
  P.work = 0;
  P.built_hist = 0;
  P.sib_hist = -1;
  P.src_buf = 0;
  P.dst_buf = 0;
  P.begin = 0;
  P.count = n_local;
  P.tile0 = 0;
  P.cursor_left = (unsigned long long)n_local;
  P.cursor_right = 0;
}

__device__ __forceinline__ bool goes_left(const BatchItem& P, int bin) {
  if (P.is_cat) {
    if (bin <= 0 || bin >= 256) return false;
    return (P.bits[bin >> 6] >> (bin & 63)) & 1ull;
  }
  if (bin == P.missing_bin) return P.default_left != 0;
  return bin <= P.threshold;
}

// Partition of every expanded leaf's range into this device's left rows (from
// the front, each tile's rows in order) and right rows (from the back), into
// the other ping-pong buffer.  Tiles of all items are one flat index space.
// Also zeroes the work slots the built children accumulate into.
// Programmatic dependent launch.  The iteration kernels (partition ->
// histogram -> scan -> commit -> next partition) can be launched with the
// programmatic-stream-serialization attribute (MOJOTREES_PDL=1), so a
// kernel's CTAs may be scheduled while its predecessor still runs.  Each first waits here for the
// predecessor grid to complete and its memory to be visible, before touching
// any data, and then lets its own dependents be scheduled.  Without the
// attribute both instructions return at once.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename PairT, int ITEMS>
__global__ void __launch_bounds__(256) k_partition(TreeState* ts, const uint8_t* __restrict__ bins_cm, long long n,
                                                   int* __restrict__ rows0, int* __restrict__ rows1,
                                                   PairT* __restrict__ pairs0, PairT* __restrict__ pairs1,
                                                   int* __restrict__ hist, long long slot_cells, int work_base) {
  pdl_enter();
  Batch& Bt = ts->batch;
  const int n_items = Bt.n_items;
  if (n_items == 0) return;
  {
    int* hs = hist + (long long)work_base * slot_cells;
    long long total = (long long)n_items * slot_cells;
    long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = tid; i < total; i += stride) hs[i] = 0;
  }
  if (Bt.root) return;  // the root's rows are already in place
  // the batch's items, staged with one coalesced copy: every tile looks up
  // its item and reads its split (from global memory each lookup would be a
  // chain of dependent L2 round trips)
  __shared__ BatchItem s_items[kMaxBatch];
  {
    const int* src = reinterpret_cast<const int*>(Bt.items);
    int* dst = reinterpret_cast<int*>(s_items);
    const int words = n_items * (int)(sizeof(BatchItem) / sizeof(int));
    for (int i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();
  constexpr int TILE = 256 * ITEMS;
  // Per-warp left/right counts of each item row of a tile, and the tile's
  // cursor bases; double-buffered by tile parity, so a tile needs two block
  // barriers: counts written -> cursors claimed -> scatter.  (A warp can only
  // refill a buffer after both barriers of the next tile, which every warp
  // reaches only after finishing its reads of this one.)
  __shared__ int s_cl[2][ITEMS][8], s_cr[2][ITEMS][8];
  __shared__ unsigned long long s_base_l[2], s_base_r[2];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const unsigned below = (1u << lane) - 1u;
  int par = 0;
  // exclusive prefixes of the (item row, warp) counts in element order,
  // written over the counts by warp 0 between the two barriers
  constexpr int E = ITEMS * 8;
  constexpr int PER = (E + 31) / 32;
  // The tile loop is software-pipelined: the next tile's row ids and pairs
  // are loaded while this tile's ballots, cursor atomics and scatter run.
  auto item_of = [&](long long tile) {
    int it = 0, hi = n_items - 1;  // the last item whose first tile is <= tile
    while (it < hi) {
      const int mid = (it + hi + 1) >> 1;
      if (s_items[mid].tile0 <= tile) it = mid;
      else hi = mid - 1;
    }
    return it;
  };
  int rr[ITEMS], nrr[ITEMS] = {};
  PairT pp[ITEMS], npp[ITEMS] = {};
  auto load_tile = [&](long long tile, int (&r)[ITEMS], PairT (&q)[ITEMS]) {
    const BatchItem& P = s_items[item_of(tile)];
    const int* src_rows = P.src_buf ? rows1 : rows0;
    const PairT* src_pairs = P.src_buf ? pairs1 : pairs0;
    const long long end = P.begin + P.count;
    const long long t0 = P.begin + (tile - P.tile0) * TILE;
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {  // every gather in flight before the first ballot
      const long long i = t0 + (long long)j * 256 + threadIdx.x;
      if (i < end) {
        r[j] = src_rows[i];
        q[j] = src_pairs[i];
      }
    }
  };
  if ((long long)blockIdx.x < Bt.n_tiles) load_tile(blockIdx.x, nrr, npp);
  for (long long tile = blockIdx.x; tile < Bt.n_tiles; tile += gridDim.x, par ^= 1) {
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
      rr[j] = nrr[j];
      pp[j] = npp[j];
    }
    if (tile + gridDim.x < Bt.n_tiles) load_tile(tile + gridDim.x, nrr, npp);
    const int it = item_of(tile);
    const BatchItem& P = s_items[it];
    BatchItem& PG = Bt.items[it];  // the item's cursors live in global memory
    const int src_buf = P.src_buf;
    int* dst_rows = src_buf ? rows0 : rows1;
    PairT* dst_pairs = src_buf ? pairs0 : pairs1;
    const uint8_t* col = bins_cm + (long long)P.feature * n;
    const long long begin = P.begin, end = P.begin + P.count;
    const long long t0 = begin + (tile - P.tile0) * TILE;
    const bool is_cat = P.is_cat != 0;
    const int thr = P.threshold, mbin = P.missing_bin;
    const bool dleft = P.default_left != 0;
    unsigned bl[ITEMS], br[ITEMS];
    bool valid[ITEMS], left[ITEMS];
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) valid[j] = t0 + (long long)j * 256 + threadIdx.x < end;
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
      left[j] = false;
      if (valid[j]) {
        const int bin = col[rr[j]];
        left[j] = is_cat ? goes_left(P, bin) : (bin == mbin ? dleft : bin <= thr);
      }
    }
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
      bl[j] = __ballot_sync(0xffffffffu, left[j]);
      br[j] = __ballot_sync(0xffffffffu, valid[j]) & ~bl[j];
      if (lane == 0) {
        s_cl[par][j][w] = __popc(bl[j]);
        s_cr[par][j][w] = __popc(br[j]);
      }
    }
    __syncthreads();
    if (w == 0) {
      int* fl = &s_cl[par][0][0];
      int* fr = &s_cr[par][0][0];
      int vl[PER], vr[PER];
      int sl = 0, sr = 0;
#pragma unroll
      for (int q = 0; q < PER; ++q) {
        const int e = lane * PER + q;
        vl[q] = e < E ? fl[e] : 0;
        vr[q] = e < E ? fr[e] : 0;
        sl += vl[q];
        sr += vr[q];
      }
      int il = sl, ir = sr;
#pragma unroll
      for (int k = 1; k < 32; k <<= 1) {
        const int ol = __shfl_up_sync(0xffffffffu, il, k), orr = __shfl_up_sync(0xffffffffu, ir, k);
        if (lane >= k) {
          il += ol;
          ir += orr;
        }
      }
      int rl = il - sl, rrr = ir - sr;
#pragma unroll
      for (int q = 0; q < PER; ++q) {
        const int e = lane * PER + q;
        if (e < E) {
          fl[e] = rl;
          fr[e] = rrr;
        }
        rl += vl[q];
        rrr += vr[q];
      }
      const int tl = __shfl_sync(0xffffffffu, il, 31), tr = __shfl_sync(0xffffffffu, ir, 31);
      if (lane == 0) {
        s_base_l[par] = atomicAdd(&PG.cursor_left, (unsigned long long)tl);
        const unsigned long long o = atomicAdd(&PG.cursor_right, (unsigned long long)tr);
        s_base_r[par] = (unsigned long long)end - o - (unsigned long long)tr;  // rights fill from the back
      }
    }
    __syncthreads();
    // ranks in element order (item row j major, then warp, then lane)
    const long long base_l = begin + (long long)s_base_l[par], base_r = (long long)s_base_r[par];
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
      const unsigned m = 1u << lane;
      if ((bl[j] | br[j]) & m) {
        const long long dst = (bl[j] & m) ? base_l + s_cl[par][j][w] + __popc(bl[j] & below)
                                          : base_r + s_cr[par][j][w] + __popc(br[j] & below);
        dst_rows[dst] = rr[j];
        dst_pairs[dst] = pp[j];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Histograms of the batch's built children: privatised shared-memory integer
// cells per CTA, merged across a thread-block cluster through DSMEM, flushed
// with int32 global atomics into each item's work slot.
// ---------------------------------------------------------------------------

// Shared-memory cells use 32-bit atomics only; one CTA owns FG features.
// Global cells are int32 [slot][F][3][B] (g, h, count): every sum is bounded
// by 2^30 + n (FIXED, quantized_gradient.mojo:98-99) or by B * n (QUANT).
constexpr int kQuantCountBits = 15;

// Shared-memory cell layouts of the histogram kernel.
//   HL_QUANT     plane 0: g * 2^15 + count (exact while a flush covers
//                < 32768 rows and |sum g| < 2^16), plane 1: h
//   HL_QUANT16   plane A: (g + g_lim) | count << 16 per cell; plane B (half
//                size): h of features 2k (low half) and 2k+1 (high half).
//                Every field is a 16-bit unsigned sum, exact while a flush
//                covers at most 65535 / max(2 g_lim, h_lim) rows; 6 bytes a
//                cell, so twice the features of HL_QUANT fit one CTA.
//   HL_FIXED_CH  plane 0: g, plane 1: count (hessian constant)
//   HL_FIXED     planes g, h, count
//   HL_QUANT16R  the cells of HL_QUANT16; a chunk's row id, g + g_lim and h
//                travel as one shuffled word (row << 6 | h << 3 | g + g_lim),
//                for fewer than 2^26 rows and 2 g_lim, h_lim <= 7
//   HL_W52       fixed point with the 2^52 bound (Int64 global cells): 64-bit
//                g and h planes and a 32-bit count plane (red.shared.add.u64
//                has no native shared-memory unit on sm_100: it costs about six
//                32-bit atomics, acceptable for a precision mode)
//   HL_W52CH     HL_W52 with a constant hessian: g and count planes
enum HistLayout : int {
  HL_QUANT = 0, HL_QUANT16 = 1, HL_FIXED_CH = 2, HL_FIXED = 3, HL_QUANT16R = 4, HL_W52 = 9, HL_W52CH = 10
};


// 32-bit words of shared memory a CTA's cells take (cells = lane cells of one plane)
__host__ __device__ constexpr int hist_layout_words(int layout, int cells) {
  return (layout == HL_QUANT16 || layout == HL_QUANT16R) ? cells + cells / 2
         : layout == HL_W52                              ? 5 * cells
         : (layout == HL_FIXED || layout == HL_W52CH) ? 3 * cells
                                                                           : 2 * cells;
}

__device__ __forceinline__ void built_range(const BatchItem& P, long long& b, long long& cnt) {
  long long nl = (long long)P.cursor_left;
  if (P.built_is_left) {
    b = P.begin;
    cnt = nl;
  } else {
    b = P.begin + nl;
    cnt = P.count - nl;
  }
}

// Shared-memory layout, one bank per lane.  A warp takes one row at a time;
// lane l owns the NPL consecutive features f0 + l*NPL + j (j < NPL) of the
// CTA's feature group (FG = 32*NPL features) and loads their NPL bin bytes
// with one load.  Cell (feature l*NPL + j, bin b) of plane p is word
//   ((p * NPL + j) * B + b) * 32 + l
// so the 32 atomics of one warp instruction fall in 32 different banks
// whatever the bin values are: no bank conflicts and no same-address
// collisions inside an instruction.
template <int NPL>
__device__ __forceinline__ int lane_cell(int j, int b, int B, int lane) {
  return (j * B + b) * 32 + lane;
}

template <int NPL>
struct BinWord;
template <>
struct BinWord<1> {
  static __device__ __forceinline__ unsigned int load(const uint8_t* p) { return __ldg(p); }
};
template <>
struct BinWord<2> {
  static __device__ __forceinline__ unsigned int load(const uint8_t* p) {
    return __ldg(reinterpret_cast<const unsigned short*>(p));
  }
};
template <>
struct BinWord<4> {
  static __device__ __forceinline__ unsigned int load(const uint8_t* p) {
    return __ldg(reinterpret_cast<const unsigned int*>(p));
  }
};

#ifndef MTB_HIST_RED_CLOBBER
#define MTB_HIST_RED_CLOBBER 0
#endif
#ifndef MTB_HIST_PIPELINE
#define MTB_HIST_PIPELINE 0
#endif
#ifndef MTB_HIST_UNROLL
#define MTB_HIST_UNROLL 8
#endif
constexpr int kHistUnroll = MTB_HIST_UNROLL;  // bin loads in flight per warp (divides 32)
#ifndef MTB_HIST_THREADS
#define MTB_HIST_THREADS 1024
#endif
constexpr int kHistThreads = MTB_HIST_THREADS;
constexpr int kHistBinsPad = 256;  // bins per feature in the shared-memory layout
// shared memory after the cells: the staged batch items and their built-row prefix sums
// (and 64 words of reduction scratch)
// rows per CTA that one merged segment costs about as much as (the split of
// a launch's rows over clusters weighs merges against rows with it)
constexpr long long kHistMergeRows = 4500;
constexpr int kHistBatchSmem =
    (int)((sizeof(BatchItem) * kMaxBatch + sizeof(long long) * (kMaxBatch + 1) + 64 * sizeof(unsigned int) + 15) /
          16 * 16);

// Atomic add to a shared-memory word whose result is not needed.  No memory
// clobber: the cells are read only after a block or cluster barrier (which
// orders them), and without it the compiler may issue the next rows' global
// loads ahead of these atomics.
__device__ __forceinline__ void shared_red_add(uint32_t addr, unsigned int v) {
#if MTB_HIST_RED_CLOBBER
  asm volatile("red.shared.add.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
#else
  asm volatile("red.shared.add.u32 [%0], %1;" ::"r"(addr), "r"(v));
#endif
}

// One cluster accumulates rows [seg_b, seg_b + seg_n) of one item's built
// child into the item's work slot.
template <int NPL, int LAYOUT>
__device__ void hist_segment(cooperative_groups::cluster_group& cluster, const BatchItem& P, long long seg_b,
                             long long seg_n, const uint8_t* __restrict__ bins_rm, int Fp, int F, int B,
                             const int* __restrict__ rows0, const int* __restrict__ rows1,
                             const void* __restrict__ pairs0, const void* __restrict__ pairs1, int* hs,
                             long long rows_per_flush, int g_lim, unsigned int* p0, unsigned int* s_red) {
  constexpr bool PR = LAYOUT == HL_QUANT16R;          // row id packed with the gradient pair
  constexpr bool Q16 = LAYOUT == HL_QUANT16 || PR;     // 16-bit packed cells
  static_assert(!Q16 || NPL % 2 == 0, "packed cells pair features");
  static_assert(!(PR && MTB_HIST_PIPELINE), "the pipelined walk does not unpack row words");
  constexpr int FG = 32 * NPL;
  constexpr int MODE = (LAYOUT == HL_QUANT || Q16) ? MODE_QUANT : MODE_FIXED;
  constexpr bool CONST_H = LAYOUT == HL_FIXED_CH;
  constexpr int U = kHistUnroll;
  const int cs = (int)cluster.num_blocks();
  const int crank = (int)cluster.block_rank();
  const long long sub = (seg_n + cs - 1) / cs;  // rows per CTA, identical across the cluster
  const long long s = seg_b + crank * sub;
  long long e = s + sub;
  if (e > seg_b + seg_n) e = seg_b + seg_n;
  // 16-bit packed cells take the segment in one pass: the rows go in windows
  // the cells' headroom allows (below), so the cluster merges once
  const long long pass_rows = Q16 ? (1ll << 40) : rows_per_flush;
  const long long n_pass = (sub + pass_rows - 1) / pass_rows;
  const int f0 = blockIdx.x * FG;
  // cells are laid out for 256 bins whatever B is, so every plane and
  // feature offset below is a compile-time constant
  constexpr int cells = NPL * kHistBinsPad * 32;  // words per full plane
  constexpr int words = hist_layout_words(LAYOUT, cells);
  const int* rows = P.dst_buf ? rows1 : rows0;
  const void* pairs = P.dst_buf ? pairs1 : pairs0;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int n_warps = blockDim.x >> 5;
  // A lane past the padded row width reads the row's first bytes instead (a
  // valid address) and accumulates them into cells of features >= Fp, which
  // the merge never reads; so the row loop needs no per-lane test.
  const bool lane_ok = f0 + lane * NPL < Fp;
  const uint8_t* bcol = bins_rm + (lane_ok ? f0 + lane * NPL : 0);
  const int slice = (cells + cs - 1) / cs;
  const int m0 = crank * slice;
  const int m1 = m0 + slice < cells ? m0 + slice : cells;
  // Shared-memory byte address of this lane's cell (feature 0, bin 0) of
  // plane A; cell (j, bin) of a plane is that plus a constant plus bin * 128
  // (32 lanes x 4 bytes).
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(p0) + 4u * lane;
  constexpr uint32_t kFeat = 128u * kHistBinsPad;  // bytes between features of a plane
  // one row of this lane's features: NPL cells in each plane
  auto add_row = [&](unsigned int bw, unsigned int x0, unsigned int x1) {
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
      const uint32_t a = sbase + (((bw >> (8 * j)) & 0xffu) << 7);
      shared_red_add(a + j * kFeat, x0);
      if (Q16) {
        // plane B: features 2k and 2k+1 share a word (low and high half)
        shared_red_add(a + 4u * cells + (j >> 1) * kFeat, (j & 1) ? x1 << 16 : x1);
      } else {
        shared_red_add(a + 4u * cells + j * kFeat, x1);
        if (LAYOUT == HL_FIXED) shared_red_add(a + 8u * cells + j * kFeat, 1u);
      }
    }
  };
  // Q16: after a window of rows, every cell word of a real feature whose
  // largest field passed half its range goes to the work slot (its fields
  // added with int32 atomics, the word zeroed); the largest field left then
  // bounds the rows the next window may take without a carry (a row adds at
  // most 2 g_lim to a g + g_lim or h field and 1 to a count).  Cells of
  // padding features (>= F) are never read and are left to wrap.
  auto headroom = [&]() -> long long {
    constexpr unsigned int kHot = 32767u;
    __syncthreads();
    unsigned int mx = 0u;
    const long long step = 2ll * (g_lim > 0 ? g_lim : 1);
    for (int c = threadIdx.x; c < cells; c += blockDim.x) {  // plane A: g + g_lim | count << 16
      const int l = c & 31, jb = c >> 5, j = jb / kHistBinsPad, bin = jb % kHistBinsPad;
      const int f = f0 + l * NPL + j;
      if (f >= F) continue;
      const unsigned int x = p0[c];
      const unsigned int g = x & 0xffffu, cnt = x >> 16;
      // the count field's load in units of the g field's per-row step
      const long long cl_ = (long long)cnt * step;
      const unsigned int load = max(g, (unsigned int)(cl_ < 65535ll ? cl_ : 65535ll));
      if (load > kHot) {
        if (bin < B) {
          int* cellp = hs + (f * 3) * B + bin;
          atomicAdd(cellp, (int)g - g_lim * (int)cnt);
          atomicAdd(cellp + 2 * B, (int)cnt);
        }
        p0[c] = 0u;
      } else {
        mx = max(mx, load);
      }
    }
    for (int c = threadIdx.x; c < cells / 2; c += blockDim.x) {  // plane B: h of features 2k, 2k+1
      const int l = c & 31, jb = c >> 5, j2 = jb / kHistBinsPad, bin = jb % kHistBinsPad;
      const int fa = f0 + l * NPL + 2 * j2;
      if (fa >= F) continue;
      const unsigned int x = p0[cells + c];
      const unsigned int ha = x & 0xffffu, hb = x >> 16;
      if (ha > kHot || hb > kHot) {
        if (bin < B) {
          atomicAdd(hs + (fa * 3 + 1) * B + bin, (int)ha);
          if (fa + 1 < F) atomicAdd(hs + ((fa + 1) * 3 + 1) * B + bin, (int)hb);
        }
        p0[cells + c] = 0u;
      } else {
        mx = max(mx, max(ha, hb));
      }
    }
    mx = __reduce_max_sync(0xffffffffu, mx);
    if (lane == 0) s_red[warp] = mx;
    __syncthreads();
    mx = 0u;
    for (int w = 0; w < n_warps; ++w) mx = max(mx, s_red[w]);
    __syncthreads();  // zeroed words and s_red reads complete before the next window
    // mx <= kHot, so every window takes at least (65535 - kHot) / step >= 1024 rows
    const long long ok = (65535ll - (long long)mx) / step;
    return ok > 1 ? ok : 1;
  };
  for (long long pass = 0; pass < n_pass; ++pass) {
    const long long ps0 = s + pass * pass_rows;
    const long long pe0 = ps0 + pass_rows < e ? ps0 + pass_rows : e;
    for (int c = threadIdx.x; c < words; c += blockDim.x) p0[c] = 0u;
    __syncthreads();
    long long window = rows_per_flush;  // rows the cells take before the next headroom check
    for (long long ps = ps0; ps < pe0;) {
    const long long pe = Q16 && ps + window < pe0 ? ps + window : pe0;
    // Each warp takes chunks of 32 consecutive positions: lane k loads the
    // row id and gradient pair of position k (coalesced; the next chunk's are
    // fetched while this one is processed), then the warp walks the chunk with
    // U bin loads in flight before their atomics.
    const long long stride = (long long)n_warps * 32;
    long long c0 = ps + (long long)warp * 32;
    int nr = 0;
    unsigned int na0 = 0u, na1 = 0u;
    auto fetch = [&](long long base, int& r, unsigned int& x0, unsigned int& x1) {
      const long long i = base + lane;
      r = 0;
      x0 = 0u;
      x1 = 0u;
      if (i < pe) {
        r = __ldg(rows + i);
        if (MODE == MODE_QUANT) {
          uint16_t pr = __ldg(reinterpret_cast<const uint16_t*>(pairs) + i);
          int g = (int)(int8_t)(pr & 0xff);
          if (PR) {
            x0 = ((unsigned int)r << 6) | ((unsigned int)(pr >> 8) << 3) | (unsigned int)(g + g_lim);
          } else if (Q16) {
            // g + g_lim and h both fit 8 bits here: carry both in one word
            // (bits 0-7 and 8-15) so the chunk walk needs one shuffle for them
            x0 = (unsigned int)(g + g_lim) | ((unsigned int)(pr >> 8) << 8) | (1u << 16);
          } else {
            x0 = (unsigned int)(g * (1 << kQuantCountBits) + 1);
            x1 = (unsigned int)(pr >> 8);
          }
        } else {
          int2 pr = __ldg(reinterpret_cast<const int2*>(pairs) + i);
          x0 = (unsigned int)pr.x;
          x1 = CONST_H ? 1u : (unsigned int)pr.y;
        }
      }
    };
    if (c0 < pe) fetch(c0, nr, na0, na1);
    for (; c0 < pe; c0 += stride) {
      const int cr = nr;
      const unsigned int ca0 = na0, ca1 = na1;
      if (c0 + stride < pe) fetch(c0 + stride, nr, na0, na1);
      if (pe - c0 >= 32) {
        // full chunk: no bounds tests
#if MTB_HIST_PIPELINE
        // the next group's bin loads are issued before this group's atomics
        unsigned int bw[U], nb[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int r = __shfl_sync(0xffffffffu, cr, u);
          bw[u] = BinWord<NPL>::load(bcol + (size_t)(unsigned int)r * (unsigned int)Fp);
        }
#pragma unroll
        for (int u0 = 0; u0 < 32; u0 += U) {
          if (u0 + U < 32) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
              const int r = __shfl_sync(0xffffffffu, cr, u0 + U + u);
              nb[u] = BinWord<NPL>::load(bcol + (size_t)(unsigned int)r * (unsigned int)Fp);
            }
          }
#pragma unroll
          for (int u = 0; u < U; ++u) {
            unsigned int x0 = __shfl_sync(0xffffffffu, ca0, u0 + u), x1;
            if (Q16) {
              x1 = (x0 >> 8) & 0xffu;
              x0 &= 0xffff00ffu;
            } else {
              x1 = (MODE == MODE_FIXED && CONST_H) ? 1u : __shfl_sync(0xffffffffu, ca1, u0 + u);
            }
            add_row(bw[u], x0, x1);
          }
#pragma unroll
          for (int u = 0; u < U; ++u) bw[u] = nb[u];
        }
#else
#pragma unroll
        for (int u0 = 0; u0 < 32; u0 += U) {
          unsigned int bw[U], pw[U];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            int r;
            if (PR) {
              pw[u] = __shfl_sync(0xffffffffu, ca0, u0 + u);
              r = (int)(pw[u] >> 6);
            } else {
              r = __shfl_sync(0xffffffffu, cr, u0 + u);
            }
            bw[u] = BinWord<NPL>::load(bcol + (size_t)(unsigned int)r * (unsigned int)Fp);
          }
#pragma unroll
          for (int u = 0; u < U; ++u) {
            unsigned int x0, x1;
            if (PR) {
              x0 = (pw[u] & 7u) | (1u << 16);
              x1 = (pw[u] >> 3) & 7u;
              add_row(bw[u], x0, x1);
              continue;
            }
            x0 = __shfl_sync(0xffffffffu, ca0, u0 + u);
            if (Q16) {
              x1 = (x0 >> 8) & 0xffu;
              x0 &= 0xffff00ffu;
            } else {
              x1 = (MODE == MODE_FIXED && CONST_H) ? 1u : __shfl_sync(0xffffffffu, ca1, u0 + u);
            }
            add_row(bw[u], x0, x1);
          }
        }
#endif
      } else {
        const int n_in = (int)(pe - c0);
        for (int u = 0; u < n_in; ++u) {
          if (PR) {
            const unsigned int w = __shfl_sync(0xffffffffu, ca0, u);
            add_row(BinWord<NPL>::load(bcol + (size_t)(w >> 6) * (unsigned int)Fp), (w & 7u) | (1u << 16),
                    (w >> 3) & 7u);
            continue;
          }
          const int r = __shfl_sync(0xffffffffu, cr, u);
          unsigned int x0 = __shfl_sync(0xffffffffu, ca0, u), x1;
          if (Q16) {
            x1 = (x0 >> 8) & 0xffu;
            x0 &= 0xffff00ffu;
          } else {
            x1 = __shfl_sync(0xffffffffu, ca1, u);
          }
          add_row(BinWord<NPL>::load(bcol + (size_t)(unsigned int)r * (unsigned int)Fp), x0, x1);
        }
      }
    }
    ps = pe;
    if (ps < pe0) window = headroom();
    }
    cluster.sync();
    // Merge: the work units are (tile, plane), one per warp at a time.  A
    // tile is 16 consecutive bins of one feature slot j for all 32 lanes
    // (512 consecutive words).  A unit's values are summed over the
    // cluster's CTAs (DSMEM) with lane = feature, transposed in registers
    // within each half-warp to lane = bin, and added to the work slot with
    // int32 atomics whose lanes hit two runs of 16 consecutive cells (4
    // sectors a warp instruction instead of 32; about 5x faster through L2
    // than the lane = feature order).  With 16-bit packed cells one unit
    // reads the (g + g_lim | count) words once for both of their planes.
    {
      constexpr int kPlanes = (MODE == MODE_FIXED && CONST_H) ? 2 : 3;  // g, [h,] count
      constexpr int kUnits = Q16 ? 2 : kPlanes;
      const int tiles = (m1 - m0) >> 9;
      const int half = lane >> 4, hl = lane & 15;
      auto transpose16 = [&](int (&v)[16]) {
        // lane 16 h + m, v[i] = cell (lane 16 h + m, bin i) becomes
        // lane 16 h + i, v[m] = cell (lane 16 h + m, bin i)
#pragma unroll
        for (int sft = 8; sft >= 1; sft >>= 1) {
          const bool upper = (lane & sft) != 0;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if ((i & sft) == 0) {
              const int send = upper ? v[i] : v[i + sft];
              const int recv = __shfl_xor_sync(0xffffffffu, send, sft);
              if (upper)
                v[i] = recv;
              else
                v[i + sft] = recv;
            }
          }
        }
      };
      auto emit = [&](int (&v)[16], int j, int bin0, int out_plane) {
        transpose16(v);
        const int bin = bin0 + hl;
#pragma unroll
        for (int m = 0; m < 16; ++m) {
          const int f = f0 + (16 * half + m) * NPL + j;
          if (f < F && bin < B && v[m] != 0) atomicAdd(hs + (f * 3 + out_plane) * B + bin, v[m]);
        }
      };
      for (int wu = warp; wu < tiles * kUnits; wu += n_warps) {
        const int t = wu / kUnits, plane = wu - t * kUnits;
        const int c0 = m0 + (t << 9);
        const int j = (c0 >> 5) / kHistBinsPad, bin0 = (c0 >> 5) % kHistBinsPad;
        int v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0;
        if (Q16 && plane == 0) {
          int vc[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) vc[i] = 0;
          for (int rk = 0; rk < cs; ++rk) {
            const unsigned int* q0 = cluster.map_shared_rank(p0, rk);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const unsigned int x = q0[c0 + (i << 5) + lane];
              v[i] += (int)(x & 0xffffu);
              vc[i] += (int)(x >> 16);
            }
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] -= g_lim * vc[i];
          emit(v, j, bin0, 0);
          emit(vc, j, bin0, 2);
          continue;
        }
        const int out_plane = Q16 ? 1 : (kPlanes == 2 && plane == 1) ? 2 : plane;  // constant hessian: g, count
        for (int rk = 0; rk < cs; ++rk) {
          const unsigned int* q0 = cluster.map_shared_rank(p0, rk);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int c = c0 + (i << 5) + lane;
            if (Q16) {  // plane B: h of features 2k (low half) and 2k + 1
              const unsigned int x = q0[cells + ((((j >> 1) * kHistBinsPad + bin0 + i) << 5) + lane)];
              v[i] += (int)((x >> (16 * (j & 1))) & 0xffffu);
            } else if (LAYOUT == HL_QUANT) {
              if (plane == 1) {
                v[i] += (int)q0[cells + c];
              } else {
                const unsigned int x = q0[c];
                v[i] += plane == 0 ? ((int)x >> kQuantCountBits) : (int)(x & ((1u << kQuantCountBits) - 1u));
              }
            } else {
              // fixed point: planes g, h, count (constant hessian: g, count)
              v[i] += (int)q0[plane * cells + c];
            }
          }
        }
        emit(v, j, bin0, out_plane);
      }
    }
    cluster.sync();  // peers finished reading before anyone re-zeroes
  }
}

__device__ __forceinline__ void shared_red_add64(uint32_t addr, unsigned long long v) {
  asm volatile("red.shared.add.u64 [%0], %1;" ::"r"(addr), "l"(v));
}

// hist_segment for the fixed-point mode with the 2^52 bound (HL_W52,
// HL_W52CH): Int64 gradient and hessian values, 64-bit shared cells for g
// (and h), a 32-bit count plane, Int64 global cells.  Same bank-per-lane
// geometry as hist_segment64.  A precision mode: one row id and two 64-bit
// values broadcast per row.
template <int NPL, int LAYOUT>
__device__ void hist_segment_w52(cooperative_groups::cluster_group& cluster, const BatchItem& P, long long seg_b,
                                 long long seg_n, const uint8_t* __restrict__ bins_rm, int Fp, int F, int B,
                                 const int* __restrict__ rows0, const int* __restrict__ rows1,
                                 const void* __restrict__ pairs0, const void* __restrict__ pairs1, int* hs_words,
                                 long long rows_per_flush, unsigned char* smem) {
  constexpr bool CH = LAYOUT == HL_W52CH;
  constexpr int FG = 32 * NPL;
  constexpr int U = 4;
  constexpr int CELLS = NPL * kHistBinsPad * 32;
  constexpr int PLANES64 = CH ? 1 : 2;
  constexpr int BYTES = CELLS * (8 * PLANES64 + 4);
  long long* hs = reinterpret_cast<long long*>(hs_words);
  const int cs = (int)cluster.num_blocks();
  const int crank = (int)cluster.block_rank();
  const long long sub = (seg_n + cs - 1) / cs;
  const long long s = seg_b + crank * sub;
  long long e = s + sub;
  if (e > seg_b + seg_n) e = seg_b + seg_n;
  const long long n_pass = (sub + rows_per_flush - 1) / rows_per_flush;
  const int f0 = blockIdx.x * FG;
  const int* rows = P.dst_buf ? rows1 : rows0;
  const longlong2* pairs = reinterpret_cast<const longlong2*>(P.dst_buf ? pairs1 : pairs0);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int n_warps = blockDim.x >> 5;
  const bool lane_ok = f0 + lane * NPL < Fp;
  const uint8_t* bcol = bins_rm + (lane_ok ? f0 + lane * NPL : 0);
  const uint32_t gbase = (uint32_t)__cvta_generic_to_shared(smem) + 8u * lane;
  const uint32_t cbase = (uint32_t)__cvta_generic_to_shared(smem) + 8u * PLANES64 * CELLS + 4u * lane;
  auto add_row = [&](unsigned int bw, long long g, long long h) {
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
      const uint32_t b = (bw >> (8 * j)) & 0xffu;
      shared_red_add64(gbase + (b << 8) + j * (256u * 256u), (unsigned long long)g);
      if (!CH) shared_red_add64(gbase + 8u * CELLS + (b << 8) + j * (256u * 256u), (unsigned long long)h);
      shared_red_add(cbase + (b << 7) + j * (128u * 256u), 1u);
    }
  };
  for (long long pass = 0; pass < n_pass; ++pass) {
    const long long ps = s + pass * rows_per_flush;
    const long long pe = ps + rows_per_flush < e ? ps + rows_per_flush : e;
    for (int c = threadIdx.x; c < BYTES / 16; c += blockDim.x) reinterpret_cast<uint4*>(smem)[c] = make_uint4(0, 0, 0, 0);
    __syncthreads();
    const long long stride = (long long)n_warps * 32;
    for (long long c0 = ps + (long long)warp * 32; c0 < pe; c0 += stride) {
      const long long i = c0 + lane;
      int r = 0;
      long long g = 0, h = 0;
      if (i < pe) {
        r = __ldg(rows + i);
        const longlong2 pr = __ldg(pairs + i);
        g = pr.x;
        h = pr.y;
      }
      const int n_in = pe - c0 >= 32 ? 32 : (int)(pe - c0);
      for (int u0 = 0; u0 < n_in; u0 += U) {
        unsigned int bw[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int rr = __shfl_sync(0xffffffffu, r, (u0 + u) & 31);
          bw[u] = u0 + u < n_in ? BinWord<NPL>::load(bcol + (size_t)(unsigned int)rr * (unsigned int)Fp) : 0u;
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const long long gg = __shfl_sync(0xffffffffu, g, (u0 + u) & 31);
          const long long hh = CH ? 0ll : __shfl_sync(0xffffffffu, h, (u0 + u) & 31);
          if (u0 + u < n_in) add_row(bw[u], gg, hh);
        }
      }
    }
    cluster.sync();
    const int slice = (CELLS + cs - 1) / cs;
    const int m0 = crank * slice;
    const int m1 = m0 + slice < CELLS ? m0 + slice : CELLS;
    const unsigned long long* g64 = reinterpret_cast<const unsigned long long*>(smem);
    const unsigned int* c32 = reinterpret_cast<const unsigned int*>(smem + 8 * PLANES64 * CELLS);
    for (int c = m0 + threadIdx.x; c < m1; c += blockDim.x) {
      const int l = c & 31;
      const int jb = c >> 5;
      const int j = jb / kHistBinsPad;
      const int bin = jb % kHistBinsPad;
      const int f = f0 + l * NPL + j;
      if (f >= F || bin >= B) continue;
      unsigned long long g = 0, h = 0;
      long long cnt = 0;
      for (int rk = 0; rk < cs; ++rk) {
        const unsigned long long* q = cluster.map_shared_rank(g64, rk);
        g += q[c];
        if (!CH) h += q[CELLS + c];
        cnt += (long long)cluster.map_shared_rank(c32, rk)[c];
      }
      if (cnt == 0) continue;
      unsigned long long* cellp = reinterpret_cast<unsigned long long*>(hs + (long long)(f * 3) * B + bin);
      atomicAdd(cellp, g);
      if (!CH) atomicAdd(cellp + B, h);
      atomicAdd(cellp + 2 * B, (unsigned long long)cnt);
    }
    cluster.sync();
  }
}

// Calls seg(item, first position, positions) for every segment cluster cid
// of n_clusters (of cs CTAs each) accumulates in a launch over the staged
// batch (s_pre: prefix sums of the items' built rows).  Every thread of the
// block calls it; s_asg is 34 ints of shared scratch.
template <typename Seg>
__device__ void for_each_segment(int n_items, const BatchItem* s_items, const long long* s_pre, long long cid,
                                 long long n_clusters, int cs, int min_rows_per_cta, int allow_owned, int* s_asg,
                                 Seg&& seg) {
  const long long S = s_pre[n_items];
  if (S == 0) return;
  const long long per_cluster = (long long)min_rows_per_cta * cs;
  long long cap = (S + per_cluster - 1) / per_cluster;
  if (cap > n_clusters) cap = n_clusters;
  if (cid >= cap) return;  // the whole cluster leaves together
  // Rows to clusters, two ways.  Contiguous: cluster c takes rows
  // [S c / cap, S (c + 1) / cap) of the batch in item order and merges one
  // segment for every item its range meets.  Owned: every item with rows gets
  // k_i = ceil(rows_i / R) clusters of its own, R the smallest row count per
  // cluster with sum k_i <= cap, and each cluster merges one segment.  The
  // launch takes the way whose costliest cluster is cheaper, a merged segment
  // counting as kHistMergeRows rows per CTA (per-launch traces of configs[1]
  // fit 32 us a merged segment against 3.6 ns a row for a cluster of two).
  // Every CTA computes the same choice from the same staged items.
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const long long mr = (long long)kHistMergeRows * cs;
    // contiguous: the largest cluster cost, lanes over clusters
    long long cost_a = 0;
    for (long long c = lane; c < cap; c += 32) {
      const long long lo = S * c / cap, hi = S * (c + 1) / cap;
      if (hi <= lo) continue;
      int first = 0, last = n_items - 1;  // items meeting [lo, hi): s_pre[i + 1] > lo and s_pre[i] < hi
      while (first < n_items && s_pre[first + 1] <= lo) ++first;
      while (last > first && s_pre[last] >= hi) --last;
      const long long cost = (hi - lo) + (long long)(last - first + 1) * mr;
      cost_a = cost > cost_a ? cost : cost_a;
    }
    for (int k = 16; k > 0; k >>= 1) {
      const long long o = __shfl_xor_sync(0xffffffffu, cost_a, k);
      cost_a = o > cost_a ? o : cost_a;
    }
    // owned: binary search of the row count R per cluster (lane = item)
    const long long rows_i = lane < n_items ? s_pre[lane + 1] - s_pre[lane] : 0;
    long long r_lo = (S + cap - 1) / cap, r_hi = rows_i;
    for (int k = 16; k > 0; k >>= 1) {
      const long long o = __shfl_xor_sync(0xffffffffu, r_hi, k);
      r_hi = o > r_hi ? o : r_hi;
    }
    const int nonempty = __popc(__ballot_sync(0xffffffffu, rows_i > 0));
    bool owned = false;
    long long k_i = 0;
    if (nonempty <= cap) {
      if (r_lo > r_hi) r_lo = r_hi;
      while (r_lo < r_hi) {
        const long long mid = (r_lo + r_hi) / 2;
        long long need = rows_i > 0 ? (rows_i + mid - 1) / mid : 0;
        for (int k = 16; k > 0; k >>= 1) need += __shfl_xor_sync(0xffffffffu, need, k);
        if (need <= cap) r_hi = mid;
        else r_lo = mid + 1;
      }
      owned = allow_owned && r_lo + mr < cost_a;
      k_i = rows_i > 0 ? (rows_i + r_lo - 1) / r_lo : 0;
    }
    // exclusive prefix of the clusters per item
    long long inc = k_i;
    for (int k = 1; k < 32; k <<= 1) {
      const long long o = __shfl_up_sync(0xffffffffu, inc, k);
      if (lane >= k) inc += o;
    }
    if (lane < n_items) s_asg[2 + lane] = (int)inc;
    if (lane == 0) {
      s_asg[0] = owned ? 1 : 0;
      s_asg[1] = 0;
    }
  }
  __syncthreads();
  if (s_asg[0]) {
    int i = 0;
    while (i < n_items && s_asg[2 + i] <= cid) ++i;
    if (i >= n_items) return;  // a cluster no item needs
    const BatchItem& P = s_items[i];
    const long long k = s_asg[2 + i] - s_asg[1 + i], r = cid - s_asg[1 + i];
    long long b, c;
    built_range(P, b, c);
    const long long s0 = c * r / k, s1 = c * (r + 1) / k;
    if (s1 > s0) seg(P, b + s0, s1 - s0);
    return;
  }
  const long long lo = S * cid / cap, hi = S * (cid + 1) / cap;
  for (int i = 0; i < n_items && s_pre[i] < hi; ++i) {
    const BatchItem& P = s_items[i];
    const long long acc = s_pre[i];
    long long b, c;
    built_range(P, b, c);
    const long long s0 = lo > acc ? lo : acc;
    const long long s1 = hi < acc + c ? hi : acc + c;
    if (s1 > s0) seg(P, b + (s0 - acc), s1 - s0);
  }
}

// CTAs of one feature group form clusters of CS along grid y.  The batch's
// built rows, taken as one sequence (item after item), are split evenly among
// ceil(rows / (min_rows_per_cta * CS)) clusters at most; a cluster whose share
// spans several items accumulates one segment per item.
template <int NPL, int LAYOUT>
__global__ void __launch_bounds__(kHistThreads) k_hist(const Batch* __restrict__ batch, const uint8_t* __restrict__ bins_rm,
                                               int Fp, int F, int B, const int* __restrict__ rows0,
                                               const int* __restrict__ rows1, const void* __restrict__ pairs0,
                                               const void* __restrict__ pairs1, int* __restrict__ hist,
                                               long long slot_cells, long long rows_per_flush, int g_lim,
                                               int work_base, int min_rows_per_cta, int allow_owned) {
  pdl_enter();
  namespace cg = cooperative_groups;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned int* p0 = reinterpret_cast<unsigned int*>(smem_raw);
  // After the cells: the batch's items and the prefix sums of their built
  // rows, staged with one coalesced copy (the item records are read many
  // times below; from global memory each read is a dependent L2 round trip).
  constexpr int kCellBytes = 4 * hist_layout_words(LAYOUT, NPL * kHistBinsPad * 32);
  BatchItem* s_items = reinterpret_cast<BatchItem*>(smem_raw + kCellBytes);
  long long* s_pre = reinterpret_cast<long long*>(s_items + kMaxBatch);
  unsigned int* s_red = reinterpret_cast<unsigned int*>(s_pre + kMaxBatch + 1);  // 64 words
  const int n_items = batch->n_items;  // uniform across the grid
  if (n_items == 0) return;
  {
    const int* src = reinterpret_cast<const int*>(batch->items);
    int* dst = reinterpret_cast<int*>(s_items);
    const int words = n_items * (int)(sizeof(BatchItem) / sizeof(int));
    for (int i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    long long carry = 0;
    for (int base = 0; base < n_items; base += 32) {
      long long b, c = 0;
      if (base + lane < n_items) built_range(s_items[base + lane], b, c);
#pragma unroll
      for (int k = 1; k < 32; k <<= 1) {
        const long long o = __shfl_up_sync(0xffffffffu, c, k);
        if (lane >= k) c += o;
      }
      if (base + lane < n_items) s_pre[base + lane + 1] = carry + c;
      carry += __shfl_sync(0xffffffffu, c, 31);
    }
    if (lane == 0) s_pre[0] = 0;
  }
  __syncthreads();
  cg::cluster_group cluster = cg::this_cluster();
  const int cs = (int)cluster.num_blocks();
  const long long n_clusters = gridDim.y / cs;
  const long long cid = blockIdx.y / cs;
  const long long S = s_pre[n_items];
  if (S == 0) return;
  for_each_segment(n_items, s_items, s_pre, cid, n_clusters, cs, min_rows_per_cta, allow_owned,
                   reinterpret_cast<int*>(s_red), [&](const BatchItem& P, long long seg_b, long long seg_n) {
                     if constexpr (LAYOUT == HL_W52 || LAYOUT == HL_W52CH)
                       hist_segment_w52<NPL, LAYOUT>(cluster, P, seg_b, seg_n, bins_rm, Fp, F, B, rows0, rows1,
                                                     pairs0, pairs1,
                                                     hist + (long long)(work_base + P.work) * slot_cells,
                                                     rows_per_flush, smem_raw);
                     else
                       hist_segment<NPL, LAYOUT>(cluster, P, seg_b, seg_n, bins_rm, Fp, F, B, rows0, rows1, pairs0,
                                                 pairs1, hist + (long long)(work_base + P.work) * slot_cells,
                                                 rows_per_flush, g_lim, p0, s_red);
                   });
}

// ---------------------------------------------------------------------------
// Subtract + split scan: one block per (child, active feature).
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

// The correctly rounded quotient a / b from y = RN(1 / b), without a divide:
// two residual corrections q' = RN(q + RN(a - b q) y), the residual exact by
// FMA (P. Markstein, "IA-64 and Elementary Functions", Prentice Hall 2000,
// ch. 8: one correction of a faithful q yields RN(a / b); the first
// correction makes RN(a y) faithful).  Valid while a / b and the residuals
// stay normal, as they do for histogram sums over quantizer units
// (mojotrees_b200_check_quotients verifies it against the divide).
__device__ __forceinline__ double quot_exact(double a, double b, double y) {
  double q = __dmul_rn(a, y);
  double r = __fma_rn(-q, b, a);
  q = __fma_rn(r, y, q);
  r = __fma_rn(-q, b, a);
  return __fma_rn(r, y, q);
}

// Dequantize an exact integer sum: FIXED multiplies by the power-of-two
// inverse scale (exact); QUANT divides by the units (quantized_gradient.mojo:
// 1324), with inv = RN(1 / units).
__device__ __forceinline__ double deq(long long q, int mode, double inv, double units) {
  return mode == MODE_FIXED ? (double)q * inv : quot_exact((double)q, units, inv);
}

// Called by every (child, feature) warp once its FeatBest is written; the
// warp that completes child c folds the child's per-feature bests (ascending
// feature, strict >: the first maximum), applies the leaf guards and writes
// the child's split, value, global count and local row range, and its gain
// in the per-leaf table.
// FeatBest and totals written by other SMs in this launch are read through
// L2 (__ldcg): L1 is not coherent inside a kernel.
__device__ void scan_pair_done(TreeState* __restrict__ ts, int c, const FeatBest* __restrict__ fbs,
                               const int* __restrict__ feats, const RoundScales* __restrict__ sc,
                               const ScanParams& sp) {
  const int lane = threadIdx.x & 31;
  unsigned int last = 0;
  if (lane == 0) {
    __threadfence();
    last = atomicAdd(&ts->child_done[c], 1u) == (unsigned int)(sp.n_active - 1) ? 1u : 0u;
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return;
  __threadfence();
  const Batch& Bt = ts->batch;
  const int item = c >> 1, side = c & 1;
  const bool root = Bt.root != 0;
  const BatchItem& P = Bt.items[item];
  const FeatBest* fc = fbs + (long long)c * sp.n_active;
  double bg = 0.0;
  int bj = -1;
  for (int j = lane; j < sp.n_active; j += 32) {
    const int flags = __ldcg(&fc[j].flags);
    const double g = __ldcg(&fc[j].gain);
    if ((flags & 1) && g > bg) {
      bg = g;
      bj = j;
    }
  }
  for (int k = 16; k > 0; k >>= 1) {
    const double og = __shfl_xor_sync(0xffffffffu, bg, k);
    const int oj = __shfl_xor_sync(0xffffffffu, bj, k);
    if (oj >= 0 && (bj < 0 || og > bg || (og == bg && oj < bj))) {
      bg = og;
      bj = oj;
    }
  }
  if (lane != 0) return;
  ts->child_done[c] = 0;
  const int leaf = P.child[side];
  LeafRec& L = ts->pool[leaf];
  const long long tg = __ldcg(&ts->totals[c].g), th = __ldcg(&ts->totals[c].h), n_rows = __ldcg(&ts->totals[c].c);
  SplitRec sr;
  clear_split(sr);
  if (bj >= 0 && !(n_rows < 2 * (long long)sp.min_data_in_leaf || n_rows < 2)) {
    const FeatBest* fb = fc + bj;
    sr.found = 1;
    sr.gain = __ldcg(&fb->gain);
    sr.feature = feats[bj];
    sr.bin = __ldcg(&fb->bin);
    const int flags = __ldcg(&fb->flags);
    sr.default_left = (flags & 2) ? 1 : 0;
    sr.is_cat = (flags & 4) ? 1 : 0;
    sr.n_left = __ldcg(&fb->n_left);
    for (int q = 0; q < 4; ++q) sr.bits[q] = __ldcg(&fb->bits[q]);
  }
  L.split = sr;
  const double gd = sp.mode == MODE_FIXED ? (double)tg * sc->g_inv : (double)tg / sc->g_units;
  const double hd = sp.mode == MODE_FIXED ? (double)th * sc->h_inv : (double)th / sc->h_units;
  L.value = -soft_l1(gd, sp.lambda_l1) / (hd + sp.lambda_l2);
  L.gcount = n_rows;
  LeafInfo& I = ts->info[leaf];
  I.gain = (sr.found && sr.gain > 0.0) ? sr.gain : -1.0;
  I.child[0] = I.child[1] = -1;
  I.expanded = 0;
  I.pad = 0;
  if (root) {
    NodeRec& nd = ts->nodes[L.node];
    nd.value = L.value;
    nd.count = n_rows;
  } else {
    const long long nl = (long long)P.cursor_left;
    L.begin = side == 0 ? P.begin : P.begin + nl;
    L.count = side == 0 ? nl : P.count - nl;
    ts->info[P.leaf].child[side] = leaf;
  }
}

// One warp per (child, active feature), 8 bins per lane: sibling
// subtraction, exact integer prefix sums, the reference gain per candidate
// threshold, and a warp arg-max that keeps the serial scan's tie rule (first
// maximum in bin order, missing-left candidate before default-right).  Pair
// p = child * n_active + j, child = 2 * item + side.
// The feature-sharded exchange's end of a child: the warp that completes
// child c folds this rank's per-feature bests exactly as scan_pair_done does
// (ascending active feature, strict >, the first maximum) and writes the
// result and the child's totals to rec[c]; the leaf itself is written by
// k_merge_children once every rank's record is gathered.
__device__ void scan_pair_done_exchange(TreeState* __restrict__ ts, int c, const FeatBest* __restrict__ fbs,
                                        const int* __restrict__ feats, const ScanParams& sp,
                                        ChildRec* __restrict__ rec) {
  const int lane = threadIdx.x & 31;
  unsigned int last = 0;
  if (lane == 0) {
    __threadfence();
    last = atomicAdd(&ts->child_done[c], 1u) == (unsigned int)(sp.n_active - 1) ? 1u : 0u;
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return;
  __threadfence();
  const FeatBest* fc = fbs + (long long)c * sp.n_active;
  double bg = 0.0;
  int bj = -1;
  for (int j = lane; j < sp.n_active; j += 32) {
    const int flags = __ldcg(&fc[j].flags);
    const double g = __ldcg(&fc[j].gain);
    if ((flags & 1) && g > bg) {
      bg = g;
      bj = j;
    }
  }
  for (int k = 16; k > 0; k >>= 1) {
    const double og = __shfl_xor_sync(0xffffffffu, bg, k);
    const int oj = __shfl_xor_sync(0xffffffffu, bj, k);
    if (oj >= 0 && (bj < 0 || og > bg || (og == bg && oj < bj))) {
      bg = og;
      bj = oj;
    }
  }
  if (lane != 0) return;
  ts->child_done[c] = 0;
  ChildRec& R = rec[c];
  R.tg = __ldcg(&ts->totals[c].g);
  R.th = __ldcg(&ts->totals[c].h);
  R.tc = __ldcg(&ts->totals[c].c);
  R.has_totals = 1;
  R.found = bj >= 0 ? 1 : 0;
  if (bj >= 0) {
    const FeatBest* fb = fc + bj;
    R.gain = __ldcg(&fb->gain);
    R.feature = feats[bj];
    R.bin = __ldcg(&fb->bin);
    R.flags = __ldcg(&fb->flags);
    R.n_left = __ldcg(&fb->n_left);
    for (int q = 0; q < 4; ++q) R.bits[q] = __ldcg(&fb->bits[q]);
  }
}

// One numerical split candidate (left sums Dg, Dh, Dc): the leaf guards and
// the gain, exactly the inline arithmetic of k_scan (same operations in the
// same order; the file is compiled without FMA contraction), or -infinity
// when a guard rejects it.  Out of line so the correctly rounded divisions
// appear once in the code rather than at every unrolled candidate site: the
// inline form makes k_scan instruction-fetch bound.
struct ScanCandCtx {
  int mode;
  double g_inv, h_inv, gu, hu, tg, th, l1, l2, mch, parent, parent_q;
  long long Tg, Th, Tc, mdl;
};

__device__ __noinline__ double scan_candidate_gain(long long Dg, long long Dh, long long Dc,
                                                   const ScanCandCtx& c) {
  const double dlg = deq(Dg, c.mode, c.g_inv, c.gu), dlh = deq(Dh, c.mode, c.h_inv, c.hu);
  const double drg = c.mode == MODE_FIXED ? c.tg - dlg : deq(c.Tg - Dg, c.mode, c.g_inv, c.gu);
  const double drh = c.mode == MODE_FIXED ? c.th - dlh : deq(c.Th - Dh, c.mode, c.h_inv, c.hu);
  if (dlh < c.mch || drh < c.mch || Dc < c.mdl || c.Tc - Dc < c.mdl) return -INFINITY;
  if (c.mode == MODE_FIXED) {
    const double tl = soft_l1(dlg, c.l1), tr = soft_l1(drg, c.l1);
    return tl * tl / (dlh + c.l2) + tr * tr / (drh + c.l2) - c.parent;
  }
  return leaf_score(dlg, dlh, c.l1, c.l2) + leaf_score(drg, drh, c.l1, c.l2) - c.parent_q;
}

constexpr int kScanWarps = 8;    // pairs per block
constexpr int kBinsPerLane = 8;  // 32 x 8 = 256 bins at most

template <bool COMPACT, bool EXCHANGE, bool WIDE = false>
__global__ void __launch_bounds__(kScanWarps * 32, 3) k_scan_t(TreeState* __restrict__ ts, int* __restrict__ hist,
                                                          long long slot_cells, const int* __restrict__ feats,
                                                          const int* __restrict__ missing_bin,
                                                          const int* __restrict__ n_cats,
                                                          const RoundScales* __restrict__ sc, ScanParams sp,
                                                          FeatBest* __restrict__ out, int work_base,
                                                          ChildRec* __restrict__ rec) {
  pdl_enter();
  using CT = typename std::conditional<WIDE, long long, int>::type;  // histogram cell type
  __shared__ CT s_cells[kScanWarps][3][256];  // categorical searches only
  const Batch& Bt = ts->batch;
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const long long pair = (long long)blockIdx.x * kScanWarps + wib;
  const int c = (int)(pair / sp.n_active);
  const int j = (int)(pair - (long long)c * sp.n_active);
  const int item = c >> 1, side = c & 1;
  if (item >= Bt.n_items) return;  // warp-uniform; the kernel has no block barrier
  if (Bt.root && side) return;
  const BatchItem& P = Bt.items[item];
  const int B = sp.B;
  const int f = feats[j];
  const bool built = Bt.root || side == (P.built_is_left ? 0 : 1);
  CT* hs = reinterpret_cast<CT*>(hist + (long long)(built ? P.built_hist : P.sib_hist) * slot_cells) + (long long)f * 3 * B;
  const CT* wk = reinterpret_cast<const CT*>(hist + (long long)(work_base + P.work) * slot_cells) + (long long)f * 3 * B;
  const int mode = sp.mode;
  const bool ch_fixed = sp.const_hess && mode == MODE_FIXED;
  const long long hq = ch_fixed ? (WIDE ? sc->hq_const64 : (long long)sc->hq_const) : 0;
  const int b0 = lane * kBinsPerLane;
  // built child: the (reduced) work slot; sibling: parent - built, in place
  CT vg[kBinsPerLane], vh[kBinsPerLane], vc[kBinsPerLane];
  long long sg = 0, sh = 0, scn = 0;
#pragma unroll
  for (int q = 0; q < kBinsPerLane; ++q) {
    const int b = b0 + q;
    vg[q] = 0;
    vh[q] = 0;
    vc[q] = 0;
    if (b < B) {
      const CT wg = wk[b], wh = wk[B + b], wc = wk[2 * B + b];
      if (built) {
        vg[q] = wg;
        vh[q] = wh;
        vc[q] = wc;
      } else {
        vg[q] = hs[b] - wg;
        vh[q] = hs[B + b] - wh;
        vc[q] = hs[2 * B + b] - wc;
      }
      hs[b] = vg[q];
      hs[B + b] = vh[q];
      hs[2 * B + b] = vc[q];
      if (ch_fixed) vh[q] = (CT)(hq * (long long)vc[q]);
    }
    sg += vg[q];
    sh += vh[q];
    scn += vc[q];
  }
  // warp scan of the lane totals: exclusive prefix = sums of earlier lanes
  long long ig = sg, ih = sh, ic = scn;
#pragma unroll
  for (int k = 1; k < 32; k <<= 1) {
    const long long og = __shfl_up_sync(0xffffffffu, ig, k);
    const long long oh = __shfl_up_sync(0xffffffffu, ih, k);
    const long long oc = __shfl_up_sync(0xffffffffu, ic, k);
    if (lane >= k) {
      ig += og;
      ih += oh;
      ic += oc;
    }
  }
  const long long Tg = __shfl_sync(0xffffffffu, ig, 31);
  const long long Th = __shfl_sync(0xffffffffu, ih, 31);
  const long long Tc = __shfl_sync(0xffffffffu, ic, 31);
  if (j == 0 && lane == 0) {
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
  CT(*cw)[256] = s_cells[wib];
  if (n_cats[f] >= 0) {
#pragma unroll
    for (int q = 0; q < kBinsPerLane; ++q) {
      cw[0][b0 + q] = vg[q];
      cw[1][b0 + q] = vh[q];
      cw[2][b0 + q] = vc[q];
    }
    __syncwarp();
    // categorical: serial search on thread 0 (categorical.mojo:478-780) over
    // the exact per-category sums
    if (lane == 0) {
      int n_cat = n_cats[f];
      double parent = leaf_score(tg, th, l1, l2);
      if (n_cat >= 2 && n_cat + 1 <= sp.max_cat_to_onehot) {
        for (int q = 1; q <= n_cat && q < B; ++q) {
          long long qg = cw[0][q], qh = cw[1][q], cc = cw[2][q];
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
          if (!((double)cw[2][q] >= sp.cat_smooth)) continue;
          double gv = deq(cw[0][q], mode, g_inv, gu);
          double hv = deq(cw[1][q], mode, h_inv, hu);
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
              qg += cw[0][q];
              qh += cw[1][q];
              qc += cw[2][q];
              cnt_group += cw[2][q];
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
    if (EXCHANGE) scan_pair_done_exchange(ts, c, out, feats, sp, rec);
    else scan_pair_done(ts, c, out, feats, sc, sp);
    return;
  }
  const int mb = missing_bin[f];
  const int n_scan = mb >= 0 ? mb : B;
  long long mg = 0, mh = 0, mc = 0;
  if (mb >= 0) {
    CT xg = 0, xh = 0, xc = 0;
#pragma unroll
    for (int q = 0; q < kBinsPerLane; ++q)
      if (b0 + q == mb) {
        xg = vg[q];
        xh = vh[q];
        xc = vc[q];
      }
    const int src = mb / kBinsPerLane;
    mg = __shfl_sync(0xffffffffu, xg, src);
    mh = __shfl_sync(0xffffffffu, xh, src);
    mc = __shfl_sync(0xffffffffu, xc, src);
  }
  const double pg = soft_l1(tg, l1);
  const double parent = pg * pg / (th + l2);
  const double parent_q = leaf_score(tg, th, l1, l2);
  double best_gain = 0.0;
  int best_key = 0x7fffffff;  // 2*bin + order
  long long best_nl = 0;
  long long Lg = ig - sg, Lh = ih - sh, Lc = ic - scn;  // prefix before this lane's bins
  const ScanCandCtx cx{mode, g_inv, h_inv, gu, hu, tg, th, l1, l2, mch, parent, parent_q, Tg, Th, Tc, mdl};
#pragma unroll
  for (int q = 0; q < kBinsPerLane; ++q) {
    const int b = b0 + q;
    Lg += vg[q];  // inclusive prefix through bin b
    Lh += vh[q];
    Lc += vc[q];
    if (!(b < n_scan && !(b == n_scan - 1 && mc == 0))) continue;
    if (COMPACT) {
      if (mb >= 0) {
        const double gain = scan_candidate_gain(Lg + mg, Lh + mh, Lc + mc, cx);
        if (gain > best_gain) {
          best_gain = gain;
          best_key = 2 * b;
          best_nl = Lc + mc;
        }
      }
      if (mb < 0 || mc > 0) {
        const double gain = scan_candidate_gain(Lg, Lh, Lc, cx);
        if (gain > best_gain) {
          best_gain = gain;
          best_key = 2 * b + 1;
          best_nl = Lc;
        }
      }
      continue;
    }
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
  // warp arg-max: higher gain, then lower key (earlier in the serial scan)
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
    if (best_key != 0x7fffffff && best_gain > 0.0) {
      fb.gain = best_gain;
      fb.bin = best_key >> 1;
      fb.flags = 1 | ((best_key & 1) ? 0 : 2);
      fb.n_left = best_nl;
    }
    out[(long long)c * sp.n_active + j] = fb;
  }
  if (EXCHANGE) scan_pair_done_exchange(ts, c, out, feats, sp, rec);
  else scan_pair_done(ts, c, out, feats, sc, sp);
}

// Feature-sharded exchange: every rank's ChildRec of this iteration, gathered
// rank-major (all[r * stride + c]).  One thread per child folds the ranks in
// ascending order with a strict > (ranks own ascending feature blocks, so this
// keeps the first maximum over all features, the single-device rule), takes
// the totals from the first rank that has them, and writes the child's leaf
// exactly as scan_pair_done does.  Every rank runs it on the same gathered
// records, so every rank holds the same tree.
__global__ void k_merge_children(TreeState* __restrict__ ts, const ChildRec* __restrict__ all, int world,
                                 int stride, const RoundScales* __restrict__ sc, ScanParams sp) {
  const Batch& Bt = ts->batch;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= 2 * Bt.n_items) return;
  const int item = c >> 1, side = c & 1;
  const bool root = Bt.root != 0;
  if (root && side) return;
  int best = -1, tot = -1;
  double bg = 0.0;
  for (int r = 0; r < world; ++r) {
    const ChildRec& R = all[(long long)r * stride + c];
    if (tot < 0 && R.has_totals) tot = r;
    if (R.found && R.gain > bg) {
      bg = R.gain;
      best = r;
    }
  }
  if (tot < 0) {  // no rank scanned this child: nothing to build its leaf from
    ts->hdr.error = 1;
    ts->hdr.done = 1;
    return;
  }
  const ChildRec& T = all[(long long)tot * stride + c];
  const BatchItem& P = Bt.items[item];
  const int leaf = P.child[side];
  LeafRec& L = ts->pool[leaf];
  const long long tg = T.tg, th = T.th, n_rows = T.tc;
  SplitRec sr;
  clear_split(sr);
  if (best >= 0 && !(n_rows < 2 * (long long)sp.min_data_in_leaf || n_rows < 2)) {
    const ChildRec& R = all[(long long)best * stride + c];
    sr.found = 1;
    sr.gain = R.gain;
    sr.feature = R.feature;
    sr.bin = R.bin;
    sr.default_left = (R.flags & 2) ? 1 : 0;
    sr.is_cat = (R.flags & 4) ? 1 : 0;
    sr.n_left = R.n_left;
    for (int q = 0; q < 4; ++q) sr.bits[q] = R.bits[q];
  }
  L.split = sr;
  const double gd = sp.mode == MODE_FIXED ? (double)tg * sc->g_inv : (double)tg / sc->g_units;
  const double hd = sp.mode == MODE_FIXED ? (double)th * sc->h_inv : (double)th / sc->h_units;
  L.value = -soft_l1(gd, sp.lambda_l1) / (hd + sp.lambda_l2);
  L.gcount = n_rows;
  LeafInfo& I = ts->info[leaf];
  I.gain = (sr.found && sr.gain > 0.0) ? sr.gain : -1.0;
  I.child[0] = I.child[1] = -1;
  I.expanded = 0;
  I.pad = 0;
  if (root) {
    NodeRec& nd = ts->nodes[L.node];
    nd.value = L.value;
    nd.count = n_rows;
  } else {
    const long long nl = (long long)P.cursor_left;
    L.begin = side == 0 ? P.begin : P.begin + nl;
    L.count = side == 0 ? nl : P.count - nl;
    ts->info[P.leaf].child[side] = leaf;
  }
}

// ---------------------------------------------------------------------------
// Commit: one 1024-thread block after every scan.
//
// 1. Fold each new child's per-feature bests (ascending feature, strict >),
//    apply the leaf guards, write its split, value and local row range.
// 2. Replay the reference's pick loop (growth_policy.mojo:659-677: largest
//    gain > 0, lowest frontier slot on ties) over the frontier, committing
//    every pick whose children are already computed, until the leaf budget is
//    spent, no leaf has a positive gain (tree done), or the pick still needs
//    its expansion.
// 3. Select the next batch: the first m frontier leaves in pick order,
//    m = min(batch capacity, leaves still to add); those not yet expanded
//    become the batch (the current pick is always among them).
// ---------------------------------------------------------------------------

constexpr int kCommitThreads = 1024;

struct CommitParams {
  int num_leaves;
  int batch_cap;       // leaves expanded per iteration at most (<= kMaxBatch)
  int hist_slots;      // histogram slots available for leaves
  int tile_rows;       // rows per partition tile
  int ranked_select;   // choose the next batch by bottleneck keys (block-parallel) instead of a pick-loop replay
};


__device__ __forceinline__ double frontier_gain(const LeafRec& L) {
  return (L.split.found && L.split.gain > 0.0) ? L.split.gain : -1.0;
}

// Shared memory of k_commit (dynamic): per leaf of the budget, the frontier
// (slot -> leaf, gain), the commit list (slot, leaf) and the simulated
// frontier (leaf, gain); then the per-leaf table for the first leaf records
// (records beyond it are read from global memory).
constexpr int kCommitSlotBytes = 8 + 4 + 4 + 4 + 4 + 8 + 4 + 4;

// Per leaf record kept in shared memory: its table entry and its bottleneck key
// (ranked batch selection).
constexpr int kCommitInfoBytes = (int)sizeof(LeafInfo) + 8;

// Leaf records whose table entries k_commit keeps in shared memory: every
// record a tree of num_leaves can allocate, within about 200 KB.
inline int commit_info_cap(int num_leaves) {
  const long long slots = (long long)num_leaves * kCommitSlotBytes;
  const long long fit = (200ll * 1024 - slots) / (long long)kCommitInfoBytes;
  const long long want = 4ll * num_leaves + 2 * kMaxBatch + 2;
  return (int)std::max(0ll, std::min(want, fit));
}

inline size_t commit_smem_bytes(int num_leaves) {
  return (size_t)num_leaves * kCommitSlotBytes + (size_t)commit_info_cap(num_leaves) * kCommitInfoBytes;
}

__global__ void __launch_bounds__(kCommitThreads) k_commit(TreeState* __restrict__ ts,
                                                           const int* __restrict__ missing_bin, CommitParams cp,
                                                           int info_cap, int* __restrict__ host_done,
                                                           int host_done_index) {
  pdl_enter();
  if (ts->hdr.done) {  // an iteration the host launched ahead after the tree was finished
    if (threadIdx.x == 0 && host_done) {
      volatile int* hd = host_done;
      hd[host_done_index] = 1;
    }
    return;
  }
  extern __shared__ __align__(16) unsigned char commit_smem[];
  const int L_max = cp.num_leaves;
  double* s_g = reinterpret_cast<double*>(commit_smem);   // slot -> gain (-1: cannot split)
  double* s_vg = s_g + L_max;                              // simulated frontier: gain
  double* s_key = s_vg + L_max;                            // leaf record -> bottleneck key (ranked selection)
  LeafInfo* s_info = reinterpret_cast<LeafInfo*>(s_key + info_cap);  // leaf records [0, info_cap)
  int* s_slot_leaf = reinterpret_cast<int*>(s_info + info_cap);  // slot -> leaf
  int* s_cslot = s_slot_leaf + L_max;                      // commit k: slot ...
  int* s_cpar = s_cslot + L_max;                           // ... and the leaf split there
  int* s_vleaf = s_cpar + L_max;                           // simulated frontier: leaf
  int* s_slot_node = s_vleaf + L_max;                      // slot -> node id of its leaf
  int* s_cnode = s_slot_node + L_max;                      // commit k: node id of the split leaf
  __shared__ int s_block, s_changed;
  __shared__ int s_ncommit, s_stop, s_nl, s_nsel;
  __shared__ int s_sel[kMaxBatch];
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  TreeHeader& H = ts->hdr;
  Batch& Bt = ts->batch;
  const int n_items = Bt.n_items;
  const bool root = Bt.root != 0;
  const int n_pool = H.n_pool;
  const int cap = n_pool < info_cap ? n_pool : info_cap;
  auto info = [&](int leaf) -> LeafInfo& { return leaf < cap ? s_info[leaf] : ts->info[leaf]; };

  // ---- 1. leaf table and frontier into shared memory; this iteration's
  // expanded leaves (whose children the scan just folded) are marked
  for (int i = t; i < cap; i += kCommitThreads) s_info[i] = ts->info[i];
  const int nl0 = H.n_leaves;
  for (int i = t; i < nl0; i += kCommitThreads) s_slot_leaf[i] = ts->slot_leaf[i];
  __syncthreads();
  if (!root && t < n_items) {
    const int leaf = Bt.items[t].leaf;
    info(leaf).expanded = 1;
    ts->info[leaf].expanded = 1;
    ts->pool[leaf].state = 1;
  }
  __syncthreads();
  for (int i = t; i < nl0; i += kCommitThreads) {
    s_g[i] = info(s_slot_leaf[i]).gain;
    s_slot_node[i] = ts->pool[s_slot_leaf[i]].node;
  }
  __syncthreads();

  // Arg-max of the pick order over gains g[0, n) (larger gain, then lower
  // slot; only gains > 0 count), on one warp.  A positive double orders like
  // its bit pattern, so the warp reduces 64-bit keys with two max reductions
  // of 32-bit halves and takes the lowest slot holding the maximum.
  auto warp_pick = [&](const double* g, int n) -> int {
    unsigned long long best = 0ull;
    int best_i = 0x7fffffff;
    for (int i0 = 0; i0 < n; i0 += 256) {
      double x[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int i = i0 + q * 32 + lane;
        x[q] = i < n ? g[i] : -1.0;
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const unsigned long long k = x[q] > 0.0 ? (unsigned long long)__double_as_longlong(x[q]) : 0ull;
        if (k > best) {  // strict: the lane's lowest slot wins ties
          best = k;
          best_i = i0 + q * 32 + lane;
        }
      }
    }
    const unsigned int hi = __reduce_max_sync(0xffffffffu, (unsigned int)(best >> 32));
    const unsigned int lo =
        __reduce_max_sync(0xffffffffu, (unsigned int)(best >> 32) == hi ? (unsigned int)best : 0u);
    const unsigned long long top = ((unsigned long long)hi << 32) | lo;
    if (top == 0ull) return -1;
    return __reduce_min_sync(0xffffffffu, best == top ? best_i : 0x7fffffff);
  };

  // Up to 256 frontier slots the pick loops keep in warp 0's registers
  // instead: slot s is key[s >> 5] of lane s & 31, its gain's bit pattern (0
  // when the gain is not > 0), so a pick is three warp reductions with no
  // shared-memory traffic and an update is two predicated moves.
  const bool reg_frontier = L_max <= 256;
  unsigned long long k0 = 0, k1 = 0, k2 = 0, k3 = 0, k4 = 0, k5 = 0, k6 = 0, k7 = 0;
  auto key_of = [](double g) -> unsigned long long {
    return g > 0.0 ? (unsigned long long)__double_as_longlong(g) : 0ull;
  };
#define MTB_FRONTIER_SET(SLOT, G)                              \
  do {                                                         \
    const int s_ = (SLOT);                                     \
    const unsigned long long k_ = key_of(G);                   \
    if (lane == (s_ & 31)) {                                   \
      const int q_ = s_ >> 5;                                  \
      k0 = q_ == 0 ? k_ : k0;                                  \
      k1 = q_ == 1 ? k_ : k1;                                  \
      k2 = q_ == 2 ? k_ : k2;                                  \
      k3 = q_ == 3 ? k_ : k3;                                  \
      k4 = q_ == 4 ? k_ : k4;                                  \
      k5 = q_ == 5 ? k_ : k5;                                  \
      k6 = q_ == 6 ? k_ : k6;                                  \
      k7 = q_ == 7 ? k_ : k7;                                  \
    }                                                          \
  } while (0)
  auto reg_pick = [&]() -> int {
    // the lane's best slot by a depth-3 tournament; on equal keys the lower
    // slot (lower q) wins, so the lane's lowest slot holding its maximum
    auto better = [](unsigned long long ka, int qa, unsigned long long kb, int qb, unsigned long long& k, int& q) {
      const bool a = ka >= kb;
      k = a ? ka : kb;
      q = a ? qa : qb;
    };
    unsigned long long k01, k23, k45, k67, k03, k47, best;
    int q01, q23, q45, q67, q03, q47, qb;
    better(k0, 0, k1, 1, k01, q01);
    better(k2, 2, k3, 3, k23, q23);
    better(k4, 4, k5, 5, k45, q45);
    better(k6, 6, k7, 7, k67, q67);
    better(k01, q01, k23, q23, k03, q03);
    better(k45, q45, k67, q67, k47, q47);
    better(k03, q03, k47, q47, best, qb);
    const int best_i = best > 0ull ? qb * 32 + lane : 0x7fffffff;
    const unsigned int hi = __reduce_max_sync(0xffffffffu, (unsigned int)(best >> 32));
    const unsigned int lo =
        __reduce_max_sync(0xffffffffu, (unsigned int)(best >> 32) == hi ? (unsigned int)best : 0u);
    const unsigned long long top = ((unsigned long long)hi << 32) | lo;
    if (top == 0ull) return -1;
    return (int)__reduce_min_sync(0xffffffffu, best == top ? (unsigned int)best_i : 0x7fffffffu);
  };
  if (w == 0 && reg_frontier) {
    for (int q = 0; q < 8; ++q) {
      const int slot = q * 32 + lane;
      MTB_FRONTIER_SET(slot, slot < nl0 ? s_g[slot] : -1.0);
    }
  }

  // ---- 2. the pick loop (growth_policy.mojo:659-677), on one warp over
  // shared memory: commit every pick whose children are computed
  if (w == 0) {
    int nl = nl0;
    int n_commit = 0;
    int stop = H.done;
    while (!stop && nl < L_max) {
      const int bs = reg_frontier ? reg_pick() : warp_pick(s_g, nl);
      if (bs < 0) {
        stop = 1;
        break;
      }
      const int leaf = s_slot_leaf[bs];
      const LeafInfo I = info(leaf);
      if (!I.expanded) {  // the pick still needs its expansion
        if (lane == 0) s_block = leaf;
        break;
      }
      if (reg_frontier) {
        MTB_FRONTIER_SET(bs, info(I.child[0]).gain);
        MTB_FRONTIER_SET(nl, info(I.child[1]).gain);
      }
      if (lane == 0) {
        // node ids are assigned here, in commit order: a child committed in
        // the same launch as its parent finds its id in s_slot_node
        s_cslot[n_commit] = bs;
        s_cpar[n_commit] = leaf;
        s_cnode[n_commit] = s_slot_node[bs];
        s_slot_leaf[bs] = I.child[0];
        s_g[bs] = info(I.child[0]).gain;
        s_slot_node[bs] = H.n_nodes + 2 * n_commit;
        s_slot_leaf[nl] = I.child[1];
        s_g[nl] = info(I.child[1]).gain;
        s_slot_node[nl] = H.n_nodes + 2 * n_commit + 1;
      }
      __syncwarp();
      ++n_commit;
      ++nl;
    }
    if (nl >= L_max) stop = 1;
    if (lane == 0) {
      H.pick_steps += n_commit + 1;
      s_ncommit = n_commit;
      s_nl = nl;
      s_stop = stop;
    }
  }
  __syncthreads();

  // ---- 3. the commits' writes, one thread each, and the frontier back
  const int n_commit = s_ncommit;
  const int nl = s_nl;
  const int nodes0 = H.n_nodes;
  // children's node records first: a leaf committed in the same launch as
  // its parent has its record reset here and its split written below
  for (int k = t; k < n_commit; k += kCommitThreads) {
    LeafRec& L = ts->pool[s_cpar[k]];
    const int left_node = nodes0 + 2 * k, right_node = left_node + 1;
    LeafRec& CL = ts->pool[L.child[0]];
    LeafRec& CR = ts->pool[L.child[1]];
    CL.node = left_node;
    CR.node = right_node;
    clear_node(ts->nodes[left_node], CL.value, CL.gcount);
    clear_node(ts->nodes[right_node], CR.value, CR.gcount);
  }
  __syncthreads();
  for (int k = t; k < n_commit; k += kCommitThreads) {
    LeafRec& L = ts->pool[s_cpar[k]];
    const SplitRec& s = L.split;
    const int left_node = nodes0 + 2 * k, right_node = left_node + 1;
    NodeRec& pn = ts->nodes[s_cnode[k]];
    pn.feature = s.feature;
    pn.gain = s.gain;
    pn.left = left_node;
    pn.right = right_node;
    pn.is_cat = s.is_cat;
    if (s.is_cat) {
      pn.thr = -1;
      pn.dleft = 0;
      pn.mbin = -1;
      for (int q = 0; q < 4; ++q) pn.bits[q] = s.bits[q];
    } else {
      pn.thr = s.bin;
      pn.dleft = s.default_left;
      pn.mbin = missing_bin[s.feature];
    }
    L.state = 2;
  }
  for (int i = t; i < nl; i += kCommitThreads) ts->slot_leaf[i] = s_slot_leaf[i];
  if (t == 0) {
    H.n_nodes = nodes0 + 2 * n_commit;
    H.n_leaves = nl;
  }

  // ---- 4. next batch: the leaves the pick loop will need next, in order.
  // By default they are ranked by bottleneck keys (below).  Otherwise the
  // loop is simulated past this point on a copy of the frontier: an
  // expanded leaf is committed virtually (its children, with their known
  // gains, take its slot and the next one), an unexpanded one is taken into
  // the batch and leaves the simulated frontier.  The first leaf taken is the
  // one the real loop stopped at, so every iteration commits a split.
  if (s_stop) {
    if (t == 0) {
      H.done = 1;
      Bt.n_items = 0;
      Bt.root = 0;
      Bt.n_tiles = 0;
    }
  } else {
    if (cp.ranked_select && cap == n_pool) {
      // Block-parallel selection.  A best-first replay takes the virtual tree's
      // nodes in decreasing order of their bottleneck key, the smallest gain on
      // the path from the frontier (a node is only available once its parent is
      // taken), so the leaves it would expand next are the unexpanded nodes
      // reachable through expanded ones with the largest keys (ties by leaf id
      // here, which only decides speculation, never the tree).  The leaf the
      // commit loop stopped at goes first, so every iteration commits a split.
      for (int i = t; i < cap; i += kCommitThreads) s_key[i] = -2.0;
      __syncthreads();
      for (int i = t; i < nl; i += kCommitThreads) s_key[s_slot_leaf[i]] = s_g[i];
      for (;;) {
        __syncthreads();
        if (t == 0) s_changed = 0;
        __syncthreads();
        for (int i = t; i < cap; i += kCommitThreads) {
          const double k = s_key[i];
          if (k > 0.0 && s_info[i].expanded)
            for (int side = 0; side < 2; ++side) {
              const int c = s_info[i].child[side];
              const double g = s_info[c].gain;
              const double kc = g < k ? g : k;
              if (s_key[c] != kc) {
                s_key[c] = kc;
                s_changed = 1;
              }
            }
        }
        __syncthreads();
        if (!s_changed) break;
      }
      const int blk = s_block;
      if (t == 0) s_nsel = 1;
      // A candidate's replay step is the nodes taken before it: the stopped
      // leaf, the candidates ranked above it and the expanded nodes whose key
      // is not below its own (each adds a leaf).  It is selected when the
      // replay reaches it before the tree is full and within the batch.
      __syncthreads();
      const int room = L_max - nl;
      for (int i = t; i < cap; i += kCommitThreads) {
        const double ka = s_key[i];
        if (!(ka > 0.0) || s_info[i].expanded || i == blk) continue;
        int r = 0, e = 0;
        for (int b = 0; b < cap; ++b) {
          const double kb = s_key[b];
          if (!(kb >= ka)) continue;
          if (s_info[b].expanded) ++e;
          else if (b != blk && (kb > ka || b < i)) ++r;
        }
        if (1 + r < cp.batch_cap && 1 + r + e < room) {
          s_sel[1 + r] = i;
          atomicAdd(&s_nsel, 1);
        }
      }
      if (t == 0) s_sel[0] = blk;
    } else {
      for (int i = t; i < nl; i += kCommitThreads) {
        s_vleaf[i] = s_slot_leaf[i];
        s_vg[i] = s_g[i];
      }
      __syncthreads();
      if (w == 0) {
        int vn = nl, vleaves = nl, n_sel = 0;
        while (n_sel < cp.batch_cap && vleaves < L_max) {
          const int bs = reg_frontier ? reg_pick() : warp_pick(s_vg, vn);
          if (bs < 0) break;
          const int leaf = s_vleaf[bs];
          const LeafInfo I = info(leaf);
          if (reg_frontier) {
            if (I.expanded) {
              MTB_FRONTIER_SET(bs, info(I.child[0]).gain);
              MTB_FRONTIER_SET(vn, info(I.child[1]).gain);
            } else {
              MTB_FRONTIER_SET(bs, -1.0);
            }
          }
          if (lane == 0) {
            if (I.expanded) {
              s_vleaf[bs] = I.child[0];
              s_vg[bs] = info(I.child[0]).gain;
              s_vleaf[vn] = I.child[1];
              s_vg[vn] = info(I.child[1]).gain;
            } else {
              s_sel[n_sel] = leaf;
              s_vg[bs] = -1.0;
            }
          }
          __syncwarp();
          if (I.expanded) ++vn;
          else ++n_sel;
          ++vleaves;
        }
        if (lane == 0) {
          s_nsel = n_sel;
          H.pick_steps += vleaves - nl;
        }
      }
    }
    __syncthreads();
    if (w == 0) {
      const int n_sel = s_nsel;
      // histogram slots: every later real commit may need one expansion, so
      // speculative items only use slots beyond that reserve; leaf records
      // take two per item
      const int pool0 = H.n_pool, hist0 = H.n_hist;
      const int free_slots = cp.hist_slots - hist0;
      const int reserve = cp.num_leaves - nl;
      int n_new = n_sel;
      const int spec = free_slots - reserve;
      if (n_new > 1 + (spec > 0 ? spec : 0)) n_new = 1 + (spec > 0 ? spec : 0);
      if (n_new > free_slots) n_new = free_slots;
      if (n_new > (kMaxPool - pool0) / 2) n_new = (kMaxPool - pool0) / 2;
      if (n_new < 0) n_new = 0;
      // item set-up, lane per item, 32 items per pass; the items' partition
      // tiles get an exclusive prefix (tile0) over all passes
      auto setup = [&](int idx) -> long long {
        const int leaf = s_sel[idx];
        LeafRec& L = ts->pool[leaf];
        const SplitRec& s = L.split;
        BatchItem& P = Bt.items[idx];
        const long long n_left = s.n_left, n_right = L.gcount - s.n_left;
        P.leaf = leaf;
        P.child[0] = pool0 + 2 * idx;
        P.child[1] = pool0 + 2 * idx + 1;
        P.built_is_left = n_left <= n_right ? 1 : 0;
        P.work = idx;
        P.built_hist = hist0 + idx;
        P.sib_hist = L.hist_slot;
        P.feature = s.feature;
        P.threshold = s.bin;
        P.default_left = s.default_left;
        P.missing_bin = s.is_cat ? -1 : missing_bin[s.feature];
        P.is_cat = s.is_cat;
        for (int q = 0; q < 4; ++q) P.bits[q] = s.bits[q];
        P.src_buf = L.buf;
        P.dst_buf = 1 - L.buf;
        P.begin = L.begin;
        P.count = L.count;
        P.cursor_left = 0;
        P.cursor_right = 0;
        L.child[0] = P.child[0];
        L.child[1] = P.child[1];
        L.exp_buf = P.dst_buf;
        for (int side = 0; side < 2; ++side) {
          LeafRec& C = ts->pool[P.child[side]];
          C.node = -1;
          C.parent = leaf;
          C.buf = P.dst_buf;
          C.hist_slot = (side == 0) == (P.built_is_left != 0) ? P.built_hist : P.sib_hist;
          C.state = 0;
          C.child[0] = C.child[1] = -1;
          C.exp_buf = 0;
          C.begin = 0;
          C.count = 0;
          C.gcount = 0;
          C.value = 0.0;
          clear_split(C.split);
          LeafInfo& CI = ts->info[P.child[side]];
          CI.gain = -1.0;
          CI.child[0] = CI.child[1] = -1;
          CI.expanded = 0;
          CI.pad = 0;
        }
        return (L.count + cp.tile_rows - 1) / cp.tile_rows;
      };
      long long total = 0;
      for (int base = 0; base < n_new; base += 32) {
        const int idx = base + lane;
        const bool take = idx < n_new;
        const long long tiles = take ? setup(idx) : 0;
        long long incl = tiles;
        for (int k = 1; k < 32; k <<= 1) {
          const long long o = __shfl_up_sync(0xffffffffu, incl, k);
          if (lane >= k) incl += o;
        }
        if (take) Bt.items[idx].tile0 = total + incl - tiles;
        total += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) {
        if (n_new == 0) {
          H.error = 1;  // reserved space exhausted (cannot happen within the bounds above)
          H.done = 1;
        }
        Bt.n_items = n_new;
        Bt.root = 0;
        Bt.n_tiles = total;
        H.n_pool = pool0 + 2 * n_new;
        H.n_hist = hist0 + n_new;
      }
    }
  }
  __syncthreads();
  if (t == 0) {
    H.iterations += 1;
    if (host_done) {
      // mapped host memory: the host learns without a copy in the stream
      volatile int* hd = host_done;
      hd[host_done_index] = H.done ? 1 : 0;  // read after the host synchronises on this iteration's event
    }
  }
}
#undef MTB_FRONTIER_SET

// After the last iteration: the row -> leaf-value map.  The unexpanded leaf
// records (committed leaves and speculative children) tile this device's rows:
// an unexpanded record's range in its own buffer was written by its parent's
// partition and nothing has written there since.  A committed leaf that was
// expanded but never split may have lost its own buffer to a speculative
// grandchild's partition, so its rows are taken from its unexpanded
// descendants, each of which takes the value of its nearest committed
// ancestor (the first record up the chain with a node id).  The table holds
// the non-empty records sorted by range start (their starts are distinct).
__global__ void __launch_bounds__(1024) k_leaf_table(TreeState* __restrict__ ts, long long* __restrict__ begins,
                                                     int* __restrict__ bufs, double* __restrict__ values,
                                                     int stage_cap) {
  // the leaf records' range starts, staged once when they fit (the rank of a
  // record is the number of non-empty unexpanded records that start before it)
  extern __shared__ long long s_begin[];  // n_pool entries, or none
  __shared__ int s_n;
  const int n_pool = ts->hdr.n_pool;
  const bool staged = n_pool <= stage_cap;
  auto begin_of = [&](int k) -> long long {
    if (staged) return s_begin[k];
    const LeafRec& Lk = ts->pool[k];
    return (Lk.state == 0 && Lk.count > 0) ? Lk.begin : -1;
  };
  if (threadIdx.x == 0) s_n = 0;
  if (staged)
    for (int k = threadIdx.x; k < n_pool; k += blockDim.x) {
      const LeafRec& Lk = ts->pool[k];
      s_begin[k] = (Lk.state == 0 && Lk.count > 0) ? Lk.begin : -1;
    }
  __syncthreads();
  for (int i = threadIdx.x; i < n_pool; i += blockDim.x) {
    const long long bi = begin_of(i);
    if (bi < 0) continue;
    int rank = 0;
    for (int k = 0; k < n_pool; ++k) {
      const long long bk = begin_of(k);
      if (bk >= 0 && bk < bi) ++rank;
    }
    int a = i;
    while (ts->pool[a].node < 0) a = ts->pool[a].parent;
    begins[rank] = bi;
    bufs[rank] = ts->pool[i].buf;
    values[rank] = ts->pool[a].value;
    atomicAdd(&s_n, 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) ts->hdr.n_table = s_n;
}

// raw[row * K + k] = fma(lr, value(leaf of row), raw[row * K + k])
// (boosting.mojo:1991-2111, explicit fused multiply-add), in two passes.
// The leaf table lists rows by buffer position, so updating raw in position
// order is a scattered 8-byte read-modify-write of the score array (each
// touching its own 32-byte sector).  Instead, k_row_slots walks the positions
// and scatters each row's table entry as a 2-byte slot into an N-entry array
// small enough to stay in L2, and k_update_raw then walks the rows in order:
// the slot and score loads and the score store are coalesced.  Every row gets
// the same fma of the same operands, so the scores are bit-identical to a
// position-order update.  Every row sits in exactly one table range, so every
// slot is rewritten each tree and the array needs no clearing.
__global__ void __launch_bounds__(256) k_row_slots(const TreeState* __restrict__ ts,
                                                   const long long* __restrict__ begins,
                                                   const int* __restrict__ bufs, const int* __restrict__ rows0,
                                                   const int* __restrict__ rows1,
                                                   unsigned short* __restrict__ slot_of_row, long long n,
                                                   int stage_cap) {
  extern __shared__ long long s_tab[];  // stage_cap entries: begin, buffer
  long long* s_begin = s_tab;
  int* s_buf = reinterpret_cast<int*>(s_tab + stage_cap);
  const int nt = ts->hdr.n_table;
  const bool staged = nt <= stage_cap;
  if (staged)
    for (int t = threadIdx.x; t < nt; t += blockDim.x) {
      s_begin[t] = begins[t];
      s_buf[t] = bufs[t];
    }
  __syncthreads();
  if (!staged) {
    s_begin = const_cast<long long*>(begins);
    s_buf = const_cast<int*>(bufs);
  }
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int lo = 0, hi = nt - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_begin[mid] <= i) lo = mid;
      else hi = mid - 1;
    }
    const int* rows = s_buf[lo] ? rows1 : rows0;
    slot_of_row[rows[i]] = (unsigned short)lo;
  }
}

__global__ void __launch_bounds__(256) k_update_raw(const TreeState* __restrict__ ts,
                                                    const double* __restrict__ values,
                                                    const unsigned short* __restrict__ slot_of_row,
                                                    double* __restrict__ raw, long long n, int K, int k, double lr,
                                                    int stage_cap) {
  extern __shared__ double s_val[];  // stage_cap leaf values
  const int nt = ts->hdr.n_table;
  const bool staged = nt <= stage_cap;
  if (staged)
    for (int t = threadIdx.x; t < nt; t += blockDim.x) s_val[t] = values[t];
  __syncthreads();
  const double* vals = staged ? s_val : values;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += stride) {
    double* p = raw + r * K + k;
    *p = fma(lr, vals[slot_of_row[r]], *p);
  }
}

}  // namespace
}  // namespace mtb
