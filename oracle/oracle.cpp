// ORACLE -- test infrastructure only.  Nothing in the product links, imports
// or executes this file; only tests/, __graft_entry__.smoke() and bench.py's
// CPU-baseline leg do, as the checker.
//
// A plain C++ restatement of the reference (ajhendel/mojoboost, "mojotrees")
// CPU training path for dense binned data, used for three things:
//   1. pinned against the reference's own golden bit patterns
//      (tests/test_golden_bits.mojo, fixtures at :7920-8120) in MODE_CPU;
//   2. the parity oracle for the GPU trainer's two integer histogram modes,
//      MODE_FIXED (the reference's shipped device semantics: pow2 fixed-point
//      Int32 cells, histogram.mojo:3457-3700) and MODE_QUANT (LightGBM-style
//      int8 gradients with seeded stochastic rounding, quantized_gradient.mojo
//      composed as its STATUS section prescribes, :194-256);
//   3. the timed CPU baseline (OpenMP over features), labelled as a C++
//      restatement of the reference CPU path, not the reference binary.
//
// Reference line map (all paths under src/mojotrees/):
//   boosting.mojo:521-577    _base_score
//   boosting.mojo:676-812    per-row derivatives, narrowed to Float32 (:462-480 of histogram.mojo)
//   boosting.mojo:2416-3008  the round loop (_boost_rounds); :1991-2111 fma raw update by leaf;
//                            :1947-1988 raw update by traversal (bagged rounds)
//   boosting.mojo:3876-4249  multiclass rounds, softmax :3515-3572, derivatives :3621-3677
//   tree.mojo:3125-4289      leaf-wise grower (grow_tree_leaves_profiled)
//   tree.mojo:733-826        stable partition;  tree.mojo:1961-1995 _leaf_value
//   tree.mojo:2011-2113      _search guards
//   histogram.mojo:1617-2010, 2257-2440, 2845-3453  Float64 accumulation and row-block fold
//   apple_cpu_policy.mojo:778-924  row-block plan (blocks = rows // (16 * n_bins), <= 64, <= 16 MiB)
//   histogram.mojo:3760-3960 sibling subtraction
//   split.mojo:601-1360      find_best_split (SIMD-lane totals, strict > scans and fold)
//   categorical.mojo:478-780 one-hot and sorted categorical searches; tree_parameters_extra.mojo:985-1042
//   growth_policy.mojo:659-677 leaf pick (max gain, lowest frontier slot on ties)
//   bagging.mojo:81-150, sampling.mojo:319-463 bags and per-tree feature sampling
//   quantized_gradient.mojo:762-815, 1343-1453, 1479-1545, 2487-2566, 2947-3195 quantized mode
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <stdexcept>
#include <string>
#include <vector>

#include "../mojoboost_b200/csrc/mt_math.h"

extern "C" {

typedef struct {
  int objective;  // 0 = L2 (squared error), 1 = binary logistic, 2 = multiclass softmax
  int n_classes;
  int num_rounds;
  double learning_rate;
  int num_leaves;
  int min_data_in_leaf;
  double lambda_l2;
  double min_child_hess;
  double lambda_l1;
  double feature_fraction;
  int feature_fraction_seed;
  double bagging_fraction;
  int bagging_freq;
  int bagging_seed;
  int max_cat_to_onehot;
  int max_cat_threshold;
  double cat_smooth;
  double cat_l2;
  int min_data_per_group;
  int mode;            // 0 = CPU Float64 histograms, 1 = fixed-point Int32, 2 = quantized int8
  int exp_kind;        // 0 = libm exp, 1 = mt_exp (the GPU trainer's exp)
  int quant_bins;      // num_grad_quant_bins (4)
  int quant_seed;      // 11
  int simd_lanes;      // SIMD_LANES of split.mojo feature totals (8 on arm64)
  int lane_reduce;     // 0 = pairwise halving, 1 = sequential
  int traversal_fma;   // bagged raw update: 1 = fma(lr, v, raw), 0 = raw + lr * v
  int n_threads;       // 0 = all
  const double* base_override;  // [n_classes] initial scores to use instead of the computed ones, or NULL
} mt_oracle_params;

typedef struct {
  int n_trees;
  int max_nodes;          // capacity per tree
  int* n_nodes;           // [n_trees_cap]
  int* feature;           // [n_trees_cap * max_nodes]
  int* threshold_bin;
  int* left;
  int* right;
  int* default_left;
  int* missing_bin;
  uint64_t* cat_bits;     // [n_trees_cap * max_nodes * 4]
  double* value;
  double* gain;
  int64_t* count;
  double* raw;            // [n_rows * n_classes]
  double* base_scores;    // [n_classes]
  double* round_seconds;  // [num_rounds] wall-clock seconds at the end of each round since the fit
                          // began (the CPU baseline's per-round timing), or NULL
} mt_oracle_out;

}  // extern "C"

namespace {

enum { MODE_CPU = 0, MODE_FIXED = 1, MODE_QUANT = 2, MODE_FIXED52 = 3 };
// MODE_FIXED52: the fixed-point mode with the scale bound raised from 2^30 to
// 2^52 (Int64 cells): every dequantized sum is still exact in Float64, and the
// per-row rounding error drops to 2^-53 of the |g| total.
inline bool fixed_point(int mode) { return mode == MODE_FIXED || mode == MODE_FIXED52; }
enum { OBJ_L2 = 0, OBJ_LOGISTIC = 1, OBJ_SOFTMAX = 2 };

struct Data {
  const uint8_t* bins;  // feature-major bins[f * n + r]
  int64_t n;
  int F;
  int B;
  const int* missing_bin;  // [F], -1 = none
  const int* n_cats;       // [F], -1 numeric, else number of kept categories
};

struct Hist {
  std::vector<double> gh;    // interleaved (g, h) per cell
  std::vector<int64_t> cnt;
  std::vector<int64_t> qg, qh;  // integer cells (MODE_FIXED / MODE_QUANT)
  void init(int F, int B, bool integer) {
    gh.assign((size_t)2 * F * B, 0.0);
    cnt.assign((size_t)F * B, 0);
    if (integer) {
      qg.assign((size_t)F * B, 0);
      qh.assign((size_t)F * B, 0);
    }
  }
};

struct Split {
  int feature = -1;
  int bin = -1;
  double gain = 0.0;
  bool found = false;
  bool default_left = false;
  bool is_cat = false;
  uint64_t bits[4] = {0, 0, 0, 0};
};

struct Tree {
  std::vector<int> feature, thr, left, right, dleft, mbin, cat;
  std::vector<uint64_t> bits;  // 4 words per node
  std::vector<double> value, gain;
  std::vector<int64_t> count;
  int add_node(double v, int64_t c) {
    feature.push_back(-1);
    thr.push_back(-1);
    left.push_back(-1);
    right.push_back(-1);
    dleft.push_back(0);
    mbin.push_back(-1);
    cat.push_back(0);
    for (int w = 0; w < 4; ++w) bits.push_back(0);
    value.push_back(v);
    gain.push_back(0.0);
    count.push_back(c);
    return (int)feature.size() - 1;
  }
  bool goes_left(int node, int bin) const {
    if (cat[node]) {
      if (bin <= 0 || bin >= 256) return false;
      return (bits[(size_t)4 * node + (bin >> 6)] >> (bin & 63)) & 1;
    }
    if (bin == mbin[node]) return dleft[node] != 0;
    return bin <= thr[node];
  }
  double predict(const Data& d, int64_t r) const {
    int node = 0;
    while (feature[node] >= 0) {
      int b = d.bins[(int64_t)feature[node] * d.n + r];
      node = goes_left(node, b) ? left[node] : right[node];
    }
    return value[node];
  }
};

struct Ctx {
  const Data& d;
  const mt_oracle_params& p;
  Ctx(const Data& dd, const mt_oracle_params& pp) : d(dd), p(pp) {}
  double ex(double x) const { return p.exp_kind == 1 ? mt_exp(x) : ::exp(x); }
  double sigmoid(double x) const {
    if (x >= 0.0) {
      double e = ex(-x);
      return 1.0 / (1.0 + e);
    }
    double e = ex(x);
    return e / (1.0 + e);
  }
};

inline double narrow(double v) { return (double)(float)v; }

// ---------------------------------------------------------------------------
// Row-block plan of apple_cpu_policy.mojo:808-924 (machine-independent).
// ---------------------------------------------------------------------------
struct BlockPlan {
  int64_t blocks;
  int64_t chunk;
};

BlockPlan plan_blocks(int64_t rows, int n_bins, int n_active) {
  BlockPlan bp{1, rows};
  if (rows <= 0 || n_bins <= 0 || n_active <= 0) return bp;
  int64_t cells = (int64_t)n_active * n_bins;
  int64_t by_bytes = (16ll * 1024 * 1024) / (cells * 3 * 8);
  if (by_bytes < 1) by_bytes = 1;
  int64_t ceiling = by_bytes < 64 ? by_bytes : 64;
  int64_t min_rows = (2ll * 8 * n_bins) / 1;
  if (min_rows <= 0) min_rows = 1;
  int64_t blocks = rows / min_rows;
  if (blocks > ceiling) blocks = ceiling;
  if (blocks > rows) blocks = rows;
  if (blocks < 2) return bp;
  int64_t chunk = (rows + blocks - 1) / blocks;
  blocks = (rows + chunk - 1) / chunk;
  if (blocks <= 1) return bp;
  bp.blocks = blocks;
  bp.chunk = chunk;
  return bp;
}

// ---------------------------------------------------------------------------
// Per-round derivative state.
// ---------------------------------------------------------------------------
struct RoundState {
  std::vector<double> grad, hess;   // Float32-narrowed values held in Float64
  bool const_h = false;
  // MODE_FIXED
  float gsf = 1.0f, hsf = 1.0f;
  // MODE_QUANT
  double g_units = 1.0, h_units = 1.0;
  std::vector<int64_t> qg, qh;      // per-row integer derivatives (both integer modes)
};

// Pairwise sum over the row index: a power-of-two tree with zero padding.
// This is the GPU trainer's reduction order for the fixed-point scale totals.
double pairwise_abs_sum(const double* v, int64_t lo, int64_t hi, int64_t n) {
  if (hi - lo == 1) return lo < n ? fabs(v[lo]) : 0.0;
  if (lo >= n) return 0.0;
  int64_t mid = lo + (hi - lo) / 2;
  return pairwise_abs_sum(v, lo, mid, n) + pairwise_abs_sum(v, mid, hi, n);
}

double pow2_abs_total(const std::vector<double>& v) {
  int64_t n = (int64_t)v.size();
  int64_t span = 1;
  while (span < n) span <<= 1;
  return pairwise_abs_sum(v.data(), 0, span, n);
}

void prepare_integer_round(const Ctx& c, RoundState& st, int round_index, int class_index) {
  int64_t n = c.d.n;
  st.qg.assign((size_t)n, 0);
  st.qh.assign((size_t)n, 0);
  if (c.p.mode == MODE_FIXED52) {
    st.gsf = mt_fixed_point_scale52(pow2_abs_total(st.grad));
    st.hsf = mt_fixed_point_scale52(pow2_abs_total(st.hess));
    const int64_t hq_const = (int64_t)nearbyint(1.0 * (double)st.hsf);
    for (int64_t r = 0; r < n; ++r) {
      st.qg[r] = (int64_t)nearbyint(st.grad[r] * (double)st.gsf);
      st.qh[r] = st.const_h ? hq_const : (int64_t)nearbyint(st.hess[r] * (double)st.hsf);
    }
  } else if (c.p.mode == MODE_FIXED) {
    // histogram_gpu.mojo:1199 scale refresh; quantized_gradient.mojo:908 rule;
    // histogram.mojo:3624-3637 per-row Int32(round(x_f32 * s_f32)), ties to even.
    st.gsf = mt_fixed_point_scale(pow2_abs_total(st.grad));
    st.hsf = mt_fixed_point_scale(pow2_abs_total(st.hess));
    int32_t hq_const = (int32_t)nearbyintf(1.0f * st.hsf);
    for (int64_t r = 0; r < n; ++r) {
      float g = (float)st.grad[r];
      st.qg[r] = (int32_t)nearbyintf(g * st.gsf);
      st.qh[r] = st.const_h ? hq_const : (int32_t)nearbyintf((float)st.hess[r] * st.hsf);
    }
  } else {
    // quantized_gradient.mojo:762-815 stats, :1343-1453 max-abs scales,
    // :2487-2566 once-per-round stochastic quantization.
    double gmax = 0.0, hmax = 0.0;
    for (int64_t r = 0; r < n; ++r) {
      double g = fabs(st.grad[r]), h = fabs(st.hess[r]);
      if (g > gmax) gmax = g;
      if (h > hmax) hmax = h;
    }
    if (gmax < 1e-12) gmax = 1e-12;
    if (hmax < 1e-12) hmax = 1e-12;
    double g_lim = (double)(c.p.quant_bins / 2);
    double h_lim = st.const_h ? 1.0 : (double)c.p.quant_bins;
    st.g_units = g_lim / gmax;
    st.h_units = st.const_h ? 1.0 / hmax : h_lim / hmax;
    uint64_t gs = mt_quant_stream(c.p.quant_seed, round_index, class_index, 0);
    uint64_t hs = mt_quant_stream(c.p.quant_seed, round_index, class_index, 1);
    for (int64_t r = 0; r < n; ++r) {
      st.qg[r] = mt_quantize_stochastic(st.grad[r], st.g_units, g_lim, gs + (uint64_t)r);
      st.qh[r] = mt_quantize_stochastic(st.hess[r], st.h_units, h_lim, hs + (uint64_t)r);
    }
  }
}

// ---------------------------------------------------------------------------
// Histogram construction.
// ---------------------------------------------------------------------------
void dequantize(const Ctx& c, const RoundState& st, Hist& h, const std::vector<int>& feats) {
  int B = c.d.B;
  double g_inv, h_inv;
  if (fixed_point(c.p.mode)) {
    g_inv = 1.0 / (double)st.gsf;
    h_inv = 1.0 / (double)st.hsf;
  } else {
    for (int f : feats)
      for (int b = 0; b < B; ++b) {
        size_t i = (size_t)f * B + b;
        h.gh[2 * i] = (double)h.qg[i] / st.g_units;
        h.gh[2 * i + 1] = (double)h.qh[i] / st.h_units;
      }
    return;
  }
  for (int f : feats)
    for (int b = 0; b < B; ++b) {
      size_t i = (size_t)f * B + b;
      h.gh[2 * i] = (double)h.qg[i] * g_inv;
      h.gh[2 * i + 1] = (double)h.qh[i] * h_inv;
    }
}

void build_hist(const Ctx& c, const RoundState& st, const std::vector<int64_t>& rows,
                const std::vector<int>& feats, Hist& h) {
  const Data& d = c.d;
  int B = d.B;
  int64_t n_sub = (int64_t)rows.size();
  bool integer = c.p.mode != MODE_CPU;
  h.init(d.F, B, integer);
  int nf = (int)feats.size();
  if (integer) {
#pragma omp parallel for schedule(dynamic, 1) num_threads(c.p.n_threads > 0 ? c.p.n_threads : omp_get_max_threads())
    for (int j = 0; j < nf; ++j) {
      int f = feats[j];
      const uint8_t* col = d.bins + (int64_t)f * d.n;
      int64_t* qg = h.qg.data() + (size_t)f * B;
      int64_t* qh = h.qh.data() + (size_t)f * B;
      int64_t* cn = h.cnt.data() + (size_t)f * B;
      for (int64_t i = 0; i < n_sub; ++i) {
        int64_t r = rows[i];
        int b = col[r];
        qg[b] += st.qg[r];
        qh[b] += st.qh[r];
        cn[b] += 1;
      }
    }
    dequantize(c, st, h, feats);
    return;
  }
  BlockPlan bp = plan_blocks(n_sub, B, nf);
#pragma omp parallel for schedule(dynamic, 1) num_threads(c.p.n_threads > 0 ? c.p.n_threads : omp_get_max_threads())
  for (int j = 0; j < nf; ++j) {
    int f = feats[j];
    const uint8_t* col = d.bins + (int64_t)f * d.n;
    double* gh = h.gh.data() + (size_t)2 * f * B;
    int64_t* cn = h.cnt.data() + (size_t)f * B;
    if (bp.blocks <= 1) {
      for (int64_t i = 0; i < n_sub; ++i) {
        int64_t r = rows[i];
        int b = col[r];
        gh[2 * b] = gh[2 * b] + st.grad[r];
        if (!st.const_h) gh[2 * b + 1] = gh[2 * b + 1] + st.hess[r];
        cn[b] += 1;
      }
      if (st.const_h)
        for (int b = 0; b < B; ++b) gh[2 * b + 1] = (double)cn[b];
    } else {
      // Row-block private partials folded in ascending block order
      // (histogram.mojo:2845-3453).  Counts ride along as Float64 sums of 1.0.
      std::vector<double> acc_g(B, 0.0), acc_h(B, 0.0), acc_c(B, 0.0);
      std::vector<double> pg(B), ph(B), pc(B);
      for (int64_t blk = 0; blk < bp.blocks; ++blk) {
        int64_t r0 = blk * bp.chunk, r1 = std::min(n_sub, r0 + bp.chunk);
        std::fill(pg.begin(), pg.end(), 0.0);
        std::fill(ph.begin(), ph.end(), 0.0);
        std::fill(pc.begin(), pc.end(), 0.0);
        for (int64_t i = r0; i < r1; ++i) {
          int64_t r = rows[i];
          int b = col[r];
          pg[b] = pg[b] + st.grad[r];
          if (st.const_h) ph[b] = ph[b] + 1.0;
          else {
            ph[b] = ph[b] + st.hess[r];
            pc[b] = pc[b] + 1.0;
          }
        }
        if (blk == 0) {
          acc_g = pg;
          acc_h = ph;
          acc_c = pc;
        } else {
          for (int b = 0; b < B; ++b) {
            acc_g[b] = acc_g[b] + pg[b];
            acc_h[b] = acc_h[b] + ph[b];
            acc_c[b] = acc_c[b] + pc[b];
          }
        }
      }
      for (int b = 0; b < B; ++b) {
        gh[2 * b] = acc_g[b];
        gh[2 * b + 1] = acc_h[b];
        cn[b] = st.const_h ? (int64_t)(acc_h[b] * 1.0 + 0.5) : (int64_t)acc_c[b];
      }
    }
  }
}

void subtract_hist(const Ctx& c, const RoundState& st, const Hist& parent, const Hist& child,
                   const std::vector<int>& feats, Hist& out) {
  int B = c.d.B;
  bool integer = c.p.mode != MODE_CPU;
  out.init(c.d.F, B, integer);
  for (int f : feats)
    for (int b = 0; b < B; ++b) {
      size_t i = (size_t)f * B + b;
      out.cnt[i] = parent.cnt[i] - child.cnt[i];
      if (integer) {
        out.qg[i] = parent.qg[i] - child.qg[i];
        out.qh[i] = parent.qh[i] - child.qh[i];
      } else {
        out.gh[2 * i] = parent.gh[2 * i] - child.gh[2 * i];
        out.gh[2 * i + 1] = st.const_h ? (double)out.cnt[i] : parent.gh[2 * i + 1] - child.gh[2 * i + 1];
      }
    }
  if (integer) dequantize(c, st, out, feats);
}

// ---------------------------------------------------------------------------
// Split search (split.mojo:601-1360, categorical.mojo:478-780).
// ---------------------------------------------------------------------------
double lane_reduce(const std::vector<double>& lanes, int kind) {
  if (kind == 1) {
    double s = lanes[0];
    for (size_t i = 1; i < lanes.size(); ++i) s = s + lanes[i];
    return s;
  }
  std::vector<double> v = lanes;
  while (v.size() > 1) {
    size_t half = v.size() / 2;
    std::vector<double> nv(half);
    for (size_t i = 0; i < half; ++i) nv[i] = v[i] + v[i + half];
    v.swap(nv);
  }
  return v[0];
}

struct Totals {
  double g, h;
  int64_t c;
};

Totals feature_totals(const Ctx& c, const Hist& h, int f) {
  int B = c.d.B, W = c.p.simd_lanes;
  const double* gh = h.gh.data() + (size_t)2 * f * B;
  const int64_t* cn = h.cnt.data() + (size_t)f * B;
  std::vector<double> lg(W, 0.0), lh(W, 0.0);
  int64_t tc = 0;
  int b = 0;
  while (b + W <= B) {
    for (int k = 0; k < W; ++k) {
      lg[k] = lg[k] + gh[2 * (b + k)];
      lh[k] = lh[k] + gh[2 * (b + k) + 1];
      tc += cn[b + k];
    }
    b += W;
  }
  double tg = lane_reduce(lg, c.p.lane_reduce);
  double th = lane_reduce(lh, c.p.lane_reduce);
  while (b < B) {
    tg = tg + gh[2 * b];
    th = th + gh[2 * b + 1];
    tc += cn[b];
    ++b;
  }
  return {tg, th, tc};
}

inline double soft_l1(double s, double l1) {
  if (l1 <= 0.0) return s;
  double mag = fabs(s) - l1;
  if (mag <= 0.0) return 0.0;
  return s > 0.0 ? mag : -mag;
}

inline double leaf_score(double g, double h, double l1, double l2) {
  double t = soft_l1(g, l1);
  return t * t / (h + l2);
}

struct CatResult {
  double gain = 0.0;
  uint64_t bits[4] = {0, 0, 0, 0};
  bool found = false;
};

inline void cat_add(uint64_t* bits, int bin) { bits[bin >> 6] |= 1ull << (bin & 63); }

CatResult categorical_split(const Ctx& c, const Hist& h, int f, int n_cat, Totals t) {
  CatResult best;
  if (n_cat < 2) return best;
  const mt_oracle_params& p = c.p;
  int B = c.d.B;
  const double* gh = h.gh.data() + (size_t)2 * f * B;
  const int64_t* cn = h.cnt.data() + (size_t)f * B;
  double parent = leaf_score(t.g, t.h, p.lambda_l1, p.lambda_l2);
  if (n_cat + 1 <= p.max_cat_to_onehot) {
    for (int tt = 1; tt <= n_cat; ++tt) {
      double lg = gh[2 * tt], lh = gh[2 * tt + 1];
      int64_t lc = cn[tt];
      if (lc < p.min_data_in_leaf || lh < p.min_child_hess) continue;
      int64_t rc = t.c - lc;
      if (rc < p.min_data_in_leaf) continue;
      double rh = t.h - lh;
      if (rh < p.min_child_hess) continue;
      double rg = t.g - lg;
      double l2 = p.lambda_l2;
      double gain = leaf_score(lg, lh, p.lambda_l1, l2) + leaf_score(rg, rh, p.lambda_l1, l2) - parent;
      if (gain > best.gain) {
        best = CatResult();
        best.gain = gain;
        cat_add(best.bits, tt);
        best.found = true;
      }
    }
    return best;
  }
  std::vector<int> cand;
  std::vector<double> keys;
  for (int tt = 1; tt <= n_cat; ++tt) {
    if (!((double)cn[tt] >= p.cat_smooth)) continue;
    cand.push_back(tt);
    keys.push_back(gh[2 * tt] / (gh[2 * tt + 1] + p.cat_smooth));
  }
  int used = (int)cand.size();
  if (used < 2) return best;
  std::vector<int> order(used);
  for (int i = 0; i < used; ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return keys[a] < keys[b]; });
  std::vector<int> sorted_bins(used);
  for (int i = 0; i < used; ++i) sorted_bins[i] = cand[order[i]];
  int max_num_cat = std::min(p.max_cat_threshold, (used + 1) / 2);
  if (max_num_cat < 0) max_num_cat = 0;
  double l2 = p.lambda_l2 + p.cat_l2;
  for (int dd = 0; dd < 2; ++dd) {
    int dir = dd == 0 ? 1 : -1;
    int start = dd == 0 ? 0 : used - 1;
    int pos = start;
    int64_t cnt_group = 0;
    double lg = 0.0, lh = 0.0;
    int64_t lc = 0;
    int steps = used < max_num_cat ? used : max_num_cat;
    for (int i = 0; i < steps; ++i) {
      int tt = sorted_bins[pos];
      pos += dir;
      lg = lg + gh[2 * tt];
      lh = lh + gh[2 * tt + 1];
      lc += cn[tt];
      cnt_group += cn[tt];
      if (lc < p.min_data_in_leaf || lh < p.min_child_hess) continue;
      int64_t rc = t.c - lc;
      if (rc < p.min_data_in_leaf || rc < p.min_data_per_group) break;
      double rh = t.h - lh;
      if (rh < p.min_child_hess) break;
      if (cnt_group < p.min_data_per_group) continue;
      cnt_group = 0;
      double rg = t.g - lg;
      double gain = leaf_score(lg, lh, p.lambda_l1, l2) + leaf_score(rg, rh, p.lambda_l1, l2) - parent;
      if (gain > best.gain) {
        best = CatResult();
        best.gain = gain;
        int q = start;
        for (int k = 0; k <= i; ++k) {
          cat_add(best.bits, sorted_bins[q]);
          q += dir;
        }
        best.found = true;
      }
    }
  }
  return best;
}

// MODE_QUANT split scan: the reference's quantized gain
// (quantized_gradient.mojo:3252-3309, dequant f64(q) / units at :1324-1328)
// evaluated on exact integer prefix sums; the threshold loop, guards, missing
// handling and tie rules are find_best_split's.
inline double dq(int64_t q, double units) { return (double)q / units; }

Split find_best_split_quant(const Ctx& c, const RoundState& st, const Hist& h, const std::vector<int>& feats) {
  const mt_oracle_params& p = c.p;
  int B = c.d.B;
  int nf = (int)feats.size();
  const double gu = st.g_units, hu = st.h_units, l1 = p.lambda_l1, l2 = p.lambda_l2, mch = p.min_child_hess;
  std::vector<Split> res(nf);
  for (int j = 0; j < nf; ++j) {
    int f = feats[j];
    const int64_t* qg = h.qg.data() + (size_t)f * B;
    const int64_t* qh = h.qh.data() + (size_t)f * B;
    const int64_t* cn = h.cnt.data() + (size_t)f * B;
    int64_t Tg = 0, Th = 0, Tc = 0;
    for (int b = 0; b < B; ++b) {
      Tg += qg[b];
      Th += qh[b];
      Tc += cn[b];
    }
    double tg = dq(Tg, gu), th = dq(Th, hu);
    Split s;
    if (c.d.n_cats[f] >= 0) {
      int n_cat = c.d.n_cats[f];
      double parent = leaf_score(tg, th, l1, l2);
      CatResult best;
      if (n_cat >= 2 && n_cat + 1 <= p.max_cat_to_onehot) {
        for (int t = 1; t <= n_cat && t < B; ++t) {
          double lgv = dq(qg[t], gu), lhv = dq(qh[t], hu);
          if (cn[t] < p.min_data_in_leaf || lhv < mch) continue;
          if (Tc - cn[t] < p.min_data_in_leaf) continue;
          double rh = dq(Th - qh[t], hu);
          if (rh < mch) continue;
          double rg = dq(Tg - qg[t], gu);
          double gain = leaf_score(lgv, lhv, l1, l2) + leaf_score(rg, rh, l1, l2) - parent;
          if (gain > best.gain) {
            best = CatResult();
            best.gain = gain;
            cat_add(best.bits, t);
            best.found = true;
          }
        }
      } else if (n_cat >= 2) {
        std::vector<int> cand;
        std::vector<double> keys;
        for (int t = 1; t <= n_cat && t < B; ++t) {
          if (!((double)cn[t] >= p.cat_smooth)) continue;
          cand.push_back(t);
          keys.push_back(dq(qg[t], gu) / (dq(qh[t], hu) + p.cat_smooth));
        }
        int used = (int)cand.size();
        if (used >= 2) {
          std::vector<int> order(used);
          for (int i = 0; i < used; ++i) order[i] = i;
          std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return keys[a] < keys[b]; });
          std::vector<int> sb(used);
          for (int i = 0; i < used; ++i) sb[i] = cand[order[i]];
          int max_num_cat = std::min(p.max_cat_threshold, (used + 1) / 2);
          if (max_num_cat < 0) max_num_cat = 0;
          double cl2 = l2 + p.cat_l2;
          for (int dd = 0; dd < 2; ++dd) {
            int dir = dd == 0 ? 1 : -1, start = dd == 0 ? 0 : used - 1, pos = start;
            int64_t cnt_group = 0, lq = 0, lh = 0, lc = 0;
            int steps = used < max_num_cat ? used : max_num_cat;
            for (int i = 0; i < steps; ++i) {
              int t = sb[pos];
              pos += dir;
              lq += qg[t];
              lh += qh[t];
              lc += cn[t];
              cnt_group += cn[t];
              double lgv = dq(lq, gu), lhv = dq(lh, hu);
              if (lc < p.min_data_in_leaf || lhv < mch) continue;
              int64_t rc = Tc - lc;
              if (rc < p.min_data_in_leaf || rc < p.min_data_per_group) break;
              double rh = dq(Th - lh, hu);
              if (rh < mch) break;
              if (cnt_group < p.min_data_per_group) continue;
              cnt_group = 0;
              double rg = dq(Tg - lq, gu);
              double gain = leaf_score(lgv, lhv, l1, cl2) + leaf_score(rg, rh, l1, cl2) - parent;
              if (gain > best.gain) {
                best = CatResult();
                best.gain = gain;
                int q = start;
                for (int k = 0; k <= i; ++k) {
                  cat_add(best.bits, sb[q]);
                  q += dir;
                }
                best.found = true;
              }
            }
          }
        }
      }
      if (best.found) {
        s.feature = f;
        s.gain = best.gain;
        s.found = true;
        s.is_cat = true;
        memcpy(s.bits, best.bits, sizeof s.bits);
      }
      res[j] = s;
      continue;
    }
    int mb = c.d.missing_bin[f];
    int n_scan = mb >= 0 ? mb : B;
    int64_t mg = 0, mh = 0, mc = 0;
    if (mb >= 0) {
      mg = qg[mb];
      mh = qh[mb];
      mc = cn[mb];
    }
    int64_t Lg = 0, Lh = 0, Lc = 0;
    double f_gain = 0.0;
    for (int b = 0; b < n_scan; ++b) {
      if (b == n_scan - 1 && mc == 0) break;
      Lg += qg[b];
      Lh += qh[b];
      Lc += cn[b];
      if (mb >= 0) {
        int64_t Dg = Lg + mg, Dh = Lh + mh, Dc = Lc + mc;
        double dlg = dq(Dg, gu), dlh = dq(Dh, hu), drg = dq(Tg - Dg, gu), drh = dq(Th - Dh, hu);
        if (!(dlh < mch || drh < mch || Dc < p.min_data_in_leaf || Tc - Dc < p.min_data_in_leaf)) {
          double gain = leaf_score(dlg, dlh, l1, l2) + leaf_score(drg, drh, l1, l2) - leaf_score(tg, th, l1, l2);
          if (gain > f_gain) {
            f_gain = gain;
            s.bin = b;
            s.default_left = true;
            s.found = true;
          }
        }
      }
      if (mb < 0 || mc > 0) {
        double lgv = dq(Lg, gu), lhv = dq(Lh, hu), rg = dq(Tg - Lg, gu), rh = dq(Th - Lh, hu);
        if (!(lhv < mch || rh < mch || Lc < p.min_data_in_leaf || Tc - Lc < p.min_data_in_leaf)) {
          double gain = leaf_score(lgv, lhv, l1, l2) + leaf_score(rg, rh, l1, l2) - leaf_score(tg, th, l1, l2);
          if (gain > f_gain) {
            f_gain = gain;
            s.bin = b;
            s.default_left = false;
            s.found = true;
          }
        }
      }
    }
    if (s.found) {
      s.feature = f;
      s.gain = f_gain;
    }
    res[j] = s;
  }
  Split best;
  for (int j = 0; j < nf; ++j)
    if (res[j].found && res[j].gain > best.gain) best = res[j];
  return best;
}

Split find_best_split(const Ctx& c, const Hist& h, const std::vector<int>& feats) {
  const mt_oracle_params& p = c.p;
  int B = c.d.B;
  int nf = (int)feats.size();
  std::vector<Split> res(nf);
#pragma omp parallel for schedule(dynamic, 4) num_threads(c.p.n_threads > 0 ? c.p.n_threads : omp_get_max_threads())
  for (int j = 0; j < nf; ++j) {
    int f = feats[j];
    Totals t = feature_totals(c, h, f);
    Split s;
    if (c.d.n_cats[f] >= 0) {
      CatResult cr = categorical_split(c, h, f, c.d.n_cats[f], t);
      if (cr.found) {
        s.feature = f;
        s.gain = cr.gain;
        s.found = true;
        s.is_cat = true;
        memcpy(s.bits, cr.bits, sizeof s.bits);
      }
      res[j] = s;
      continue;
    }
    const double* gh = h.gh.data() + (size_t)2 * f * B;
    const int64_t* cn = h.cnt.data() + (size_t)f * B;
    int missing_bin = c.d.missing_bin[f];
    double pg = soft_l1(t.g, p.lambda_l1);
    double parent = pg * pg / (t.h + p.lambda_l2);
    int n_scan = missing_bin >= 0 ? missing_bin : B;
    double mg = 0.0, mh = 0.0;
    int64_t mc = 0;
    if (missing_bin >= 0) {
      mg = gh[2 * missing_bin];
      mh = gh[2 * missing_bin + 1];
      mc = cn[missing_bin];
    }
    double lg = 0.0, lh = 0.0;
    int64_t lc = 0;
    double f_gain = 0.0;
    int f_bin = -1;
    bool f_dl = false, f_found = false;
    for (int b = 0; b < n_scan; ++b) {
      if (b == n_scan - 1 && mc == 0) break;
      lg = lg + gh[2 * b];
      lh = lh + gh[2 * b + 1];
      lc += cn[b];
      if (missing_bin >= 0) {
        double dlg = lg + mg, dlh = lh + mh;
        int64_t dlc = lc + mc;
        double drg = t.g - dlg, drh = t.h - dlh;
        if (!(dlh < p.min_child_hess || drh < p.min_child_hess || dlc < p.min_data_in_leaf ||
              t.c - dlc < p.min_data_in_leaf)) {
          double tl = soft_l1(dlg, p.lambda_l1), tr = soft_l1(drg, p.lambda_l1);
          double gain = tl * tl / (dlh + p.lambda_l2) + tr * tr / (drh + p.lambda_l2) - parent;
          if (gain > f_gain) {
            f_gain = gain;
            f_bin = b;
            f_dl = true;
            f_found = true;
          }
        }
      }
      if (missing_bin < 0 || mc > 0) {
        double rg = t.g - lg, rh = t.h - lh;
        if (!(lh < p.min_child_hess || rh < p.min_child_hess || lc < p.min_data_in_leaf ||
              t.c - lc < p.min_data_in_leaf)) {
          double tl = soft_l1(lg, p.lambda_l1), tr = soft_l1(rg, p.lambda_l1);
          double gain = tl * tl / (lh + p.lambda_l2) + tr * tr / (rh + p.lambda_l2) - parent;
          if (gain > f_gain) {
            f_gain = gain;
            f_bin = b;
            f_dl = false;
            f_found = true;
          }
        }
      }
    }
    if (f_found) {
      s.feature = f;
      s.bin = f_bin;
      s.gain = f_gain;
      s.found = true;
      s.default_left = f_dl;
    }
    res[j] = s;
  }
  Split best;
  for (int j = 0; j < nf; ++j)
    if (res[j].found && res[j].gain > best.gain) best = res[j];
  return best;
}

double leaf_value(const Ctx& c, const RoundState& st, const Hist& h, int value_feature) {
  int B = c.d.B;
  if (c.p.mode == MODE_QUANT) {
    // quantized_leaf_output (quantized_gradient.mojo:3312-3333) on the node totals
    int64_t G = 0, H = 0;
    for (int b = 0; b < B; ++b) {
      G += h.qg[(size_t)value_feature * B + b];
      H += h.qh[(size_t)value_feature * B + b];
    }
    return -soft_l1(dq(G, st.g_units), c.p.lambda_l1) / (dq(H, st.h_units) + c.p.lambda_l2);
  }
  const double* gh = h.gh.data() + (size_t)2 * value_feature * B;
  double g = 0.0, hh = 0.0;
  for (int b = 0; b < B; ++b) {
    g = g + gh[2 * b];
    hh = hh + gh[2 * b + 1];
  }
  return -soft_l1(g, c.p.lambda_l1) / (hh + c.p.lambda_l2);
}

bool goes_left(const Split& s, int missing_bin, int bin) {
  if (s.is_cat) {
    if (bin <= 0 || bin >= 256) return false;
    return (s.bits[bin >> 6] >> (bin & 63)) & 1;
  }
  if (bin == missing_bin) return s.default_left;
  return bin <= s.bin;
}

// ---------------------------------------------------------------------------
// Leaf-wise grower.
// ---------------------------------------------------------------------------
struct Leaf {
  int node;
  std::vector<int64_t> rows;
  Hist hist;
  Split split;
};

Split search(const Ctx& c, const RoundState& st, const Hist& h, int64_t n_rows, const std::vector<int>& feats) {
  if (n_rows < 2 * (int64_t)c.p.min_data_in_leaf || n_rows < 2) return Split();
  if (c.p.mode == MODE_QUANT) return find_best_split_quant(c, st, h, feats);
  return find_best_split(c, h, feats);
}

Tree grow_tree(const Ctx& c, const RoundState& st, const std::vector<int64_t>& bag,
               const std::vector<int>& feats, std::vector<std::vector<int64_t>>& leaf_rows,
               std::vector<int>& leaf_nodes) {
  const mt_oracle_params& p = c.p;
  Tree tree;
  std::vector<Leaf> frontier;
  frontier.emplace_back();
  Leaf& root = frontier.back();
  if (bag.empty()) {
    root.rows.resize((size_t)c.d.n);
    for (int64_t r = 0; r < c.d.n; ++r) root.rows[r] = r;
  } else {
    root.rows = bag;
  }
  build_hist(c, st, root.rows, feats, root.hist);
  int value_feature = feats[0];
  root.node = tree.add_node(leaf_value(c, st, root.hist, value_feature), (int64_t)root.rows.size());
  root.split = search(c, st, root.hist, (int64_t)root.rows.size(), feats);
  int n_leaves = 1;
  while (n_leaves < p.num_leaves) {
    int best_i = -1;
    double best_gain = 0.0;
    for (size_t i = 0; i < frontier.size(); ++i) {
      const Split& s = frontier[i].split;
      if (s.found && s.gain > 0.0 && s.gain > best_gain) {
        best_gain = s.gain;
        best_i = (int)i;
      }
    }
    if (best_i < 0) break;
    Leaf parent = std::move(frontier[best_i]);
    const Split& split = parent.split;
    int mbin = split.is_cat ? -1 : c.d.missing_bin[split.feature];
    Leaf L, R;
    const uint8_t* col = c.d.bins + (int64_t)split.feature * c.d.n;
    for (int64_t r : parent.rows) {
      if (goes_left(split, mbin, col[r])) L.rows.push_back(r);
      else R.rows.push_back(r);
    }
    bool builds_left = L.rows.size() <= R.rows.size();
    if (builds_left) {
      build_hist(c, st, L.rows, feats, L.hist);
      subtract_hist(c, st, parent.hist, L.hist, feats, R.hist);
    } else {
      build_hist(c, st, R.rows, feats, R.hist);
      subtract_hist(c, st, parent.hist, R.hist, feats, L.hist);
    }
    double lv = leaf_value(c, st, L.hist, value_feature);
    double rv = leaf_value(c, st, R.hist, value_feature);
    L.node = tree.add_node(lv, (int64_t)L.rows.size());
    R.node = tree.add_node(rv, (int64_t)R.rows.size());
    int pn = parent.node;
    tree.left[pn] = L.node;
    tree.right[pn] = R.node;
    tree.feature[pn] = split.feature;
    tree.gain[pn] = split.gain;
    if (split.is_cat) {
      tree.thr[pn] = -1;
      tree.dleft[pn] = 0;
      tree.mbin[pn] = -1;
      tree.cat[pn] = 1;
      for (int w = 0; w < 4; ++w) tree.bits[(size_t)4 * pn + w] = split.bits[w];
    } else {
      tree.thr[pn] = split.bin;
      tree.dleft[pn] = split.default_left;
      tree.mbin[pn] = mbin;
    }
    L.split = search(c, st, L.hist, (int64_t)L.rows.size(), feats);
    R.split = search(c, st, R.hist, (int64_t)R.rows.size(), feats);
    frontier[best_i] = std::move(L);
    frontier.push_back(std::move(R));
    ++n_leaves;
  }
  leaf_rows.clear();
  leaf_nodes.clear();
  for (auto& lf : frontier) {
    leaf_nodes.push_back(lf.node);
    leaf_rows.push_back(std::move(lf.rows));
  }
  return tree;
}

// sampling.mojo:319-463
std::vector<int> select_tree_features(int F, double fraction, int seed, int tree_index) {
  std::vector<int> pool(F);
  for (int f = 0; f < F; ++f) pool[f] = f;
  if (fraction >= 1.0) return pool;
  const uint64_t mask = 0x7FFFFFFFFFFFFFFFull;
  uint64_t h = mt_splitmix64((uint64_t)(int64_t)seed & mask);
  h = mt_splitmix64(h ^ ((uint64_t)(int64_t)tree_index & mask));
  uint64_t stream = mt_splitmix64(h ^ 0ull);
  int count = (int)((double)F * fraction + 0.5);
  int floor_count = F >= 2 ? 2 : F;
  if (count < floor_count) count = floor_count;
  if (count > F) count = F;
  if (count >= F) return pool;
  std::vector<int> out;
  int chosen = 0;
  for (int i = 0; i < F && chosen < count; ++i) {
    double prob = (double)(count - chosen) / (double)(F - i);
    if (mt_uniform(stream + (uint64_t)i) < prob) {
      out.push_back(pool[i]);
      ++chosen;
    }
  }
  return out;
}

// bagging.mojo:81-150
bool refresh_bag(const mt_oracle_params& p, int64_t n, int iteration, std::vector<int64_t>& bag) {
  if (!(p.bagging_freq > 0 && p.bagging_fraction < 1.0)) return false;
  if (iteration % p.bagging_freq != 0) return true;
  int64_t bag_index = iteration / p.bagging_freq;
  uint64_t stream = mt_splitmix64(((uint64_t)(int64_t)p.bagging_seed & 0x7FFFFFFFFFFFFFFFull) ^
                                  ((uint64_t)bag_index * MT_GOLDEN));
  bag.clear();
  double min_draw = 2.0;
  int64_t min_row = 0;
  for (int64_t r = 0; r < n; ++r) {
    double u = mt_uniform(stream + (uint64_t)r);
    if (u < p.bagging_fraction) bag.push_back(r);
    if (u < min_draw) {
      min_draw = u;
      min_row = r;
    }
  }
  if (bag.empty()) bag.push_back(min_row);
  return true;
}

void fill_grad(const Ctx& c, const std::vector<double>& raw, const double* y, RoundState& st) {
  int64_t n = c.d.n;
  st.grad.resize((size_t)n);
  st.hess.resize((size_t)n);
  if (c.p.objective == OBJ_LOGISTIC) {
    for (int64_t r = 0; r < n; ++r) {
      double pr = c.sigmoid(raw[r]);
      st.grad[r] = narrow(1.0 * (pr - y[r]));
      double h = pr * (1.0 - pr);
      if (h < 1e-16) h = 1e-16;
      st.hess[r] = narrow(1.0 * h);
    }
  } else {
    for (int64_t r = 0; r < n; ++r) {
      st.grad[r] = narrow(1.0 * (raw[r] - y[r]));
      st.hess[r] = narrow(1.0);
    }
  }
}

void store_tree(const Tree& t, int ti, mt_oracle_out* out) {
  int nn = (int)t.feature.size();
  if (nn > out->max_nodes) throw std::runtime_error("tree node capacity exceeded");
  out->n_nodes[ti] = nn;
  size_t base = (size_t)ti * out->max_nodes;
  for (int i = 0; i < nn; ++i) {
    out->feature[base + i] = t.feature[i];
    out->threshold_bin[base + i] = t.thr[i];
    out->left[base + i] = t.left[i];
    out->right[base + i] = t.right[i];
    out->default_left[base + i] = t.dleft[i];
    out->missing_bin[base + i] = t.mbin[i];
    out->value[base + i] = t.value[i];
    out->gain[base + i] = t.gain[i];
    out->count[base + i] = t.count[i];
    for (int w = 0; w < 4; ++w) out->cat_bits[(base + i) * 4 + w] = t.bits[(size_t)4 * i + w];
  }
}

void train(const Data& d, const double* y, const mt_oracle_params& p, mt_oracle_out* out) {
  const double t_start = omp_get_wtime();
  auto mark_round = [&](int it) {
    if (out->round_seconds) out->round_seconds[it] = omp_get_wtime() - t_start;
  };
  Ctx c(d, p);
  int64_t n = d.n;
  int K = p.objective == OBJ_SOFTMAX ? p.n_classes : 1;
  std::vector<double> raw((size_t)n * K);
  std::vector<int> all(d.F);
  for (int f = 0; f < d.F; ++f) all[f] = f;
  int n_trees = 0;
  RoundState st;
  std::vector<std::vector<int64_t>> leaf_rows;
  std::vector<int> leaf_nodes;
  if (K == 1) {
    // boosting.mojo:521-577
    double mean = 0.0, tw = 0.0;
    for (int64_t r = 0; r < n; ++r) {
      mean += 1.0 * y[r];
      tw += 1.0;
    }
    mean /= tw;
    double base = mean;
    if (p.objective == OBJ_LOGISTIC) {
      double pr = mean < 1e-15 ? 1e-15 : (mean > 1.0 - 1e-15 ? 1.0 - 1e-15 : mean);
      base = log(pr / (1.0 - pr));
    }
    if (p.base_override) base = p.base_override[0];
    out->base_scores[0] = base;
    for (int64_t r = 0; r < n; ++r) raw[r] = base;
    st.const_h = p.objective == OBJ_L2;
    std::vector<int64_t> bag;
    for (int it = 0; it < p.num_rounds; ++it) {
      bool bagged = refresh_bag(p, n, it, bag);
      fill_grad(c, raw, y, st);
      if (p.mode != MODE_CPU) prepare_integer_round(c, st, it, 0);
      std::vector<int> feats = select_tree_features(d.F, p.feature_fraction, p.feature_fraction_seed, it);
      Tree t = grow_tree(c, st, bagged ? bag : std::vector<int64_t>(), feats, leaf_rows, leaf_nodes);
      int nl = (int)leaf_nodes.size();
      if (nl == 1 && fabs(t.value[0]) < 1e-12) {
        mark_round(it);
        if (bagged) continue;
        break;
      }
      if (!bagged) {
        for (size_t l = 0; l < leaf_nodes.size(); ++l) {
          double v = t.value[leaf_nodes[l]];
          for (int64_t r : leaf_rows[l]) raw[r] = fma(p.learning_rate, v, raw[r]);
        }
      } else {
        for (int64_t r = 0; r < n; ++r) {
          double v = t.predict(d, r);
          raw[r] = p.traversal_fma ? fma(p.learning_rate, v, raw[r]) : raw[r] + p.learning_rate * v;
        }
      }
      store_tree(t, n_trees++, out);
      mark_round(it);
    }
  } else {
    // boosting.mojo:4167-4249 and :3876-4164
    std::vector<double> cw(K, 0.0);
    double tw = 0.0;
    for (int64_t r = 0; r < n; ++r) {
      cw[(int)y[r]] += 1.0;
      tw += 1.0;
    }
    for (int k = 0; k < K; ++k) {
      double q = cw[k] / tw;
      q = q < 1e-15 ? 1e-15 : (q > 1.0 - 1e-15 ? 1.0 - 1e-15 : q);
      out->base_scores[k] = p.base_override ? p.base_override[k] : log(q);
    }
    for (int64_t r = 0; r < n; ++r)
      for (int k = 0; k < K; ++k) raw[(size_t)r * K + k] = out->base_scores[k];
    std::vector<double> prob((size_t)n * K);
    double factor = (double)K / (double)(K - 1);
    st.const_h = false;
    for (int it = 0; it < p.num_rounds; ++it) {
      for (int64_t r = 0; r < n; ++r) {
        double* pp = prob.data() + (size_t)r * K;
        const double* rp = raw.data() + (size_t)r * K;
        double m = rp[0];
        for (int k = 1; k < K; ++k)
          if (rp[k] > m) m = rp[k];
        double total = 0.0;
        for (int k = 0; k < K; ++k) {
          double e = c.ex(rp[k] - m);
          pp[k] = e;
          total += e;
        }
        for (int k = 0; k < K; ++k) pp[k] = pp[k] / total;
      }
      bool progress = false;
      int first = n_trees;
      for (int k = 0; k < K; ++k) {
        st.grad.resize((size_t)n);
        st.hess.resize((size_t)n);
        for (int64_t r = 0; r < n; ++r) {
          double pr = prob[(size_t)r * K + k];
          double yy = (int)y[r] == k ? 1.0 : 0.0;
          st.grad[r] = narrow(1.0 * (pr - yy));
          double h = factor * pr * (1.0 - pr);
          if (h < 1e-16) h = 1e-16;
          st.hess[r] = narrow(1.0 * h);
        }
        if (p.mode != MODE_CPU) prepare_integer_round(c, st, it, k);
        Tree t = grow_tree(c, st, std::vector<int64_t>(), all, leaf_rows, leaf_nodes);
        if ((int)leaf_nodes.size() > 1 || fabs(t.value[0]) >= 1e-12) progress = true;
        for (size_t l = 0; l < leaf_nodes.size(); ++l) {
          double v = t.value[leaf_nodes[l]];
          for (int64_t r : leaf_rows[l]) {
            size_t s = (size_t)r * K + k;
            raw[s] = fma(p.learning_rate, v, raw[s]);
          }
        }
        store_tree(t, n_trees++, out);
      }
      if (!progress) {
        n_trees = first;
        break;
      }
      mark_round(it);
    }
  }
  out->n_trees = n_trees;
  memcpy(out->raw, raw.data(), sizeof(double) * raw.size());
}

}  // namespace

extern "C" {

// Returns 0 on success, -1 on invalid input (message in err, if non-null).
int mt_oracle_train(const uint8_t* bins, int64_t n_rows, int n_features, int n_bins,
                    const int* missing_bin, const int* n_cats, const double* labels,
                    const mt_oracle_params* params, mt_oracle_out* out, char* err, int err_len) {
  try {
    if (!bins || !labels || !params || !out || !missing_bin || !n_cats)
      throw std::runtime_error("null pointer argument");
    Data d{bins, n_rows, n_features, n_bins, missing_bin, n_cats};
    train(d, labels, *params, out);
    return 0;
  } catch (const std::exception& e) {
    if (err && err_len > 0) {
      strncpy(err, e.what(), (size_t)err_len - 1);
      err[err_len - 1] = 0;
    }
    return -1;
  }
}

// Pairwise |x| total in the GPU trainer's order (exposed for tests).
double mt_oracle_pow2_abs_total(const double* v, int64_t n) {
  std::vector<double> x(v, v + n);
  return pow2_abs_total(x);
}

double mt_oracle_exp(double x) { return mt_exp(x); }

// The quantizer primitives the device kernels share (mt_math.h), exposed for
// the known-answer tests ported from the reference's quantized-gradient tests.
uint64_t mt_oracle_splitmix64(uint64_t state) { return mt_splitmix64(state); }
double mt_oracle_uniform(uint64_t counter) { return mt_uniform(counter); }
uint64_t mt_oracle_quant_stream(long long seed, long long round_index, long long class_index, int plane) {
  return mt_quant_stream(seed, round_index, class_index, plane);
}
long long mt_oracle_quantize_stochastic(double value, double units, double lim, uint64_t counter) {
  return mt_quantize_stochastic(value, units, lim, counter);
}
double mt_oracle_fixed_point_scale(double total) { return (double)mt_fixed_point_scale(total); }

}  // extern "C"
