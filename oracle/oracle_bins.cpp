// ORACLE -- test infrastructure only.  Nothing in the product links, imports
// or executes this file; only tests/ and bench.py's reference/CPU-baseline
// legs do, as the checker and the CPU baseline's binner.
//
// A plain C++ restatement of the reference's default quantile binner
// (src/mojotrees/binning.mojo), independent of the product's binner
// (mojoboost_b200/csrc/binning.cpp: block-parallel draws, radix sorts): serial
// draws, std::sort, one feature per thread.  Line map:
//   binning.mojo:1745-1786  bin_construct_sample_rows (Knuth selection sampling,
//                           uniform(seed * GOLDEN + r) per row)
//   binning.mojo:1531-1655  distinct levels, merged to min_data_in_bin
//   binning.mojo:558-580    quantile_boundary_indices (idx = b * n_valid // n_ordinary)
//   binning.mojo:583-631    emit_quantile_edges (midpoint, strictly increasing, clamped)
//   binning.mojo:3565-4047  fit_bins (missing bin reserved when a sampled value is NaN)
//   binning.mojo:3242-3455  transform (bin = number of edges below v; NaN -> missing bin,
//                           or 0.0 when none is reserved)
//   categorical.mojo:298-462 kept categorical codes (the max_bins - 1 most frequent,
//                           ties by ascending code; bins 1.. in code order, 0 unseen)
#include <math.h>
#include <stdint.h>

#include <algorithm>
#include <map>
#include <vector>

#include "../mojoboost_b200/csrc/mt_math.h"

namespace {

double clamp_edge(double x) {  // binning.mojo _avoid_inf
  if (x != x) return 0.0;
  if (x >= 1e300) return 1e300;
  if (x <= -1e300) return -1e300;
  return x;
}

std::vector<int64_t> sample_rows(int64_t n, int64_t cnt, int seed) {
  std::vector<int64_t> out;
  if (n < 1 || cnt <= 0 || cnt >= n) return out;
  uint64_t base = (uint64_t)(int64_t)seed * MT_GOLDEN;
  int64_t need = cnt;
  for (int64_t r = 0; r < n && need > 0; ++r) {
    int64_t left = n - r;
    if (need >= left || mt_uniform(base + (uint64_t)r) * (double)left < (double)need) {
      out.push_back(r);
      --need;
    }
  }
  return out;
}

std::vector<double> numeric_edges(std::vector<double> col, int64_t n_sample, int max_bins, int min_data_in_bin,
                                  bool use_missing, bool* reserve_out) {
  const int64_t n_valid = (int64_t)col.size();
  const bool reserve = use_missing && n_valid < n_sample;
  *reserve_out = reserve;
  const int n_ordinary = reserve ? max_bins - 1 : max_bins;
  std::sort(col.begin(), col.end());
  std::vector<double> below, above;
  // distinct levels (0.0 and -0.0 are one level)
  std::vector<double> lv;
  std::vector<int64_t> lc;
  bool fits = n_valid >= 1;
  for (int64_t i = 0; i < n_valid; ++i) {
    double v = col[i] == 0.0 ? 0.0 : col[i];
    if (!lv.empty() && lv.back() == v) {
      lc.back() += 1;
      continue;
    }
    if ((int)lv.size() >= n_ordinary) {
      fits = false;
      break;
    }
    lv.push_back(v);
    lc.push_back(1);
  }
  if (fits) {
    int64_t acc = 0;
    for (size_t j = 0; j + 1 < lv.size(); ++j) {
      acc += lc[j];
      if (min_data_in_bin <= 1 || acc >= min_data_in_bin) {
        below.push_back(lv[j]);
        above.push_back(lv[j + 1]);
        acc = 0;
      }
    }
  } else {
    int64_t nb = n_ordinary;
    if (min_data_in_bin > 1) nb = std::max<int64_t>(1, std::min<int64_t>(nb, n_valid / min_data_in_bin));
    for (int64_t b = 1; b < nb; ++b) {
      int64_t idx = b * n_valid / nb;
      if (idx <= 0 || idx >= n_valid) continue;
      double w = col[idx - 1];
      below.push_back(w);
      // the smallest value strictly greater than w, or w when none
      int64_t k = idx;
      while (k < n_valid && !(col[k] > w)) ++k;
      above.push_back(k < n_valid ? col[k] : w);
    }
  }
  std::vector<double> edges;
  for (size_t j = 0; j < below.size() && j < above.size(); ++j) {
    if (!(above[j] > below[j])) continue;
    double e = clamp_edge((below[j] + above[j]) / 2.0);
    if (!edges.empty() && e <= edges.back()) continue;
    edges.push_back(e);
  }
  return edges;
}

}  // namespace

extern "C" {

// x is column-major float64 [F][n]; cat_flags[f] != 0 marks a categorical
// feature (may be NULL).  Writes feature-major bins out[f * n + r], and per
// feature the missing bin (-1 when none) and the kept category count (-1 for
// numeric features).  Returns 0, or -1 on invalid arguments.
int mt_oracle_bin_dense(const double* x, int64_t n, int F, int max_bins, int min_data_in_bin, int64_t sample_cnt,
                        int seed, int use_missing, const int* cat_flags, uint8_t* out, int* missing_bin,
                        int* n_cats) {
  if (max_bins < 2 || max_bins > 256 || n < 1 || F < 1 || min_data_in_bin < 1) return -1;
  std::vector<int64_t> sample = sample_rows(n, sample_cnt, seed);
  const bool sampled = !sample.empty();
  const int64_t n_sample = sampled ? (int64_t)sample.size() : n;
  int bad = 0;
  // features are independent: one per thread (the result does not depend on
  // the thread count)
#pragma omp parallel for schedule(dynamic, 1) reduction(| : bad)
  for (int f = 0; f < F; ++f) {
    const double* c = x + (int64_t)f * n;
    uint8_t* o = out + (int64_t)f * n;
    if (cat_flags && cat_flags[f]) {
      std::map<int64_t, int64_t> count;
      for (int64_t r = 0; r < n; ++r)
        if (c[r] >= 0.0) {
          if (c[r] >= 2147483648.0) {
            bad = 1;
            break;
          }
          count[(int64_t)c[r]] += 1;
        }
      std::vector<std::pair<int64_t, int64_t>> byfreq(count.begin(), count.end());  // ascending code
      std::stable_sort(byfreq.begin(), byfreq.end(),
                       [](const std::pair<int64_t, int64_t>& a, const std::pair<int64_t, int64_t>& b) {
                         return a.second > b.second;
                       });
      if ((int)byfreq.size() > max_bins - 1) byfreq.resize((size_t)(max_bins - 1));
      std::vector<int64_t> kept;
      for (auto& p : byfreq) kept.push_back(p.first);
      std::sort(kept.begin(), kept.end());
      for (int64_t r = 0; r < n; ++r) {
        int b = 0;
        if (c[r] >= 0.0 && c[r] < 2147483648.0) {
          auto it = std::lower_bound(kept.begin(), kept.end(), (int64_t)c[r]);
          if (it != kept.end() && *it == (int64_t)c[r]) b = (int)(it - kept.begin()) + 1;
        }
        o[r] = (uint8_t)b;
      }
      missing_bin[f] = -1;
      n_cats[f] = (int)kept.size();
      continue;
    }
    std::vector<double> col;
    for (int64_t i = 0; i < n_sample; ++i) {
      double v = c[sampled ? sample[(size_t)i] : i];
      if (v == v) col.push_back(v);
    }
    bool reserve = false;
    std::vector<double> edges = numeric_edges(std::move(col), n_sample, max_bins, min_data_in_bin, use_missing != 0,
                                              &reserve);
    const int mb = reserve ? (int)edges.size() + 1 : -1;
    for (int64_t r = 0; r < n; ++r) {
      double v = c[r];
      if (v != v) {
        if (mb >= 0) {
          o[r] = (uint8_t)mb;
          continue;
        }
        v = 0.0;
      }
      o[r] = (uint8_t)(std::lower_bound(edges.begin(), edges.end(), v) - edges.begin());
    }
    missing_bin[f] = mb;
    n_cats[f] = -1;
  }
  return bad ? -1 : 0;
}

}  // extern "C"
