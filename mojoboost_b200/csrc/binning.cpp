// Host binning; see binning.h for the reference line map.
#include "binning.h"

#include <algorithm>
#include <cstring>
#include <exception>
#include <cmath>
#include <stdexcept>

#include "mt_math.h"

namespace mtb {

static const double kMaxEdge = 1e300;

static double avoid_inf(double x) {
  if (std::isnan(x)) return 0.0;
  if (x >= kMaxEdge) return kMaxEdge;
  if (x <= -kMaxEdge) return -kMaxEdge;
  return x;
}

// binning.mojo:1745-1786: sequential selection sampling with splitmix64 draws.
// The draw of row r depends only on r, so the draws of a block of rows are
// computed in parallel; the accept decisions then run in row order.
static std::vector<int64_t> sample_rows(int64_t n_rows, int64_t cnt, int seed) {
  std::vector<int64_t> out;
  if (n_rows < 1 || cnt <= 0 || cnt >= n_rows) return out;
  out.reserve((size_t)cnt);
  const uint64_t base = (uint64_t)(int64_t)seed * MT_GOLDEN;
  constexpr int64_t kBlock = 1 << 20;
  std::vector<double> u((size_t)std::min<int64_t>(kBlock, n_rows));
  int64_t need = cnt;
  for (int64_t b0 = 0; b0 < n_rows && need > 0; b0 += kBlock) {
    const int64_t nb = std::min<int64_t>(kBlock, n_rows - b0);
#pragma omp parallel for schedule(static) if (nb >= 65536)
    for (int64_t i = 0; i < nb; ++i) u[(size_t)i] = mt_uniform(base + (uint64_t)(b0 + i));
    for (int64_t i = 0; i < nb && need > 0; ++i) {
      const int64_t r = b0 + i;
      const int64_t left = n_rows - r;
      if (need >= left || u[(size_t)i] * (double)left < (double)need) {
        out.push_back(r);
        --need;
      }
    }
  }
  return out;
}

// Ascending sort of non-NaN doubles: LSD radix sort (11-bit digits) of keys
// whose unsigned order is the numeric order (-0.0 sorts just before +0.0,
// which compare equal).  Digits that every key shares are skipped.
static void sort_doubles(std::vector<double>& v, std::vector<uint64_t>& k0, std::vector<uint64_t>& k1) {
  const size_t n = v.size();
  if (n < 512) {
    std::sort(v.begin(), v.end());
    return;
  }
  k0.resize(n);
  k1.resize(n);
  for (size_t i = 0; i < n; ++i) {
    uint64_t b;
    memcpy(&b, &v[i], 8);
    k0[i] = (b >> 63) ? ~b : (b | 0x8000000000000000ull);
  }
  constexpr int kBits = 11, kBuckets = 1 << kBits, kPasses = (64 + kBits - 1) / kBits;
  std::vector<uint32_t> cnt((size_t)kPasses * kBuckets, 0u);
  for (size_t i = 0; i < n; ++i)
    for (int p = 0; p < kPasses; ++p) ++cnt[(size_t)p * kBuckets + ((k0[i] >> (p * kBits)) & (kBuckets - 1))];
  uint64_t* src = k0.data();
  uint64_t* dst = k1.data();
  for (int p = 0; p < kPasses; ++p) {
    uint32_t* c = &cnt[(size_t)p * kBuckets];
    const int shift = p * kBits;
    if (c[(src[0] >> shift) & (kBuckets - 1)] == n) continue;  // one digit value: order unchanged
    uint32_t acc = 0;
    for (int d = 0; d < kBuckets; ++d) {
      const uint32_t t = c[d];
      c[d] = acc;
      acc += t;
    }
    for (size_t i = 0; i < n; ++i) dst[c[(src[i] >> shift) & (kBuckets - 1)]++] = src[i];
    std::swap(src, dst);
  }
  for (size_t i = 0; i < n; ++i) {
    const uint64_t key = src[i];
    const uint64_t b = (key >> 63) ? (key & 0x7fffffffffffffffull) : ~key;
    memcpy(&v[i], &b, 8);
  }
}

static void emit_edges(const std::vector<double>& below, const std::vector<double>& above,
                       std::vector<double>& out) {
  out.clear();
  size_t n = std::min(below.size(), above.size());
  for (size_t j = 0; j < n; ++j) {
    double lo = below[j], hi = above[j];
    if (hi <= lo) continue;
    double edge = avoid_inf((lo + hi) / 2.0);
    if (!out.empty() && edge <= out.back()) continue;
    out.push_back(edge);
  }
}

// Kept categorical codes: the max_bins-1 most frequent, ties by ascending code
// (a stable sort of -count over ascending codes), stored ascending.
static std::vector<int64_t> kept_codes(const double* col, int64_t n_rows, int max_bins) {
  std::vector<int64_t> present;
  present.reserve((size_t)n_rows);
  for (int64_t r = 0; r < n_rows; ++r) {
    double v = col[r];
    if (!(v >= 0.0)) continue;
    if (v >= 2147483648.0) throw std::runtime_error("categorical code out of range (>= 2^31)");
    present.push_back((int64_t)v);
  }
  std::sort(present.begin(), present.end());
  std::vector<int64_t> codes, counts;
  for (size_t i = 0; i < present.size();) {
    size_t j = i;
    while (j + 1 < present.size() && present[j + 1] == present[i]) ++j;
    codes.push_back(present[i]);
    counts.push_back((int64_t)(j - i + 1));
    i = j + 1;
  }
  size_t keep = (size_t)(max_bins - 1);
  if (codes.size() <= keep) return codes;
  std::vector<size_t> order(codes.size());
  for (size_t i = 0; i < order.size(); ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) { return counts[a] > counts[b]; });
  std::vector<int64_t> kept;
  for (size_t i = 0; i < keep; ++i) kept.push_back(codes[order[i]]);
  std::sort(kept.begin(), kept.end());
  return kept;
}

int BinMapper::bin_value(int f, double v) const {
  if (!is_cat.empty() && is_cat[f]) {
    if (!(v >= 0.0) || v >= 2147483648.0) return 0;
    int64_t code = (int64_t)v;
    auto b = cat_codes.begin() + cat_offsets[f];
    auto e = cat_codes.begin() + cat_offsets[f + 1];
    auto it = std::lower_bound(b, e, code);
    if (it != e && *it == code) return (int)(it - b) + 1;
    return 0;
  }
  double value = v;
  if (std::isnan(value)) {
    if (missing_bin[f] >= 0) return missing_bin[f];
    value = 0.0;
  }
  int64_t lo = edge_offsets[f], hi = edge_offsets[f + 1];
  int64_t left = lo, right = hi;
  while (left < right) {
    int64_t mid = (left + right) / 2;
    if (value <= edges[mid]) right = mid;
    else left = mid + 1;
  }
  return (int)(left - lo);
}

// Edges of one numeric feature from its sampled non-NaN values `col`
// (n_sample values were sampled, NaN included); sorts col.  The missing bin
// is reserved when a sampled value was NaN (binning.mojo:3565-4047).
static void numeric_edges(std::vector<double>& col, int64_t n_sample, const BinningParams& p,
                          std::vector<double>& below, std::vector<double>& above, std::vector<double>& levels,
                          std::vector<int64_t>& level_counts, std::vector<uint64_t>& key0,
                          std::vector<uint64_t>& key1, std::vector<double>& out, int* missing) {
  int64_t n_valid = (int64_t)col.size();
  bool reserve = p.use_missing && n_valid < n_sample;
  int n_ordinary = reserve ? p.max_bins - 1 : p.max_bins;
  below.clear();
  above.clear();
  // Sort once; -0.0 and 0.0 compare equal and are one level.
  sort_doubles(col, key0, key1);
  levels.clear();
  level_counts.clear();
  bool distinct_fits = n_valid >= 1;
  for (int64_t i = 0; i < n_valid && distinct_fits; ++i) {
    double v = col[i] == 0.0 ? 0.0 : col[i];
    if (!levels.empty() && levels.back() == v) {
      level_counts.back() += 1;
      continue;
    }
    if ((int)levels.size() >= n_ordinary) {
      distinct_fits = false;
      break;
    }
    levels.push_back(v);
    level_counts.push_back(1);
  }
  if (distinct_fits) {
    // binning.mojo:3850-3868
    if (p.min_data_in_bin <= 1) {
      for (size_t j = 0; j + 1 < levels.size(); ++j) {
        below.push_back(levels[j]);
        above.push_back(levels[j + 1]);
      }
    } else {
      int64_t acc = 0;
      for (size_t j = 0; j + 1 < levels.size(); ++j) {
        acc += level_counts[j];
        if (acc >= p.min_data_in_bin) {
          below.push_back(levels[j]);
          above.push_back(levels[j + 1]);
          acc = 0;
        }
      }
    }
  } else {
    // binning.mojo:3876-3957
    int64_t n_ord = n_ordinary;
    if (p.min_data_in_bin > 1) {
      int64_t cap = n_valid / p.min_data_in_bin;
      if (cap < 1) cap = 1;
      if (cap < n_ord) n_ord = cap;
    }
    for (int64_t b = 1; b < n_ord; ++b) {
      int64_t idx = b * n_valid / n_ord;
      if (idx <= 0 || idx >= n_valid) continue;
      double w = col[idx - 1];
      below.push_back(w);
      auto it = std::upper_bound(col.begin() + idx, col.end(), w);
      above.push_back(it != col.end() ? *it : w);
    }
  }
  emit_edges(below, above, out);
  *missing = reserve ? (int)out.size() + 1 : -1;
}

BinMapper fit_bins(const double* x, int64_t n_rows, int n_features, const BinningParams& p) {
  if (p.max_bins < 2 || p.max_bins > 256) throw std::runtime_error("max_bins must be in [2, 256]");
  if (n_rows < 1) throw std::runtime_error("n_rows must be positive");
  if (p.min_data_in_bin < 1) throw std::runtime_error("min_data_in_bin must be positive");
  BinMapper m;
  m.n_features = n_features;
  m.n_bins = p.max_bins;
  m.missing_bin.assign((size_t)n_features, -1);
  m.is_cat.assign((size_t)n_features, 0);
  for (int f : p.categorical_features) {
    if (f < 0 || f >= n_features) throw std::runtime_error("categorical feature index out of range");
    if (m.is_cat[f]) throw std::runtime_error("categorical feature listed twice");
    m.is_cat[f] = 1;
  }
  // Features are independent: each one's codes or edges are computed on its
  // own thread with its own scratch, then laid out in feature order (the
  // result does not depend on the thread count).
  std::vector<std::vector<int64_t>> codes_f((size_t)n_features);
  std::vector<std::vector<double>> edges_f((size_t)n_features);
  std::vector<int> missing_f((size_t)n_features, -1);
  std::vector<int64_t> sample = sample_rows(n_rows, p.bin_construct_sample_cnt, p.data_random_seed);
  const bool sampled = !sample.empty();
  const int64_t n_sample = sampled ? (int64_t)sample.size() : n_rows;
  // an exception must not leave an OpenMP region: the first one is kept and
  // rethrown after it
  std::exception_ptr failure;
#pragma omp parallel
  {
    std::vector<double> col, below, above, out, levels;
    std::vector<int64_t> level_counts;
    std::vector<uint64_t> key0, key1;
#pragma omp for schedule(dynamic, 1)
    for (int f = 0; f < n_features; ++f) {
      if (m.is_cat[f]) {
        try {
          codes_f[f] = kept_codes(x + (int64_t)f * n_rows, n_rows, p.max_bins);
        } catch (...) {
#pragma omp critical(mtb_fit_bins_failure)
          if (!failure) failure = std::current_exception();
        }
        continue;
      }
      const double* base = x + (int64_t)f * n_rows;
      col.clear();
      if (sampled) {
        for (int64_t i = 0; i < n_sample; ++i) {
          double v = base[sample[i]];
          if (!std::isnan(v)) col.push_back(v);
        }
      } else {
        for (int64_t r = 0; r < n_rows; ++r)
          if (!std::isnan(base[r])) col.push_back(base[r]);
      }
      numeric_edges(col, n_sample, p, below, above, levels, level_counts, key0, key1, out, &missing_f[f]);
      edges_f[f] = out;
    }
  }
  if (failure) std::rethrow_exception(failure);
  m.cat_offsets.push_back(0);
  m.edge_offsets.push_back(0);
  for (int f = 0; f < n_features; ++f) {
    m.cat_codes.insert(m.cat_codes.end(), codes_f[f].begin(), codes_f[f].end());
    m.cat_offsets.push_back((int64_t)m.cat_codes.size());
    m.edges.insert(m.edges.end(), edges_f[f].begin(), edges_f[f].end());
    m.edge_offsets.push_back((int64_t)m.edges.size());
    m.missing_bin[f] = missing_f[f];
  }
  return m;
}

// Kept categorical codes of a compressed column: the stored values plus
// n_zeros implicit 0.0 entries (code 0); the rule of kept_codes.
static std::vector<int64_t> kept_codes_sparse(const double* vals, int64_t nnz_f, int64_t n_zeros, int max_bins) {
  std::vector<int64_t> present;
  present.reserve((size_t)nnz_f);
  for (int64_t i = 0; i < nnz_f; ++i) {
    double v = vals[i];
    if (!(v >= 0.0)) continue;
    if (v >= 2147483648.0) throw std::runtime_error("categorical code out of range (>= 2^31)");
    present.push_back((int64_t)v);
  }
  std::sort(present.begin(), present.end());
  std::vector<int64_t> codes, counts;
  for (size_t i = 0; i < present.size();) {
    size_t j = i;
    while (j + 1 < present.size() && present[j + 1] == present[i]) ++j;
    codes.push_back(present[i]);
    counts.push_back((int64_t)(j - i + 1));
    i = j + 1;
  }
  if (n_zeros > 0) {  // the implicit entries are code 0, the smallest code
    if (!codes.empty() && codes[0] == 0) {
      counts[0] += n_zeros;
    } else {
      codes.insert(codes.begin(), 0);
      counts.insert(counts.begin(), n_zeros);
    }
  }
  size_t keep = (size_t)(max_bins - 1);
  if (codes.size() <= keep) return codes;
  std::vector<size_t> order(codes.size());
  for (size_t i = 0; i < order.size(); ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) { return counts[a] > counts[b]; });
  std::vector<int64_t> kept;
  for (size_t i = 0; i < keep; ++i) kept.push_back(codes[order[i]]);
  std::sort(kept.begin(), kept.end());
  return kept;
}

void check_csc(const int64_t* indptr, const int64_t* indices, int64_t n_rows, int n_features) {
  if (indptr[0] != 0) throw std::invalid_argument("sparse matrix: indptr[0] must be 0");
  for (int f = 0; f < n_features; ++f) {
    if (indptr[f + 1] < indptr[f]) throw std::invalid_argument("sparse matrix: indptr is not non-decreasing");
    for (int64_t i = indptr[f]; i < indptr[f + 1]; ++i) {
      if (indices[i] < 0 || indices[i] >= n_rows) throw std::invalid_argument("sparse matrix: a row index is out of range");
      if (i > indptr[f] && indices[i] <= indices[i - 1])
        throw std::invalid_argument("sparse matrix: row indices must be strictly increasing within each column");
    }
  }
}

BinMapper fit_bins_csc(const int64_t* indptr, const int64_t* indices, const double* values, int64_t n_rows,
                       int n_features, const BinningParams& p) {
  if (p.max_bins < 2 || p.max_bins > 256) throw std::runtime_error("max_bins must be in [2, 256]");
  if (n_rows < 1) throw std::runtime_error("n_rows must be positive");
  if (p.min_data_in_bin < 1) throw std::runtime_error("min_data_in_bin must be positive");
  BinMapper m;
  m.n_features = n_features;
  m.n_bins = p.max_bins;
  m.missing_bin.assign((size_t)n_features, -1);
  m.is_cat.assign((size_t)n_features, 0);
  for (int f : p.categorical_features) {
    if (f < 0 || f >= n_features) throw std::runtime_error("categorical feature index out of range");
    if (m.is_cat[f]) throw std::runtime_error("categorical feature listed twice");
    m.is_cat[f] = 1;
  }
  std::vector<std::vector<int64_t>> codes_f((size_t)n_features);
  std::vector<std::vector<double>> edges_f((size_t)n_features);
  std::vector<int> missing_f((size_t)n_features, -1);
  std::vector<int64_t> sample = sample_rows(n_rows, p.bin_construct_sample_cnt, p.data_random_seed);
  const bool sampled = !sample.empty();
  const int64_t n_sample = sampled ? (int64_t)sample.size() : n_rows;
  std::exception_ptr failure;
#pragma omp parallel
  {
    std::vector<double> col, below, above, out, levels;
    std::vector<int64_t> level_counts;
    std::vector<uint64_t> key0, key1;
#pragma omp for schedule(dynamic, 1)
    for (int f = 0; f < n_features; ++f) {
      const int64_t b = indptr[f], e = indptr[f + 1];
      if (m.is_cat[f]) {
        try {
          codes_f[f] = kept_codes_sparse(values + b, e - b, n_rows - (e - b), p.max_bins);
        } catch (...) {
#pragma omp critical(mtb_fit_bins_csc_failure)
          if (!failure) failure = std::current_exception();
        }
        continue;
      }
      // the sampled column of the densified matrix: a stored value, or 0.0
      col.clear();
      if (sampled) {
        int64_t k = b;
        for (int64_t i = 0; i < n_sample; ++i) {
          const int64_t r = sample[i];
          while (k < e && indices[k] < r) ++k;
          const double v = (k < e && indices[k] == r) ? values[k] : 0.0;
          if (!std::isnan(v)) col.push_back(v);
        }
      } else {
        for (int64_t k = b; k < e; ++k)
          if (!std::isnan(values[k])) col.push_back(values[k]);
        col.insert(col.end(), (size_t)(n_rows - (e - b)), 0.0);
      }
      numeric_edges(col, n_sample, p, below, above, levels, level_counts, key0, key1, out, &missing_f[f]);
      edges_f[f] = out;
    }
  }
  if (failure) std::rethrow_exception(failure);
  m.cat_offsets.push_back(0);
  m.edge_offsets.push_back(0);
  for (int f = 0; f < n_features; ++f) {
    m.cat_codes.insert(m.cat_codes.end(), codes_f[f].begin(), codes_f[f].end());
    m.cat_offsets.push_back((int64_t)m.cat_codes.size());
    m.edges.insert(m.edges.end(), edges_f[f].begin(), edges_f[f].end());
    m.edge_offsets.push_back((int64_t)m.edges.size());
    m.missing_bin[f] = missing_f[f];
  }
  return m;
}

void transform_csc(const BinMapper& m, const int64_t* indptr, const int64_t* indices, const double* values,
                   int64_t n_rows, uint8_t* out) {
#pragma omp parallel for schedule(dynamic, 1)
  for (int f = 0; f < m.n_features; ++f) {
    uint8_t* dst = out + (int64_t)f * n_rows;
    memset(dst, m.bin_value(f, 0.0), (size_t)n_rows);
    for (int64_t k = indptr[f]; k < indptr[f + 1]; ++k) dst[indices[k]] = (uint8_t)m.bin_value(f, values[k]);
  }
}

void transform(const BinMapper& m, const double* x, int64_t n_rows, uint8_t* out) {
#pragma omp parallel for schedule(static)
  for (int f = 0; f < m.n_features; ++f) {
    const double* col = x + (int64_t)f * n_rows;
    uint8_t* dst = out + (int64_t)f * n_rows;
    for (int64_t r = 0; r < n_rows; ++r) dst[r] = (uint8_t)m.bin_value(f, col[r]);
  }
}

void bin_equal_width(const double* x, int64_t n_rows, int n_features, int n_bins, uint8_t* out) {
  for (int f = 0; f < n_features; ++f) {
    const double* col = x + (int64_t)f * n_rows;
    double lo = col[0], hi = col[0];
    for (int64_t r = 1; r < n_rows; ++r) {
      if (col[r] < lo) lo = col[r];
      if (col[r] > hi) hi = col[r];
    }
    double width = (hi - lo) / (double)n_bins;
    for (int64_t r = 0; r < n_rows; ++r) {
      double v = col[r];
      int64_t b;
      if (width <= 0.0 || std::isnan(v)) b = 0;
      else {
        b = (int64_t)((v - lo) / width);
        if (b >= n_bins) b = n_bins - 1;
        if (b < 0) b = 0;
      }
      out[(int64_t)f * n_rows + r] = (uint8_t)b;
    }
  }
}

}  // namespace mtb
