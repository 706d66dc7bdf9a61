// Host-side feature binning: float64 column-major matrix -> uint8 bins.
//
// Binning runs once per fit on the host in the reference too (model.mojo:518-526:
// fit_bins then BinMapper.transform) and is not on the per-round hot path.  This
// is a restatement of the reference's quantile binner for its default border
// type, written for this library:
//   * fit_bins            binning.mojo:3565-4047
//   * quantile indices    binning.mojo:558-580  (quantile_boundary_indices)
//   * edge emission       binning.mojo:583-631  (emit_quantile_edges, midpoints)
//   * distinct levels     binning.mojo:1531-1655 (collect_distinct + min_data_in_bin merge)
//   * row sample          binning.mojo:1745-1786 (bin_construct_sample_rows)
//   * transform           binning.mojo:3242-3455 (bin = #edges < v; NaN -> missing bin)
//   * categorical codes   categorical.mojo:298-462 (kept codes -> bins 1.., bin 0 unseen)
#pragma once
#include <stdint.h>
#include <string>
#include <vector>

namespace mtb {

struct BinMapper {
  int n_features = 0;
  int n_bins = 0;                   // histogram width (= max_bins)
  std::vector<double> edges;        // concatenated per-feature upper edges
  std::vector<int64_t> edge_offsets;  // n_features + 1
  std::vector<int> missing_bin;     // -1 when the feature reserves none
  std::vector<uint8_t> is_cat;      // 1 for categorical features
  std::vector<int64_t> cat_codes;   // concatenated kept codes, ascending per feature
  std::vector<int64_t> cat_offsets; // n_features + 1

  int n_categories(int f) const {
    return cat_offsets.empty() ? 0 : (int)(cat_offsets[f + 1] - cat_offsets[f]);
  }
  int bin_value(int f, double v) const;
};

struct BinningParams {
  int max_bins = 255;
  int min_data_in_bin = 3;
  int64_t bin_construct_sample_cnt = 200000;
  int data_random_seed = 1;
  bool use_missing = true;
  std::vector<int> categorical_features;
};

// Fits bin edges.  Throws std::runtime_error with a message on invalid input.
BinMapper fit_bins(const double* x, int64_t n_rows, int n_features, const BinningParams& p);

// Writes feature-major bins: out[f * n_rows + r].
void transform(const BinMapper& m, const double* x, int64_t n_rows, uint8_t* out);

// The same for a compressed-sparse-column matrix (indptr[n_features + 1],
// row indices strictly increasing within a column, values; an absent entry
// is the value 0.0, a stored NaN is missing): the bins of the densified
// matrix, without densifying it (sparse.mojo:535-570).  check_csc throws
// std::invalid_argument on a malformed matrix.
void check_csc(const int64_t* indptr, const int64_t* indices, int64_t n_rows, int n_features);
BinMapper fit_bins_csc(const int64_t* indptr, const int64_t* indices, const double* values, int64_t n_rows,
                       int n_features, const BinningParams& p);
void transform_csc(const BinMapper& m, const int64_t* indptr, const int64_t* indices, const double* values,
                   int64_t n_rows, uint8_t* out);

// Equal-width binning of the reference's test fixtures (binning.mojo:4109-4168).
void bin_equal_width(const double* x, int64_t n_rows, int n_features, int n_bins, uint8_t* out);

}  // namespace mtb
