// GPU trainer entry point (host side).
#pragma once
#include <stdexcept>
#include <string>

#include "model.h"

namespace mtb {

// A request the device path does not cover (maps to MOJOTREES_ERROR_UNSUPPORTED).
struct Unsupported : std::runtime_error {
  explicit Unsupported(const std::string& m) : std::runtime_error(m) {}
};

struct BinMapper;

struct BinnedInput {
  const uint8_t* bins_fm;   // feature-major bins[f * n_rows + r], host memory
  long long n_rows;
  int n_features;
  int n_bins;               // histogram width (<= 256)
  const int* missing_bin;   // [n_features], -1 when none
  const int* n_cats;        // [n_features], -1 numeric, else kept categories
  const double* labels;     // [n_rows]
  // Data-parallel fits (one process per GPU): this device's rows are global
  // rows [row_offset, row_offset + n_rows); every shard but the last holds a
  // multiple of 1024 rows.  coll == nullptr for a single-device fit.
  long long row_offset = 0;
  long long n_rows_global = 0;
  class Collective* coll = nullptr;
  // Dense entry point: instead of bins_fm, float64 columns dense_fm[f * n_rows
  // + r] (host memory) binned on the device with `mapper`.
  const double* dense_fm = nullptr;
  const BinMapper* mapper = nullptr;
};

// Trains on the current (or configured) CUDA device; fills model.trees,
// base_scores and stats.  Throws Unsupported or std::runtime_error.
void train_gpu(const BinnedInput& in, const TrainConfig& cfg, Model& model);

// Number of CUDA devices visible (0 when the driver or a device is absent).
int cuda_device_count();

}  // namespace mtb
