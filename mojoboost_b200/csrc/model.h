// Host-side model and training configuration shared by the trainer and the
// C ABI.  A trained model is immutable.
#pragma once
#include <stdint.h>

#include <iosfwd>
#include <memory>
#include <string>
#include <vector>

#include "binning.h"

namespace mtb {

// One node of a trained tree (layout shared with the device NodeRec).
struct HostNode {
  int feature;
  int thr;
  int left;
  int right;
  int dleft;
  int mbin;
  int is_cat;
  int pad;
  unsigned long long bits[4];
  double value;
  double gain;
  long long count;
};

enum ObjectiveKind { OBJECTIVE_L2 = 0, OBJECTIVE_BINARY = 1, OBJECTIVE_MULTICLASS = 2 };

struct TrainConfig {
  int objective = OBJECTIVE_L2;
  int num_class = 1;
  int num_iterations = 100;
  double learning_rate = 0.1;
  int num_leaves = 31;
  int min_data_in_leaf = 20;
  double lambda_l2 = 1.0;
  double lambda_l1 = 0.0;
  double min_sum_hessian_in_leaf = 1e-3;
  double feature_fraction = 1.0;
  int feature_fraction_seed = 2;
  int max_cat_to_onehot = 4;
  int max_cat_threshold = 32;
  double cat_smooth = 10.0;
  double cat_l2 = 10.0;
  int min_data_per_group = 100;
  bool use_quantized_grad = false;
  int num_grad_quant_bins = 4;
  int quant_seed = 11;
  int gpu_device_id = -1;      // -1: current device
  double dp_timeout_seconds = 300.0;
  bool hist_int64 = false;     // fixed-point histograms with the 2^52 bound and Int64 cells  // data-parallel fits: bound of every wait on the other ranks
  bool keep_training_scores = false;
  bool profile_phases = false;    // CUDA events around every kernel phase
  bool profile_histogram = false; // CUDA events around the histogram launches only
  BinningParams binning;
};

struct TrainStats {
  double fit_seconds = 0.0;         // wall time of the device loop
  double upload_seconds = 0.0;      // host->device copies and layout build
  double hist_ms = 0.0;             // summed histogram-kernel time (profile_phases)
  double partition_ms = 0.0;
  double scan_ms = 0.0;
  double grad_ms = 0.0;
  double commit_ms = 0.0;
  double binning_seconds = 0.0;     // host bin fitting + transform (dense entry point)
  double hist_rows = 0.0;           // rows read by histogram builds (built children + roots)
  double hist_bytes = 0.0;          // algorithmic bytes: hist_rows * (F + pair bytes)
  int hist_launches = 0;            // histogram launches (one per batch iteration)
  int iterations = 0;               // batch iterations that did work, summed over trees
  int expansions = 0;               // leaves whose children were computed, summed over trees
  long long pick_steps = 0;         // commit-kernel pick-loop steps, summed over trees
  double hist_sparse_entries = 0.0; // entries of the sparse histogram's row lists (0: dense histograms)
  int kernel_launches = 0;          // kernels this library launched
  int rounds = 0;
  std::vector<double> round_ms;     // device time of each round (CUDA events on the trainer's stream)
  // per round: histogram-kernel time (profile_phases), histogram launches,
  // rows read by histogram builds, kernels launched
  std::vector<double> round_hist_ms, round_hist_launches, round_hist_rows, round_launches;
};

struct Model {
  int objective = OBJECTIVE_L2;
  int num_class = 1;        // values per row (1 for single-output objectives)
  int n_features = 0;
  double learning_rate = 0.1;
  std::vector<double> base_scores;
  std::vector<std::vector<HostNode>> trees;  // multiclass: tree i*K + k is class k
  bool has_mapper = false;
  BinMapper mapper;
  std::vector<double> train_scores;  // when keep_training_scores
  TrainStats stats;
};

// Model files in the reference's token format (model_io.cpp): v4 written,
// v1-v4 read.  A model trained on pre-binned columns carries an edge-free
// mapper (its bin width, missing bins and categorical counts) and
// has_mapper = false.
void save_model_v4(const Model& m, std::ostream& os);
Model load_model_text(const std::string& content);
// The reference's inspection dump of a model, as JSON (model_io.cpp).
std::string dump_model_json(const Model& m);

}  // namespace mtb
