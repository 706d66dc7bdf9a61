// The extern "C" surface of libmojotrees_b200.so (declared in include/mojotrees.h).
//
// Mirrors the reference C ABI v3 (capi/mojotrees.h, implemented there by
// capi/mojotrees_capi.mojo:386 onward): LightGBM-style parameter strings,
// per-call error objects cleared on entry, status codes 0/-1/-2/-3/-4, no
// retained caller pointers, and no silent CPU fallback for a GPU request.
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <chrono>
#include <cctype>
#include <fstream>
#include <map>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/mojotrees.h"
#include "binning.h"
#include "capi_util.h"
#include "collective.h"
#include "model.h"
#include "predict.h"
#include "device_binning.h"
#include "trainer.h"

struct MojoTreesError {
  std::string message;
};

struct MojoTreesModel {
  mtb::Model m;
};

namespace mtb {
void capi_set_error(MojoTreesError* e, const std::string& msg) {
  if (e) e->message = msg;
}
void capi_clear_error(MojoTreesError* e) {
  if (e) e->message.clear();
}
}  // namespace mtb

namespace {

using mtb::TrainConfig;

struct InvalidArgument : std::runtime_error {
  explicit InvalidArgument(const std::string& m) : std::runtime_error(m) {}
};

void set_error(MojoTreesError* e, const std::string& msg) {
  if (e) e->message = msg;
}

void clear_error(MojoTreesError* e) {
  if (e) e->message.clear();
}

std::string lower(std::string s) {
  for (auto& c : s) c = (char)std::tolower((unsigned char)c);
  return s;
}

// primary name -> aliases (LightGBM's names)
const std::vector<std::pair<std::string, std::vector<std::string>>>& param_table() {
  static const std::vector<std::pair<std::string, std::vector<std::string>>> t = {
      {"objective", {"objective_type", "app", "application", "loss"}},
      {"num_class", {"num_classes"}},
      {"num_iterations",
       {"num_iteration", "n_iter", "num_tree", "num_trees", "num_round", "num_rounds", "nrounds", "num_boost_round",
        "n_estimators", "max_iter"}},
      {"learning_rate", {"shrinkage_rate", "eta"}},
      {"num_leaves", {"num_leaf", "max_leaves", "max_leaf", "max_leaf_nodes"}},
      {"min_data_in_leaf", {"min_data_per_leaf", "min_data", "min_child_samples", "min_samples_leaf"}},
      {"lambda_l2", {"reg_lambda", "lambda", "l2_regularization"}},
      {"lambda_l1", {"reg_alpha", "l1_regularization"}},
      {"min_sum_hessian_in_leaf", {"min_sum_hessian_per_leaf", "min_sum_hessian", "min_hessian", "min_child_weight"}},
      {"max_bin", {"max_bins"}},
      {"min_data_in_bin", {}},
      {"bin_construct_sample_cnt", {"subsample_for_bin"}},
      {"data_random_seed", {"data_seed"}},
      {"use_missing", {}},
      {"categorical_feature", {"cat_feature", "categorical_column", "cat_column", "categorical_features"}},
      {"device_type", {"device"}},
      {"gpu_device_id", {"device_id"}},
      {"gpu_histogram_precision", {}},
      {"dp_timeout_seconds", {}},
      {"use_quantized_grad", {}},
      {"num_grad_quant_bins", {}},
      {"stochastic_rounding", {}},
      {"quant_seed", {}},
      {"max_cat_to_onehot", {}},
      {"max_cat_threshold", {}},
      {"cat_smooth", {}},
      {"cat_l2", {}},
      {"min_data_per_group", {}},
      {"feature_fraction", {"sub_feature", "colsample_bytree"}},
      {"feature_fraction_seed", {}},
      {"bagging_fraction", {"sub_row", "subsample", "bagging"}},
      {"bagging_freq", {"subsample_freq"}},
      {"bagging_seed", {"bagging_fraction_seed"}},
      {"max_depth", {}},
      {"boosting", {"boosting_type", "boost"}},
      {"data_sample_strategy", {}},
      {"verbosity", {"verbose"}},
      {"seed", {"random_seed", "random_state"}},
      {"num_threads", {"num_thread", "nthread", "nthreads", "n_jobs"}},
      {"keep_training_scores", {}},
      {"profile_phases", {}},
      {"profile_histogram", {}},
  };
  return t;
}

std::map<std::string, std::string> parse_kv(const char* s) {
  std::map<std::string, std::string> out;
  if (!s) return out;
  std::istringstream is(s);
  std::string tok;
  std::map<std::string, std::string> alias;
  for (auto& e : param_table()) {
    alias[e.first] = e.first;
    for (auto& a : e.second) alias[a] = e.first;
  }
  while (is >> tok) {
    size_t eq = tok.find('=');
    if (eq == std::string::npos || eq == 0) throw InvalidArgument("malformed parameter '" + tok + "', expected key=value");
    std::string key = lower(tok.substr(0, eq)), val = tok.substr(eq + 1);
    auto it = alias.find(key);
    if (it == alias.end()) throw InvalidArgument("unknown parameter '" + key + "'");
    if (out.count(it->second)) throw InvalidArgument("parameter '" + it->second + "' given twice");
    out[it->second] = val;
  }
  return out;
}

long long to_int(const std::string& k, const std::string& v) {
  char* end = nullptr;
  long long x = strtoll(v.c_str(), &end, 10);
  if (v.empty() || *end) throw InvalidArgument("parameter '" + k + "' expects an integer, got '" + v + "'");
  return x;
}

double to_double(const std::string& k, const std::string& v) {
  char* end = nullptr;
  double x = strtod(v.c_str(), &end);
  if (v.empty() || *end) throw InvalidArgument("parameter '" + k + "' expects a number, got '" + v + "'");
  return x;
}

bool to_bool(const std::string& k, const std::string& v) {
  std::string l = lower(v);
  if (l == "true" || l == "1" || l == "yes" || l == "+") return true;
  if (l == "false" || l == "0" || l == "no" || l == "-") return false;
  throw InvalidArgument("parameter '" + k + "' expects a boolean, got '" + v + "'");
}

// Parses a parameter string into a training configuration.  Requests the
// device path does not cover throw mtb::Unsupported naming them.
TrainConfig parse_config(const char* params, bool need_training) {
  TrainConfig c;
  auto kv = parse_kv(params);
  for (auto& p : kv) {
    const std::string& k = p.first;
    const std::string& v = p.second;
    if (k == "objective") {
      std::string o = lower(v);
      if (o == "regression" || o == "regression_l2" || o == "l2" || o == "mse" || o == "mean_squared_error" ||
          o == "rmse" || o == "root_mean_squared_error" || o == "l2_root")
        c.objective = mtb::OBJECTIVE_L2;
      else if (o == "binary")
        c.objective = mtb::OBJECTIVE_BINARY;
      else if (o == "multiclass" || o == "softmax")
        c.objective = mtb::OBJECTIVE_MULTICLASS;
      else
        throw mtb::Unsupported("objective '" + v + "' is not covered by the device path (regression, binary, multiclass are)");
    } else if (k == "num_class") c.num_class = (int)to_int(k, v);
    else if (k == "num_iterations") c.num_iterations = (int)to_int(k, v);
    else if (k == "learning_rate") c.learning_rate = to_double(k, v);
    else if (k == "num_leaves") c.num_leaves = (int)to_int(k, v);
    else if (k == "min_data_in_leaf") c.min_data_in_leaf = (int)to_int(k, v);
    else if (k == "lambda_l2") c.lambda_l2 = to_double(k, v);
    else if (k == "lambda_l1") c.lambda_l1 = to_double(k, v);
    else if (k == "min_sum_hessian_in_leaf") c.min_sum_hessian_in_leaf = to_double(k, v);
    else if (k == "max_bin") c.binning.max_bins = (int)to_int(k, v);
    else if (k == "min_data_in_bin") c.binning.min_data_in_bin = (int)to_int(k, v);
    else if (k == "bin_construct_sample_cnt") c.binning.bin_construct_sample_cnt = to_int(k, v);
    else if (k == "data_random_seed") c.binning.data_random_seed = (int)to_int(k, v);
    else if (k == "use_missing") c.binning.use_missing = to_bool(k, v);
    else if (k == "categorical_feature") {
      std::string s = v;
      std::replace(s.begin(), s.end(), ',', ' ');
      std::istringstream is(s);
      std::string t;
      while (is >> t) c.binning.categorical_features.push_back((int)to_int(k, t));
    } else if (k == "device_type") {
      std::string d = lower(v);
      if (d == "cpu") throw mtb::Unsupported("device=cpu: this library implements the GPU training path only");
      if (!(d == "gpu" || d == "cuda" || d == "auto"))
        throw InvalidArgument("device must be cpu, gpu or auto, got '" + v + "'");
    } else if (k == "gpu_device_id") c.gpu_device_id = (int)to_int(k, v);
    else if (k == "gpu_histogram_precision") {
      const std::string d = lower(v);
      if (d == "int32" || d == "32") c.hist_int64 = false;
      else if (d == "int64" || d == "64") c.hist_int64 = true;
      else throw InvalidArgument("gpu_histogram_precision must be int32 or int64, got '" + v + "'");
    } else if (k == "dp_timeout_seconds") {
      c.dp_timeout_seconds = to_double(k, v);
      if (!(c.dp_timeout_seconds > 0.0)) throw InvalidArgument("dp_timeout_seconds must be positive");
    }
    else if (k == "use_quantized_grad") c.use_quantized_grad = to_bool(k, v);
    else if (k == "num_grad_quant_bins") c.num_grad_quant_bins = (int)to_int(k, v);
    else if (k == "stochastic_rounding") {
      if (!to_bool(k, v)) throw mtb::Unsupported("stochastic_rounding=false: the device quantizer rounds stochastically");
    } else if (k == "quant_seed") c.quant_seed = (int)to_int(k, v);
    else if (k == "max_cat_to_onehot") c.max_cat_to_onehot = (int)to_int(k, v);
    else if (k == "max_cat_threshold") c.max_cat_threshold = (int)to_int(k, v);
    else if (k == "cat_smooth") c.cat_smooth = to_double(k, v);
    else if (k == "cat_l2") c.cat_l2 = to_double(k, v);
    else if (k == "min_data_per_group") c.min_data_per_group = (int)to_int(k, v);
    else if (k == "feature_fraction") c.feature_fraction = to_double(k, v);
    else if (k == "feature_fraction_seed") c.feature_fraction_seed = (int)to_int(k, v);
    else if (k == "bagging_fraction") {
      if (to_double(k, v) < 1.0 && kv.count("bagging_freq") && to_int("bagging_freq", kv["bagging_freq"]) > 0)
        throw mtb::Unsupported("bagging (bagging_fraction < 1 with bagging_freq > 0) is not covered by the device path");
    } else if (k == "bagging_freq" || k == "bagging_seed") {
      to_int(k, v);
    } else if (k == "max_depth") {
      if (to_int(k, v) > 0) throw mtb::Unsupported("max_depth is not covered by the device path");
    } else if (k == "boosting") {
      std::string b = lower(v);
      if (!(b == "gbdt" || b == "gbrt")) throw mtb::Unsupported("boosting '" + v + "' is not covered by the device path");
    } else if (k == "data_sample_strategy") {
      if (lower(v) != "bagging") throw mtb::Unsupported("data_sample_strategy '" + v + "' (GOSS) is not covered by the device path");
    } else if (k == "keep_training_scores") c.keep_training_scores = to_bool(k, v);
    else if (k == "profile_phases") c.profile_phases = to_bool(k, v);
    else if (k == "profile_histogram") c.profile_histogram = to_bool(k, v);
    else if (k == "verbosity" || k == "seed" || k == "num_threads") {
      to_int(k, v);
    }
  }
  if (need_training) {
    if (c.num_iterations < 0) throw InvalidArgument("num_iterations must be non-negative");
    if (!(c.learning_rate > 0.0)) throw InvalidArgument("learning_rate must be positive");
    if (c.num_leaves < 2) throw InvalidArgument("num_leaves must be at least 2");
    if (c.min_data_in_leaf < 0) throw InvalidArgument("min_data_in_leaf must be non-negative");
    if (c.lambda_l2 < 0.0 || c.lambda_l1 < 0.0) throw InvalidArgument("lambda_l1 and lambda_l2 must be non-negative");
    if (c.objective == mtb::OBJECTIVE_MULTICLASS && c.num_class < 2)
      throw InvalidArgument("multiclass needs num_class >= 2");
    if (c.objective != mtb::OBJECTIVE_MULTICLASS) c.num_class = 1;
  }
  return c;
}

template <typename F>
int32_t guarded(MojoTreesError* err, F&& fn, int32_t fail_code = MOJOTREES_ERROR_TRAINING) {
  clear_error(err);
  try {
    return fn();
  } catch (const InvalidArgument& e) {
    set_error(err, e.what());
    return MOJOTREES_ERROR_INVALID_ARGUMENT;
  } catch (const mtb::Unsupported& e) {
    set_error(err, e.what());
    return MOJOTREES_ERROR_UNSUPPORTED;
  } catch (const std::bad_alloc&) {
    set_error(err, "out of host memory");
    return fail_code;
  } catch (const std::exception& e) {
    set_error(err, e.what());
    return fail_code;
  }
}

// Tree walk on bins (tree.mojo:483-503).
inline double tree_value(const std::vector<mtb::HostNode>& t, const uint8_t* row_bins, int64_t stride) {
  int node = 0;
  while (t[node].feature >= 0) {
    const mtb::HostNode& nd = t[node];
    int b = row_bins[(int64_t)nd.feature * stride];
    bool left;
    if (nd.is_cat) left = b > 0 && b < 256 && ((nd.bits[b >> 6] >> (b & 63)) & 1ull);
    else if (b == nd.mbin) left = nd.dleft != 0;
    else left = b <= nd.thr;
    node = left ? nd.left : nd.right;
  }
  return t[node].value;
}

// The node a row of bins reaches (the walk of tree_value).
inline int tree_leaf_node(const std::vector<mtb::HostNode>& t, const uint8_t* row_bins, int64_t stride) {
  int node = 0;
  while (t[node].feature >= 0) {
    const mtb::HostNode& nd = t[node];
    int b = row_bins[(int64_t)nd.feature * stride];
    bool left;
    if (nd.is_cat) left = b > 0 && b < 256 && ((nd.bits[b >> 6] >> (b & 63)) & 1ull);
    else if (b == nd.mbin) left = nd.dleft != 0;
    else left = b <= nd.thr;
    node = left ? nd.left : nd.right;
  }
  return node;
}

// Raw scores of feature-major bins over iterations [it0, it1)
// (boosting.mojo:1722-1727, 3747-3757; the sum is a fused multiply-add).
void raw_scores(const mtb::Model& m, const uint8_t* bins, int64_t n, int64_t it0, int64_t it1, double* out) {
  const int K = m.num_class;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < n; ++r) {
    for (int k = 0; k < K; ++k) {
      double s = it0 == 0 ? m.base_scores[k] : 0.0;
      for (int64_t i = it0; i < it1; ++i) s = fma(m.learning_rate, tree_value(m.trees[i * K + k], bins + r, n), s);
      out[r * K + k] = s;
    }
  }
}

void response(const mtb::Model& m, int64_t n, double* v) {
  if (m.objective == mtb::OBJECTIVE_BINARY) {
    for (int64_t r = 0; r < n; ++r) {
      double x = v[r];
      if (x >= 0.0) v[r] = 1.0 / (1.0 + exp(-x));
      else {
        double e = exp(x);
        v[r] = e / (1.0 + e);
      }
    }
  } else if (m.objective == mtb::OBJECTIVE_MULTICLASS) {
    const int K = m.num_class;
    for (int64_t r = 0; r < n; ++r) {
      double* p = v + r * K;
      double mx = p[0];
      for (int k = 1; k < K; ++k)
        if (p[k] > mx) mx = p[k];
      double tot = 0.0;
      for (int k = 0; k < K; ++k) {
        p[k] = exp(p[k] - mx);
        tot += p[k];
      }
      for (int k = 0; k < K; ++k) p[k] /= tot;
    }
  }
}

int32_t predict_impl(const MojoTreesModel* model, const double* data, int64_t n_rows, int64_t n_features,
                     int64_t start_iteration, int64_t num_iteration, int32_t flags, int32_t device, double* out,
                     int64_t out_len, MojoTreesError* err) {
  return guarded(
      err,
      [&]() -> int32_t {
        if (!model || !data || !out) throw InvalidArgument("null pointer argument");
        if (flags != MOJOTREES_PREDICT_RESPONSE && flags != MOJOTREES_PREDICT_RAW)
          throw InvalidArgument("unknown predict flags");
        if (device != MOJOTREES_DEVICE_CPU && device != MOJOTREES_DEVICE_GPU && device != MOJOTREES_DEVICE_AUTO) throw InvalidArgument("unknown device");
        const mtb::Model& m = model->m;
        if (n_rows < 0) throw InvalidArgument("n_rows must be non-negative");
        if (n_features != m.n_features) throw InvalidArgument("n_features does not match the model");
        if (out_len < n_rows * m.num_class) throw InvalidArgument("output buffer too small");
        if (!m.has_mapper)
          throw mtb::Unsupported("model was trained on pre-binned data; use mojotrees_b200_predict_binned_u8");
        int64_t iters = (int64_t)m.trees.size() / m.num_class;
        int64_t it0 = std::max<int64_t>(0, std::min(start_iteration, iters));
        int64_t it1 = num_iteration <= 0 ? iters : std::min(iters, it0 + num_iteration);
        std::vector<double> tmp((size_t)n_rows * m.num_class);
        if (device == MOJOTREES_DEVICE_GPU) {
          // binning and tree walks on the current CUDA device; the response
          // below stays on the host, so both devices return the same bits
          if (mtb::cuda_device_count() < 1) throw mtb::Unsupported("device=gpu prediction: no CUDA device is available");
          mtb::predict_raw_device(m, data, n_rows, it0, it1, tmp.data());
        } else {
          std::vector<uint8_t> bins((size_t)n_rows * n_features);
          mtb::transform(m.mapper, data, n_rows, bins.data());
          raw_scores(m, bins.data(), n_rows, it0, it1, tmp.data());
        }
        if (flags == MOJOTREES_PREDICT_RESPONSE) response(m, n_rows, tmp.data());
        memcpy(out, tmp.data(), sizeof(double) * tmp.size());
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

char* dup_string(const std::string& s) {
  char* p = (char*)malloc(s.size() + 1);
  if (!p) throw std::bad_alloc();
  memcpy(p, s.c_str(), s.size() + 1);
  return p;
}

int32_t train_binned(const uint8_t* bins, int64_t n_rows, int64_t n_features, int32_t n_bins,
                     const std::vector<int>& missing, const std::vector<int>& ncats, const double* labels,
                     const TrainConfig& cfg, MojoTreesModel** out_model, const mtb::BinMapper* mapper,
                     mtb::Collective* coll = nullptr, int64_t row_offset = 0, int64_t n_rows_global = 0,
                     const double* dense = nullptr) {
  for (int64_t r = 0; r < n_rows; ++r)
    if (!std::isfinite(labels[r])) throw InvalidArgument("labels must be finite");
  mtb::BinnedInput in{bins, n_rows, (int)n_features, n_bins, missing.data(), ncats.data(), labels};
  in.dense_fm = dense;
  in.mapper = dense ? mapper : nullptr;
  in.coll = coll;
  in.row_offset = row_offset;
  in.n_rows_global = coll ? n_rows_global : n_rows;
  std::unique_ptr<MojoTreesModel> h(new MojoTreesModel());
  mtb::train_gpu(in, cfg, h->m);
  if (mapper) {
    h->m.has_mapper = true;
    h->m.mapper = *mapper;
  } else {
    // pre-binned columns: an edge-free mapper records the bin width, the
    // missing bins and the categorical bins 1..n (codes 0..n-1), so the
    // model can be written to a model file; raw values cannot be binned
    mtb::BinMapper& mp = h->m.mapper;
    mp.n_features = (int)n_features;
    mp.n_bins = n_bins;
    mp.edge_offsets.assign((size_t)n_features + 1, 0);
    mp.missing_bin = missing;
    mp.is_cat.assign((size_t)n_features, 0);
    mp.cat_offsets.assign(1, 0);
    for (int64_t f = 0; f < n_features; ++f) {
      if (ncats[f] >= 0) {
        mp.is_cat[f] = 1;
        for (int c = 0; c < ncats[f]; ++c) mp.cat_codes.push_back(c);
      }
      mp.cat_offsets.push_back((int64_t)mp.cat_codes.size());
    }
  }
  *out_model = h.release();
  return MOJOTREES_OK;
}

}  // namespace

extern "C" {

int32_t mojotrees_abi_version(void) { return MOJOTREES_ABI_VERSION; }

void mojotrees_library_version(int32_t* major, int32_t* minor, int32_t* patch) {
  if (major) *major = 0;
  if (minor) *minor = 1;
  if (patch) *patch = 0;
}

int32_t mojotrees_gpu_available(void) { return mtb::cuda_device_count() > 0 ? 1 : 0; }

MojoTreesError* mojotrees_error_create(void) { return new (std::nothrow) MojoTreesError(); }

void mojotrees_error_free(MojoTreesError* error) { delete error; }

const char* mojotrees_error_message(const MojoTreesError* error) { return error ? error->message.c_str() : nullptr; }

int32_t mojotrees_train_dense(const double* data, int64_t n_rows, int64_t n_features, const double* labels,
                              const double* weights, const char* parameters, MojoTreesModel** out_model,
                              MojoTreesError* error) {
  return guarded(error, [&]() -> int32_t {
    if (!data || !labels || !out_model) throw InvalidArgument("null pointer argument");
    if (n_rows < 1 || n_features < 1) throw InvalidArgument("n_rows and n_features must be positive");
    TrainConfig cfg = parse_config(parameters, true);
    if (weights) throw mtb::Unsupported("sample weights are not covered by the device path");
    // bin edges are fitted on the host from a row sample; the columns
    // themselves are binned on the device (device_binning.cu)
    auto t0 = std::chrono::steady_clock::now();
    mtb::BinMapper mapper = mtb::fit_bins(data, n_rows, (int)n_features, cfg.binning);
    const double bin_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    std::vector<int> ncats(n_features, -1);
    for (int f = 0; f < n_features; ++f)
      if (mapper.is_cat[f]) ncats[f] = mapper.n_categories(f);
    int32_t rc = train_binned(nullptr, n_rows, n_features, mapper.n_bins, mapper.missing_bin, ncats, labels, cfg,
                              out_model, &mapper, nullptr, 0, 0, data);
    if (rc == MOJOTREES_OK && *out_model) (*out_model)->m.stats.binning_seconds = bin_s;
    return rc;
  });
}

int32_t mojotrees_b200_train_binned_u8(const uint8_t* bins, int64_t n_rows, int64_t n_features, int32_t n_bins,
                                       const int32_t* missing_bin, const int32_t* n_categories, const double* labels,
                                       const double* weights, const char* parameters, MojoTreesModel** out_model,
                                       MojoTreesError* error) {
  return guarded(error, [&]() -> int32_t {
    if (!bins || !labels || !out_model) throw InvalidArgument("null pointer argument");
    if (n_rows < 1 || n_features < 1) throw InvalidArgument("n_rows and n_features must be positive");
    if (n_bins < 2 || n_bins > 256) throw InvalidArgument("n_bins must be in [2, 256]");
    TrainConfig cfg = parse_config(parameters, true);
    if (weights) throw mtb::Unsupported("sample weights are not covered by the device path");
    std::vector<int> missing(n_features, -1), ncats(n_features, -1);
    for (int64_t f = 0; f < n_features; ++f) {
      if (missing_bin) missing[f] = missing_bin[f];
      if (n_categories) ncats[f] = n_categories[f];
      if (missing[f] >= n_bins) throw InvalidArgument("missing_bin out of range");
    }
    return train_binned(bins, n_rows, n_features, n_bins, missing, ncats, labels, cfg, out_model, nullptr);
  });
}

int32_t mojotrees_b200_nccl_unique_id(uint8_t* out_id, MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!out_id) throw InvalidArgument("null pointer argument");
        std::string why;
        if (!mtb::Collective::load(&why)) throw mtb::Unsupported(why);
        mtb::Collective::unique_id(out_id);
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_UNSUPPORTED);
}

int32_t mojotrees_b200_train_binned_u8_dp(const uint8_t* bins, int64_t n_rows, int64_t n_features, int32_t n_bins,
                                          const int32_t* missing_bin, const int32_t* n_categories,
                                          const double* labels, const double* weights, const char* parameters,
                                          const uint8_t* nccl_id, int32_t rank, int32_t world, int64_t row_offset,
                                          int64_t n_rows_global, MojoTreesModel** out_model, MojoTreesError* error) {
  return guarded(error, [&]() -> int32_t {
    if (!bins || !labels || !out_model || !nccl_id) throw InvalidArgument("null pointer argument");
    if (n_rows < 1 || n_features < 1) throw InvalidArgument("n_rows and n_features must be positive");
    if (n_bins < 2 || n_bins > 256) throw InvalidArgument("n_bins must be in [2, 256]");
    if (world < 1 || rank < 0 || rank >= world) throw InvalidArgument("invalid rank / world size");
    if (row_offset < 0 || row_offset + n_rows > n_rows_global) throw InvalidArgument("row_offset out of range");
    TrainConfig cfg = parse_config(parameters, true);
    if (weights) throw mtb::Unsupported("sample weights are not covered by the device path");
    std::vector<int> missing(n_features, -1), ncats(n_features, -1);
    for (int64_t f = 0; f < n_features; ++f) {
      if (missing_bin) missing[f] = missing_bin[f];
      if (n_categories) ncats[f] = n_categories[f];
      if (missing[f] >= n_bins) throw InvalidArgument("missing_bin out of range");
    }
    if (mtb::cuda_device_count() < 1) throw mtb::Unsupported("no CUDA device is available");
    if (cfg.gpu_device_id >= 0 && cudaSetDevice(cfg.gpu_device_id) != cudaSuccess)
      throw mtb::Unsupported("cannot select the CUDA device");
    mtb::Collective coll(nccl_id, rank, world, cfg.dp_timeout_seconds);
    try {
      return train_binned(bins, n_rows, n_features, n_bins, missing, ncats, labels, cfg, out_model, nullptr, &coll,
                          row_offset, n_rows_global);
    } catch (...) {
      // the other ranks may be gone or waiting: end this rank's share of the
      // communicator without waiting for them
      coll.abort();
      throw;
    }
  });
}

int32_t mojotrees_b200_round_times(const MojoTreesModel* model, double* out_values, int64_t out_len, int64_t* out_n,
                                   MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!model || !out_n) throw InvalidArgument("null pointer argument");
        const auto& r = model->m.stats.round_ms;
        *out_n = (int64_t)r.size();
        if (out_values) {
          int64_t n = std::min<int64_t>(out_len, (int64_t)r.size());
          for (int64_t i = 0; i < n; ++i) out_values[i] = r[i];
        }
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}


int32_t mojotrees_b200_round_stats(const MojoTreesModel* model, double* out_values, int64_t out_len, int64_t* out_n,
                                   MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!model || !out_n) throw InvalidArgument("null pointer argument");
        const mtb::TrainStats& s = model->m.stats;
        const size_t n = s.round_ms.size();
        *out_n = (int64_t)n;
        if (out_values) {
          auto at = [](const std::vector<double>& v, size_t i) { return i < v.size() ? v[i] : 0.0; };
          for (size_t i = 0; i < n && (int64_t)(5 * i + 4) < out_len; ++i) {
            out_values[5 * i + 0] = s.round_ms[i];
            out_values[5 * i + 1] = at(s.round_hist_ms, i);
            out_values[5 * i + 2] = at(s.round_hist_launches, i);
            out_values[5 * i + 3] = at(s.round_hist_rows, i);
            out_values[5 * i + 4] = at(s.round_launches, i);
          }
        }
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

int32_t mojotrees_b200_model_categorical(const MojoTreesModel* model, int32_t* out_flags, int64_t out_len,
                                         MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!model || !out_flags) throw InvalidArgument("null pointer argument");
        const mtb::Model& m = model->m;
        if (out_len < m.n_features) throw InvalidArgument("output buffer too small");
        for (int f = 0; f < m.n_features; ++f)
          out_flags[f] = (f < (int)m.mapper.is_cat.size() && m.mapper.is_cat[f]) ? 1 : 0;
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

// Host ingestion of a caller's float64 matrix (the reference's
// ingest_column_major / buffer_has_infinite, bindings/_mojotrees.mojo:682-739):
// a tiled row-major -> column-major transpose on all host threads that also
// reports whether any value is +inf or -inf (NaN marks missing values and is
// not reported).
int32_t mojotrees_b200_ingest_column_major(const double* src, double* dst, int64_t n_rows, int64_t n_features,
                                           int32_t* out_has_infinite, MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (n_rows < 0 || n_features < 0) throw InvalidArgument("n_rows and n_features must be non-negative");
        if ((!src || !dst) && n_rows > 0 && n_features > 0) throw InvalidArgument("null pointer argument");
        constexpr int64_t kTile = 64;  // 32 KB read and 32 KB written per tile
        const int64_t rt = (n_rows + kTile - 1) / kTile, ft = (n_features + kTile - 1) / kTile;
        int found = 0;
#pragma omp parallel for schedule(static) reduction(| : found)
        for (int64_t t = 0; t < rt * ft; ++t) {
          const int64_t r0 = (t / ft) * kTile, f0 = (t % ft) * kTile;
          const int64_t r1 = std::min(n_rows, r0 + kTile), f1 = std::min(n_features, f0 + kTile);
          for (int64_t f = f0; f < f1; ++f) {
            double* col = dst + f * n_rows;
            for (int64_t r = r0; r < r1; ++r) {
              const double v = src[r * n_features + f];
              found |= std::isinf(v) ? 1 : 0;
              col[r] = v;
            }
          }
        }
        if (out_has_infinite) *out_has_infinite = found;
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

int32_t mojotrees_b200_buffer_has_infinite(const double* data, int64_t n, int32_t* out_has_infinite,
                                           MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!out_has_infinite || (!data && n > 0)) throw InvalidArgument("null pointer argument");
        if (n < 0) throw InvalidArgument("n must be non-negative");
        int found = 0;
#pragma omp parallel for schedule(static) reduction(| : found)
        for (int64_t i = 0; i < n; ++i) found |= std::isinf(data[i]) ? 1 : 0;
        *out_has_infinite = found;
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

// Leaf ordinals (a leaf's rank among its tree's leaves in node order,
// tree.mojo:558-580) of column-major float64 rows over iterations
// [it0, it0 + n): out[r * (n * K) + i * K + k] is class k's tree of the
// range's iteration i (bindings/_mojotrees.mojo:3960-4010).  Host walk.
int32_t mojotrees_b200_predict_leaf(const MojoTreesModel* model, const double* data, int64_t n_rows,
                                    int64_t n_features, int64_t start_iteration, int64_t num_iteration,
                                    double* out_values, int64_t out_len, MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!model || (!data && n_rows > 0) || (!out_values && n_rows > 0)) throw InvalidArgument("null pointer argument");
        const mtb::Model& m = model->m;
        if (n_rows < 0) throw InvalidArgument("n_rows must be non-negative");
        if (n_features != m.n_features) throw InvalidArgument("n_features does not match the model");
        if (!m.has_mapper)
          throw mtb::Unsupported("model was trained on pre-binned data; raw values cannot be binned");
        const int K = m.num_class;
        const int64_t iters = (int64_t)m.trees.size() / K;
        const int64_t it0 = std::max<int64_t>(0, std::min(start_iteration, iters));
        const int64_t it1 = num_iteration <= 0 ? iters : std::min(iters, it0 + num_iteration);
        const int64_t cols = (it1 - it0) * K;
        if (out_len < n_rows * cols) throw InvalidArgument("output buffer too small");
        if (n_rows == 0 || cols == 0) return MOJOTREES_OK;
        std::vector<std::vector<int>> ord((size_t)cols);
        for (int64_t j = 0; j < cols; ++j) {
          const auto& t = m.trees[(size_t)(it0 * K + j)];
          ord[(size_t)j].assign(t.size(), -1);
          int next = 0;
          for (size_t i = 0; i < t.size(); ++i)
            if (t[i].feature < 0) ord[(size_t)j][i] = next++;
        }
        std::vector<uint8_t> bins((size_t)n_rows * n_features);
        mtb::transform(m.mapper, data, n_rows, bins.data());
#pragma omp parallel for schedule(static)
        for (int64_t r = 0; r < n_rows; ++r)
          for (int64_t j = 0; j < cols; ++j) {
            const auto& t = m.trees[(size_t)(it0 * K + j)];
            out_values[r * cols + j] = (double)ord[(size_t)j][(size_t)tree_leaf_node(t, bins.data() + r, n_rows)];
          }
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

// Rows binned with the model's own mapper, feature-major
// (out[f * n_rows + r]), for repeated scoring of one matrix.
int32_t mojotrees_b200_model_bin(const MojoTreesModel* model, const double* data, int64_t n_rows, int64_t n_features,
                                 uint8_t* out_bins, int64_t out_len, MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!model || ((!data || !out_bins) && n_rows > 0)) throw InvalidArgument("null pointer argument");
        const mtb::Model& m = model->m;
        if (n_rows < 0) throw InvalidArgument("n_rows must be non-negative");
        if (n_features != m.n_features) throw InvalidArgument("n_features does not match the model");
        if (!m.has_mapper)
          throw mtb::Unsupported("model was trained on pre-binned data; raw values cannot be binned");
        if (out_len < n_rows * n_features) throw InvalidArgument("output buffer too small");
        if (n_rows > 0) mtb::transform(m.mapper, data, n_rows, out_bins);
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

// raw[r * K + k] = fma(learning_rate, tree(iteration * K + k)(row r),
// raw[r * K + k]) for feature-major bins: one step of the host predictor's
// sum, so adding iterations 0..i-1 to the base scores gives the raw scores
// of the first i iterations bit for bit.
int32_t mojotrees_b200_add_iteration_raw(const MojoTreesModel* model, const uint8_t* bins, int64_t n_rows,
                                         int64_t n_features, int64_t iteration, double* raw_inout, int64_t len,
                                         MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!model || ((!bins || !raw_inout) && n_rows > 0)) throw InvalidArgument("null pointer argument");
        const mtb::Model& m = model->m;
        if (n_features != m.n_features) throw InvalidArgument("n_features does not match the model");
        const int K = m.num_class;
        const int64_t iters = (int64_t)m.trees.size() / K;
        if (iteration < 0 || iteration >= iters) throw InvalidArgument("iteration out of range");
        if (n_rows < 0 || len < n_rows * K) throw InvalidArgument("raw buffer too small");
#pragma omp parallel for schedule(static)
        for (int64_t r = 0; r < n_rows; ++r)
          for (int k = 0; k < K; ++k)
            raw_inout[r * K + k] =
                fma(m.learning_rate, tree_value(m.trees[(size_t)(iteration * K + k)], bins + r, n_rows),
                    raw_inout[r * K + k]);
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

// A new model holding the first n_iterations iterations of `model` (the cut
// early stopping makes); `model` itself is unchanged.
int32_t mojotrees_b200_model_prefix(const MojoTreesModel* model, int64_t n_iterations, MojoTreesModel** out_model,
                                    MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!model || !out_model) throw InvalidArgument("null pointer argument");
        const mtb::Model& m = model->m;
        const int64_t iters = (int64_t)m.trees.size() / m.num_class;
        if (n_iterations < 0 || n_iterations > iters) throw InvalidArgument("n_iterations out of range");
        std::unique_ptr<MojoTreesModel> h(new MojoTreesModel());
        h->m = m;
        h->m.trees.resize((size_t)(n_iterations * m.num_class));
        h->m.train_scores.clear();
        *out_model = h.release();
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

int32_t mojotrees_b200_bin_dense(const double* data, int64_t n_rows, int64_t n_features, const char* parameters,
                                 uint8_t* out_bins, int32_t* out_missing_bin, int32_t* out_n_categories,
                                 int32_t* out_n_bins, MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!data || !out_bins) throw InvalidArgument("null pointer argument");
        if (n_rows < 1 || n_features < 1) throw InvalidArgument("n_rows and n_features must be positive");
        TrainConfig cfg = parse_config(parameters, false);
        mtb::BinMapper m = mtb::fit_bins(data, n_rows, (int)n_features, cfg.binning);
        mtb::transform(m, data, n_rows, out_bins);
        for (int64_t f = 0; f < n_features; ++f) {
          if (out_missing_bin) out_missing_bin[f] = m.missing_bin[f];
          if (out_n_categories) out_n_categories[f] = m.is_cat[f] ? m.n_categories((int)f) : -1;
        }
        if (out_n_bins) *out_n_bins = m.n_bins;
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}


int32_t mojotrees_b200_bin_csc(const int64_t* indptr, const int64_t* indices, const double* values, int64_t n_rows,
                               int64_t n_features, const char* parameters, uint8_t* out_bins,
                               int32_t* out_missing_bin, int32_t* out_n_categories, int32_t* out_n_bins,
                               MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!indptr || !out_bins) throw InvalidArgument("null pointer argument");
        if (indptr[n_features] > 0 && (!indices || !values)) throw InvalidArgument("null pointer argument");
        if (n_rows < 1 || n_features < 1) throw InvalidArgument("n_rows and n_features must be positive");
        TrainConfig cfg = parse_config(parameters, false);
        try {
          mtb::check_csc(indptr, indices, n_rows, (int)n_features);
        } catch (const std::invalid_argument& e) {
          throw InvalidArgument(e.what());
        }
        mtb::BinMapper m = mtb::fit_bins_csc(indptr, indices, values, n_rows, (int)n_features, cfg.binning);
        mtb::transform_csc(m, indptr, indices, values, n_rows, out_bins);
        for (int64_t f = 0; f < n_features; ++f) {
          if (out_missing_bin) out_missing_bin[f] = m.missing_bin[f];
          if (out_n_categories) out_n_categories[f] = m.is_cat[f] ? m.n_categories((int)f) : -1;
        }
        if (out_n_bins) *out_n_bins = m.n_bins;
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

int32_t mojotrees_b200_train_csc(const int64_t* indptr, const int64_t* indices, const double* values, int64_t n_rows,
                                 int64_t n_features, const double* labels, const double* weights,
                                 const char* parameters, MojoTreesModel** out_model, MojoTreesError* error) {
  return guarded(error, [&]() -> int32_t {
    if (!indptr || !labels || !out_model) throw InvalidArgument("null pointer argument");
    if (n_rows < 1 || n_features < 1) throw InvalidArgument("n_rows and n_features must be positive");
    if (indptr[n_features] > 0 && (!indices || !values)) throw InvalidArgument("null pointer argument");
    TrainConfig cfg = parse_config(parameters, true);
    if (weights) throw mtb::Unsupported("sample weights are not covered by the device path");
    try {
      mtb::check_csc(indptr, indices, n_rows, (int)n_features);
    } catch (const std::invalid_argument& e) {
      throw InvalidArgument(e.what());
    }
    // bins of the densified matrix from the compressed columns: the host
    // holds n_rows x n_features bytes of bins, never the float64 matrix
    auto t0 = std::chrono::steady_clock::now();
    mtb::BinMapper mapper = mtb::fit_bins_csc(indptr, indices, values, n_rows, (int)n_features, cfg.binning);
    std::vector<uint8_t> bins((size_t)n_rows * (size_t)n_features);
    mtb::transform_csc(mapper, indptr, indices, values, n_rows, bins.data());
    const double bin_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    std::vector<int> ncats(n_features, -1);
    for (int f = 0; f < n_features; ++f)
      if (mapper.is_cat[f]) ncats[f] = mapper.n_categories(f);
    int32_t rc = train_binned(bins.data(), n_rows, n_features, mapper.n_bins, mapper.missing_bin, ncats, labels, cfg,
                              out_model, &mapper);
    if (rc == MOJOTREES_OK && *out_model) (*out_model)->m.stats.binning_seconds = bin_s;
    return rc;
  });
}

int32_t mojotrees_b200_bin_dense_gpu(const double* data, int64_t n_rows, int64_t n_features, const char* parameters,
                                     uint8_t* out_bins, int32_t* out_missing_bin, int32_t* out_n_categories,
                                     int32_t* out_n_bins, MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!data || !out_bins) throw InvalidArgument("null pointer argument");
        if (n_rows < 1 || n_features < 1) throw InvalidArgument("n_rows and n_features must be positive");
        TrainConfig cfg = parse_config(parameters, false);
        if (mtb::cuda_device_count() < 1) throw mtb::Unsupported("no CUDA device is available");
        mtb::BinMapper m = mtb::fit_bins(data, n_rows, (int)n_features, cfg.binning);
        const size_t bytes = (size_t)n_rows * (size_t)n_features;
        uint8_t* d_bins = nullptr;
        if (cudaMalloc(&d_bins, bytes) != cudaSuccess) throw std::runtime_error("cudaMalloc failed");
        struct Free {
          uint8_t* p;
          ~Free() { cudaFree(p); }
        } fr{d_bins};
        mtb::transform_on_device(m, data, n_rows, d_bins, 0);
        if (cudaMemcpy(out_bins, d_bins, bytes, cudaMemcpyDeviceToHost) != cudaSuccess)
          throw std::runtime_error("cudaMemcpy failed");
        for (int64_t f = 0; f < n_features; ++f) {
          if (out_missing_bin) out_missing_bin[f] = m.missing_bin[f];
          if (out_n_categories) out_n_categories[f] = m.is_cat[f] ? m.n_categories((int)f) : -1;
        }
        if (out_n_bins) *out_n_bins = m.n_bins;
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

int32_t mojotrees_predict(const MojoTreesModel* model, const double* data, int64_t n_rows, int64_t n_features,
                          double* out_values, int64_t out_len, MojoTreesError* error) {
  return predict_impl(model, data, n_rows, n_features, 0, 0, MOJOTREES_PREDICT_RESPONSE, MOJOTREES_DEVICE_CPU,
                      out_values, out_len, error);
}

int32_t mojotrees_predict_raw(const MojoTreesModel* model, const double* data, int64_t n_rows, int64_t n_features,
                              double* out_values, int64_t out_len, MojoTreesError* error) {
  return predict_impl(model, data, n_rows, n_features, 0, 0, MOJOTREES_PREDICT_RAW, MOJOTREES_DEVICE_CPU, out_values,
                      out_len, error);
}

int32_t mojotrees_predict_ex(const MojoTreesModel* model, const double* data, int64_t n_rows, int64_t n_features,
                             int64_t start_iteration, int64_t num_iteration, int32_t flags, int32_t device,
                             double* out_values, int64_t out_len, MojoTreesError* error) {
  return predict_impl(model, data, n_rows, n_features, start_iteration, num_iteration, flags, device, out_values,
                      out_len, error);
}

int32_t mojotrees_b200_predict_binned_u8(const MojoTreesModel* model, const uint8_t* bins, int64_t n_rows,
                                         int64_t n_features, double* out_values, int64_t out_len,
                                         MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!model || !bins || !out_values) throw InvalidArgument("null pointer argument");
        const mtb::Model& m = model->m;
        if (n_features != m.n_features) throw InvalidArgument("n_features does not match the model");
        if (out_len < n_rows * m.num_class) throw InvalidArgument("output buffer too small");
        raw_scores(m, bins, n_rows, 0, (int64_t)m.trees.size() / m.num_class, out_values);
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

static const char kMagic[] = "mojotrees-b200 v1";

// Model files use the reference's text format v4 (serialize.mojo:999-1119):
// floats as their IEEE-754 bit patterns, so a round trip is bit-exact.
int32_t mojotrees_save_model(const MojoTreesModel* model, const char* path, MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!model || !path) throw InvalidArgument("null pointer argument");
        std::ostringstream os;
        mtb::save_model_v4(model->m, os);
        std::ofstream f(path);
        if (!f) throw std::runtime_error(std::string("cannot open '") + path + "' for writing");
        f << os.str();
        f.flush();
        if (!f) throw std::runtime_error("write failed");
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_IO);
}

static double read_double(std::istream& is) {
  std::string s;
  is >> s;
  return strtod(s.c_str(), nullptr);
}

int32_t mojotrees_load_model(const char* path, MojoTreesModel** out_model, MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!path || !out_model) throw InvalidArgument("null pointer argument");
        std::ifstream is(path);
        if (!is) throw std::runtime_error(std::string("cannot open '") + path + "'");
        std::string magic;
        std::getline(is, magic);
        if (magic != kMagic) {
          // the reference's token format (v1-v4)
          std::ostringstream all;
          all << magic << '\n' << is.rdbuf();
          std::unique_ptr<MojoTreesModel> h(new MojoTreesModel());
          h->m = mtb::load_model_text(all.str());
          *out_model = h.release();
          return MOJOTREES_OK;
        }
        // this library's earlier private format
        std::unique_ptr<MojoTreesModel> h(new MojoTreesModel());
        mtb::Model& m = h->m;
        size_t n_trees;
        int has_mapper;
        is >> m.objective >> m.num_class >> m.n_features;
        m.learning_rate = read_double(is);
        is >> n_trees >> has_mapper;
        m.base_scores.resize(m.num_class);
        for (auto& b : m.base_scores) b = read_double(is);
        if (has_mapper) {
          mtb::BinMapper& mp = m.mapper;
          size_t ne, nc;
          is >> mp.n_bins >> ne >> nc;
          mp.n_features = m.n_features;
          mp.edges.resize(ne);
          for (auto& e : mp.edges) e = read_double(is);
          mp.edge_offsets.resize(m.n_features + 1);
          for (auto& o : mp.edge_offsets) is >> o;
          mp.missing_bin.resize(m.n_features);
          for (auto& v : mp.missing_bin) is >> v;
          mp.is_cat.resize(m.n_features);
          for (auto& v : mp.is_cat) {
            int x;
            is >> x;
            v = (uint8_t)x;
          }
          mp.cat_codes.resize(nc);
          for (auto& v : mp.cat_codes) is >> v;
          mp.cat_offsets.resize(m.n_features + 1);
          for (auto& v : mp.cat_offsets) is >> v;
          m.has_mapper = true;
        }
        m.trees.resize(n_trees);
        for (auto& t : m.trees) {
          size_t nn;
          is >> nn;
          t.resize(nn);
          for (auto& nd : t) {
            is >> nd.feature >> nd.thr >> nd.left >> nd.right >> nd.dleft >> nd.mbin >> nd.is_cat >> nd.bits[0] >>
                nd.bits[1] >> nd.bits[2] >> nd.bits[3];
            nd.value = read_double(is);
            nd.gain = read_double(is);
            is >> nd.count;
            nd.pad = 0;
          }
        }
        if (!is) throw std::runtime_error("truncated or malformed model file");
        *out_model = h.release();
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_IO);
}

#define MTB_ACCESSOR(name, expr)                                                                          \
  int32_t name(const MojoTreesModel* model, int64_t* out_value, MojoTreesError* error) {                  \
    return guarded(                                                                                       \
        error,                                                                                            \
        [&]() -> int32_t {                                                                                \
          if (!model || !out_value) throw InvalidArgument("null pointer argument");                       \
          const mtb::Model& m = model->m;                                                                 \
          *out_value = (expr);                                                                            \
          return MOJOTREES_OK;                                                                            \
        },                                                                                                \
        MOJOTREES_ERROR_INVALID_ARGUMENT);                                                                \
  }

MTB_ACCESSOR(mojotrees_model_num_features, m.n_features)
MTB_ACCESSOR(mojotrees_model_num_classes, m.num_class)
MTB_ACCESSOR(mojotrees_model_num_trees, (int64_t)m.trees.size())
MTB_ACCESSOR(mojotrees_model_num_iterations, (int64_t)m.trees.size() / m.num_class)

int32_t mojotrees_model_dump_json(const MojoTreesModel* model, char** out_text, MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!model || !out_text) throw InvalidArgument("null pointer argument");
        *out_text = dup_string(mtb::dump_model_json(model->m));
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

int32_t mojotrees_feature_importance(const MojoTreesModel* model, int32_t importance_type, double* out_values,
                                     int64_t out_len, MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!model || !out_values) throw InvalidArgument("null pointer argument");
        if (importance_type != MOJOTREES_IMPORTANCE_SPLIT && importance_type != MOJOTREES_IMPORTANCE_GAIN)
          throw InvalidArgument("unknown importance type");
        const mtb::Model& m = model->m;
        if (out_len < m.n_features) throw InvalidArgument("output buffer too small");
        std::vector<double> imp(m.n_features, 0.0);
        for (auto& t : m.trees)
          for (auto& nd : t)
            if (nd.feature >= 0) imp[nd.feature] += importance_type == MOJOTREES_IMPORTANCE_SPLIT ? 1.0 : nd.gain;
        memcpy(out_values, imp.data(), sizeof(double) * imp.size());
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

int32_t mojotrees_parameter_keys(char** out_text, MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!out_text) throw InvalidArgument("null pointer argument");
        std::string s;
        for (auto& e : param_table()) s += (s.empty() ? "" : ",") + e.first;
        *out_text = dup_string(s);
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

void mojotrees_string_free(char* text) { free(text); }

void mojotrees_model_free(MojoTreesModel* model) { delete model; }

int32_t mojotrees_b200_tree_nodes(const MojoTreesModel* model, int64_t tree, int32_t* out_ints, double* out_doubles,
                                  int64_t* out_counts, uint64_t* out_cat_bits, int64_t capacity, int64_t* out_n_nodes,
                                  MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!model || !out_n_nodes) throw InvalidArgument("null pointer argument");
        const mtb::Model& m = model->m;
        if (tree < 0 || tree >= (int64_t)m.trees.size()) throw InvalidArgument("tree index out of range");
        const auto& t = m.trees[tree];
        *out_n_nodes = (int64_t)t.size();
        if (capacity < (int64_t)t.size()) throw InvalidArgument("capacity too small for the tree");
        for (size_t i = 0; i < t.size(); ++i) {
          const auto& nd = t[i];
          if (out_ints) {
            int32_t* p = out_ints + 7 * i;
            p[0] = nd.feature;
            p[1] = nd.thr;
            p[2] = nd.left;
            p[3] = nd.right;
            p[4] = nd.dleft;
            p[5] = nd.mbin;
            p[6] = nd.is_cat;
          }
          if (out_doubles) {
            out_doubles[2 * i] = nd.value;
            out_doubles[2 * i + 1] = nd.gain;
          }
          if (out_counts) out_counts[i] = nd.count;
          if (out_cat_bits)
            for (int w = 0; w < 4; ++w) out_cat_bits[4 * i + w] = nd.bits[w];
        }
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

int32_t mojotrees_b200_base_scores(const MojoTreesModel* model, double* out_values, int64_t out_len,
                                   MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!model || !out_values) throw InvalidArgument("null pointer argument");
        const mtb::Model& m = model->m;
        if (out_len < (int64_t)m.base_scores.size()) throw InvalidArgument("output buffer too small");
        memcpy(out_values, m.base_scores.data(), sizeof(double) * m.base_scores.size());
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

int32_t mojotrees_b200_training_scores(const MojoTreesModel* model, double* out_values, int64_t out_len,
                                       MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!model || !out_values) throw InvalidArgument("null pointer argument");
        const mtb::Model& m = model->m;
        if (m.train_scores.empty()) throw InvalidArgument("the fit did not keep training scores (keep_training_scores=true)");
        if (out_len < (int64_t)m.train_scores.size()) throw InvalidArgument("output buffer too small");
        memcpy(out_values, m.train_scores.data(), sizeof(double) * m.train_scores.size());
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

int32_t mojotrees_b200_train_stats(const MojoTreesModel* model, double* out_values, int64_t out_len, int64_t* out_n,
                                   MojoTreesError* error) {
  return guarded(
      error,
      [&]() -> int32_t {
        if (!model || !out_values) throw InvalidArgument("null pointer argument");
        const mtb::TrainStats& s = model->m.stats;
        const double v[] = {s.fit_seconds, s.upload_seconds, s.hist_ms,   s.partition_ms,
                            s.scan_ms,     s.grad_ms,        s.hist_rows, s.hist_bytes,
                            (double)s.hist_launches, (double)s.kernel_launches, (double)s.rounds,
                            s.commit_ms,   (double)s.iterations, (double)s.expansions, s.binning_seconds,
                            (double)s.pick_steps, s.hist_sparse_entries};
        int64_t n = std::min<int64_t>(out_len, (int64_t)(sizeof v / sizeof v[0]));
        for (int64_t i = 0; i < n; ++i) out_values[i] = v[i];
        if (out_n) *out_n = n;
        return MOJOTREES_OK;
      },
      MOJOTREES_ERROR_INVALID_ARGUMENT);
}

}  // extern "C"
