/* mojotrees C ABI, served by the B200-native training library
 * (libmojotrees_b200.so).
 *
 * This header declares the same entry points, with the same signatures,
 * status codes and ownership rules, as the reference's C ABI v3
 * (ajhendel/mojoboost capi/mojotrees.h), so a caller built against that
 * header links against this library unchanged.  Each declaration cites the
 * reference line it replaces.  Entry points prefixed `mojotrees_b200_` are
 * extensions with no counterpart in the reference header.
 *
 * Rules callers may rely on (reference capi/mojotrees.h:8-35):
 *   - Only C scalars, C strings and opaque handles cross the boundary.
 *   - Hyperparameters are a LightGBM-style "key=value key=value" string.
 *   - Fallible calls return MOJOTREES_OK (0) or a negative code; the reason
 *     is written into the caller's error object, cleared on entry.
 *   - The library copies what it needs and never retains caller pointers.
 *   - Every returned handle is freed exactly once; free functions accept NULL.
 *   - A NULL required pointer is MOJOTREES_ERROR_INVALID_ARGUMENT, not a crash.
 *
 * Device policy of this library: training runs on a CUDA device (sm_100a).
 * "device=gpu" (the default here) never falls back to the CPU; a request the
 * device path does not cover returns MOJOTREES_ERROR_UNSUPPORTED naming what
 * is uncovered.  "device=cpu" is MOJOTREES_ERROR_UNSUPPORTED as well: this
 * library is the accelerated path only.  Prediction runs on the host unless
 * mojotrees_predict_ex asks for MOJOTREES_DEVICE_GPU (the same bits; an error
 * without a CUDA device, never a host fallback).
 */
#ifndef MOJOTREES_H
#define MOJOTREES_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* reference capi/mojotrees.h:84 */
#define MOJOTREES_ABI_VERSION 3

/* reference capi/mojotrees.h:87-91 */
#define MOJOTREES_OK 0
#define MOJOTREES_ERROR_INVALID_ARGUMENT (-1)
#define MOJOTREES_ERROR_TRAINING (-2)
#define MOJOTREES_ERROR_IO (-3)
#define MOJOTREES_ERROR_UNSUPPORTED (-4)

/* reference capi/mojotrees.h:101-103 */
#define MOJOTREES_DEVICE_CPU 0
#define MOJOTREES_DEVICE_GPU 1
#define MOJOTREES_DEVICE_AUTO 2

/* reference capi/mojotrees.h:108-109 */
#define MOJOTREES_PREDICT_RESPONSE 0
#define MOJOTREES_PREDICT_RAW 1

/* reference capi/mojotrees.h:115-116 */
#define MOJOTREES_IMPORTANCE_SPLIT 0
#define MOJOTREES_IMPORTANCE_GAIN 1

/* reference capi/mojotrees.h:119-122 */
typedef struct MojoTreesModel MojoTreesModel;
typedef struct MojoTreesError MojoTreesError;

/* reference capi/mojotrees.h:127 */
int32_t mojotrees_abi_version(void);
/* reference capi/mojotrees.h:130-131 */
void mojotrees_library_version(int32_t *major, int32_t *minor, int32_t *patch);
/* reference capi/mojotrees.h:142.  1 when a CUDA device is visible. */
int32_t mojotrees_gpu_available(void);

/* reference capi/mojotrees.h:147-161 */
MojoTreesError *mojotrees_error_create(void);
void mojotrees_error_free(MojoTreesError *error);
const char *mojotrees_error_message(const MojoTreesError *error);

/* reference capi/mojotrees.h:181-185.  data is column-major
 * (data[f * n_rows + r]), NaN is missing.  weights must be NULL on the
 * device path (weighted fits return MOJOTREES_ERROR_UNSUPPORTED). */
int32_t mojotrees_train_dense(const double *data, int64_t n_rows, int64_t n_features, const double *labels,
                              const double *weights, const char *parameters, MojoTreesModel **out_model,
                              MojoTreesError *error);

/* reference capi/mojotrees.h:197-200 */
int32_t mojotrees_predict(const MojoTreesModel *model, const double *data, int64_t n_rows, int64_t n_features,
                          double *out_values, int64_t out_len, MojoTreesError *error);
/* reference capi/mojotrees.h:205-208 */
int32_t mojotrees_predict_raw(const MojoTreesModel *model, const double *data, int64_t n_rows,
                              int64_t n_features, double *out_values, int64_t out_len, MojoTreesError *error);
/* reference capi/mojotrees.h:227-233.  device CPU or AUTO: host; GPU: rows binned
 * and trees walked on the current CUDA device, bit-identical to the host. */
int32_t mojotrees_predict_ex(const MojoTreesModel *model, const double *data, int64_t n_rows, int64_t n_features,
                             int64_t start_iteration, int64_t num_iteration, int32_t flags, int32_t device,
                             double *out_values, int64_t out_len, MojoTreesError *error);

/* reference capi/mojotrees.h:238-246.  The file is this library's own text
 * format ("mojotrees-b200 v1"), not the reference's format v4. */
int32_t mojotrees_save_model(const MojoTreesModel *model, const char *path, MojoTreesError *error);
int32_t mojotrees_load_model(const char *path, MojoTreesModel **out_model, MojoTreesError *error);

/* reference capi/mojotrees.h:251-274 */
int32_t mojotrees_model_num_features(const MojoTreesModel *model, int64_t *out_value, MojoTreesError *error);
int32_t mojotrees_model_num_classes(const MojoTreesModel *model, int64_t *out_value, MojoTreesError *error);
int32_t mojotrees_model_num_trees(const MojoTreesModel *model, int64_t *out_value, MojoTreesError *error);
int32_t mojotrees_model_num_iterations(const MojoTreesModel *model, int64_t *out_value, MojoTreesError *error);

/* reference capi/mojotrees.h:287-288 */
int32_t mojotrees_model_dump_json(const MojoTreesModel *model, char **out_text, MojoTreesError *error);
/* reference capi/mojotrees.h:307-310 */
int32_t mojotrees_feature_importance(const MojoTreesModel *model, int32_t importance_type, double *out_values,
                                     int64_t out_len, MojoTreesError *error);
/* reference capi/mojotrees.h:323 */
int32_t mojotrees_parameter_keys(char **out_text, MojoTreesError *error);

/* reference capi/mojotrees.h:331-336 */
void mojotrees_string_free(char *text);
void mojotrees_model_free(MojoTreesModel *model);

/* ------------------------------------------------------------ extensions */

/* Train on pre-binned data: bins is feature-major uint8 (bins[f * n_rows + r])
 * with values < n_bins.  missing_bin (NULL = none) gives per feature the bin
 * that holds missing values or -1; n_categories (NULL = all numeric) gives
 * per feature -1 for numeric or the number of category bins (bins 1..n,
 * bin 0 = unseen).  For inputs too large for a float64 matrix, such as
 * 200M x 128.  Replaces the reference's binned Dataset route
 * (bindings/dataset_bindings.mojo). */
int32_t mojotrees_b200_train_binned_u8(const uint8_t *bins, int64_t n_rows, int64_t n_features, int32_t n_bins,
                                       const int32_t *missing_bin, const int32_t *n_categories,
                                       const double *labels, const double *weights, const char *parameters,
                                       MojoTreesModel **out_model, MojoTreesError *error);

/* Host binning exactly as mojotrees_train_dense bins its input: writes
 * feature-major bins (n_rows * n_features bytes), the per-feature missing bin
 * and category count.  Parameters: max_bin, min_data_in_bin,
 * bin_construct_sample_cnt, data_random_seed, use_missing, categorical_feature. */
int32_t mojotrees_b200_bin_dense(const double *data, int64_t n_rows, int64_t n_features, const char *parameters,
                                 uint8_t *out_bins, int32_t *out_missing_bin, int32_t *out_n_categories,
                                 int32_t *out_n_bins, MojoTreesError *error);

/* The same bins as mojotrees_b200_bin_dense, with the columns binned on the
 * current CUDA device (the transform mojotrees_train_dense uses): edges are
 * fitted on the host, the float64 columns are copied in feature chunks and
 * binned by a kernel.  MOJOTREES_ERROR_UNSUPPORTED without a device. */
int32_t mojotrees_b200_bin_dense_gpu(const double *data, int64_t n_rows, int64_t n_features,
                                     const char *parameters, uint8_t *out_bins, int32_t *out_missing_bin,
                                     int32_t *out_n_categories, int32_t *out_n_bins, MojoTreesError *error);

/* Measured roofline of the histogram kernel's inner loop: the rate (lane
 * atomics per second, whole GPU) at which the SMs sustain conflict-free
 * red.shared.add.u32 in the histogram's shared-memory layout and launch
 * geometry, with no global traffic.  Runs a few short kernels on the current
 * device. */
int32_t mojotrees_b200_shared_atomic_peak(double *out_lane_atomics_per_s, MojoTreesError *error);

/* Raw-score prediction on pre-binned feature-major data (any model). */
int32_t mojotrees_b200_predict_binned_u8(const MojoTreesModel *model, const uint8_t *bins, int64_t n_rows,
                                         int64_t n_features, double *out_values, int64_t out_len,
                                         MojoTreesError *error);

/* Node table of one tree: per node feature, threshold_bin, left, right,
 * default_left, missing_bin, is_categorical (7 int32 per node, node-major),
 * value, gain (2 doubles per node) and count (int64), plus 4 uint64 words of
 * categorical set per node.  Any out pointer may be NULL.  *out_n_nodes
 * receives the node count; capacities are in nodes. */
int32_t mojotrees_b200_tree_nodes(const MojoTreesModel *model, int64_t tree, int32_t *out_ints, double *out_doubles,
                                  int64_t *out_counts, uint64_t *out_cat_bits, int64_t capacity,
                                  int64_t *out_n_nodes, MojoTreesError *error);

/* Initial scores (num_classes doubles). */
int32_t mojotrees_b200_base_scores(const MojoTreesModel *model, double *out_values, int64_t out_len,
                                   MojoTreesError *error);

/* Training-set raw scores after the last round, when the fit was run with
 * keep_training_scores=true: n_rows * num_classes doubles, row-major. */
int32_t mojotrees_b200_training_scores(const MojoTreesModel *model, double *out_values, int64_t out_len,
                                       MojoTreesError *error);

/* Training statistics: fills up to out_len doubles in this order:
 * fit_seconds, upload_seconds, hist_ms, partition_ms, scan_ms, grad_ms,
 * hist_rows, hist_bytes, hist_launches, kernel_launches, rounds, commit_ms,
 * iterations (batch iterations that did work), expansions (leaves whose
 * children were computed; exceeds the splits by the speculative ones),
 * binning_seconds (host bin fitting and transform of mojotrees_train_dense).  The phase
 * times are measured with CUDA events only when the fit ran with
 * profile_phases=true.  Returns the number of values written via *out_n. */
int32_t mojotrees_b200_train_stats(const MojoTreesModel *model, double *out_values, int64_t out_len,
                                   int64_t *out_n, MojoTreesError *error);

/* Device time of each boosting round of the fit, in milliseconds, measured
 * with CUDA events on the trainer's stream (one round = the K trees of a
 * multiclass iteration).  *out_n receives the number of rounds. */
int32_t mojotrees_b200_round_times(const MojoTreesModel *model, double *out_values, int64_t out_len,
                                   int64_t *out_n, MojoTreesError *error);

/* Per-round statistics of the fit, 5 doubles per round (row-major, *out_n =
 * rounds): device time (ms, CUDA events), histogram-kernel time (ms; CUDA
 * events around every histogram launch, only when the fit ran with
 * profile_phases=true, else 0), histogram launches, rows read by histogram
 * builds (the root and the smaller child of every split), kernels launched.
 * out_values may be NULL to query the count. */
int32_t mojotrees_b200_round_stats(const MojoTreesModel *model, double *out_values, int64_t out_len,
                                   int64_t *out_n, MojoTreesError *error);
/* Which features the model splits by category set, from its bin mapper: one
 * flag (1 categorical, 0 numerical) per feature into out_flags[0, n_features).
 * The reference's `categorical_features` (bindings/_mojotrees.mojo:4802). */
int32_t mojotrees_b200_model_categorical(const MojoTreesModel *model, int32_t *out_flags, int64_t out_len,
                                         MojoTreesError *error);

/* Row-major float64 (src[r * n_features + f]) into a caller-allocated
 * column-major buffer (dst[f * n_rows + r]) on all host threads, with
 * *out_has_infinite (may be NULL) = 1 when any value is +inf or -inf (NaN is
 * not reported).  The reference's `ingest_column_major`
 * (bindings/_mojotrees.mojo:682). */
int32_t mojotrees_b200_ingest_column_major(const double *src, double *dst, int64_t n_rows, int64_t n_features,
                                           int32_t *out_has_infinite, MojoTreesError *error);
/* *out_has_infinite = 1 when data[0, n) holds +inf or -inf.  The reference's
 * `buffer_has_infinite` (bindings/_mojotrees.mojo:722). */
int32_t mojotrees_b200_buffer_has_infinite(const double *data, int64_t n, int32_t *out_has_infinite,
                                           MojoTreesError *error);
/* Leaf ordinals (a leaf's rank among its tree's leaves in node order) of
 * column-major rows over iterations [start_iteration, start_iteration +
 * num_iteration) (num_iteration <= 0: to the end), as float64:
 * out[r * (n * K) + i * K + k] for class k's tree of iteration i.  On the
 * host.  The reference's `predict_leaf` / `predict_leaf_multiclass`
 * (bindings/_mojotrees.mojo:3960-4010, tree.mojo:558-580). */
int32_t mojotrees_b200_predict_leaf(const MojoTreesModel *model, const double *data, int64_t n_rows,
                                    int64_t n_features, int64_t start_iteration, int64_t num_iteration,
                                    double *out_values, int64_t out_len, MojoTreesError *error);

/* Validation scoring, the round loop of the reference's metric fits
 * (custom_metric.mojo:1087-1280, which scores validation sets after every
 * tree): bin the rows once with the model's mapper (feature-major uint8,
 * out_bins[f * n_rows + r]), then add one iteration at a time to raw scores
 * that start at the base scores.  Each step is the host predictor's
 * raw = fma(learning_rate, leaf, raw), so after i steps the scores equal
 * mojotrees_predict_ex's raw scores of the first i iterations bit for bit. */
int32_t mojotrees_b200_model_bin(const MojoTreesModel *model, const double *data, int64_t n_rows,
                                 int64_t n_features, uint8_t *out_bins, int64_t out_len, MojoTreesError *error);
int32_t mojotrees_b200_add_iteration_raw(const MojoTreesModel *model, const uint8_t *bins, int64_t n_rows,
                                         int64_t n_features, int64_t iteration, double *raw_inout, int64_t len,
                                         MojoTreesError *error);
/* A new model with the first n_iterations iterations of `model` (the
 * early-stopping cut, custom_metric.mojo:1270-1280); free it with
 * mojotrees_model_free. */
int32_t mojotrees_b200_model_prefix(const MojoTreesModel *model, int64_t n_iterations, MojoTreesModel **out_model,
                                    MojoTreesError *error);

/* Data-parallel training (one process per GPU, rows sharded): a fresh
 * 128-byte NCCL unique id, created on one rank and broadcast by the caller. */
int32_t mojotrees_b200_nccl_unique_id(uint8_t *out_id, MojoTreesError *error);

/* Data-parallel fit over row shards.  Every rank calls this collectively with
 * the same parameters and nccl_id; rank r passes its rows
 * [row_offset, row_offset + n_rows) of n_rows_global, shards other than the
 * last holding a multiple of 1024 rows.  Histograms are summed across GPUs
 * with NCCL (exact int32), so every rank grows the same trees, identical to
 * a single-GPU fit on all rows.  Replaces the reference's CPU data-parallel
 * strategy (bindings/distributed_bindings.mojo, distributed.mojo:1286-1520). */
int32_t mojotrees_b200_train_binned_u8_dp(const uint8_t *bins, int64_t n_rows, int64_t n_features, int32_t n_bins,
                                          const int32_t *missing_bin, const int32_t *n_categories,
                                          const double *labels, const double *weights, const char *parameters,
                                          const uint8_t *nccl_id, int32_t rank, int32_t world, int64_t row_offset,
                                          int64_t n_rows_global, MojoTreesModel **out_model, MojoTreesError *error);

/* One quantized-gradient histogram, built by the trainer's per-leaf kernel:
 * for the selected rows (rows = NULL: all rows), per feature and bin, the
 * sums of grad_q and hess_q and the row count.  bins is feature-major
 * (bins[f * n_rows + r] < n_bins); grad_q[r] in [-q/2, q/2] and hess_q[r] in
 * [0, q] for q = num_grad_quant_bins (the int8 packer's range).  out_hist
 * receives n_features * 3 * n_bins int32, laid out [feature][g, h, count][bin].
 * Host buffers; the call allocates device memory.  The device kernel behind
 * gpu_active_rows.mojo:3903 (_range_hist_atomic_kernel) in the reference. */
int32_t mojotrees_b200_histogram_u8(const uint8_t *bins, int64_t n_rows, int64_t n_features, int32_t n_bins,
                                    const int32_t *rows, int64_t n_sel, const int8_t *grad_q,
                                    const uint8_t *hess_q, int32_t num_grad_quant_bins, int32_t *out_hist,
                                    MojoTreesError *error);

/* The histogram of mojotrees_b200_histogram_u8 for callers that cannot
 * allocate GPU memory: callers whose own pool allocator owns the device
 * memory and forbids others from taking any, and latency-critical paths that
 * must not take the allocator's locks.  It has no counterpart in the
 * reference.  Everything is device memory the caller owns: bins_rm is
 * row-major uint8 with a row stride of n_features rounded up to 16 bytes,
 * rows holds n_sel row ids, pairs holds n_sel packed gradients (low byte the
 * int8 gradient, high byte the hessian, in the order of rows), out_hist
 * receives n_features * 3 * n_bins int32 as in mojotrees_b200_histogram_u8.
 * Preconditions the call cannot check (the data is on the device): every
 * rows[i] is in [0, n_rows), every bin is below n_bins, and with
 * q = num_grad_quant_bins every gradient is in [-q/2, q/2] and every hessian
 * in [0, q]; values outside these ranges read out of bounds or carry into
 * neighbouring packed counters.
 * The work runs on `stream` (a cudaStream_t; NULL = the legacy stream).
 * The library keeps the job descriptor and the accumulation cells in one
 * fixed device array (about 385 KB, held by every GPU that loads the library
 * until exit), so n_features * n_bins may not exceed 128 * 256; larger
 * requests return MOJOTREES_ERROR_INVALID_ARGUMENT.  The first call on a
 * device looks up the array's device address.  Every call shares the array
 * and clears the cells it uses; calls whose GPU work overlaps (two streams,
 * two threads) race on it. */
int32_t mojotrees_b200_histogram_u8_noalloc(const uint8_t *bins_rm, int64_t n_rows, int64_t n_features,
                                            int32_t n_bins, const int32_t *rows, int64_t n_sel,
                                            const uint16_t *pairs, int32_t num_grad_quant_bins, int32_t *out_hist,
                                            void *stream, MojoTreesError *error);

/* Training on a compressed-sparse-column matrix: indptr[n_features + 1]
 * offsets, row indices strictly increasing within each column, values; an
 * absent entry is the value 0.0 and a stored NaN is missing.  The bins are
 * those of the densified matrix (the reference's sparse fit bins them
 * identically, sparse.mojo:535-570), computed from the compressed columns:
 * the host holds n_rows x n_features bytes of bins, never the dense float64
 * matrix.  Replaces the sparse fit of bindings/_mojotrees.mojo:3335-3420
 * (fit_csc); the model predicts raw feature values like a dense fit's.
 * mojotrees_b200_bin_csc returns those bins (feature-major), missing bins,
 * category counts (-1 for numeric features) and the bin count. */
int32_t mojotrees_b200_train_csc(const int64_t *indptr, const int64_t *indices, const double *values,
                                 int64_t n_rows, int64_t n_features, const double *labels, const double *weights,
                                 const char *parameters, MojoTreesModel **out_model, MojoTreesError *error);
int32_t mojotrees_b200_bin_csc(const int64_t *indptr, const int64_t *indices, const double *values, int64_t n_rows,
                               int64_t n_features, const char *parameters, uint8_t *out_bins,
                               int32_t *out_missing_bin, int32_t *out_n_categories, int32_t *out_n_bins,
                               MojoTreesError *error);

/* Diagnostic: n random (integer sum, quantizer units) pairs dequantized on
 * the device by the trainer's divide-free quotient and by the divide; the
 * number of results whose bits differ goes to out_mismatches (0 expected).
 * No counterpart in the reference. */
int32_t mojotrees_b200_check_quotients(int64_t n, uint64_t seed, int64_t *out_mismatches, MojoTreesError *error);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* MOJOTREES_H */
