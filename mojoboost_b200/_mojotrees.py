"""The subset of the reference's `_mojotrees` extension the estimators use for
`fit(device="gpu")`, over ctypes and libmojotrees_b200.so.

Reference: bindings/_mojotrees.mojo:2094-2102 (`fit`) and its multiclass twin
`fit_multiclass`; objective codes python/mojotrees/sklearn.py:33-55.  Buffers
cross as integer addresses of float64 arrays, X column-major, as the reference
wrapper passes them (`_addr(Xb)`).  Hooks this library does not implement
raise NotImplementedError naming the hook.
"""
import ctypes

import numpy as np

from . import _capi
from ._registry import (metric_code_of_name, objective_code_of_name, objective_name_status_of,  # noqa: F401
                        registry_metric_aliases, registry_metrics, registry_objective_aliases,
                        registry_objective_unimplemented, registry_objectives, registry_vocabulary)

# objective codes of the reference package (python/mojotrees/sklearn.py:33-55)
SQUARED_ERROR = 0
BINARY_LOGISTIC = 1
MULTICLASS = -1
_OBJECTIVE_NAMES = {SQUARED_ERROR: "regression", BINARY_LOGISTIC: "binary", MULTICLASS: "multiclass"}

# reference params-dict keys (python/mojotrees/sklearn.py `_Base._params`)
# -> parameter-string keys of the C ABI
_KEY_MAP = {
    "n_estimators": "num_iterations", "learning_rate": "learning_rate", "num_leaves": "num_leaves",
    "min_data_in_leaf": "min_data_in_leaf", "lambda_l2": "lambda_l2", "lambda_l1": "lambda_l1",
    "min_child_hess": "min_sum_hessian_in_leaf", "feature_fraction": "feature_fraction",
    "feature_fraction_seed": "feature_fraction_seed", "max_bin": "max_bin", "min_data_in_bin": "min_data_in_bin",
    "bin_construct_sample_cnt": "bin_construct_sample_cnt", "data_random_seed": "data_random_seed",
    "use_missing": "use_missing", "max_cat_to_onehot": "max_cat_to_onehot",
    "max_cat_threshold": "max_cat_threshold", "cat_smooth": "cat_smooth", "cat_l2": "cat_l2",
    "min_data_per_group": "min_data_per_group", "use_quantized_grad": "use_quantized_grad",
    "num_grad_quant_bins": "num_grad_quant_bins", "stochastic_rounding": "stochastic_rounding",
    "num_class": "num_class",
}
# Options that change training and that the device path does not implement:
# they must stay at the value meaning "off", and anything else is refused by
# name rather than silently trained without.
_MUST_BE = {
    "bagging_fraction": 1.0, "bagging_freq": 0, "bootstrap_type": "no", "goss": 0, "boosting": "gbdt",
    "max_depth": -1, "linear_tree": 0, "ordered": 0, "feature_fraction_bynode": 1.0, "enable_bundle": 0,
    "ctr": "off", "catboost_mode_defaults": 0, "grow_policy": "lossguide", "score_function": "l2",
    "random_strength": 0.0, "leaf_estimation_iterations": 1, "auto_learning_rate": 0, "boost_from_average": 1,
    "min_gain_to_split": 0.0, "max_delta_step": 0.0, "path_smooth": 0.0, "extra_trees": 0,
    "monotone_penalty": 0.0, "cegb_tradeoff": 1.0, "cegb_penalty_split": 0.0, "forced_splits": "",
    "monotone_addr": 0, "interaction_flat_addr": 0, "interaction_flat_len": 0, "interaction_offsets_addr": 0,
    "interaction_offsets_len": 0, "feature_contri_addr": 0, "cegb_penalty_feature_coupled_addr": 0,
    "cegb_penalty_feature_lazy_addr": 0, "sample_weight_addr": 0, "derivative_precision": "float32",
}
# Keys that only matter when one of the options above is on (their seeds and
# knobs), or for objectives this library does not train: read and ignored.
_INERT = {
    "alpha", "bagging_seed", "bagging_temperature", "boost_from_average_set", "bootstrap_explicit",
    "bootstrap_seed", "bootstrap_subsample", "bundle_missing", "ctr_set", "ctr_target_border_count",
    "ctr_target_border_type", "drop_rate", "drop_seed", "extra_seed", "fold_len_multiplier",
    "fold_permutation_block", "goss_seed", "goss_warmup_rounds", "linear_lambda", "max_bundle_bins",
    "max_bundle_size", "max_conflict_rate", "max_drop", "max_nondefault_rate", "min_reduction",
    "monotone_constraints_method", "mvs_reg", "one_hot_max_size", "ordered_seed", "other_rate",
    "permutation_count", "random_strength_seed", "random_strength_set", "skip_drop", "top_rate", "uniform_drop",
    "xgboost_dart_mode", "leaf_estimation_iterations_set", "auto_learning_rate_l2_set",
    "auto_learning_rate_leaf_iters_set", "auto_learning_rate_required", "device", "categorical_addr",
    "categorical_len", "categorical_features", "categorical_feature", "objective", "fair_c",
    "tweedie_variance_power",
}


def _f64(addr, n):
    buf = (ctypes.c_double * n).from_address(addr)
    return np.frombuffer(buf, dtype=np.float64, count=n)


def _same(value, default):
    if isinstance(default, str):
        return str(value).lower() == default
    try:
        return float(value) == float(default)
    except (TypeError, ValueError):
        return False


def param_string(objective, params):
    """The C ABI parameter string for the reference estimators' params dict.
    Every key is mapped, checked to be off, or known to be inert; an option
    the device path does not cover, or a key this mapping does not know, is
    refused by name."""
    if objective not in _OBJECTIVE_NAMES:
        raise NotImplementedError(f"objective code {objective} is not covered by the B200 device path")
    device = str(params.get("device", "gpu")).lower()
    if device == "cpu":
        raise NotImplementedError("device='cpu': the B200 library is the GPU path only")
    out = {"objective": _OBJECTIVE_NAMES[objective], "device": "gpu"}
    for k, v in params.items():
        if v is None:
            continue
        if k in _KEY_MAP:
            out[_KEY_MAP[k]] = v
        elif k in _MUST_BE:
            if not _same(v, _MUST_BE[k]):
                raise NotImplementedError(f"{k}={v!r} is not covered by the B200 device path")
        elif k not in _INERT:
            raise NotImplementedError(f"parameter {k!r} is not covered by the B200 device path")
    cats = params.get("categorical_features") or params.get("categorical_feature")
    if params.get("categorical_addr") and params.get("categorical_len"):
        cats = [int(c) for c in _f64(int(params["categorical_addr"]), int(params["categorical_len"]))]
    if cats:
        out["categorical_feature"] = ",".join(str(int(c)) for c in cats)
    return _capi.params_string(out)


def fit(x_addr, n_rows, n_features, y_addr, objective, params):
    """Train a single-output model (bindings/_mojotrees.mojo:2094)."""
    n_rows, n_features = int(n_rows), int(n_features)
    X = _f64(int(x_addr), n_rows * n_features)
    y = _f64(int(y_addr), n_rows)
    e = _capi._Err()
    h = ctypes.c_void_p()
    e.check(_capi.lib().mojotrees_train_dense(X.ctypes.data_as(ctypes.c_void_p), n_rows, n_features,
                                              y.ctypes.data_as(ctypes.c_void_p), None,
                                              param_string(int(objective), dict(params)), ctypes.byref(h), e.h))
    return _capi.Model(h.value)


def fit_multiclass(x_addr, n_rows, n_features, y_addr, n_classes, params):
    """Train a softmax model (the multiclass twin of `fit`)."""
    p = dict(params)
    p["num_class"] = int(n_classes)
    return fit(x_addr, n_rows, n_features, y_addr, MULTICLASS, p)


# ---- fits scored on validation sets (bindings/_mojotrees.mojo:2709-3060;
# the round loop and early stopping of custom_metric.mojo:1000-1290) --------

_METRIC_PARAM_KEYS = {"valid_sets", "n_valid", "metrics", "n_metrics", "primary_metric", "early_stopping_rounds",
                      "min_delta", "pred_addr", "reset_addr", "evals_addr", "callback", "has_callback"}


def _fit_scored(x_addr, n_rows, n_features, y_addr, objective, bridge, params):
    """Train on the device, then score the validation sets after every
    iteration on the host.  Training is deterministic and no round depends on
    a later one, so the first i iterations of the full fit are the model the
    reference's round loop holds after i trees; scoring them in order,
    stopping when any flagged (set, metric) pair has gone
    early_stopping_rounds rounds without a strict improvement beyond
    min_delta, and cutting to the primary metric's best round on the first
    set is the reference's metric fit.  Callbacks can change a round's
    hyperparameters and are not covered."""
    if int(params.get("has_callback", 0)):
        raise NotImplementedError("training callbacks are not covered by the B200 device path")
    esr = int(params.get("early_stopping_rounds", 0))
    min_delta = float(params.get("min_delta", 0.0))
    if esr < 0:
        raise ValueError("early_stopping_rounds must not be negative")
    if min_delta < 0.0:
        raise ValueError("min_delta must not be negative")
    metrics = [tuple(params["metrics"][m]) for m in range(int(params["n_metrics"]))]
    valid = [tuple(params["valid_sets"][v]) for v in range(int(params["n_valid"]))]
    primary = int(params.get("primary_metric", 0))
    if metrics and not 0 <= primary < len(metrics):
        raise ValueError("primary_metric out of range")
    train_params = {k: v for k, v in params.items() if k not in _METRIC_PARAM_KEYS}
    model = fit(x_addr, n_rows, n_features, y_addr, objective, train_params)
    K = model.num_classes
    n_features = int(n_features)
    pred = _f64(int(params["pred_addr"]), max([int(v[2]) for v in valid] + [0]) * K)
    bins, raws = [], []
    for name, vx, vn, vy in valid:
        vn = int(vn)
        X = _f64(int(vx), vn * n_features).reshape(n_features, vn).T  # column-major rows
        bins.append(model.bin_rows(X))
        raws.append(np.tile(model.base_scores(), vn))
    n_v, n_m = len(valid), len(metrics)
    values, best_value, best_round = [], [0.0] * (n_v * n_m), [0] * (n_v * n_m)

    def score(rnd):
        for v in range(n_v):
            pred[: raws[v].size] = raws[v]
            for m in range(n_m):
                value = float(bridge(m, v))
                if not np.isfinite(value):
                    raise ValueError(f"metric {metrics[m][0]} returned a non-finite value on validation set "
                                     f"{valid[v][0]} at round {rnd}")
                values.append(value)
                i = v * n_m + m
                if rnd == 0:
                    best_value[i], best_round[i] = value, 0
                elif (value > best_value[i] + min_delta) if int(metrics[m][1]) else \
                        (value < best_value[i] - min_delta):
                    best_value[i], best_round[i] = value, rnd

    score(0)
    stopped = False
    iters = model.num_iterations
    for it in range(iters):
        for v in range(n_v):
            model.add_iteration_raw(bins[v], it, raws[v])
        score(it + 1)
        if esr > 0 and any(int(metrics[i % n_m][2]) and (it + 1) - best_round[i] >= esr
                           for i in range(n_v * n_m)):
            stopped = True
            break
    best = best_round[primary] if n_m else 0
    best_score = best_value[primary] if n_m else 0.0
    if esr > 0 and best < iters:
        model = model.prefix(best)
    n_rounds = len(values) // (n_v * n_m) if n_v * n_m else 0
    return [model, values, n_rounds, best, best_score, int(stopped)]


def fit_with_metrics(x_addr, n_rows, n_features, y_addr, objective, bridge, params):
    return _fit_scored(x_addr, n_rows, n_features, y_addr, int(objective), bridge, dict(params))


def fit_multiclass_with_metrics(x_addr, n_rows, n_features, y_addr, n_classes, bridge, params):
    p = dict(params)
    p["num_class"] = int(n_classes)
    return _fit_scored(x_addr, n_rows, n_features, y_addr, MULTICLASS, bridge, p)


# ---- sparse input (bindings/_mojotrees.mojo:3335-3510) --------------------

_SPARSE_KEYS = {"sparse_data_addr", "sparse_indices_addr", "sparse_indptr_addr", "sparse_nnz", "n_rows",
                "n_features"}


def _i64(addr, n):
    if n == 0:
        return np.zeros(0, np.int64)
    buf = (ctypes.c_int64 * n).from_address(int(addr))
    return np.frombuffer(buf, dtype=np.int64, count=n)


def _densify(params, compressed_columns):
    """The dense float64 matrix [n_rows, n_features] (column-major) of a CSC
    (compressed_columns) or CSR matrix given by buffer addresses: absent
    entries are the value 0.0 and a stored NaN is missing, the semantics the
    reference's sparse path shares with its dense one (sparse.mojo:535-570:
    bit-identical bins to the densified matrix).  Needs n_rows x n_features
    x 8 bytes of host memory."""
    n, f, nnz = int(params["n_rows"]), int(params["n_features"]), int(params["sparse_nnz"])
    if n < 0 or f < 0 or nnz < 0:
        raise ValueError("sparse matrix: negative shape or nnz")
    n_major = f if compressed_columns else n
    n_minor = n if compressed_columns else f
    indptr = _i64(params["sparse_indptr_addr"], n_major + 1)
    indices = _i64(params["sparse_indices_addr"], nnz)
    data = _f64(int(params["sparse_data_addr"]), nnz) if nnz else np.zeros(0)
    if indptr[0] != 0 or indptr[-1] != nnz or np.any(np.diff(indptr) < 0):
        raise ValueError("sparse matrix: indptr is not a valid offset array")
    if nnz and (indices.min() < 0 or indices.max() >= n_minor):
        raise ValueError("sparse matrix: an index is out of range")
    major = np.repeat(np.arange(n_major), np.diff(indptr))
    if nnz > 1:
        same = major[1:] == major[:-1]
        if np.any(same & (indices[1:] <= indices[:-1])):
            raise ValueError("sparse matrix: indices must be strictly increasing within each "
                             + ("column" if compressed_columns else "row"))
    dense = np.zeros((n, f), order="F")
    if compressed_columns:
        dense[indices, major] = data
    else:
        dense[major, indices] = data
    return dense


def _dense_params(params):
    return {k: v for k, v in params.items() if k not in _SPARSE_KEYS}


def _csc_buffers(params):
    """The CSC matrix's (indptr, indices, data) at the given addresses."""
    f, nnz = int(params["n_features"]), int(params["sparse_nnz"])
    if f < 0 or nnz < 0:
        raise ValueError("sparse matrix: negative shape or nnz")
    indptr = _i64(params["sparse_indptr_addr"], f + 1)
    indices = _i64(params["sparse_indices_addr"], nnz)
    data = _f64(int(params["sparse_data_addr"]), nnz) if nnz else np.zeros(0)
    return indptr, indices, data


def fit_csc(y_addr, objective, params):
    """A fit on a CSC matrix (bindings/_mojotrees.mojo:3335): the compressed
    columns are binned as the densified matrix would be
    (mojotrees_b200_train_csc), so the host holds bins, not the dense
    float64 matrix, and the trees equal the dense fit's."""
    n = int(params["n_rows"])
    indptr, indices, data = _csc_buffers(params)
    y = _f64(int(y_addr), n)
    e = _capi._Err()
    h = ctypes.c_void_p()
    e.check(_capi.lib().mojotrees_b200_train_csc(
        indptr.ctypes.data_as(ctypes.c_void_p), indices.ctypes.data_as(ctypes.c_void_p),
        data.ctypes.data_as(ctypes.c_void_p), n, indptr.size - 1, y.ctypes.data_as(ctypes.c_void_p), None,
        param_string(int(objective), _dense_params(params)), ctypes.byref(h), e.h))
    return _capi.Model(h.value)


def fit_multiclass_csc(y_addr, n_classes, params):
    p = dict(params)
    p["num_class"] = int(n_classes)
    return fit_csc(y_addr, MULTICLASS, p)


def _predict_csr(model, params, out_addr, raw):
    device = str(params.get("device", "cpu")).lower()
    if device in ("gpu", "cuda"):
        # as the reference does (`_refuse_gpu_sparse`): sparse prediction
        # has no device walk, and densifying behind the caller is not done
        raise NotImplementedError("device='gpu' prediction of sparse input: the sparse walk runs on the host")
    X = _densify(params, False)
    n, f = X.shape
    return _predict_into(model, X.ctypes.data, n, f, {"device": "cpu", "start": 0, "stop": model.num_iterations,
                                                      "raw_score": int(raw)}, out_addr)


def predict_csr(model, params, out_addr):
    _predict_csr(model, params, out_addr, False)


def predict_raw_csr(model, params, out_addr):
    _predict_csr(model, params, out_addr, True)


def predict_proba_csr(model, params, out_addr):
    _predict_csr(model, params, out_addr, bool(int(params.get("raw_score", 0))))


# ---- the LightGBM-style Dataset / train API (python/mojotrees/basic.py over
# bindings/_mojotrees.mojo:4993-5310, dataset_bindings.mojo:263) ------------

class _Dataset:
    """A constructed training set: a copy of the column-major float64 matrix,
    the label and the binning parameters.  Binning itself happens in the
    device fit, from the same parameters, so the trees are those a fit of the
    matrix grows."""

    def __init__(self, X, label, max_bin, use_missing, categorical, names):
        self.X, self.label = X, label
        self.max_bin, self.use_missing = int(max_bin), int(use_missing)
        self.categorical, self.names = list(categorical), list(names)

    @property
    def n_rows(self):
        return self.X.shape[0]

    @property
    def n_features(self):
        return self.X.shape[1]


def dataset_create(x_addr, n_rows, n_features, params):
    n, f = int(n_rows), int(n_features)
    for key, what in (("weight_addr", "sample weights"), ("init_score_addr", "init scores"),
                      ("group_addr", "query groups")):
        if int(params.get(key, 0) or 0):
            raise NotImplementedError(f"a Dataset with {what} is not covered by the B200 device path")
    if str(params.get("ctr", "off")).lower() != "off":
        raise NotImplementedError("ctr: CatBoost target statistics are not covered by the B200 device path")
    X = _f64(int(x_addr), n * f).reshape(f, n).T.copy(order="F")  # column-major, owned
    label = _f64(int(params["label_addr"]), n).copy() if int(params.get("label_addr", 0) or 0) else None
    cats = []
    if params.get("categorical_addr") and params.get("categorical_len"):
        cats = [int(c) for c in _f64(int(params["categorical_addr"]), int(params["categorical_len"]))]
    names = [str(x) for x in (params.get("feature_names") or [])][: int(params.get("n_names", 0) or 0)]
    return _Dataset(X, label, params.get("max_bin", 255), params.get("use_missing", 1), cats, names)


def dataset_metadata(dataset):
    d = dataset
    return {"num_data": d.n_rows, "num_feature": d.n_features, "num_bin": d.max_bin, "max_bin": d.max_bin,
            "is_sparse": False, "nnz": d.n_rows * d.n_features, "has_raw": False, "use_missing": d.use_missing,
            "n_groups": 0, "n_categorical": len(d.categorical), "has_names": bool(d.names),
            "n_label": 0 if d.label is None else d.n_rows, "n_weight": 0, "n_init_score": 0}


def dataset_num_data(dataset):
    return dataset.n_rows


def dataset_num_feature(dataset):
    return dataset.n_features


def dataset_feature_names(dataset):
    return list(dataset.names)


def dataset_categorical_features(dataset):
    return list(dataset.categorical)


def _dataset_fit(dataset, params, multiclass):
    if dataset.label is None:
        raise ValueError("the Dataset has no label to train on")
    model = _dataset_fit_once(dataset, params, multiclass)
    # what booster_update needs to continue this fit exactly
    model._continue = (dataset, multiclass, _without_rounds(params))
    return model


def _without_rounds(params):
    return {k: v for k, v in params.items() if k != "n_estimators"}


def _dataset_fit_once(dataset, params, multiclass):
    p = dict(params)
    objective = int(p.pop("objective", 0))
    n_classes = int(p.pop("n_classes", 0) or 0)
    for k in ("categorical_addr", "categorical_len"):
        p.pop(k, None)
    p["max_bin"], p["use_missing"] = dataset.max_bin, dataset.use_missing
    if dataset.categorical:
        p["categorical_features"] = dataset.categorical
    X, y = dataset.X, np.ascontiguousarray(dataset.label)
    if multiclass:
        return fit_multiclass(X.ctypes.data, dataset.n_rows, dataset.n_features, y.ctypes.data, n_classes, p)
    return fit(X.ctypes.data, dataset.n_rows, dataset.n_features, y.ctypes.data, objective, p)


def _booster_update(model, dataset, params, multiclass):
    """Append params["n_estimators"] more rounds to a model trained on
    `dataset` through train_dataset, returning how many were added
    (bindings/_mojotrees.mojo:5406-5560).  The reference continues from the
    existing trees; training here is deterministic and no round depends on a
    later one, so a fresh fit of (current + n) rounds holds the same first
    rounds and is that continued model.  Exact only when nothing but the
    round count changed, so any other change is refused."""
    state = getattr(model, "_continue", None)
    if state is None or state[0] is not dataset or state[1] != multiclass:
        raise NotImplementedError("continued training needs a model trained on this Dataset through "
                                  "mojotrees.train() with the B200 library")
    if _without_rounds(params) != state[2]:
        raise NotImplementedError("continued training with changed parameters is not covered by the B200 "
                                  "device path (only the round count may change)")
    before = model.num_iterations
    grown = _dataset_fit_once(dataset, dict(params, n_estimators=before + int(params["n_estimators"])),
                              multiclass)
    model.h, grown.h = grown.h, model.h  # the booster's handle now holds the longer model
    return model.num_iterations - before


def booster_update(model, dataset, params):
    return _booster_update(model, dataset, params, False)


def booster_update_multiclass(model, dataset, params):
    return _booster_update(model, dataset, params, True)


# ---- built-in metrics (bindings/_mojotrees.mojo:3168-3270, metrics.mojo) ----

def _seq_sum(terms):
    """Left-to-right double sum, the reference metrics' accumulation order."""
    return float(np.cumsum(terms)[-1]) if len(terms) else 0.0


def _metric_weight(weight, n):
    """check_metric_weight (metrics.mojo:112-130): the weight total."""
    if weight is None:
        return float(n)
    if not np.all(np.isfinite(weight)) or np.any(weight < 0.0):
        raise ValueError("weights must be finite and nonnegative")
    total = _seq_sum(weight)
    if total <= 0.0:
        raise ValueError("weights must have a positive sum")
    return total


def _sigmoid(x):
    """boosting.mojo:261-268, the sign-split logistic."""
    out = np.empty_like(x)
    pos = x >= 0.0
    out[pos] = 1.0 / (1.0 + np.exp(-x[pos]))
    e = np.exp(x[~pos])
    out[~pos] = e / (1.0 + e)
    return out


def _clamp(p):
    return np.minimum(np.maximum(p, 1e-15), 1.0 - 1e-15)


def eval_metric(code, params):
    """One built-in metric over the caller's raw predictions, after the
    objective's link (bindings/_mojotrees.mojo:3168): l2, rmse, l1,
    binary_logloss, binary_error, auc, multi_logloss and multi_error, the
    metrics of the objectives this library trains.  Sums run left to right
    as metrics.mojo's loops do; log and exp are the platform's."""
    code = int(code)
    n = int(params["n_rows"])
    if n <= 0:
        raise ValueError("metrics need at least one row")
    w_addr = int(params.get("weight_addr", 0) or 0)
    weight = _f64(w_addr, n).copy() if w_addr else None
    total_w = _metric_weight(weight, n)
    w = np.ones(n) if weight is None else weight
    y = _f64(int(params["y_addr"]), n).copy()
    if code in (8, 9):  # multi_logloss, multi_error
        k = int(params["n_classes"])
        raw = _f64(int(params["pred_addr"]), n * k).reshape(n, k).copy()
        labels = y.astype(np.int64)
        if np.any(labels < 0) or np.any(labels >= k):
            raise ValueError("label out of range")
        # _softmax_inplace (boosting.mojo:3515): max, exp, sequential total
        e = np.exp(raw - raw.max(axis=1, keepdims=True))
        tot = np.cumsum(e, axis=1)[:, -1:]
        prob = e / tot
        if code == 8:
            return _seq_sum(-(w * np.log(_clamp(prob[np.arange(n), labels])))) / total_w
        correct = np.where(np.argmax(prob, axis=1) == labels, w, 0.0)
        return 1.0 - _seq_sum(correct) / total_w
    raw = _f64(int(params["pred_addr"]), n).copy()
    objective = int(params.get("objective", 0))
    pred = _sigmoid(raw) if objective == BINARY_LOGISTIC else raw  # response_scale
    if code in (0, 1):  # l2, rmse
        d = pred - y
        v = _seq_sum((w * d) * d) / total_w
        return float(np.sqrt(v)) if code == 1 else v
    if code == 2:  # l1
        return _seq_sum(w * np.abs(pred - y)) / total_w
    if code == 5:  # binary_logloss
        p = _clamp(pred)
        return _seq_sum(-(w * np.where(y > 0.5, np.log(p), np.log(1.0 - p)))) / total_w
    if code == 6:  # binary_error: 1 - accuracy at threshold 0.5
        predicted = np.where(pred >= 0.5, 1.0, 0.0)
        return 1.0 - _seq_sum(np.where(np.abs(predicted - y) < 0.5, w, 0.0)) / total_w
    if code == 7:  # auc (metrics.mojo binary_auc): stable ascending order, tie blocks
        pos = y > 0.5
        w_pos, w_neg = _seq_sum(np.where(pos, w, 0.0)), _seq_sum(np.where(pos, 0.0, w))
        if w_pos <= 0.0 or w_neg <= 0.0:
            raise ValueError("AUC needs at least one positive and one negative")
        order = np.argsort(pred, kind="stable")
        seen_neg, total, i = 0.0, 0.0, 0
        while i < n:
            j = i
            while j + 1 < n and pred[order[j + 1]] == pred[order[i]]:
                j += 1
            block_pos = block_neg = 0.0
            for t in range(i, j + 1):
                if pos[order[t]]:
                    block_pos += w[order[t]]
                else:
                    block_neg += w[order[t]]
            total += block_pos * (seen_neg + 0.5 * block_neg)
            seen_neg += block_neg
            i = j + 1
        return total / (w_pos * w_neg)
    raise NotImplementedError(f"metric code {code} is not covered by the B200 library's metrics")


def train_dataset(dataset, params):
    """A single-output fit on a constructed Dataset (bindings/_mojotrees.mojo:5122)."""
    return _dataset_fit(dataset, params, False)


def train_dataset_multiclass(dataset, params):
    return _dataset_fit(dataset, params, True)


def resolve_device(device, n_rows=0, n_features=0, n_outputs=1):
    """`gpu` when a CUDA device is present; an explicit `gpu` request without
    one raises instead of falling back (capi/mojotrees.h:99-106)."""
    d = str(device).lower()
    if d in ("gpu", "cuda", "auto"):
        if _capi.gpu_available():
            return "gpu"
        raise RuntimeError(f"device='{device}': no CUDA device is available and this library has no CPU path")
    raise NotImplementedError("device='cpu': the B200 library is the GPU path only")


def gpu_available():
    return bool(_capi.gpu_available())


# ---- prediction (bindings/_mojotrees.mojo:4223-4296) ----------------------

_DEVICES = {"cpu": _capi.DEVICE_CPU, "gpu": _capi.DEVICE_GPU, "cuda": _capi.DEVICE_GPU, "auto": _capi.DEVICE_AUTO}


def _predict_into(model, x_addr, n_rows, n_features, params, out_addr):
    """Predictions of a column-major float64 batch over the half-open
    iteration range [start, stop) (clamped to the ensemble), written to the
    float64 buffer at out_addr ([r * n_classes + k]).  Returns the backend
    that ran, or None for an empty batch."""
    n_rows, n_features = int(n_rows), int(n_features)
    if n_rows == 0:
        return None
    device = str(params.get("device", "cpu")).lower()
    if device not in _DEVICES:
        raise ValueError(f"unknown device {device!r}")
    k = model.num_classes
    iters = model.num_iterations
    start = min(max(int(params.get("start", 0)), 0), iters)
    stop = params.get("stop", iters)
    stop = iters if stop is None or int(stop) < 0 else min(int(stop), iters)
    raw = int(params.get("raw_score", 0)) != 0
    out = _f64(int(out_addr), n_rows * k)
    if stop <= start:
        # an empty range scores no tree: from iteration 0 that is the base
        # scores, answered by the C predictor on a zero-iteration copy (so
        # the response is its arithmetic); from a later start, raw scores of
        # zero, whose responses are exact (sigmoid 0.5, softmax 1/K)
        if start == 0:
            X = _f64(int(x_addr), n_rows * n_features).reshape(n_features, n_rows).T
            out[:] = model.prefix(0).predict(X, raw_score=raw).reshape(-1)
        elif raw or model.objective_name == "regression":
            out[:] = 0.0
        else:
            out[:] = 0.5 if k == 1 else 1.0 / k
        return "cpu" if _DEVICES[device] != _capi.DEVICE_GPU else "gpu"
    X = _f64(int(x_addr), n_rows * n_features)
    e = _capi._Err()
    e.check(_capi.lib().mojotrees_predict_ex(model.h, X.ctypes.data_as(ctypes.c_void_p), n_rows, n_features, start,
                                             stop - start, _capi.PREDICT_RAW if raw else _capi.PREDICT_RESPONSE,
                                             _DEVICES[device], out.ctypes.data_as(ctypes.c_void_p), out.size, e.h))
    return "gpu" if _DEVICES[device] == _capi.DEVICE_GPU else "cpu"


def predict_leaf(model, x_addr, n_rows, n_features, start, stop, out_addr):
    """Per-tree leaf ordinals over [start, stop), row-major and round-major
    within a row (bindings/_mojotrees.mojo:3960-4010), on the host."""
    n_rows, n_features = int(n_rows), int(n_features)
    iters = model.num_iterations
    start = min(max(int(start), 0), iters)
    stop = iters if stop is None or int(stop) < 0 else min(int(stop), iters)
    if n_rows == 0 or stop <= start:
        return None
    cols = (stop - start) * model.num_classes
    X = _f64(int(x_addr), n_rows * n_features)
    out = _f64(int(out_addr), n_rows * cols)
    e = _capi._Err()
    e.check(_capi.lib().mojotrees_b200_predict_leaf(model.h, X.ctypes.data_as(ctypes.c_void_p), n_rows, n_features,
                                                    start, stop - start, out.ctypes.data_as(ctypes.c_void_p),
                                                    out.size, e.h))
    return None


predict_leaf_multiclass = predict_leaf


def predict_leaf_batch(model, x_addr, n_rows, n_features, params, out_addr):
    """Leaf ordinals for a batch; the walk runs on the host, so an explicit
    device request is refused rather than answered from the host."""
    device = str(params.get("device", "cpu")).lower()
    if device in ("gpu", "cuda"):
        raise NotImplementedError("leaf prediction runs on the host in the B200 library")
    if int(n_rows) == 0:
        return None
    predict_leaf(model, x_addr, n_rows, n_features, params.get("start", 0), params.get("stop", -1), out_addr)
    return "cpu"


predict_leaf_multiclass_batch = predict_leaf_batch


def predict_batch(model, x_addr, n_rows, n_features, params, out_addr):
    """Single-output predictions (response, or raw with params["raw_score"])."""
    return _predict_into(model, x_addr, n_rows, n_features, params, out_addr)


def predict_proba_batch(model, x_addr, n_rows, n_features, params, out_addr):
    """Multiclass probabilities (or per-class raw scores), row-major."""
    return _predict_into(model, x_addr, n_rows, n_features, params, out_addr)


# ---- model accessors -------------------------------------------------------

def n_features(model):
    return model.num_features


def n_classes(model):
    return model.num_classes


def num_iterations(model):
    return model.num_iterations


def num_trees(model):
    return model.num_trees


n_features_multiclass = n_features
num_iterations_multiclass = num_iterations
num_trees_multiclass = num_trees


def feature_importance(model, n_features, kind, out_addr):
    """Split-count (kind 0) or total-gain (kind 1) importance into the float64
    buffer at out_addr (bindings/_mojotrees.mojo:4881)."""
    vals = model.feature_importance("gain" if int(kind) == 1 else "split")
    _f64(int(out_addr), int(n_features))[:] = vals[: int(n_features)]
    return None


feature_importance_multiclass = feature_importance


def categorical_features(model):
    """Indices of the features the model splits by category set
    (bindings/_mojotrees.mojo:4802)."""
    return model.categorical_features()


categorical_features_multiclass = categorical_features


def extra_params_check(params, shape):
    """The extra tree options (min_gain_to_split, max_delta_step, path_smooth,
    extra_trees, monotone penalty, CEGB, forced splits): the device path
    implements none of them, so any value other than "off" is refused; with
    all of them off nothing is active (bindings/basic_bindings.mojo:268)."""
    for k in ("min_gain_to_split", "max_delta_step", "path_smooth", "extra_trees", "monotone_penalty",
              "cegb_tradeoff", "cegb_penalty_split", "forced_splits", "feature_contri_addr",
              "cegb_penalty_feature_coupled_addr", "cegb_penalty_feature_lazy_addr"):
        if k in params and params[k] is not None and not _same(params[k], _MUST_BE[k]):
            raise NotImplementedError(f"{k}={params[k]!r} is not covered by the B200 device path")
    return {"is_active": False, "needs_leaf_finish": False, "needs_node_identity": False,
            "needs_grower_support": False}


def efb_check(params, cpu=0):
    """Exclusive feature bundling is not part of the device path."""
    if params.get("enable_bundle") and not _same(params["enable_bundle"], 0):
        raise NotImplementedError("enable_bundle: exclusive feature bundling is not covered by the B200 device path")
    return None


def extra_option_supported(name):
    """Every other LightGBM option name: not this function's to refuse."""
    return None


def efb_defaults():
    """Exclusive-feature-bundling knob defaults (EfbParams.default,
    efb.mojo:373).  Bundling itself is not part of the device path."""
    return {"max_conflict_rate": 0.0, "max_bundle_bins": 256, "max_bundle_size": 0,
            "max_nondefault_rate": 0.95, "min_reduction": 0.0, "bundle_missing": False}


# ---- host ingestion (bindings/_mojotrees.mojo:682-739) ---------------------

def ingest_column_major(src_addr, dst_addr, n_rows, n_features):
    """Row-major float64 at src_addr into the column-major buffer at
    dst_addr, on all host threads; 1 when any value is +inf or -inf."""
    found = ctypes.c_int32(0)
    e = _capi._Err()
    e.check(_capi.lib().mojotrees_b200_ingest_column_major(ctypes.c_void_p(int(src_addr)), ctypes.c_void_p(int(dst_addr)),
                                                           int(n_rows), int(n_features), ctypes.byref(found), e.h))
    return int(found.value)


def buffer_has_infinite(addr, n):
    """1 when the float64 buffer at addr holds +inf or -inf."""
    found = ctypes.c_int32(0)
    e = _capi._Err()
    e.check(_capi.lib().mojotrees_b200_buffer_has_infinite(ctypes.c_void_p(int(addr)), int(n), ctypes.byref(found),
                                                           e.h))
    return int(found.value)


# ---- model files (src/mojotrees/serialize.mojo) ----------------------------

_ESC = {" ": "\\s", "\t": "\\t", "\n": "\\n", "\r": "\\r", "\\": "\\\\"}
_UNESC = {"s": " ", "t": "\t", "n": "\n", "r": "\r", "\\": "\\"}


def _escape_name(name):
    """serialize.mojo:276-318: one whitespace-free token per name."""
    if name == "":
        return "\\e"
    out = []
    for ch in name:
        if ch in _ESC:
            out.append(_ESC[ch])
        elif ord(ch) < 32 or ord(ch) == 127:
            raise ValueError(f"feature name contains control byte {ord(ch)}, which the model file format cannot carry")
        else:
            out.append(ch)
    return "".join(out)


def _unescape_name(token):
    """serialize.mojo:321-355, the inverse of _escape_name."""
    if token == "\\e":
        return ""
    out, i = [], 0
    while i < len(token):
        if token[i] != "\\":
            out.append(token[i])
            i += 1
            continue
        if i + 1 >= len(token) or token[i + 1] not in _UNESC:
            raise ValueError("corrupt feature name escape")
        out.append(_UNESC[token[i + 1]])
        i += 2
    return "".join(out)


def save(model, path, names=(), n_names=None):
    """Format v4 through mojotrees_save_model, with the optional
    feature_names section (serialize.mojo:389-398) when names are given."""
    names = [str(n) for n in (names or [])]
    if names and len(names) != model.num_features:
        raise ValueError(f"{len(names)} feature names for {model.num_features} features")
    model.save(str(path))
    if names:
        with open(path) as f:
            head, rest = f.read().split("\n", 1)
        section = f"feature_names {len(names)}\n" + "".join(_escape_name(n) + " " for n in names) + "\n"
        with open(path, "w") as f:
            f.write(head + "\n" + section + rest)


save_multiclass = save


def load(path):
    return _capi.Model.load(str(path))


load_multiclass = load


def model_file_kind(path):
    """Which loader a saved model needs, "objective" or "multiclass", from
    the file header (serialize.mojo:1408-1428)."""
    with open(path) as f:
        tok = f.read(1 << 20).split()
    if tok and tok[0] == "mojotrees-dataset":
        raise ValueError("this is a prepared dataset file, not a model; read it with load_dataset")
    if len(tok) < 2 or tok[0] != "mojotrees" or tok[1] not in ("v1", "v2", "v3", "v4", "v5"):
        raise ValueError("not a mojotrees model file")
    i = 2
    if i < len(tok) and tok[i] == "feature_names":
        i += 2 + int(tok[i + 1])
    kind = tok[i] if i < len(tok) else ""
    if kind not in ("objective", "multiclass"):
        raise ValueError("corrupt model file: unknown model kind")
    return kind


def file_kind(path):
    with open(path) as f:
        head = f.read(64).split()
    if head and head[0] == "mojotrees-dataset":
        return "dataset"
    return model_file_kind(path)


def model_feature_names(path):
    """The names a model file carries (serialize.mojo:1448), or []."""
    with open(path) as f:
        tok = f.read().split()
    if len(tok) < 4 or tok[2] != "feature_names":
        return []
    n = int(tok[3])
    return [_unescape_name(t) for t in tok[4:4 + n]]


class HookNotProvided(AttributeError, NotImplementedError):
    """An extension hook this library does not provide.  An AttributeError,
    so the estimators' optional-hook probes (getattr(_mojotrees, name, None))
    fall back, and a NotImplementedError for direct calls."""


def __getattr__(name):
    raise HookNotProvided(f"_mojotrees.{name} is not provided by the B200 training library")
