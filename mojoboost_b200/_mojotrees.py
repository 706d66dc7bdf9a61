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

# objective codes of the reference package (python/mojotrees/sklearn.py:33-55)
SQUARED_ERROR = 0
BINARY_LOGISTIC = 1
MULTICLASS = -1
_OBJECTIVE_NAMES = {SQUARED_ERROR: "regression", BINARY_LOGISTIC: "binary", MULTICLASS: "multiclass"}

# reference params-dict keys -> parameter-string keys of the C ABI
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
# keys whose value must stay at the default for the device path
_MUST_BE = {"bagging_fraction": 1.0, "bagging_freq": 0, "max_depth": -1, "goss": 0, "linear_tree": 0,
            "ordered": 0, "feature_fraction_bynode": 1.0}


def _f64(addr, n):
    buf = (ctypes.c_double * n).from_address(addr)
    return np.frombuffer(buf, dtype=np.float64, count=n)


def param_string(objective, params):
    if objective not in _OBJECTIVE_NAMES:
        raise NotImplementedError(f"objective code {objective} is not covered by the B200 device path")
    device = str(params.get("device", "gpu")).lower()
    if device == "cpu":
        raise NotImplementedError("device='cpu': the B200 library is the GPU path only")
    out = {"objective": _OBJECTIVE_NAMES[objective], "device": "gpu"}
    for k, v in params.items():
        if k in _KEY_MAP and v is not None:
            out[_KEY_MAP[k]] = v
        elif k in _MUST_BE and v is not None and float(v) != float(_MUST_BE[k]):
            raise NotImplementedError(f"{k}={v} is not covered by the B200 device path")
    cats = params.get("categorical_features") or params.get("categorical_feature")
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


def resolve_device(device, n_rows=0, n_features=0, n_outputs=1):
    """`gpu` when a CUDA device is present; an explicit `gpu` request without
    one raises instead of falling back (capi/mojotrees.h:99-106)."""
    d = str(device).lower()
    if d in ("gpu", "cuda", "auto"):
        if _capi.gpu_available():
            return "gpu"
        raise RuntimeError(f"device='{device}': no CUDA device is available and this library has no CPU path")
    raise NotImplementedError("device='cpu': the B200 library is the GPU path only")


def __getattr__(name):
    raise NotImplementedError(f"_mojotrees.{name} is not provided by the B200 training library")
