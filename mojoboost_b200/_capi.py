"""ctypes binding of libmojotrees_b200.so (the C ABI in include/mojotrees.h).

The library is built in-tree (``make -C mojoboost_b200``).  Loading fails
loudly when it is missing: there is no Python or CPU fallback for training.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmojotrees_b200.so")

OK = 0
ERROR_INVALID_ARGUMENT = -1
ERROR_TRAINING = -2
ERROR_IO = -3
ERROR_UNSUPPORTED = -4

DEVICE_CPU, DEVICE_GPU, DEVICE_AUTO = 0, 1, 2
PREDICT_RESPONSE, PREDICT_RAW = 0, 1
IMPORTANCE_SPLIT, IMPORTANCE_GAIN = 0, 1

STAT_NAMES = ("fit_seconds", "upload_seconds", "hist_ms", "partition_ms", "scan_ms", "grad_ms",
              "hist_rows", "hist_bytes", "hist_launches", "kernel_launches", "rounds",
              "commit_ms", "iterations", "expansions", "binning_seconds", "pick_steps", "hist_sparse_entries")

# Every symbol include/mojotrees.h declares, with its ctypes signature.
_P, _I32, _I64, _D = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_double
SIGNATURES = {
    "mojotrees_abi_version": (_I32, []),
    "mojotrees_library_version": (None, [_P, _P, _P]),
    "mojotrees_gpu_available": (_I32, []),
    "mojotrees_error_create": (_P, []),
    "mojotrees_error_free": (None, [_P]),
    "mojotrees_error_message": (ctypes.c_char_p, [_P]),
    "mojotrees_train_dense": (_I32, [_P, _I64, _I64, _P, _P, ctypes.c_char_p, _P, _P]),
    "mojotrees_predict": (_I32, [_P, _P, _I64, _I64, _P, _I64, _P]),
    "mojotrees_predict_raw": (_I32, [_P, _P, _I64, _I64, _P, _I64, _P]),
    "mojotrees_predict_ex": (_I32, [_P, _P, _I64, _I64, _I64, _I64, _I32, _I32, _P, _I64, _P]),
    "mojotrees_save_model": (_I32, [_P, ctypes.c_char_p, _P]),
    "mojotrees_load_model": (_I32, [ctypes.c_char_p, _P, _P]),
    "mojotrees_model_num_features": (_I32, [_P, _P, _P]),
    "mojotrees_model_num_classes": (_I32, [_P, _P, _P]),
    "mojotrees_model_num_trees": (_I32, [_P, _P, _P]),
    "mojotrees_model_num_iterations": (_I32, [_P, _P, _P]),
    "mojotrees_model_dump_json": (_I32, [_P, _P, _P]),
    "mojotrees_feature_importance": (_I32, [_P, _I32, _P, _I64, _P]),
    "mojotrees_parameter_keys": (_I32, [_P, _P]),
    "mojotrees_string_free": (None, [_P]),
    "mojotrees_model_free": (None, [_P]),
    "mojotrees_b200_train_binned_u8": (_I32, [_P, _I64, _I64, _I32, _P, _P, _P, _P, ctypes.c_char_p, _P, _P]),
    "mojotrees_b200_bin_dense": (_I32, [_P, _I64, _I64, ctypes.c_char_p, _P, _P, _P, _P, _P]),
    "mojotrees_b200_bin_dense_gpu": (_I32, [_P, _I64, _I64, ctypes.c_char_p, _P, _P, _P, _P, _P]),
    "mojotrees_b200_shared_atomic_peak": (_I32, [_P, _P]),
    "mojotrees_b200_check_quotients": (_I32, [_I64, ctypes.c_uint64, _P, _P]),
    "mojotrees_b200_train_csc": (_I32, [_P, _P, _P, _I64, _I64, _P, _P, ctypes.c_char_p, _P, _P]),
    "mojotrees_b200_bin_csc": (_I32, [_P, _P, _P, _I64, _I64, ctypes.c_char_p, _P, _P, _P, _P, _P]),
    "mojotrees_b200_predict_binned_u8": (_I32, [_P, _P, _I64, _I64, _P, _I64, _P]),
    "mojotrees_b200_tree_nodes": (_I32, [_P, _I64, _P, _P, _P, _P, _I64, _P, _P]),
    "mojotrees_b200_base_scores": (_I32, [_P, _P, _I64, _P]),
    "mojotrees_b200_training_scores": (_I32, [_P, _P, _I64, _P]),
    "mojotrees_b200_train_stats": (_I32, [_P, _P, _I64, _P, _P]),
    "mojotrees_b200_round_times": (_I32, [_P, _P, _I64, _P, _P]),
    "mojotrees_b200_round_stats": (_I32, [_P, _P, _I64, _P, _P]),
    "mojotrees_b200_model_categorical": (_I32, [_P, _P, _I64, _P]),
    "mojotrees_b200_ingest_column_major": (_I32, [_P, _P, _I64, _I64, _P, _P]),
    "mojotrees_b200_buffer_has_infinite": (_I32, [_P, _I64, _P, _P]),
    "mojotrees_b200_predict_leaf": (_I32, [_P, _P, _I64, _I64, _I64, _I64, _P, _I64, _P]),
    "mojotrees_b200_model_bin": (_I32, [_P, _P, _I64, _I64, _P, _I64, _P]),
    "mojotrees_b200_add_iteration_raw": (_I32, [_P, _P, _I64, _I64, _I64, _P, _I64, _P]),
    "mojotrees_b200_model_prefix": (_I32, [_P, _I64, _P, _P]),
    "mojotrees_b200_nccl_unique_id": (_I32, [_P, _P]),
    "mojotrees_b200_histogram_u8": (_I32, [_P, _I64, _I64, _I32, _P, _I64, _P, _P, _I32, _P, _P]),
    "mojotrees_b200_histogram_u8_noalloc": (_I32, [_P, _I64, _I64, _I32, _P, _I64, _P, _I32, _P, _P, _P]),
    "mojotrees_b200_train_binned_u8_dp": (_I32, [_P, _I64, _I64, _I32, _P, _P, _P, _P, ctypes.c_char_p, _P, _I32,
                                                 _I32, _I64, _I64, _P, _P]),
}

_lib = None


class MojoTreesError(RuntimeError):
    """A failed C ABI call: `code` is the negative status, `args[0]` the reason."""

    def __init__(self, code, message):
        super().__init__(message)
        self.code = code


class UnsupportedError(MojoTreesError, NotImplementedError):
    pass


def lib():
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `make -C {HERE}` (nvcc, sm_100a). "
                "This package has no CPU or Python training fallback.")
        lb = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lb, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lb
    return _lib


class _Err:
    def __init__(self):
        self.h = lib().mojotrees_error_create()

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.mojotrees_error_free(self.h)
            self.h = None

    def check(self, rc):
        if rc != OK:
            msg = lib().mojotrees_error_message(self.h).decode()
            cls = UnsupportedError if rc == ERROR_UNSUPPORTED else MojoTreesError
            raise cls(rc, msg)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def params_string(params):
    if params is None:
        return b""
    if isinstance(params, (bytes, str)):
        return params.encode() if isinstance(params, str) else params
    parts = []
    for k, v in params.items():
        if isinstance(v, bool):
            v = "true" if v else "false"
        elif isinstance(v, (list, tuple)):
            v = ",".join(str(x) for x in v)
        parts.append(f"{k}={v}")
    return " ".join(parts).encode()


class Model:
    """A trained model handle (immutable)."""

    def __init__(self, handle):
        self.h = handle

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.mojotrees_model_free(self.h)
            self.h = None

    def _int(self, fn):
        e = _Err()
        v = ctypes.c_int64(0)
        e.check(getattr(lib(), fn)(self.h, ctypes.byref(v), e.h))
        return v.value

    @property
    def num_features(self):
        return self._int("mojotrees_model_num_features")

    @property
    def num_classes(self):
        return self._int("mojotrees_model_num_classes")

    @property
    def num_trees(self):
        return self._int("mojotrees_model_num_trees")

    @property
    def num_iterations(self):
        return self._int("mojotrees_model_num_iterations")

    def predict(self, X, raw_score=False, start_iteration=0, num_iteration=0, device="cpu"):
        """X: float64 array [n_rows, n_features] (any layout).  device "gpu"
        bins the rows and walks the trees on the current CUDA device (the
        same bits as "cpu"); there is no fallback between the two."""
        dev = {"cpu": DEVICE_CPU, "gpu": DEVICE_GPU, "auto": DEVICE_AUTO}[device]
        X = np.asarray(X, dtype=np.float64)
        n, f = X.shape
        Xc = np.asfortranarray(X)  # column-major: data[f * n + r]
        k = self.num_classes
        out = np.empty(n * k, np.float64)
        e = _Err()
        e.check(lib().mojotrees_predict_ex(self.h, Xc.ctypes.data_as(ctypes.c_void_p), n, f, start_iteration,
                                           num_iteration, PREDICT_RAW if raw_score else PREDICT_RESPONSE,
                                           dev, _ptr(out), out.size, e.h))
        return out.reshape(n, k) if k > 1 else out

    def predict_binned(self, bins_fm):
        """Raw scores for feature-major uint8 bins [n_features, n_rows]."""
        bins_fm = np.ascontiguousarray(bins_fm, dtype=np.uint8)
        f, n = bins_fm.shape
        k = self.num_classes
        out = np.empty(n * k, np.float64)
        e = _Err()
        e.check(lib().mojotrees_b200_predict_binned_u8(self.h, _ptr(bins_fm), n, f, _ptr(out), out.size, e.h))
        return out.reshape(n, k) if k > 1 else out

    def tree(self, t):
        """Node table of tree t as a dict of numpy arrays."""
        e = _Err()
        nn = ctypes.c_int64(0)
        rc = lib().mojotrees_b200_tree_nodes(self.h, t, None, None, None, None, 0, ctypes.byref(nn), e.h)
        n = nn.value
        ints = np.zeros((n, 7), np.int32)
        dbl = np.zeros((n, 2), np.float64)
        cnt = np.zeros(n, np.int64)
        bits = np.zeros((n, 4), np.uint64)
        e.check(lib().mojotrees_b200_tree_nodes(self.h, t, _ptr(ints), _ptr(dbl), _ptr(cnt), _ptr(bits), n,
                                                ctypes.byref(nn), e.h))
        return {"feature": ints[:, 0], "threshold_bin": ints[:, 1], "left": ints[:, 2], "right": ints[:, 3],
                "default_left": ints[:, 4], "missing_bin": ints[:, 5], "is_categorical": ints[:, 6],
                "value": dbl[:, 0], "gain": dbl[:, 1], "count": cnt, "cat_bits": bits}

    def base_scores(self):
        out = np.zeros(self.num_classes, np.float64)
        e = _Err()
        e.check(lib().mojotrees_b200_base_scores(self.h, _ptr(out), out.size, e.h))
        return out

    def training_scores(self, n_rows):
        out = np.zeros(n_rows * self.num_classes, np.float64)
        e = _Err()
        e.check(lib().mojotrees_b200_training_scores(self.h, _ptr(out), out.size, e.h))
        return out

    def stats(self):
        out = np.zeros(len(STAT_NAMES), np.float64)
        n = ctypes.c_int64(0)
        e = _Err()
        e.check(lib().mojotrees_b200_train_stats(self.h, _ptr(out), out.size, ctypes.byref(n), e.h))
        return dict(zip(STAT_NAMES, out[: n.value].tolist()))

    def round_stats(self):
        """Per round: (device ms, histogram ms, histogram launches, histogram rows, kernel launches)."""
        n = ctypes.c_int64(0)
        e = _Err()
        e.check(lib().mojotrees_b200_round_stats(self.h, None, 0, ctypes.byref(n), e.h))
        out = np.zeros((n.value, 5), np.float64)
        e.check(lib().mojotrees_b200_round_stats(self.h, _ptr(out), out.size, ctypes.byref(n), e.h))
        return out

    def round_times_ms(self):
        n = ctypes.c_int64(0)
        e = _Err()
        e.check(lib().mojotrees_b200_round_times(self.h, None, 0, ctypes.byref(n), e.h))
        out = np.zeros(n.value, np.float64)
        e.check(lib().mojotrees_b200_round_times(self.h, _ptr(out), out.size, ctypes.byref(n), e.h))
        return out

    def feature_importance(self, importance_type="split"):
        out = np.zeros(self.num_features, np.float64)
        e = _Err()
        t = IMPORTANCE_GAIN if importance_type == "gain" else IMPORTANCE_SPLIT
        e.check(lib().mojotrees_feature_importance(self.h, t, _ptr(out), out.size, e.h))
        return out

    def bin_rows(self, X):
        """Feature-major uint8 bins [n_features, n_rows] of float64 rows,
        with this model's mapper."""
        X = np.asfortranarray(np.asarray(X, dtype=np.float64))
        n, f = X.shape
        out = np.empty((f, n), np.uint8)
        e = _Err()
        e.check(lib().mojotrees_b200_model_bin(self.h, X.ctypes.data_as(ctypes.c_void_p), n, f, _ptr(out), out.size,
                                               e.h))
        return out

    def add_iteration_raw(self, bins_fm, iteration, raw):
        """raw (float64 [n_rows * num_classes]) += iteration's trees, in
        place, with the predictor's fused multiply-add."""
        f, n = bins_fm.shape
        e = _Err()
        e.check(lib().mojotrees_b200_add_iteration_raw(self.h, _ptr(bins_fm), n, f, int(iteration), _ptr(raw),
                                                       raw.size, e.h))

    def prefix(self, n_iterations):
        """A new model with the first n_iterations iterations."""
        e = _Err()
        h = ctypes.c_void_p()
        e.check(lib().mojotrees_b200_model_prefix(self.h, int(n_iterations), ctypes.byref(h), e.h))
        return Model(h.value)

    def categorical_features(self):
        """Indices of the features the model splits by category set."""
        out = np.zeros(self.num_features, np.int32)
        e = _Err()
        e.check(lib().mojotrees_b200_model_categorical(self.h, _ptr(out), out.size, e.h))
        return [int(i) for i in np.flatnonzero(out)]

    @property
    def objective_name(self):
        """'regression', 'binary' or 'multiclass'."""
        import json
        code = json.loads(self.dump_json())["objective_code"]
        return "multiclass" if code is None else {0: "regression", 1: "binary"}[int(code)]

    def dump_json(self):
        e = _Err()
        p = ctypes.c_void_p()
        e.check(lib().mojotrees_model_dump_json(self.h, ctypes.byref(p), e.h))
        try:
            return ctypes.string_at(p.value).decode()
        finally:
            lib().mojotrees_string_free(p)

    def save(self, path):
        e = _Err()
        e.check(lib().mojotrees_save_model(self.h, path.encode(), e.h))

    @staticmethod
    def load(path):
        e = _Err()
        h = ctypes.c_void_p()
        e.check(lib().mojotrees_load_model(path.encode(), ctypes.byref(h), e.h))
        return Model(h.value)


def train_dense(X, y, params=None, weights=None):
    """Train on a float64 matrix [n_rows, n_features] through mojotrees_train_dense."""
    X = np.asarray(X, dtype=np.float64)
    n, f = X.shape
    Xc = np.asfortranarray(X)
    y = np.ascontiguousarray(y, dtype=np.float64)
    w = None if weights is None else np.ascontiguousarray(weights, dtype=np.float64)
    e = _Err()
    h = ctypes.c_void_p()
    e.check(lib().mojotrees_train_dense(Xc.ctypes.data_as(ctypes.c_void_p), n, f, _ptr(y), _ptr(w),
                                        params_string(params), ctypes.byref(h), e.h))
    return Model(h.value)


def train_binned(bins_fm, n_bins, y, params=None, missing_bin=None, n_categories=None):
    """Train on feature-major uint8 bins [n_features, n_rows]."""
    bins_fm = np.ascontiguousarray(bins_fm, dtype=np.uint8)
    f, n = bins_fm.shape
    y = np.ascontiguousarray(y, dtype=np.float64)
    mb = None if missing_bin is None else np.ascontiguousarray(missing_bin, dtype=np.int32)
    nc = None if n_categories is None else np.ascontiguousarray(n_categories, dtype=np.int32)
    e = _Err()
    h = ctypes.c_void_p()
    e.check(lib().mojotrees_b200_train_binned_u8(_ptr(bins_fm), n, f, n_bins, _ptr(mb), _ptr(nc), _ptr(y), None,
                                                 params_string(params), ctypes.byref(h), e.h))
    return Model(h.value)


def histogram_u8(bins_fm, n_bins, grad_q, hess_q, rows=None, num_grad_quant_bins=4):
    """Quantized histogram [n_features, 3, n_bins] (sum g, sum h, count) of the selected rows."""
    bins_fm = np.ascontiguousarray(bins_fm, dtype=np.uint8)
    f, n = bins_fm.shape
    g = np.ascontiguousarray(grad_q, dtype=np.int8)
    h = np.ascontiguousarray(hess_q, dtype=np.uint8)
    r = None if rows is None else np.ascontiguousarray(rows, dtype=np.int32)
    out = np.zeros((f, 3, n_bins), np.int32)
    e = _Err()
    e.check(lib().mojotrees_b200_histogram_u8(_ptr(bins_fm), n, f, n_bins, _ptr(r), 0 if r is None else r.size,
                                              _ptr(g), _ptr(h), num_grad_quant_bins, _ptr(out), e.h))
    return out


def nccl_unique_id():
    """128 bytes identifying a new NCCL communicator (create on one rank)."""
    out = np.zeros(128, np.uint8)
    e = _Err()
    e.check(lib().mojotrees_b200_nccl_unique_id(_ptr(out), e.h))
    return out


def train_binned_dp(bins_fm, n_bins, y, nccl_id, rank, world, row_offset, n_rows_global, params=None,
                    missing_bin=None, n_categories=None):
    """Data-parallel fit: this rank's feature-major bins [n_features, n_local]."""
    bins_fm = np.ascontiguousarray(bins_fm, dtype=np.uint8)
    f, n = bins_fm.shape
    y = np.ascontiguousarray(y, dtype=np.float64)
    mb = None if missing_bin is None else np.ascontiguousarray(missing_bin, dtype=np.int32)
    nc = None if n_categories is None else np.ascontiguousarray(n_categories, dtype=np.int32)
    nid = np.ascontiguousarray(nccl_id, dtype=np.uint8)
    e = _Err()
    h = ctypes.c_void_p()
    e.check(lib().mojotrees_b200_train_binned_u8_dp(_ptr(bins_fm), n, f, n_bins, _ptr(mb), _ptr(nc), _ptr(y), None,
                                                    params_string(params), _ptr(nid), rank, world, row_offset,
                                                    n_rows_global, ctypes.byref(h), e.h))
    return Model(h.value)


def bin_dense(X, params=None, device=False):
    """Binning as train_dense does it: (bins [F, N] uint8, missing_bin, n_categories, n_bins).
    device=True bins the columns on the GPU (mojotrees_b200_bin_dense_gpu)."""
    X = np.asarray(X, dtype=np.float64)
    n, f = X.shape
    Xc = np.asfortranarray(X)
    bins = np.zeros((f, n), np.uint8)
    mb = np.zeros(f, np.int32)
    nc = np.zeros(f, np.int32)
    nb = ctypes.c_int32(0)
    e = _Err()
    fn = lib().mojotrees_b200_bin_dense_gpu if device else lib().mojotrees_b200_bin_dense
    e.check(fn(Xc.ctypes.data_as(ctypes.c_void_p), n, f, params_string(params), _ptr(bins), _ptr(mb), _ptr(nc),
               ctypes.byref(nb), e.h))
    return bins, mb, nc, nb.value


def shared_atomic_peak():
    """Lane atomics per second the GPU sustains in the histogram's shared-memory layout."""
    v = ctypes.c_double(0.0)
    e = _Err()
    e.check(lib().mojotrees_b200_shared_atomic_peak(ctypes.byref(v), e.h))
    return v.value


def _csc_arrays(indptr, indices, values):
    return (np.ascontiguousarray(indptr, dtype=np.int64), np.ascontiguousarray(indices, dtype=np.int64),
            np.ascontiguousarray(values, dtype=np.float64))


def train_csc(indptr, indices, values, n_rows, y, params=None):
    """Train on a CSC matrix (n_rows x len(indptr) - 1) through mojotrees_b200_train_csc."""
    ip, ix, vv = _csc_arrays(indptr, indices, values)
    y = np.ascontiguousarray(y, dtype=np.float64)
    e = _Err()
    h = ctypes.c_void_p()
    e.check(lib().mojotrees_b200_train_csc(_ptr(ip), _ptr(ix), _ptr(vv), n_rows, ip.size - 1, _ptr(y), None,
                                           params_string(params), ctypes.byref(h), e.h))
    return Model(h.value)


def bin_csc(indptr, indices, values, n_rows, params=None):
    """The bins train_csc trains on: (bins [F, N] uint8, missing_bin, n_categories, n_bins)."""
    ip, ix, vv = _csc_arrays(indptr, indices, values)
    f = ip.size - 1
    bins = np.zeros((f, n_rows), np.uint8)
    mb = np.zeros(f, np.int32)
    nc = np.zeros(f, np.int32)
    nb = ctypes.c_int32(0)
    e = _Err()
    e.check(lib().mojotrees_b200_bin_csc(_ptr(ip), _ptr(ix), _ptr(vv), n_rows, f, params_string(params), _ptr(bins),
                                         _ptr(mb), _ptr(nc), ctypes.byref(nb), e.h))
    return bins, mb, nc, nb.value


def check_quotients(n, seed=1):
    """Bits that differ between the trainer's divide-free dequantization and
    the divide, over n random (sum, units) pairs on the device (0 expected)."""
    out = ctypes.c_int64(-1)
    e = _Err()
    e.check(lib().mojotrees_b200_check_quotients(n, seed, ctypes.byref(out), e.h))
    return out.value


def gpu_available():
    return bool(lib().mojotrees_gpu_available())


def abi_version():
    return lib().mojotrees_abi_version()
