"""ctypes binding of the CPU oracle (oracle/liboracle.so) -- test infrastructure.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load this.
"""
import ctypes
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_SO = os.path.join(ROOT, "oracle", "liboracle.so")

MODE_CPU, MODE_FIXED, MODE_QUANT, MODE_FIXED52 = 0, 1, 2, 3
OBJ_L2, OBJ_LOGISTIC, OBJ_SOFTMAX = 0, 1, 2


class OracleParams(ctypes.Structure):
    _fields_ = [
        ("objective", ctypes.c_int),
        ("n_classes", ctypes.c_int),
        ("num_rounds", ctypes.c_int),
        ("learning_rate", ctypes.c_double),
        ("num_leaves", ctypes.c_int),
        ("min_data_in_leaf", ctypes.c_int),
        ("lambda_l2", ctypes.c_double),
        ("min_child_hess", ctypes.c_double),
        ("lambda_l1", ctypes.c_double),
        ("feature_fraction", ctypes.c_double),
        ("feature_fraction_seed", ctypes.c_int),
        ("bagging_fraction", ctypes.c_double),
        ("bagging_freq", ctypes.c_int),
        ("bagging_seed", ctypes.c_int),
        ("max_cat_to_onehot", ctypes.c_int),
        ("max_cat_threshold", ctypes.c_int),
        ("cat_smooth", ctypes.c_double),
        ("cat_l2", ctypes.c_double),
        ("min_data_per_group", ctypes.c_int),
        ("mode", ctypes.c_int),
        ("exp_kind", ctypes.c_int),
        ("quant_bins", ctypes.c_int),
        ("quant_seed", ctypes.c_int),
        ("simd_lanes", ctypes.c_int),
        ("lane_reduce", ctypes.c_int),
        ("traversal_fma", ctypes.c_int),
        ("n_threads", ctypes.c_int),
        ("base_override", ctypes.c_void_p),
    ]


class OracleOut(ctypes.Structure):
    _fields_ = [
        ("n_trees", ctypes.c_int),
        ("max_nodes", ctypes.c_int),
        ("n_nodes", ctypes.c_void_p),
        ("feature", ctypes.c_void_p),
        ("threshold_bin", ctypes.c_void_p),
        ("left", ctypes.c_void_p),
        ("right", ctypes.c_void_p),
        ("default_left", ctypes.c_void_p),
        ("missing_bin", ctypes.c_void_p),
        ("cat_bits", ctypes.c_void_p),
        ("value", ctypes.c_void_p),
        ("gain", ctypes.c_void_p),
        ("count", ctypes.c_void_p),
        ("raw", ctypes.c_void_p),
        ("base_scores", ctypes.c_void_p),
        ("round_seconds", ctypes.c_void_p),
    ]


def build():
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        _lib = ctypes.CDLL(ORACLE_SO)
        _lib.mt_oracle_train.restype = ctypes.c_int
        _lib.mt_oracle_pow2_abs_total.restype = ctypes.c_double
        _lib.mt_oracle_pow2_abs_total.argtypes = [ctypes.c_void_p, ctypes.c_int64]
        _lib.mt_oracle_exp.restype = ctypes.c_double
        _lib.mt_oracle_exp.argtypes = [ctypes.c_double]
        _lib.mt_oracle_splitmix64.restype = ctypes.c_uint64
        _lib.mt_oracle_splitmix64.argtypes = [ctypes.c_uint64]
        _lib.mt_oracle_uniform.restype = ctypes.c_double
        _lib.mt_oracle_uniform.argtypes = [ctypes.c_uint64]
        _lib.mt_oracle_quant_stream.restype = ctypes.c_uint64
        _lib.mt_oracle_quant_stream.argtypes = [ctypes.c_longlong, ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int]
        _lib.mt_oracle_quantize_stochastic.restype = ctypes.c_longlong
        _lib.mt_oracle_quantize_stochastic.argtypes = [ctypes.c_double, ctypes.c_double, ctypes.c_double,
                                                       ctypes.c_uint64]
        _lib.mt_oracle_fixed_point_scale.restype = ctypes.c_double
        _lib.mt_oracle_fixed_point_scale.argtypes = [ctypes.c_double]
    return _lib


def default_params(**kw):
    p = dict(
        objective=OBJ_L2, n_classes=1, num_rounds=10, learning_rate=0.1,
        num_leaves=31, min_data_in_leaf=20, lambda_l2=1.0, min_child_hess=1e-3,
        lambda_l1=0.0, feature_fraction=1.0, feature_fraction_seed=2,
        bagging_fraction=1.0, bagging_freq=0, bagging_seed=3,
        max_cat_to_onehot=4, max_cat_threshold=32, cat_smooth=10.0, cat_l2=10.0,
        min_data_per_group=100, mode=MODE_CPU, exp_kind=0, quant_bins=4,
        quant_seed=11, simd_lanes=8, lane_reduce=0, traversal_fma=0, n_threads=0,
        base_override=None,
    )
    p.update(kw)
    return p


class OracleModel:
    """Trees as numpy arrays: tree t has n_nodes[t] nodes in row t."""

    def __init__(self, n_trees, n_nodes, arrays, raw, base_scores):
        self.n_trees = n_trees
        self.n_nodes = n_nodes[:n_trees].copy()
        for k, v in arrays.items():
            setattr(self, k, v[:n_trees].copy())
        self.raw = raw
        self.base_scores = base_scores


def train(bins_fm, n_bins, labels, missing_bin=None, n_cats=None, **kw):
    """bins_fm: uint8 array [F, N] (feature-major)."""
    bins_fm = np.ascontiguousarray(bins_fm, dtype=np.uint8)
    F, N = bins_fm.shape
    labels = np.ascontiguousarray(labels, dtype=np.float64)
    missing_bin = np.ascontiguousarray(
        np.full(F, -1) if missing_bin is None else missing_bin, dtype=np.int32)
    n_cats = np.ascontiguousarray(np.full(F, -1) if n_cats is None else n_cats, dtype=np.int32)
    p = default_params(**kw)
    keep = None
    if p["base_override"] is not None:
        keep = np.ascontiguousarray(p["base_override"], dtype=np.float64)
        p["base_override"] = keep.ctypes.data
    params = OracleParams(**p)
    K = p["n_classes"] if p["objective"] == OBJ_SOFTMAX else 1
    T = p["num_rounds"] * K
    M = 2 * p["num_leaves"] - 1
    n_nodes = np.zeros(T, np.int32)
    arrs = {
        "feature": np.full((T, M), -1, np.int32),
        "threshold_bin": np.full((T, M), -1, np.int32),
        "left": np.full((T, M), -1, np.int32),
        "right": np.full((T, M), -1, np.int32),
        "default_left": np.zeros((T, M), np.int32),
        "missing_bin": np.full((T, M), -1, np.int32),
        "cat_bits": np.zeros((T, M, 4), np.uint64),
        "value": np.zeros((T, M), np.float64),
        "gain": np.zeros((T, M), np.float64),
        "count": np.zeros((T, M), np.int64),
    }
    raw = np.zeros(N * K, np.float64)
    base = np.zeros(K, np.float64)
    round_s = np.full(p["num_rounds"], np.nan)
    out = OracleOut(0, M, n_nodes.ctypes.data, *(arrs[k].ctypes.data for k in (
        "feature", "threshold_bin", "left", "right", "default_left", "missing_bin",
        "cat_bits", "value", "gain", "count")), raw.ctypes.data, base.ctypes.data, round_s.ctypes.data)
    err = ctypes.create_string_buffer(512)
    rc = lib().mt_oracle_train(
        bins_fm.ctypes.data_as(ctypes.c_void_p), ctypes.c_int64(N), ctypes.c_int(F),
        ctypes.c_int(n_bins), missing_bin.ctypes.data_as(ctypes.c_void_p),
        n_cats.ctypes.data_as(ctypes.c_void_p), labels.ctypes.data_as(ctypes.c_void_p),
        ctypes.byref(params), ctypes.byref(out), err, 512)
    if rc != 0:
        raise RuntimeError("oracle: " + err.value.decode())
    m = OracleModel(out.n_trees, n_nodes, arrs, raw.reshape(N, K) if K > 1 else raw, base)
    m.round_seconds = round_s  # wall-clock seconds since the fit began, at the end of each round
    return m


def bin_dense(X, max_bin=255, categorical=(), min_data_in_bin=3, sample_cnt=200_000, seed=1, use_missing=True):
    """The oracle's restatement of the reference binner: X [N, F] float64 ->
    (bins [F, N] uint8, missing_bin, n_categories, n_bins)."""
    X = np.asarray(X, dtype=np.float64)
    n, f = X.shape
    Xc = np.asfortranarray(X)
    cats = np.zeros(f, np.int32)
    for c in categorical:
        cats[c] = 1
    bins = np.zeros((f, n), np.uint8)
    mb = np.zeros(f, np.int32)
    nc = np.zeros(f, np.int32)
    P = ctypes.c_void_p
    rc = lib().mt_oracle_bin_dense(Xc.ctypes.data_as(P), ctypes.c_int64(n), ctypes.c_int(f), ctypes.c_int(max_bin),
                                   ctypes.c_int(min_data_in_bin), ctypes.c_int64(sample_cnt), ctypes.c_int(seed),
                                   ctypes.c_int(1 if use_missing else 0), cats.ctypes.data_as(P),
                                   bins.ctypes.data_as(P), mb.ctypes.data_as(P), nc.ctypes.data_as(P))
    if rc != 0:
        raise ValueError("oracle binning: invalid arguments")
    return bins, mb, nc, max_bin


def predict_raw_bins(model, bins_fm, fma=False):
    """Sum of learning-rate-scaled tree outputs per row, in tree order.

    Mirrors Booster.predict_raw_row (boosting.mojo:1722-1727) for one class.
    """
    raise NotImplementedError
