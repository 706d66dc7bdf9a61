"""C ABI surface on the host (no GPU needed): exports, errors, parsing, binning.

Mirrors the reference's capi/test_capi.c checks of status codes, NULL
handling and error objects, plus this library's device policy (a GPU request
never falls back; device=cpu is unsupported here).
"""
import ctypes
import os
import re

import numpy as np
import pytest

from golden_fixtures import fixture

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "mojotrees.h")).read()
    return sorted(set(re.findall(r"\b(mojotrees_\w+)\s*\(", text)))


def test_every_declared_symbol_is_exported(mtlib):
    from mojoboost_b200 import _capi
    syms = declared_symbols()
    assert len(syms) >= 30
    for s in syms:
        assert hasattr(mtlib.lib(), s), s
    assert set(syms) == set(_capi.SIGNATURES), "ctypes table and header disagree"


def test_versions(mtlib):
    lib = mtlib.lib()
    assert lib.mojotrees_abi_version() == 3
    a, b, c = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    lib.mojotrees_library_version(ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
    lib.mojotrees_library_version(None, None, None)


def test_error_object_lifecycle(mtlib):
    lib = mtlib.lib()
    e = lib.mojotrees_error_create()
    assert lib.mojotrees_error_message(e) == b""
    assert lib.mojotrees_error_message(None) is None
    lib.mojotrees_error_free(e)
    lib.mojotrees_error_free(None)
    lib.mojotrees_model_free(None)
    lib.mojotrees_string_free(None)


def _train(lib, params, data=True, labels=True, out=True, n_rows=4):
    X = np.zeros(n_rows * 2)
    y = np.zeros(n_rows)
    h = ctypes.c_void_p()
    e = lib.mojotrees_error_create()
    try:
        rc = lib.mojotrees_train_dense(X.ctypes.data if data else None, n_rows, 2, y.ctypes.data if labels else None,
                                       None, params, ctypes.byref(h) if out else None, e)
        return rc, lib.mojotrees_error_message(e).decode(), h
    finally:
        lib.mojotrees_error_free(e)


def test_null_pointers_are_invalid_argument(mtlib):
    lib = mtlib.lib()
    for kw in (dict(data=False), dict(labels=False), dict(out=False)):
        rc, msg, _ = _train(lib, b"", **kw)
        assert rc == -1 and "null" in msg


@pytest.mark.parametrize("params,code,needle", [
    (b"no_such_key=1", -1, "unknown parameter"),
    (b"num_leaves", -1, "malformed"),
    (b"num_leaves=abc", -1, "integer"),
    (b"num_leaves=1", -1, "num_leaves"),
    (b"device=cpu", -4, "GPU training path only"),
    (b"objective=poisson", -4, "not covered"),
    (b"boosting=dart", -4, "not covered"),
    (b"bagging_fraction=0.5 bagging_freq=1", -4, "bagging"),
    (b"max_depth=6", -4, "max_depth"),
    (b"learning_rate=0.1 eta=0.2", -1, "given twice"),
])
def test_parameter_errors(mtlib, params, code, needle):
    rc, msg, _ = _train(mtlib.lib(), params)
    assert rc == code, msg
    assert needle in msg


def test_weights_unsupported(mtlib):
    lib = mtlib.lib()
    X, y, w = np.zeros(8), np.zeros(4), np.ones(4)
    h = ctypes.c_void_p()
    e = lib.mojotrees_error_create()
    rc = lib.mojotrees_train_dense(X.ctypes.data, 4, 2, y.ctypes.data, w.ctypes.data, b"", ctypes.byref(h), e)
    assert rc == -4 and b"weights" in lib.mojotrees_error_message(e)
    lib.mojotrees_error_free(e)


def test_no_silent_cpu_fallback(mtlib):
    """Without a CUDA device a valid fit fails with UNSUPPORTED; it never trains on the CPU."""
    if mtlib.gpu_available():
        pytest.skip("a GPU is present")
    rc, msg, h = _train(mtlib.lib(), b"num_iterations=2", n_rows=50)
    assert rc == -4 and "CUDA" in msg
    assert not h.value


def test_parameter_keys(mtlib):
    lib = mtlib.lib()
    p = ctypes.c_void_p()
    e = lib.mojotrees_error_create()
    assert lib.mojotrees_parameter_keys(ctypes.byref(p), e) == 0
    keys = ctypes.string_at(p.value).decode().split(",")
    lib.mojotrees_string_free(p)
    lib.mojotrees_error_free(e)
    for k in ("objective", "num_leaves", "max_bin", "use_quantized_grad", "num_grad_quant_bins", "device_type"):
        assert k in keys


def test_bin_dense_matches_reference_fixture_bins(mtlib):
    """Host binning reproduces the missing-bin and categorical layout of the
    reference's misscat fixture (its golden trees depend on it)."""
    fx = fixture("misscat")
    bins, mb, nc, nb = mtlib.bin_dense(fx["x"].T, {"max_bin": 32, "categorical_feature": "2"})
    assert nb == 32
    assert list(mb) == [-1, 31, -1, -1, -1]
    assert list(nc) == [-1, -1, 6, -1, -1]
    assert np.all(bins[1][np.isnan(fx["x"][1])] == 31)
    assert bins[2].min() >= 1 and bins[2].max() <= 6


def test_bin_dense_edges_monotone_and_sampled(mtlib):
    rng = np.random.default_rng(0)
    X = rng.normal(size=(300_000, 2))  # above bin_construct_sample_cnt: sampled edges
    bins, mb, nc, nb = mtlib.bin_dense(X, {"max_bin": 255})
    for f in range(2):
        order = np.argsort(X[:, f], kind="stable")
        assert np.all(np.diff(bins[f][order].astype(int)) >= 0)
        assert bins[f].max() <= 254
    assert list(mb) == [-1, -1]


def test_bin_dense_reports_bad_categorical_code(mtlib):
    """A categorical code beyond int32 is an input error (raised on one of the
    binning threads, reported through the error object)."""
    X = np.zeros((100, 3))
    X[:, 1] = np.arange(100) % 5
    X[7, 1] = 3e9
    with pytest.raises(mtlib.MojoTreesError):
        mtlib.bin_dense(X, {"categorical_feature": "1"})


def test_extension_argument_checks(mtlib, tmp_path):
    """The host-side extensions refuse bad arguments with a status, never a
    crash: null pointers, short buffers, out-of-range iterations, a model
    without a raw-value mapper."""
    from test_model_io import X_A, model_a, write
    lib = mtlib.lib()
    m = mtlib.Model.load(write(tmp_path, "a.mbst", model_a(4)))
    e = lib.mojotrees_error_create()
    X = np.asfortranarray(X_A)
    out = np.zeros(1)
    try:
        assert lib.mojotrees_b200_predict_leaf(m.h, X.ctypes.data, len(X), 2, 0, 0, out.ctypes.data, 1, e) == -1
        assert lib.mojotrees_b200_predict_leaf(m.h, X.ctypes.data, len(X), 3, 0, 0, out.ctypes.data, 99, e) == -1
        assert lib.mojotrees_b200_model_bin(m.h, None, 5, 2, None, 10, e) == -1
        raw = np.zeros(len(X))
        bins = m.bin_rows(X)
        assert lib.mojotrees_b200_add_iteration_raw(m.h, bins.ctypes.data, len(X), 2, 1, raw.ctypes.data, raw.size,
                                                    e) == -1  # iteration 1 of a 1-iteration model
        assert lib.mojotrees_b200_add_iteration_raw(m.h, bins.ctypes.data, len(X), 2, 0, raw.ctypes.data, 3, e) == -1
        h = ctypes.c_void_p()
        assert lib.mojotrees_b200_model_prefix(m.h, 2, ctypes.byref(h), e) == -1
        assert lib.mojotrees_b200_model_prefix(m.h, -1, ctypes.byref(h), e) == -1
        assert lib.mojotrees_b200_ingest_column_major(None, None, -1, 2, None, e) == -1
        assert lib.mojotrees_b200_buffer_has_infinite(None, 4, None, e) == -1
        assert lib.mojotrees_b200_model_categorical(m.h, out.ctypes.data, 1, e) == -1  # 2 features, room for 1
    finally:
        lib.mojotrees_error_free(e)
