"""Sparse input through the shim: CSC fits and CSR predictions take the dense
path on the densified matrix (absent entries 0.0, stored NaN missing)."""
import numpy as np
import pytest
import scipy.sparse as sp

from test_model_io import RAW_A, X_A, model_a, write


@pytest.fixture()
def shim(mtlib):
    from mojoboost_b200 import _mojotrees
    return _mojotrees


def _params(M):
    M.sort_indices()
    data = np.ascontiguousarray(M.data, dtype=np.float64)
    indices = np.ascontiguousarray(M.indices, dtype=np.int64)
    indptr = np.ascontiguousarray(M.indptr, dtype=np.int64)
    keep = (data, indices, indptr)
    return {"sparse_data_addr": data.ctypes.data, "sparse_indices_addr": indices.ctypes.data,
            "sparse_indptr_addr": indptr.ctypes.data, "sparse_nnz": int(M.nnz), "n_rows": M.shape[0],
            "n_features": M.shape[1]}, keep


def test_densify_matches_scipy(shim):
    rng = np.random.default_rng(4)
    for n, f, d in ((1, 1, 1.0), (50, 7, 0.2), (300, 40, 0.05), (10, 3, 0.0)):
        M = sp.random(n, f, density=d, random_state=int(rng.integers(1 << 30)), format="csc")
        if M.nnz:
            M.data[::7] = np.nan
        p, keep = _params(M)
        np.testing.assert_array_equal(shim._densify(p, True), M.toarray())
        R = M.tocsr()
        p, keep = _params(R)
        np.testing.assert_array_equal(shim._densify(p, False), R.toarray())


def test_malformed_sparse_is_refused(shim):
    M = sp.csc_matrix(np.array([[1.0, 0.0], [0.0, 2.0]]))
    p, keep = _params(M)
    bad = np.array([0, 1, 5], dtype=np.int64)
    q = dict(p, sparse_indptr_addr=bad.ctypes.data)
    with pytest.raises(ValueError):
        shim._densify(q, True)
    idx = np.array([0, 7], dtype=np.int64)
    q = dict(p, sparse_indices_addr=idx.ctypes.data)
    with pytest.raises(ValueError):
        shim._densify(q, True)


def test_predict_csr_equals_dense(shim, tmp_path):
    m = shim.load(write(tmp_path, "a.mbst", model_a(4)))
    X = np.nan_to_num(X_A, nan=0.0)
    X[3, 0] = np.nan  # a stored NaN is missing
    R = sp.csr_matrix(np.where(X == 0.0, 0.0, X))
    R.data[np.isnan(R.data)] = np.nan
    p, keep = _params(R)
    out = np.zeros(len(X))
    shim.predict_raw_csr(m, dict(p, device="cpu"), out.ctypes.data)
    np.testing.assert_array_equal(out, m.predict(R.toarray(), raw_score=True))
    with pytest.raises(NotImplementedError):
        shim.predict_csr(m, dict(p, device="gpu"), out.ctypes.data)


def test_fit_csc_reaches_the_device_path(shim, mtlib, monkeypatch):
    """The densified matrix and the estimator's parameters reach `fit`."""
    seen = {}

    def fake_fit(x_addr, n, f, y_addr, objective, params):
        seen["X"] = shim._f64(x_addr, n * f).reshape(f, n).T.copy()
        seen["params"] = params
        return "model"

    monkeypatch.setattr(shim, "fit", fake_fit)
    M = sp.random(40, 5, density=0.3, random_state=1, format="csc")
    p, keep = _params(M)
    y = np.zeros(40)
    assert shim.fit_csc(y.ctypes.data, 0, dict(p, n_estimators=3)) == "model"
    np.testing.assert_array_equal(seen["X"], M.toarray())
    assert seen["params"] == {"n_estimators": 3}
