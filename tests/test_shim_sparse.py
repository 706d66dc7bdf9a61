"""Sparse input through the shim.  CSC fits bin the compressed columns as the
densified matrix would be binned (absent entries 0.0, stored NaN missing)
and train on those bins, without a dense float64 matrix on the host; CSR
predictions take the host predictor on the densified rows."""
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


def test_fit_csc_reaches_the_device_path(shim, mtlib):
    """The compressed columns go to mojotrees_b200_train_csc as they are (no
    dense float64 matrix on the host); without a CUDA device the C ABI
    refuses instead of falling back."""
    M = sp.random(40, 5, density=0.3, random_state=1, format="csc")
    p, keep = _params(M)
    y = np.zeros(40)
    if mtlib.gpu_available():
        pytest.skip("host-only check (a GPU box trains)")
    with pytest.raises(mtlib.UnsupportedError, match="CUDA device"):
        shim.fit_csc(y.ctypes.data, 0, dict(p, n_estimators=3))


def _messy_csc(seed, n, f):
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(n, f))
    X[rng.random((n, f)) < 0.85] = 0.0
    X[:, 1] = np.round(X[:, 1] * 3)
    X[::37, 2] = np.nan
    X[:, 3] = np.where(rng.random(n) < 0.6, 0.0, rng.integers(0, 400, n).astype(np.float64))
    X[rng.random(n) < 0.01, 3] = np.nan
    X[5, 0] = 0.0  # stored explicitly below
    C = sp.csc_matrix(np.where(np.isnan(X), 1.5e300, X))
    C.data[C.data == 1.5e300] = np.nan
    # an explicitly stored zero is the same value as an absent entry
    C = C.tolil()
    C[5, 0] = 0.0
    C = C.tocsc()
    C.data[C.indptr[0]] = C.data[C.indptr[0]]
    return X, C


@pytest.mark.parametrize("n,params", [(260_000, {"max_bin": 255}),
                                      (20_000, {"max_bin": 63, "categorical_feature": "3"}),
                                      (1_000, {"max_bin": 16})])
def test_bins_of_csc_equal_bins_of_the_densified_matrix(mtlib, n, params):
    X, C = _messy_csc(7, n, 5)
    dense = mtlib.bin_dense(X, params)
    sparse = mtlib.bin_csc(C.indptr, C.indices, C.data, n, params)
    assert dense[3] == sparse[3]
    for a, b in zip(dense[:3], sparse[:3]):
        np.testing.assert_array_equal(a, b)


def test_malformed_csc_is_refused(mtlib):
    with pytest.raises(mtlib.MojoTreesError, match="strictly increasing"):
        mtlib.bin_csc(np.array([0, 2]), np.array([3, 1]), np.array([1.0, 2.0]), 5)
    with pytest.raises(mtlib.MojoTreesError, match="out of range"):
        mtlib.bin_csc(np.array([0, 1]), np.array([9]), np.array([1.0]), 5)


@pytest.mark.gpu
def test_gpu_csc_fit_equals_the_dense_fit(mtlib):
    X, C = _messy_csc(8, 50_000, 5)
    y = np.nan_to_num(X[:, 0]) * 2 + np.nan_to_num(X[:, 1]) + 0.1 * np.arange(50_000) % 3
    p = {"objective": "regression", "num_iterations": 4, "num_leaves": 31, "max_bin": 63,
         "categorical_feature": "3", "keep_training_scores": True}
    dm = mtlib.train_dense(X, y, p)
    sm = mtlib.train_csc(C.indptr, C.indices, C.data, 50_000, y, p)
    assert dm.num_trees == sm.num_trees
    for t in range(dm.num_trees):
        a, b = dm.tree(t), sm.tree(t)
        for k in a:
            np.testing.assert_array_equal(np.asarray(a[k]), np.asarray(b[k]), err_msg=f"tree {t} {k}")
    np.testing.assert_array_equal(dm.training_scores(50_000), sm.training_scores(50_000))
