"""The `_mojotrees` shim's prediction, model-file and accessor hooks, called as
the reference estimators call them (raw addresses, column-major float64,
half-open iteration ranges; bindings/_mojotrees.mojo:4223-4296)."""
import numpy as np
import pytest

from test_model_io import RAW_A, X_A, model_a, write


@pytest.fixture()
def shim(mtlib):
    from mojoboost_b200 import _mojotrees
    return _mojotrees


def _predict(shim, m, X, **params):
    Xc = np.asfortranarray(X, dtype=np.float64)
    out = np.full(X.shape[0] * m.num_classes, np.nan)
    ran = shim.predict_batch(m, Xc.ctypes.data, X.shape[0], X.shape[1],
                             {"device": "cpu", "start": 0, "stop": m.num_iterations, "raw_score": 0, **params},
                             out.ctypes.data)
    return ran, out


def test_predict_batch_on_the_host(shim, tmp_path):
    m = shim.load(write(tmp_path, "a.mbst", model_a(4)))
    ran, out = _predict(shim, m, X_A)
    assert ran == "cpu"
    np.testing.assert_array_equal(out, RAW_A)  # regression: response == raw
    # an empty iteration range leaves the base score
    _, out = _predict(shim, m, X_A, stop=0)
    np.testing.assert_array_equal(out, np.full(len(X_A), 0.25))
    # an empty batch selects no backend and writes nothing
    assert shim.predict_batch(m, 0, 0, 2, {"device": "cpu", "start": 0, "stop": 1, "raw_score": 1}, 0) is None


def test_accessors_and_names(shim, tmp_path):
    m = shim.load(write(tmp_path, "a.mbst", model_a(4)))
    assert (shim.n_features(m), shim.n_classes(m), shim.num_iterations(m)) == (2, 1, 1)
    p = str(tmp_path / "named.mbst")
    names = ["x 0", "tab\there\\"]
    shim.save(m, p, names, len(names))
    assert shim.model_feature_names(p) == names
    assert open(p).read().split("\n")[1] == "feature_names 2"
    m2 = shim.load(p)
    np.testing.assert_array_equal(_predict(shim, m2, X_A)[1], RAW_A)
    assert shim.model_feature_names(write(tmp_path, "plain.mbst", model_a(4))) == []
    with pytest.raises(ValueError):
        shim.save(m, p, ["bad\x01name", "b"], 2)


def test_missing_hooks_probe_as_absent(shim):
    """The estimators probe optional hooks with getattr(..., None); a hook
    this library lacks reads as absent there and raises on a direct call."""
    assert getattr(shim, "predict_contrib", None) is None
    with pytest.raises(NotImplementedError):
        shim.predict_contrib


@pytest.mark.gpu
def test_predict_batch_on_the_device(shim, tmp_path):
    m = shim.load(write(tmp_path, "a.mbst", model_a(4)))
    ran, out = _predict(shim, m, X_A, device="gpu", raw_score=1)
    assert ran == "gpu"
    np.testing.assert_array_equal(out, RAW_A)


def test_ingest_column_major(shim):
    rng = np.random.default_rng(3)
    for n, f in ((1, 1), (65, 3), (130, 70), (1000, 1)):
        X = np.ascontiguousarray(rng.normal(size=(n, f)))
        X[rng.random((n, f)) < 0.05] = np.nan
        out = np.empty((n, f), order="F")
        assert shim.ingest_column_major(X.ctypes.data, out.ctypes.data, n, f) == 0
        np.testing.assert_array_equal(out, X)
        assert shim.buffer_has_infinite(out.ctypes.data, n * f) == 0
        X[n // 2, f - 1] = -np.inf
        assert shim.ingest_column_major(X.ctypes.data, out.ctypes.data, n, f) == 1
        assert shim.buffer_has_infinite(out.ctypes.data, n * f) == 1
    assert shim.ingest_column_major(0, 0, 0, 5) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("objective", [0, 1])
def test_gpu_fit_through_the_shim(shim, mtlib, objective):
    """`_mojotrees.fit` at raw addresses (column-major X, as the estimators
    pass it) trains the model `mojotrees_train_dense` trains for the same
    parameters, and `predict_batch` on either device returns its predictions."""
    from parity_util import make_data
    X, y = make_data(51, 5000, 6, kind="binary" if objective == 1 else "regression", nan_frac=0.05)
    Xf = np.asfortranarray(X)
    y = np.ascontiguousarray(y, dtype=np.float64)
    params = {"n_estimators": 4, "num_leaves": 15, "min_data_in_leaf": 20}
    m = shim.fit(Xf.ctypes.data, X.shape[0], X.shape[1], y.ctypes.data, objective, params)
    ref = mtlib.train_dense(X, y, dict(kv.split("=", 1) for kv in
                                       shim.param_string(objective, params).decode().split()))
    for t in range(ref.num_trees):
        for k, v in ref.tree(t).items():
            np.testing.assert_array_equal(m.tree(t)[k], v)
    for device in ("cpu", "gpu"):
        ran, out = _predict(shim, m, X, device=device)
        assert ran == device
        np.testing.assert_array_equal(out, m.predict(X))


def test_predict_leaf(shim, mtlib, tmp_path):
    """Leaf ordinals: a leaf's rank among its tree's leaves in node order
    (tree.mojo:558-580).  Tree A's leaves are nodes 2, 3, 4."""
    m = shim.load(write(tmp_path, "a.mbst", model_a(4)))
    Xc = np.asfortranarray(X_A)
    out = np.full(len(X_A), -9.0)
    assert shim.predict_leaf_batch(m, Xc.ctypes.data, len(X_A), 2, {"device": "cpu", "start": 0, "stop": 1},
                                   out.ctypes.data) == "cpu"
    np.testing.assert_array_equal(out, [1, 2, 0, 1, 1, 1, 2])
    with pytest.raises(NotImplementedError):
        shim.predict_leaf_batch(m, Xc.ctypes.data, len(X_A), 2, {"device": "gpu", "start": 0, "stop": 1},
                                out.ctypes.data)
    imp = np.zeros(2)
    shim.feature_importance(m, 2, 0, imp.ctypes.data)
    np.testing.assert_array_equal(imp, [1, 1])
    shim.feature_importance(m, 2, 1, imp.ctypes.data)
    np.testing.assert_array_equal(imp, [5.0, 2.0])


def test_predict_leaf_multiclass_range(shim, tmp_path):
    # 2 iterations x 2 classes of one-leaf trees: every ordinal is 0; the
    # range [1, 2) has K = 2 columns a row
    from test_model_io import b, row, frow
    s = "mojotrees v4\nmulticlass 2\n" + f"learning_rate {b(1.0)}\nbase_scores {b(0.0)} {b(0.0)}\n"
    s += "mapper 1 255 1\n" + frow([0.0]) + row([0, 1]) + row([-1]) + "trees 4\n"
    for v in (1.0, 2.0, 3.0, 4.0):
        s += "tree 1 1\n" + row([-1]) * 4 + frow([v]) + row([0]) + row([-1]) + "counts 0\ngains 0\n"
    m = shim.load(write(tmp_path, "mc.mbst", s))
    X = np.zeros((3, 1), order="F")
    out = np.full(3 * 2, -1.0)
    shim.predict_leaf_multiclass(m, X.ctypes.data, 3, 1, 1, 2, out.ctypes.data)
    np.testing.assert_array_equal(out, np.zeros(6))


def test_empty_range_response(shim, tmp_path):
    """An empty iteration range scores no tree: from iteration 0 the response
    of the base score (the C predictor's sigmoid), from a later start the
    response of a zero raw score."""
    import math
    m = shim.load(write(tmp_path, "b.mbst", model_a(4).replace("objective 0", "objective 1")))
    _, out = _predict(shim, m, X_A, stop=0)
    assert np.all(out == 1.0 / (1.0 + math.exp(-0.25)))
    _, out = _predict(shim, m, X_A, start=1, stop=1)
    assert np.all(out == 0.5)
    _, out = _predict(shim, m, X_A, stop=0, raw_score=1)
    assert np.all(out == 0.25)


def _metric(shim, code, pred, y, objective=0, weight=None, n_classes=0):
    pred = np.ascontiguousarray(pred, dtype=np.float64)
    y = np.ascontiguousarray(y, dtype=np.float64)
    w = None if weight is None else np.ascontiguousarray(weight, dtype=np.float64)
    return shim.eval_metric(code, {"pred_addr": pred.ctypes.data, "y_addr": y.ctypes.data, "n_rows": len(y),
                                   "weight_addr": 0 if w is None else w.ctypes.data, "objective": objective,
                                   "n_classes": n_classes, "alpha": 0.9})


def test_eval_metric_values(shim):
    """metrics.mojo's definitions on small hand-worked cases."""
    import math
    pred, y = [1.0, 2.0, 4.0], [1.0, 3.0, 2.0]
    assert _metric(shim, 0, pred, y) == (0.0 + 1.0 + 4.0) / 3                      # l2
    assert _metric(shim, 1, pred, y) == math.sqrt(5.0 / 3)                         # rmse
    assert _metric(shim, 2, pred, y) == (0.0 + 1.0 + 2.0) / 3                      # l1
    assert _metric(shim, 0, pred, y, weight=[1.0, 0.0, 2.0]) == (0.0 + 0.0 + 2.0 * 4.0) / 3.0
    raw, lab = [0.0, 2.0, -1.0, 3.0], [1.0, 0.0, 0.0, 1.0]
    p = [0.5, 1 / (1 + math.exp(-2.0)), math.exp(-1.0) / (1 + math.exp(-1.0)), 1 / (1 + math.exp(-3.0))]
    want = -(math.log(p[0]) + math.log(1 - p[1]) + math.log(1 - p[2]) + math.log(p[3])) / 4
    assert abs(_metric(shim, 5, raw, lab, objective=1) - want) < 1e-15               # binary_logloss
    assert _metric(shim, 6, raw, lab, objective=1) == 0.25                         # binary_error: row 1 wrong
    # multiclass: 2 rows x 3 classes of raw scores
    mraw = [0.0, 1.0, 2.0, 3.0, 0.0, 0.0]
    e0 = np.exp(np.array([0.0, 1.0, 2.0]) - 2.0)
    e1 = np.exp(np.array([3.0, 0.0, 0.0]) - 3.0)
    want = -(math.log(e0[1] / e0.sum()) + math.log(e1[0] / e1.sum())) / 2
    assert abs(_metric(shim, 8, mraw, [1.0, 0.0], n_classes=3) - want) < 1e-15     # multi_logloss
    assert _metric(shim, 9, mraw, [1.0, 0.0], n_classes=3) == 0.5                   # multi_error


def test_eval_metric_auc_matches_sklearn(shim):
    metrics = pytest.importorskip("sklearn.metrics")
    rng = np.random.default_rng(6)
    s = np.round(rng.normal(size=500), 1)  # many ties
    y = (rng.random(500) < 0.4).astype(float)
    w = rng.random(500)
    assert abs(_metric(shim, 7, s, y) - metrics.roc_auc_score(y, s)) < 1e-12
    assert abs(_metric(shim, 7, s, y, weight=w) - metrics.roc_auc_score(y, s, sample_weight=w)) < 1e-12
    with pytest.raises(NotImplementedError):
        _metric(shim, 10, s, y)
