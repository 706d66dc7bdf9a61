"""The reference's own Python package (python/mojotrees, unchanged) over this
library's `_mojotrees` shim: it imports (the objective/metric registry
queries), loads model files, predicts, saves with feature names, and a
`device="gpu"` fit without a CUDA device refuses instead of falling back.

Runs when MOJOTREES_REFERENCE_PYTHON names the directory that holds the
reference's `mojotrees` package (this test reads it at run time); skipped
otherwise.
"""
import os
import sys

import numpy as np
import pytest

from test_model_io import RAW_A, X_A, model_a, write

REF_PY = os.environ.get("MOJOTREES_REFERENCE_PYTHON", "")
pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF_PY, "mojotrees")),
                                reason="the reference package is not mounted")


@pytest.fixture(scope="module")
def ref():
    from mojoboost_b200 import _mojotrees as shim
    saved = {k: v for k, v in sys.modules.items() if k == "mojotrees" or k.startswith("mojotrees.")}
    for k in saved:
        del sys.modules[k]
    sys.path.insert(0, REF_PY)
    sys.modules["mojotrees._mojotrees"] = shim
    try:
        import mojotrees
        yield mojotrees
    finally:
        sys.path.remove(REF_PY)
        for k in [k for k in sys.modules if k == "mojotrees" or k.startswith("mojotrees.")]:
            del sys.modules[k]
        sys.modules.update(saved)


def test_registry_answers_the_reference_import(ref):
    from mojotrees import _eval
    assert _eval._TABLE.metric_code("l2") == 0
    assert _eval._TABLE.higher_is_better(_eval._TABLE.metric_code("auc"))
    assert _eval._TABLE.canonical_name("mse") == "l2"
    assert _eval._TABLE.default_metric("binary", "binary") == "binary_logloss"


def test_regressor_load_predict_save(ref, tmp_path):
    est = ref.MojoTreesRegressor.load(write(tmp_path, "a.mbst", model_a(4)))
    assert est.n_features_in_ == 2
    np.testing.assert_array_equal(est.predict(X_A), RAW_A)
    np.testing.assert_array_equal(est.predict(X_A, raw_score=True), RAW_A)
    out = str(tmp_path / "saved.mbst")
    est.feature_names_in_ = np.array(["alpha", "beta gamma"], dtype=object)
    est.save(out)
    back = ref.MojoTreesRegressor.load(out)
    assert list(back.feature_names_in_) == ["alpha", "beta gamma"]
    np.testing.assert_array_equal(back.predict(X_A), RAW_A)


def test_classifier_load_predict_proba(ref, tmp_path):
    text = model_a(4).replace("objective 0", "objective 1")
    est = ref.MojoTreesClassifier.load(write(tmp_path, "b.mbst", text))
    proba = est.predict_proba(X_A)
    want = 1.0 / (1.0 + np.exp(-RAW_A))
    np.testing.assert_allclose(proba[:, 1], want, rtol=1e-15, atol=0)
    np.testing.assert_allclose(proba[:, 0], 1.0 - want, rtol=1e-12, atol=1e-15)


def test_gpu_fit_without_a_device_is_refused(ref, mtlib):
    if mtlib.gpu_available():
        pytest.skip("a CUDA device is present")
    est = ref.MojoTreesRegressor(n_estimators=3, device="gpu")
    with pytest.raises(Exception) as ei:
        est.fit(np.random.default_rng(0).random((200, 3)), np.random.default_rng(1).random(200))
    assert "CUDA" in str(ei.value) or "device" in str(ei.value)


@pytest.fixture()
def captured_fit(ref, monkeypatch):
    """The estimators' call into `_mojotrees.fit` / `fit_multiclass`, stopped
    there (no device needed): (objective code, params dict)."""
    from mojoboost_b200 import _mojotrees as shim
    param_string = shim.param_string
    cap = {}

    def fake(*a):
        cap["objective"] = shim.MULTICLASS if len(a) == 6 and "num_class" in a[5] else a[4]
        cap["params"] = dict(a[5])
        # built here, as the real hook does: the categorical index buffer the
        # dict points at lives only while the estimator's fit runs
        try:
            cap["string"] = param_string(cap["objective"], cap["params"]).decode()
        except NotImplementedError as e:
            cap["refused"] = e
        raise RuntimeError("captured")

    def fake_mc(x, n, f, y, k, params):
        p = dict(params)
        p["num_class"] = k
        return fake(x, n, f, y, shim.MULTICLASS, p)

    monkeypatch.setattr(shim, "fit", fake)
    monkeypatch.setattr(shim, "fit_multiclass", fake_mc)
    monkeypatch.setattr(shim, "resolve_device", lambda *a, **k: "gpu")
    return cap


def _fit(est, X, y):
    with pytest.raises(Exception):
        est.fit(X, y)


@pytest.mark.parametrize("kind", ["regressor", "binary", "multiclass"])
def test_estimator_params_reach_the_c_abi(ref, captured_fit, mtlib, kind):
    """The params dict each estimator builds becomes a parameter string the C
    ABI's own parser accepts (without a device the call then stops at the
    device check, never at a parameter)."""
    from mojoboost_b200 import _mojotrees as shim
    rng = np.random.default_rng(0)
    X = rng.random((300, 4))
    X[:, 2] = rng.integers(0, 5, 300)
    if kind == "regressor":
        est, y = ref.MojoTreesRegressor(n_estimators=4, categorical_feature=[2]), rng.random(300)
    else:
        k = 2 if kind == "binary" else 3
        est, y = ref.MojoTreesClassifier(n_estimators=4, categorical_feature=[2]), rng.integers(0, k, 300)
    _fit(est, X, y.astype(float))
    s = captured_fit["string"]
    assert "categorical_feature=2" in s and "num_iterations=4" in s
    if kind == "multiclass":
        assert "num_class=3" in s and "objective=multiclass" in s
    if mtlib.gpu_available():
        return
    with pytest.raises(mtlib.MojoTreesError) as ei:
        mtlib.train_dense(X, y.astype(float), dict(kv.split("=", 1) for kv in s.split()))
    assert ei.value.code == -4 and "CUDA" in str(ei.value)


@pytest.mark.parametrize("kw", [dict(max_depth=5), dict(boosting="dart"), dict(min_gain_to_split=0.5),
                                dict(bagging_fraction=0.5, bagging_freq=1), dict(extra_trees=True),
                                dict(path_smooth=1.0)])
def test_uncovered_estimator_options_are_refused(ref, captured_fit, kw):
    """An option the device path does not implement is refused by name, never
    trained without."""
    from mojoboost_b200 import _mojotrees as shim
    try:
        est = ref.MojoTreesRegressor(n_estimators=3, **kw)
    except TypeError:
        pytest.skip(f"the reference estimator takes no {kw}")
    rng = np.random.default_rng(1)
    try:
        est.fit(rng.random((200, 3)), rng.random(200))
    except RuntimeError as e:
        if str(e) != "captured":
            return  # refused before the fit hook
        assert "refused" in captured_fit, "an uncovered option reached the parameter string"
    except (ValueError, NotImplementedError):
        return  # refused by the estimator's preflight through the shim


def test_regressor_leaves_and_importances(ref, tmp_path):
    est = ref.MojoTreesRegressor.load(write(tmp_path, "a.mbst", model_a(4)))
    np.testing.assert_array_equal(np.asarray(est.predict(X_A, pred_leaf=True)).reshape(-1), [1, 2, 0, 1, 1, 1, 2])
    np.testing.assert_array_equal(est.feature_importances_, [1, 1])


def test_sparse_input_through_the_estimators(ref, captured_fit, tmp_path):
    """SciPy sparse input: prediction equals the dense prediction, and a
    sparse fit reaches the device fit with the estimator's parameters."""
    sp = pytest.importorskip("scipy.sparse")
    est = ref.MojoTreesRegressor.load(write(tmp_path, "a.mbst", model_a(4)))
    X = np.nan_to_num(X_A)
    np.testing.assert_array_equal(est.predict(sp.csr_matrix(X)), est.predict(X))
    fit_est = ref.MojoTreesRegressor(n_estimators=3, device="gpu")
    _fit(fit_est, sp.random(100, 4, density=0.3, format="csc", random_state=0), np.random.default_rng(2).random(100))
    assert "num_iterations=3" in captured_fit["string"]


def test_booster_inspection(ref, tmp_path):
    """The reference Booster's inspection API over a model this library
    wrote: its own model_to_string parser reads the v4 text."""
    b = ref.MojoTreesRegressor.load(write(tmp_path, "a.mbst", model_a(4))).booster_
    assert b.num_trees() == 1 and b.num_feature() == 2 and b.current_iteration() == 1
    d = b.dump_model()
    assert d["tree_info"][0]["num_leaves"] == 3
    df = b.trees_to_dataframe()
    assert len(df) == 5


@pytest.fixture()
def captured_dataset_fit(ref, monkeypatch, tmp_path):
    """`_mojotrees.fit` / `fit_multiclass` as the Dataset route reaches them:
    the parameter string and matrix are recorded and a model file stands in
    for the device fit."""
    from mojoboost_b200 import _mojotrees as shim
    cap = {}
    path = write(tmp_path, "a.mbst", model_a(4))
    param_string = shim.param_string

    def fake(x, n, f, y, objective, params):
        cap["string"] = param_string(objective, params).decode()
        cap["X"] = shim._f64(x, n * f).reshape(f, n).T.copy()
        cap["y"] = shim._f64(y, n).copy()
        return shim.load(path)

    def fake_mc(x, n, f, y, k, params):
        return fake(x, n, f, y, shim.MULTICLASS, dict(params, num_class=k))

    monkeypatch.setattr(shim, "fit", fake)
    monkeypatch.setattr(shim, "fit_multiclass", fake_mc)
    monkeypatch.setattr(shim, "resolve_device", lambda *a, **k: "gpu")
    return cap


def test_lightgbm_style_train_over_the_shim(ref, captured_dataset_fit):
    """mojotrees.train(params, Dataset(X, label)) builds the device fit's
    parameters from the params dict and the Dataset's binning, hands over the
    matrix and label unchanged, and the Booster it returns predicts."""
    rng = np.random.default_rng(3)
    X, y = rng.normal(size=(400, 2)), rng.normal(size=400)
    bst = ref.train({"objective": "regression", "device": "gpu", "num_leaves": 7},
                    ref.Dataset(X, label=y, params={"max_bin": 63}), num_boost_round=3)
    s = captured_dataset_fit["string"]
    assert "objective=regression" in s and "num_iterations=3" in s and "num_leaves=7" in s and "max_bin=63" in s
    np.testing.assert_array_equal(captured_dataset_fit["X"], X)
    np.testing.assert_array_equal(captured_dataset_fit["y"], y)
    np.testing.assert_array_equal(bst.predict(X_A), RAW_A)


def test_lightgbm_style_train_multiclass_and_refusals(ref, captured_dataset_fit):
    rng = np.random.default_rng(4)
    X, y = rng.normal(size=(300, 2)), rng.integers(0, 3, 300).astype(float)
    try:
        ref.train({"objective": "multiclass", "num_class": 3, "device": "gpu"}, ref.Dataset(X, label=y),
                  num_boost_round=2)
    except Exception:
        pass  # the stand-in model is single-output; only the parameters matter here
    assert "objective=multiclass" in captured_dataset_fit["string"]
    assert "num_class=3" in captured_dataset_fit["string"]
    with pytest.raises(Exception) as ei:
        ref.train({"objective": "regression", "device": "gpu"},
                  ref.Dataset(X, label=y, weight=np.ones(300)), num_boost_round=2)
    assert "weight" in str(ei.value)


def test_booster_save_and_reload(ref, captured_dataset_fit, tmp_path):
    rng = np.random.default_rng(5)
    X, y = rng.normal(size=(200, 2)), rng.normal(size=200)
    bst = ref.train({"objective": "regression", "device": "gpu"}, ref.Dataset(X, label=y), num_boost_round=2)
    out = str(tmp_path / "saved.mbst")
    bst.save_model(out)
    back = ref.Booster(model_file=out)
    np.testing.assert_array_equal(back.predict(X_A), RAW_A)
    from mojoboost_b200 import _mojotrees as shim
    assert shim.model_file_kind(out) == "objective"
    mc = out.replace("saved", "mc")
    with open(mc, "w") as f:
        f.write("mojotrees v4\nfeature_names 2\na b \nmulticlass 3\n")
    assert shim.model_file_kind(mc) == "multiclass"


def test_cv_over_the_shim(ref, monkeypatch, tmp_path):
    """mojotrees.cv: folds of the Dataset trained through train_dataset and
    grown one round at a time through booster_update (a fresh fit of the
    longer run, exact because no round depends on a later one), scored with
    eval_metric.  Stand-in fits return models of the requested length."""
    import re
    from mojoboost_b200 import _mojotrees as shim
    from test_fit_with_metrics import model_text
    lengths = []

    def fake(x, n, f, y, objective, params):
        k = int(re.search(r"num_iterations=(\d+)", shim.param_string(objective, params).decode()).group(1))
        lengths.append(k)
        return shim.load(write(tmp_path, f"m{k}.mbst", model_text(k)))

    monkeypatch.setattr(shim, "fit", fake)
    monkeypatch.setattr(shim, "resolve_device", lambda *a, **k: "gpu")
    rng = np.random.default_rng(7)
    X, y = rng.normal(size=(300, 2)), rng.normal(size=300)
    res = ref.cv({"objective": "regression", "device": "gpu"}, ref.Dataset(X, label=y), num_boost_round=3, nfold=3)
    assert len(res["valid l2-mean"]) == 3 and all(np.isfinite(res["valid l2-mean"]))
    assert lengths == [0, 0, 0, 1, 1, 1, 2, 2, 2, 3, 3, 3]
    # continuing with changed parameters is refused, not trained as something else
    ds = ref.Dataset(X, label=y)
    bst = ref.train({"objective": "regression", "device": "gpu"}, ds, num_boost_round=1)
    with pytest.raises(NotImplementedError):
        shim.booster_update(bst._handle, ds._constructed(), {"n_estimators": 1, "learning_rate": 0.5})
