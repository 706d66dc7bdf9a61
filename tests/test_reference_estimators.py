"""The reference's own Python package (python/mojotrees, unchanged) over this
library's `_mojotrees` shim: it imports (the objective/metric registry
queries), loads model files, predicts, saves with feature names, and a
`device="gpu"` fit without a CUDA device refuses instead of falling back.

Runs where the reference tree is mounted (this test reads its Python package
at run time); skipped elsewhere.
"""
import os
import sys

import numpy as np
import pytest

from test_model_io import RAW_A, X_A, model_a, write

REF_PY = "/root/reference/python"
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
