"""Prediction on the device (mojotrees_predict_ex, MOJOTREES_DEVICE_GPU) equals
host prediction bit for bit: raw scores and responses, iteration ranges,
missing values and categorical features, multiclass."""
import numpy as np
import pytest

from test_model_io import RAW_A, X_A, model_a, write


def test_gpu_prediction_is_refused_without_a_device(mtlib, tmp_path):
    """No silent host fallback: a device request on a machine without a CUDA
    device is an error, not a host prediction."""
    if mtlib.gpu_available():
        pytest.skip("a CUDA device is present")
    m = mtlib.Model.load(write(tmp_path, "a.mbst", model_a(4)))
    with pytest.raises(mtlib.MojoTreesError) as ei:
        m.predict(X_A, raw_score=True, device="gpu")
    assert ei.value.code == -4


@pytest.mark.gpu
def test_gpu_prediction_of_a_model_file(mtlib, tmp_path):
    m = mtlib.Model.load(write(tmp_path, "a.mbst", model_a(4)))
    np.testing.assert_array_equal(m.predict(X_A, raw_score=True, device="gpu"), RAW_A)


@pytest.mark.gpu
@pytest.mark.parametrize("kind, quant", [("regression", False), ("binary", True), ("multiclass", False)])
def test_gpu_prediction_matches_host(mtlib, kind, quant):
    from parity_util import make_data, params_for
    nc = 4 if kind == "multiclass" else 1
    X, y = make_data(41, 30_000, 10, kind=kind, n_classes=nc, nan_frac=0.05, cat_cols=(2,), n_cat=20)
    p = params_for(kind, 6, 31, quant=quant, n_classes=nc, extra={"categorical_feature": "2"})
    m = mtlib.train_dense(X, y, p)
    Xt, _ = make_data(42, 7_001, 10, kind=kind, n_classes=nc, nan_frac=0.05, cat_cols=(2,), n_cat=25)
    for raw in (True, False):
        for s0, n in ((0, 0), (0, 2), (3, 0), (2, 3), (6, 0)):
            host = m.predict(Xt, raw_score=raw, start_iteration=s0, num_iteration=n)
            dev = m.predict(Xt, raw_score=raw, start_iteration=s0, num_iteration=n, device="gpu")
            np.testing.assert_array_equal(dev, host)
    assert m.predict(Xt[:0], device="gpu").size == 0
