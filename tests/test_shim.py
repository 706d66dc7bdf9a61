"""The `_mojotrees` extension shim: parameter mapping and refusals (host only)."""
import numpy as np
import pytest

from mojoboost_b200 import _mojotrees


def test_param_mapping():
    s = _mojotrees.param_string(1, {"n_estimators": 7, "num_leaves": 63, "min_child_hess": 0.01,
                                    "max_bin": 63, "use_quantized_grad": True, "bagging_fraction": 1.0,
                                    "categorical_features": [2, 5]}).decode()
    for part in ("objective=binary", "num_iterations=7", "num_leaves=63", "min_sum_hessian_in_leaf=0.01",
                 "max_bin=63", "use_quantized_grad=true", "categorical_feature=2,5"):
        assert part in s


@pytest.mark.parametrize("params", [{"device": "cpu"}, {"bagging_fraction": 0.5}, {"max_depth": 6}])
def test_refusals(params):
    with pytest.raises(NotImplementedError):
        _mojotrees.param_string(0, params)


def test_unknown_objective_and_hook():
    with pytest.raises(NotImplementedError):
        _mojotrees.param_string(7, {})
    with pytest.raises(NotImplementedError):
        _mojotrees.predict_leaf_index


def test_fit_without_gpu_is_unsupported(mtlib):
    if mtlib.gpu_available():
        pytest.skip("a GPU is present")
    X = np.asfortranarray(np.random.default_rng(0).normal(size=(100, 3)))
    y = np.zeros(100)
    with pytest.raises(mtlib.UnsupportedError):
        _mojotrees.fit(X.ctypes.data, 100, 3, y.ctypes.data, 0, {"n_estimators": 2})
