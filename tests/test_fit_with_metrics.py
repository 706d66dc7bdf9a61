"""The shim's validation-scored fits (`fit_with_metrics`, the reference's
custom_metric.mojo round loop): staged raw scores, per-round metric history,
early stopping and the cut to the best round.  The device fit is replaced by
a model file here, so the scoring runs without a GPU; the GPU test at the end
runs the real fit."""
import ctypes

import numpy as np
import pytest

from test_model_io import b, frow, row, write

LR = 0.3


def model_text(n_iter, K=1):
    """n_iter iterations over two features (f0 edges 0.5, 1.5 and a missing
    bin; f1 edge 0.0): iteration i splits f0 at bin i % 2 and f1 below."""
    s = "mojotrees v4\n"
    if K == 1:
        s += f"objective 0\nlearning_rate {b(LR)}\nbase_score {b(0.125)}\n"
    else:
        s += f"multiclass {K}\nlearning_rate {b(LR)}\nbase_scores" + "".join(f" {b(0.1 * k)}" for k in range(K)) + "\n"
    s += "mapper 2 255 3\n" + frow([0.5, 1.5, 0.0]) + row([0, 2, 3]) + row([3, -1]) + f"trees {n_iter * K}\n"
    for i in range(n_iter * K):
        vals = [0.0, 0.0, 1.0 + 0.37 * i, -0.5 - 0.11 * i, 0.25 * (i % 3) - 0.3]
        s += "tree 5 3\n" + row([0, 1, -1, -1, -1]) + row([i % 2, 0, -1, -1, -1]) + row([1, 3, -1, -1, -1])
        s += row([2, 4, -1, -1, -1]) + frow(vals) + row([i % 2, 0, 0, 0, 0]) + row([3, -1, -1, -1, -1])
        s += "counts 0\ngains 0\n"
    return s


@pytest.fixture()
def shim(mtlib):
    from mojoboost_b200 import _mojotrees
    return _mojotrees


def _valid(rng, n):
    X = rng.normal(size=(n, 2)) * 1.2
    X[rng.random((n, 2)) < 0.1] = np.nan
    return np.asfortranarray(X), rng.normal(size=n)


def test_staged_raw_equals_prediction(mtlib, tmp_path):
    for K in (1, 3):
        m = mtlib.Model.load(write(tmp_path, f"m{K}.mbst", model_text(6, K)))
        X, _ = _valid(np.random.default_rng(K), 500)
        bins = m.bin_rows(X)
        raw = np.tile(m.base_scores(), len(X))
        for i in range(6):
            m.add_iteration_raw(bins, i, raw)
            want = m.predict(X, raw_score=True, num_iteration=i + 1).reshape(-1)
            np.testing.assert_array_equal(raw, want)
        assert m.prefix(2).num_iterations == 2
        np.testing.assert_array_equal(m.prefix(2).predict(X, raw_score=True),
                                      m.predict(X, raw_score=True, num_iteration=2))


def _run(shim, monkeypatch, tmp_path, metric_values=None, esr=0, n_iter=8, higher=0, min_delta=0.0):
    full = shim.load(write(tmp_path, "full.mbst", model_text(n_iter)))
    monkeypatch.setattr(shim, "fit", lambda *a: full)
    rng = np.random.default_rng(5)
    (Xa, ya), (Xb, yb) = _valid(rng, 300), _valid(rng, 200)
    pred = np.zeros(300)
    calls = []

    def bridge(m, v):
        n = 300 if v == 0 else 200
        p = pred[:n].copy()
        calls.append((m, v, p))
        if metric_values is not None and m == 0:  # the same script on both sets
            return metric_values[sum(1 for c in calls if c[0] == 0 and c[1] == v) - 1]
        y = ya if v == 0 else yb
        return float(np.mean((p - y) ** 2))

    params = {"valid_sets": [("a", Xa.ctypes.data, 300, ya.ctypes.data), ("b", Xb.ctypes.data, 200, yb.ctypes.data)],
              "n_valid": 2, "metrics": [("m0", higher, 1), ("l2", 0, 0)], "n_metrics": 2, "primary_metric": 0,
              "early_stopping_rounds": esr, "min_delta": min_delta, "pred_addr": pred.ctypes.data,
              "has_callback": 0, "n_estimators": n_iter}
    out = shim.fit_with_metrics(0, 10, 2, 0, 0, bridge, params)
    return full, (Xa, ya, Xb, yb), calls, out


def test_history_is_the_staged_predictions(shim, monkeypatch, tmp_path):
    full, (Xa, ya, Xb, yb), calls, out = _run(shim, monkeypatch, tmp_path)
    model, values, n_rounds, best, best_score, stopped = out
    assert n_rounds == 9 and stopped == 0 and model.num_iterations == 8  # no early stopping: full ensemble
    assert len(values) == 9 * 2 * 2
    for r in range(9):
        pa = full.predict(Xa, raw_score=True, num_iteration=r) if r else np.full(300, 0.125)
        pb = full.predict(Xb, raw_score=True, num_iteration=r) if r else np.full(200, 0.125)
        np.testing.assert_array_equal(calls[4 * r][2], pa)
        np.testing.assert_array_equal(calls[4 * r + 2][2], pb)
        assert values[4 * r + 1] == float(np.mean((pa - ya) ** 2))
        assert values[4 * r + 3] == float(np.mean((pb - yb) ** 2))
    l2a = [values[4 * r] for r in range(9)]
    assert best == int(np.argmin(l2a)) and best_score == min(l2a)


def test_early_stopping_and_cut(shim, monkeypatch, tmp_path):
    """Any flagged (set, metric) pair going early_stopping_rounds rounds
    without a strict improvement stops the fit; the model is cut to the
    primary metric's best round on the first set."""
    seq = [5.0, 4.0, 3.0, 3.0, 3.5, 3.2, 9.0, 9.0, 9.0]
    model, values, n_rounds, best, best_score, stopped = _run(shim, monkeypatch, tmp_path, seq, esr=3)[3]
    assert (stopped, best, best_score) == (1, 2, 3.0)
    assert n_rounds == 6 and model.num_iterations == 2  # rounds 0..5 scored; 5 - 2 >= 3
    # a tie is not an improvement, and min_delta must be cleared strictly
    model, values, n_rounds, best, best_score, stopped = _run(shim, monkeypatch, tmp_path,
                                                              [5.0, 4.6, 4.5, 4.0, 3.9, 3.95, 3.6, 3.6, 3.6],
                                                              esr=3, min_delta=0.5)[3]
    assert (best, stopped, n_rounds) == (3, 1, 7)  # 4.6, 4.5 do not clear 5 - 0.5 strictly, 4.0 does; 3.6 does not clear 3.5
    # higher is better
    model, values, n_rounds, best, best_score, stopped = _run(shim, monkeypatch, tmp_path,
                                                              [1.0, 2.0, 3.0, 4.0, 4.0, 3.9, 9.0, 9.0, 9.0],
                                                              esr=2, higher=1)[3]
    assert (best, best_score, stopped, n_rounds, model.num_iterations) == (3, 4.0, 1, 6, 3)
    # no early stopping: every round scored, the full ensemble kept, best reported
    model, values, n_rounds, best, best_score, stopped = _run(shim, monkeypatch, tmp_path, seq, esr=0)[3]
    assert (best, stopped, n_rounds, model.num_iterations) == (2, 0, 9, 8)


def test_callbacks_are_refused(shim):
    with pytest.raises(NotImplementedError):
        shim.fit_with_metrics(0, 1, 1, 0, 0, None, {"has_callback": 1})


@pytest.mark.gpu
def test_gpu_fit_with_metrics(shim, mtlib):
    """The real device fit scored on a validation set: the history is the l2
    of the staged predictions and the early-stopping cut is a prefix."""
    from parity_util import make_data
    X, y = make_data(61, 4000, 5)
    Xv, yv = make_data(62, 1000, 5)
    Xf, Xvf = np.asfortranarray(X), np.asfortranarray(Xv)
    y, yv = np.ascontiguousarray(y), np.ascontiguousarray(yv)
    pred = np.zeros(1000)
    bridge = lambda m, v: float(np.mean((pred - yv) ** 2))
    params = {"n_estimators": 30, "num_leaves": 15, "valid_sets": [("v", Xvf.ctypes.data, 1000, yv.ctypes.data)],
              "n_valid": 1, "metrics": [("l2", 0, 1)], "n_metrics": 1, "primary_metric": 0,
              "early_stopping_rounds": 3, "min_delta": 0.0, "pred_addr": pred.ctypes.data, "has_callback": 0}
    model, values, n_rounds, best, best_score, stopped = shim.fit_with_metrics(
        Xf.ctypes.data, 4000, 5, y.ctypes.data, 0, bridge, params)
    assert model.num_iterations == best and values[best] == best_score == min(values)
    for r in (1, best):
        p = model.predict(Xv, raw_score=True, num_iteration=r)
        assert values[r] == float(np.mean((p - yv) ** 2))
