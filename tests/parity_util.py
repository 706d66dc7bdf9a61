"""Shared helpers for GPU-vs-oracle parity tests (test infrastructure)."""
import numpy as np

import oracle_api as oa

OBJ = {"regression": oa.OBJ_L2, "binary": oa.OBJ_LOGISTIC, "multiclass": oa.OBJ_SOFTMAX}


def make_data(seed, n, f, kind="regression", n_classes=3, nan_frac=0.0, cat_cols=(), n_cat=12, zero_frac=0.0):
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(n, f))
    if zero_frac > 0:  # features 1.. are mostly one value (a dominant bin)
        X[:, 1:][rng.random((n, f - 1)) < zero_frac] = 0.0
    for c in cat_cols:
        X[:, c] = rng.integers(0, n_cat, size=n).astype(np.float64)
    if nan_frac > 0:
        mask = rng.random((n, f)) < nan_frac
        for c in cat_cols:
            mask[:, c] = False
        X[mask] = np.nan
    Z = np.nan_to_num(X)
    if kind == "regression":
        y = np.sin(3 * Z[:, 0]) + Z[:, 1] * Z[:, min(2, f - 1)] - 0.5 * Z[:, min(3, f - 1)] ** 2
        for c in cat_cols:
            y = y + np.cos(X[:, c])
        y = y + 0.1 * rng.normal(size=n)
    elif kind == "binary":
        s = Z[:, : min(5, f)] @ rng.normal(0, 0.7, size=min(5, f)) + 0.5 * Z[:, 0] * Z[:, min(1, f - 1)]
        y = (rng.random(n) < 1 / (1 + np.exp(-s))).astype(np.float64)
    else:
        W = rng.normal(size=(f, n_classes))
        y = np.argmax(Z @ W + rng.gumbel(size=(n, n_classes)), axis=1).astype(np.float64)
    return X, y


def params_for(objective, rounds, leaves, min_data=20, quant=False, n_classes=1, extra=None):
    p = {"objective": objective, "num_iterations": rounds, "num_leaves": leaves,
         "min_data_in_leaf": min_data, "learning_rate": 0.1, "keep_training_scores": True}
    if objective == "multiclass":
        p["num_class"] = n_classes
    if quant:
        p["use_quantized_grad"] = True
    if extra:
        p.update(extra)
    return p


def oracle_kwargs(p):
    kw = dict(objective=OBJ[p["objective"]], n_classes=p.get("num_class", 1), num_rounds=p["num_iterations"],
              learning_rate=p["learning_rate"], num_leaves=p["num_leaves"],
              min_data_in_leaf=p["min_data_in_leaf"],
              mode=(oa.MODE_QUANT if p.get("use_quantized_grad")
                    else oa.MODE_FIXED52 if str(p.get("gpu_histogram_precision", "int32")) == "int64"
                    else oa.MODE_FIXED), exp_kind=1)
    for k in ("feature_fraction", "max_cat_to_onehot", "max_cat_threshold", "cat_smooth", "cat_l2",
              "min_data_per_group", "lambda_l2", "lambda_l1"):
        if k in p:
            kw[k] = p[k]
    if "min_sum_hessian_in_leaf" in p:
        kw["min_child_hess"] = p["min_sum_hessian_in_leaf"]
    if "num_grad_quant_bins" in p:
        kw["quant_bins"] = p["num_grad_quant_bins"]
    return kw


def assert_models_identical(gm, om, n_rows, check_raw=True):
    """Bit-for-bit equality of every tree array, value, gain and count, and of
    the training raw scores."""
    assert gm.num_trees == om.n_trees, f"tree count {gm.num_trees} vs oracle {om.n_trees}"
    for t in range(om.n_trees):
        g = gm.tree(t)
        nn = int(om.n_nodes[t])
        assert len(g["feature"]) == nn, f"tree {t}: {len(g['feature'])} nodes vs oracle {nn}"
        for key in ("feature", "threshold_bin", "left", "right", "default_left", "missing_bin", "count"):
            np.testing.assert_array_equal(g[key], getattr(om, key)[t, :nn], err_msg=f"tree {t} {key}")
        np.testing.assert_array_equal(g["cat_bits"], om.cat_bits[t, :nn], err_msg=f"tree {t} cat bits")
        np.testing.assert_array_equal(g["value"].view(np.uint64), om.value[t, :nn].view(np.uint64),
                                      err_msg=f"tree {t} values (bits)")
        np.testing.assert_array_equal(g["gain"].view(np.uint64), om.gain[t, :nn].view(np.uint64),
                                      err_msg=f"tree {t} gains (bits)")
    if check_raw:
        raw = gm.training_scores(n_rows)
        np.testing.assert_array_equal(raw.view(np.uint64), np.ravel(om.raw).view(np.uint64),
                                      err_msg="training raw scores (bits)")


def fp_tolerance_report(gm, om, n_rows, gain_rtol=1e-5, pred_rms=1e-5):
    """Compare a device fit with the oracle's Float64 CPU path (the reference's
    own device=cpu arithmetic) within floating-point tolerances: identical tree
    structure, split gains within gain_rtol relative, training raw scores
    within pred_rms RMS.  Returns a list of failure messages (empty = pass);
    a structural difference names the first divergent node and both gains, so
    a flipped near-tie is told apart from an error."""
    fails = []
    if gm.num_trees != om.n_trees:
        return [f"tree count {gm.num_trees} vs {om.n_trees}"]
    worst = 0.0
    for t in range(om.n_trees):
        g = gm.tree(t)
        nn = int(om.n_nodes[t])
        if len(g["feature"]) != nn:
            fails.append(f"tree {t}: {len(g['feature'])} nodes vs {nn}")
            continue
        for i in range(nn):
            same = (g["feature"][i] == om.feature[t, i] and g["threshold_bin"][i] == om.threshold_bin[t, i]
                    and g["left"][i] == om.left[t, i] and g["right"][i] == om.right[t, i])
            if not same:
                fails.append(f"tree {t} node {i}: split (feature {g['feature'][i]}, bin {g['threshold_bin'][i]}, "
                             f"gain {g['gain'][i]!r}) vs CPU (feature {om.feature[t, i]}, bin "
                             f"{om.threshold_bin[t, i]}, gain {om.gain[t, i]!r})")
                break
            if om.feature[t, i] >= 0:
                rel = abs(g["gain"][i] - om.gain[t, i]) / abs(om.gain[t, i])
                worst = max(worst, rel)
                if rel > gain_rtol:
                    fails.append(f"tree {t} node {i}: gain {g['gain'][i]!r} vs CPU {om.gain[t, i]!r} (rel {rel:.3g})")
    raw = gm.training_scores(n_rows)
    rms = float(np.sqrt(np.mean((raw - np.ravel(om.raw)) ** 2)))
    if rms > pred_rms:
        fails.append(f"training raw scores: RMS difference {rms:.3g} > {pred_rms}")
    return fails
