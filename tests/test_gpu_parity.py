"""GPU trainer (through the C ABI) vs the CPU oracle: bit-exact trees.

Both integer histogram modes are exact by construction, so every tree array,
every leaf value and gain (as IEEE bits) and every training raw score must be
identical to the oracle run in the same mode on the same bins.  Cases follow
the reference's own test strategy (tests/test_gpu_training.mojo,
tests/test_host_replica.mojo): several objectives, missing values,
categorical splits, feature sampling, tiny and ragged shapes.
"""
import os

import numpy as np
import pytest

from parity_util import assert_models_identical, make_data, oracle_kwargs, params_for

pytestmark = pytest.mark.gpu

CASES = {
    # name: (data kwargs, params kwargs, max_bin)
    "l2_fixed": (dict(seed=1, n=50_000, f=28), dict(objective="regression", rounds=4, leaves=63), 255),
    "l2_quant": (dict(seed=2, n=40_000, f=28), dict(objective="regression", rounds=4, leaves=63, quant=True), 255),
    "binary_fixed": (dict(seed=3, n=30_000, f=20, kind="binary"), dict(objective="binary", rounds=4, leaves=31), 255),
    "binary_quant": (dict(seed=4, n=30_000, f=20, kind="binary"),
                     dict(objective="binary", rounds=5, leaves=63, quant=True), 255),
    "binary_quant_large": (dict(seed=16, n=300_000, f=100, kind="binary"),
                           dict(objective="binary", rounds=2, leaves=255, quant=True), 255),
    "multiclass_fixed": (dict(seed=5, n=20_000, f=12, kind="multiclass", n_classes=4),
                         dict(objective="multiclass", rounds=3, leaves=15, n_classes=4), 255),
    "multiclass_quant": (dict(seed=6, n=20_000, f=12, kind="multiclass", n_classes=4),
                         dict(objective="multiclass", rounds=3, leaves=15, n_classes=4, quant=True), 255),
    "missing_cat_fixed": (dict(seed=7, n=20_000, f=8, nan_frac=0.1, cat_cols=(2, 5), n_cat=12),
                          dict(objective="regression", rounds=4, leaves=31,
                               extra={"categorical_feature": "2,5", "min_data_per_group": 20, "cat_smooth": 5.0}), 63),
    "missing_cat_quant": (dict(seed=8, n=20_000, f=8, nan_frac=0.1, cat_cols=(2, 5), n_cat=3, kind="binary"),
                          dict(objective="binary", rounds=4, leaves=31, quant=True,
                               extra={"categorical_feature": "2,5"}), 63),
    # quantizer widths that select each shared-memory cell layout of the
    # histogram: 16 keeps 16-bit packed cells, 64 and 254 the 32-bit ones
    "binary_quant16": (dict(seed=12, n=60_000, f=40, kind="binary"),
                       dict(objective="binary", rounds=3, leaves=63, quant=True,
                            extra={"num_grad_quant_bins": 16}), 255),
    "binary_quant64": (dict(seed=13, n=60_000, f=40, kind="binary"),
                       dict(objective="binary", rounds=3, leaves=63, quant=True,
                            extra={"num_grad_quant_bins": 64}), 255),
    "l2_quant254": (dict(seed=14, n=40_000, f=20), dict(objective="regression", rounds=3, leaves=31, quant=True,
                                                       extra={"num_grad_quant_bins": 254}), 127),
    "feature_fraction": (dict(seed=9, n=20_000, f=24), dict(objective="regression", rounds=4, leaves=31,
                                                            extra={"feature_fraction": 0.5}), 255),
    "wide_features": (dict(seed=10, n=10_000, f=150), dict(objective="regression", rounds=2, leaves=31), 255),
    "tiny_ragged": (dict(seed=11, n=37, f=3), dict(objective="regression", rounds=3, leaves=4, min_data=3), 255),
    "two_leaves": (dict(seed=12, n=5_000, f=5, kind="binary"), dict(objective="binary", rounds=3, leaves=2), 255),
    # L1 shrinkage, no L2 and a binding minimum hessian: the split scan's
    # integer hessian thresholds and its pruning bounds under soft thresholds
    "regularised_fixed": (dict(seed=17, n=30_000, f=16), dict(objective="regression", rounds=4, leaves=31, min_data=2,
                                                             extra={"lambda_l1": 0.5, "lambda_l2": 0.0,
                                                                    "min_sum_hessian_in_leaf": 40.0}), 255),
    # packed 32-bit cells with spills: quantizer widths 2 and 6 (other field
    # geometries), and features with a dominant bin (a cell takes most rows,
    # so its count field spills to the global cells many times per launch)
    "binary_quant2": (dict(seed=23, n=60_000, f=24, kind="binary"),
                      dict(objective="binary", rounds=3, leaves=63, quant=True, extra={"num_grad_quant_bins": 2}), 255),
    "binary_quant6": (dict(seed=24, n=60_000, f=24, kind="binary"),
                      dict(objective="binary", rounds=3, leaves=63, quant=True, extra={"num_grad_quant_bins": 6}), 255),
    "binary_quant_skewed": (dict(seed=25, n=400_000, f=40, kind="binary", zero_frac=0.97),
                            dict(objective="binary", rounds=3, leaves=127, quant=True), 63),
    # more than 16k rows per CTA at the root: the 16-bit cells take several
    # windows, and the dominant bins' cells go to the work slot between them
    "binary_quant_skewed_large": (dict(seed=26, n=3_000_000, f=8, kind="binary", zero_frac=0.97),
                                  dict(objective="binary", rounds=2, leaves=31, quant=True), 63),
    # fixed point with the 2^52 bound and Int64 cells (gpu_histogram_precision=int64)
    "l2_fixed52": (dict(seed=19, n=50_000, f=28), dict(objective="regression", rounds=4, leaves=63,
                                                      extra={"gpu_histogram_precision": "int64"}), 255),
    "binary_fixed52": (dict(seed=20, n=30_000, f=20, kind="binary", nan_frac=0.05),
                       dict(objective="binary", rounds=4, leaves=31, extra={"gpu_histogram_precision": "int64"}), 255),
    "multiclass_fixed52": (dict(seed=21, n=20_000, f=12, kind="multiclass", n_classes=4),
                           dict(objective="multiclass", rounds=3, leaves=15, n_classes=4,
                                extra={"gpu_histogram_precision": "int64"}), 255),
    "missing_cat_fixed52": (dict(seed=22, n=20_000, f=8, nan_frac=0.1, cat_cols=(2, 5), n_cat=12),
                            dict(objective="regression", rounds=3, leaves=31,
                                 extra={"categorical_feature": "2,5", "min_data_per_group": 20, "cat_smooth": 5.0,
                                        "gpu_histogram_precision": "int64"}), 63),
    # sparse histograms (fixed point, a row listing few bins outside its
    # features' default bins): constant hessian (g, count cells), binary with
    # missing values and categoricals (g, h, count), multiclass, and a
    # configs[2]-like width of 400 columns at 63 bins
    "sparse_l2_fixed": (dict(seed=27, n=80_000, f=60, zero_frac=0.9),
                        dict(objective="regression", rounds=4, leaves=63), 63),
    "sparse_binary_fixed": (dict(seed=28, n=60_000, f=40, kind="binary", zero_frac=0.85, nan_frac=0.03,
                                 cat_cols=(3, 7), n_cat=20),
                            dict(objective="binary", rounds=4, leaves=31, extra={"categorical_feature": "3,7"}), 255),
    "sparse_multiclass_fixed": (dict(seed=29, n=30_000, f=24, kind="multiclass", n_classes=3, zero_frac=0.9),
                                dict(objective="multiclass", rounds=3, leaves=15, n_classes=3), 63),
    "sparse_wide_fixed": (dict(seed=30, n=40_000, f=400, zero_frac=0.9),
                          dict(objective="regression", rounds=2, leaves=127), 63),
    "regularised_quant": (dict(seed=18, n=30_000, f=16, kind="binary"),
                          dict(objective="binary", rounds=4, leaves=31, quant=True, min_data=2,
                               extra={"lambda_l1": 0.2, "lambda_l2": 0.0, "min_sum_hessian_in_leaf": 3.0}), 255),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_gpu_matches_oracle(case, mtlib, oracle):
    dkw, pkw, max_bin = CASES[case]
    pkw = dict(pkw)
    X, y = make_data(**dkw)
    extra = pkw.pop("extra", {})
    p = params_for(pkw.pop("objective"), pkw.pop("rounds"), pkw.pop("leaves"), extra=extra, **pkw)
    p["max_bin"] = max_bin
    bins, mbin, ncat, nb = mtlib.bin_dense(X, {k: v for k, v in p.items() if k in ("max_bin", "categorical_feature")})
    gm = mtlib.train_binned(bins, nb, y, p, missing_bin=mbin, n_categories=ncat)
    om = oracle.train(bins, nb, y, missing_bin=mbin, n_cats=ncat, **oracle_kwargs(p))
    assert_models_identical(gm, om, len(y))


def test_gpu_no_split_single_leaf_trees(mtlib, oracle):
    """min_data_in_leaf above n/2: the root never splits; every tree is one
    leaf, identical to the oracle's (its value is the Float32-narrowed
    gradient sum, not exactly 0, so the fit does not stop early)."""
    X, y = make_data(13, 1000, 4)
    p = params_for("regression", 5, 31, min_data=600)
    bins, mbin, ncat, nb = mtlib.bin_dense(X, {"max_bin": 255})
    gm = mtlib.train_binned(bins, nb, y, p, missing_bin=mbin, n_categories=ncat)
    om = oracle.train(bins, nb, y, missing_bin=mbin, n_cats=ncat, **oracle_kwargs(p))
    assert_models_identical(gm, om, len(y))
    assert all(len(gm.tree(t)["feature"]) == 1 for t in range(gm.num_trees))


def test_gpu_constant_target_stops(mtlib, oracle):
    """A constant L2 target: gradients are exactly 0, the first tree is a
    zero-valued leaf and the fit stops with no tree (boosting.mojo:2898-2907)."""
    X, _ = make_data(15, 2000, 4)
    y = np.full(2000, 0.25)
    p = params_for("regression", 5, 31)
    bins, mbin, ncat, nb = mtlib.bin_dense(X, {"max_bin": 255})
    gm = mtlib.train_binned(bins, nb, y, p, missing_bin=mbin, n_categories=ncat)
    om = oracle.train(bins, nb, y, missing_bin=mbin, n_cats=ncat, **oracle_kwargs(p))
    assert gm.num_trees == om.n_trees == 0


def test_gpu_dense_entry_matches_binned(mtlib):
    """mojotrees_train_dense (host binning + device) equals the binned entry."""
    X, y = make_data(14, 8000, 6, kind="binary", nan_frac=0.05)
    p = params_for("binary", 3, 15)
    dm = mtlib.train_dense(X, y, p)
    bins, mbin, ncat, nb = mtlib.bin_dense(X, {})
    bm = mtlib.train_binned(bins, nb, y, p, missing_bin=mbin, n_categories=ncat)
    assert dm.num_trees == bm.num_trees
    for t in range(dm.num_trees):
        a, b = dm.tree(t), bm.tree(t)
        for k in a:
            np.testing.assert_array_equal(a[k], b[k])
    np.testing.assert_array_equal(dm.predict(X, raw_score=True), bm.predict_binned(bins))


def test_gpu_device_binning_matches_host(mtlib):
    """Columns binned on the device equal the host transform: NaNs (with and
    without a missing bin), categorical codes (kept, unseen, negative, huge,
    fractional), values on the edges, +-0 and infinities."""
    rng = np.random.default_rng(21)
    n = 70_000
    X = rng.normal(size=(n, 7))
    X[rng.random(n) < 0.1, 0] = np.nan
    X[:, 1] = np.round(rng.normal(size=n), 1)  # few distinct levels
    X[: n // 3, 1] = -0.0
    X[n // 3 : n // 2, 1] = 0.0
    X[:, 2] = rng.integers(0, 40, size=n).astype(np.float64)
    X[::97, 2] = -3.0
    X[::89, 2] = 1e6  # unseen code
    X[::83, 2] = 2.5
    X[::79, 2] = np.nan
    X[::71, 3] = np.inf
    X[::73, 3] = -np.inf
    X[:, 4] = 1.0  # constant
    X[:, 5] = rng.integers(0, 600, size=n).astype(np.float64)  # more codes than bins
    X[:, 6] = rng.exponential(size=n)
    params = {"categorical_feature": "2,5", "max_bin": 63}
    host = mtlib.bin_dense(X, params)
    dev = mtlib.bin_dense(X, params, device=True)
    for a, b in zip(host, dev):
        np.testing.assert_array_equal(a, b)
    X[5, 2] = 1e12  # a categorical code beyond int32 is an input error on both paths
    for device in (False, True):
        with pytest.raises(mtlib.MojoTreesError):
            mtlib.bin_dense(X, params, device=device)


def test_gpu_device_binning_row_chunks(mtlib):
    """Columns longer than one 32 MB staging chunk (4,194,304 float64 values)
    are streamed as row ranges of one feature; the last range is ragged.  The
    device bins equal the host transform."""
    rng = np.random.default_rng(22)
    n = 4_500_001
    X = np.empty((n, 3))
    X[:, 0] = rng.normal(size=n)
    X[:, 1] = rng.integers(0, 30, size=n).astype(np.float64)
    X[:, 2] = rng.exponential(size=n)
    X[::101, 2] = np.nan
    params = {"categorical_feature": "1", "max_bin": 255}
    host = mtlib.bin_dense(X, params)
    dev = mtlib.bin_dense(X, params, device=True)
    for a, b in zip(host, dev):
        np.testing.assert_array_equal(a, b)


def test_gpu_round_times_and_stats(mtlib):
    X, y = make_data(17, 20_000, 10, kind="binary")
    bins, mbin, ncat, nb = mtlib.bin_dense(X, {})
    m = mtlib.train_binned(bins, nb, y, params_for("binary", 4, 31, quant=True), missing_bin=mbin,
                           n_categories=ncat)
    rt = m.round_times_ms()
    assert len(rt) == 4 and np.all(rt > 0)
    st = m.stats()
    assert st["hist_rows"] >= 4 * 20_000 and st["kernel_launches"] > 0


@pytest.mark.skipif(os.environ.get("MOJOTREES_TEST_SCAN_COMPACT") != "1",
                    reason="the compact split scan is an opt-in variant; set MOJOTREES_TEST_SCAN_COMPACT=1")
@pytest.mark.parametrize("case", ["binary_quant", "missing_cat_fixed", "regularised_quant", "binary_quant_large"])
def test_gpu_compact_scan_matches_oracle(case, mtlib, oracle, monkeypatch):
    """MOJOTREES_SCAN=compact (candidate evaluation out of line) grows the
    oracle's trees bit for bit, like the default scan."""
    monkeypatch.setenv("MOJOTREES_SCAN", "compact")
    test_gpu_matches_oracle(case, mtlib, oracle)


@pytest.mark.parametrize("case", ["binary_quant", "missing_cat_fixed", "binary_quant_large"])
def test_gpu_replay_batch_selection_matches_oracle(case, mtlib, oracle, monkeypatch):
    """MOJOTREES_COMMIT_SELECT=replay (each speculative batch chosen by a
    serial replay of the pick loop instead of by bottleneck keys) decides
    only which leaves are built early; the trees stay the oracle's."""
    monkeypatch.setenv("MOJOTREES_COMMIT_SELECT", "replay")
    test_gpu_matches_oracle(case, mtlib, oracle)


@pytest.mark.parametrize("case", ["l2_fixed", "missing_cat_fixed", "sparse_l2_fixed"])
def test_gpu_forced_histogram_kind_matches_oracle(case, mtlib, oracle, monkeypatch):
    """MOJOTREES_HIST_SPARSE=1 (sparse histograms even where rows list
    nearly every bin) and =0 (dense histograms for sparse data) grow the
    oracle's trees as well."""
    for v in ("1", "0"):
        monkeypatch.setenv("MOJOTREES_HIST_SPARSE", v)
        test_gpu_matches_oracle(case, mtlib, oracle)


def test_gpu_sparse_histograms_are_chosen(mtlib):
    """Sparse data in a fixed-point mode takes the sparse histogram path, and
    its row lists hold only the entries outside the default bins."""
    X, y = make_data(31, 20_000, 30, zero_frac=0.9)
    bins, mbin, ncat, nb = mtlib.bin_dense(X, {"max_bin": 63})
    m = mtlib.train_binned(bins, nb, y, params_for("regression", 2, 15), missing_bin=mbin, n_categories=ncat)
    entries = m.stats()["hist_sparse_entries"]
    default = np.array([np.bincount(bins[f], minlength=256).argmax() for f in range(bins.shape[0])])
    assert entries == int((bins != default[:, None]).sum())
