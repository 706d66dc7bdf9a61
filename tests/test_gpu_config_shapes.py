"""GPU trainer against the CPU oracle at the benchmark configurations' shapes.

The parity cases of test_gpu_parity.py are small; these grow a few trees at
the row and feature counts of the benchmark configurations themselves, where
the launch geometry differs: full 255-leaf trees over 10M rows, ten class
planes per round, and more than 2^26 rows on one GPU (row ids no longer fit
the packed row word of the histogram kernel, so it takes its other cell
layout).  Every tree array, value and gain bit and every training raw score
must equal the oracle's, as in the small cases.

Data follows the configurations' published recipes (synthetic, seeded); the
row count of the multiclass case is reduced, its feature count, class count,
bins and leaves are those of the configuration.
"""
import numpy as np
import pytest

import bench
from parity_util import assert_models_identical, oracle_kwargs, params_for

pytestmark = pytest.mark.gpu


def config1_data(n=1_000_000, seed=0):
    """28 features, half ~N(0,1) and half ~U(0,1); y = sin(3 x0)
    + x1 x2 - 0.5 x3^2 + 0.1 N(0,1)."""
    rng = np.random.default_rng(seed)
    X = np.empty((n, 28))
    X[:, :14] = rng.standard_normal((n, 14))
    X[:, 14:] = rng.random((n, 14))
    y = np.sin(3 * X[:, 0]) + X[:, 1] * X[:, 2] - 0.5 * X[:, 3] ** 2 + 0.1 * rng.standard_normal(n)
    return X, y


def config4_data(n, seed=3, k=10, f=64):
    """class = argmax of k random linear projections plus Gumbel noise."""
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((n, f))
    W = rng.standard_normal((f, k))
    y = np.argmax(X @ W + rng.gumbel(size=(n, k)), axis=1).astype(np.float64)
    return X, y


def config5_bins(n, seed=4, f=128):
    """pre-binned uint8 uniform over 255 bins; label ~ Bernoulli(
    sigmoid(sum over 16 features of a per-bin effect ~ N(0, 0.2)))."""
    rng = np.random.default_rng(seed)
    bins = rng.integers(0, 255, size=(f, n), dtype=np.uint8)
    eff = rng.normal(0.0, 0.2, size=(16, 255))
    s = np.zeros(n)
    for j in range(16):
        s += eff[j][bins[j]]
    y = (rng.random(n) < 1.0 / (1.0 + np.exp(-s))).astype(np.float64)
    return bins, y


def _fit_both(mtlib, oracle, bins, nb, y, p, mbin=None, ncat=None):
    gm = mtlib.train_binned(bins, nb, y, p, missing_bin=mbin, n_categories=ncat)
    om = oracle.train(bins, nb, y, missing_bin=mbin, n_cats=ncat, **oracle_kwargs(p))
    return gm, om


def test_config1_shape_fixed(mtlib, oracle):
    """L2, 1M x 28, 255 bins, 255 leaves, fixed-point gradients."""
    X, y = config1_data()
    p = params_for("regression", 3, 255, extra={"max_bin": 255})
    bins, mbin, ncat, nb = mtlib.bin_dense(X, {"max_bin": 255})
    gm, om = _fit_both(mtlib, oracle, bins, nb, y, p, mbin, ncat)
    assert_models_identical(gm, om, len(y))


def test_config2_shape_quant(mtlib, oracle):
    """configs[1], the benchmark workload: binary logistic, 10M x 100, 255
    bins, 255 leaves, int8 quantized gradients."""
    X, y = bench.make_data(bench.N_ROWS, seed=1)
    bins, mbin, ncat, nb = mtlib.bin_dense(np.asfortranarray(X.T.astype(np.float64)), {"max_bin": 255})
    del X
    p = params_for("binary", 3, 255, quant=True, extra={"max_bin": 255})
    gm, om = _fit_both(mtlib, oracle, bins, nb, y, p, mbin, ncat)
    assert_models_identical(gm, om, len(y))


def test_config4_shape_multiclass(mtlib, oracle):
    """configs[3] at 1M rows: softmax K=10, 64 features, 255 bins, 63 leaves
    (ten histograms per round)."""
    X, y = config4_data(1_000_000)
    p = params_for("multiclass", 2, 63, n_classes=10, extra={"max_bin": 255})
    bins, mbin, ncat, nb = mtlib.bin_dense(X, {"max_bin": 255})
    gm, om = _fit_both(mtlib, oracle, bins, nb, y, p, mbin, ncat)
    assert_models_identical(gm, om, len(y))


def test_config5_shape_beyond_2pow26_rows(mtlib, oracle):
    """configs[4] on one GPU with 2^26 + 1M rows: pre-binned uint8 x 128,
    quantized gradients, 255 leaves."""
    n = (1 << 26) + 1_000_000
    bins, y = config5_bins(n)
    p = params_for("binary", 2, 255, quant=True)
    gm, om = _fit_both(mtlib, oracle, bins, 255, y, p)
    assert_models_identical(gm, om, n)
