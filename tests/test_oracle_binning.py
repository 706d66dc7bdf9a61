"""The oracle's serial restatement of the reference binner against the
product's host binner (block-parallel sample draws, radix sorts, OpenMP):
identical bins, missing bins and category counts.  The oracle binner is
itself pinned by the golden fixtures (test_golden.py), so this pins the
product binner to the reference's rule on inputs the fixtures do not reach:
sampled fits (more rows than the 200k sample), ties, NaN, signed zeros,
infinities, categorical codes (unseen, negative, above the kept set)."""
import numpy as np
import pytest


def _cases():
    rng = np.random.default_rng(11)
    n = 260_000  # above the 200k edge-fitting sample
    X = rng.normal(size=(n, 6))
    X[:, 1] = np.round(X[:, 1] * 3)  # heavy ties, few levels
    X[rng.random(n) < 0.05, 2] = np.nan
    X[:, 3] = np.where(rng.random(n) < 0.5, 0.0, -0.0)
    X[: 10, 3] = [np.inf, -np.inf, 1.0, 2.0, np.nan, 5.0, -5.0, 0.5, 1e308, -1e308]
    X[:, 4] = rng.integers(-3, 400, size=n).astype(np.float64)  # categorical, more codes than bins
    X[rng.random(n) < 0.01, 4] = np.nan
    X[:, 5] = rng.lognormal(size=n)
    yield "sampled", X, dict(max_bin=255, categorical=[4])
    small = rng.normal(size=(3000, 3))
    small[::7, 0] = np.nan
    yield "small63", small, dict(max_bin=63)
    yield "tiny", rng.normal(size=(37, 2)), dict(max_bin=255)
    yield "two_bins", rng.normal(size=(5000, 2)), dict(max_bin=2)


@pytest.mark.parametrize("name,X,kw", list(_cases()), ids=[c[0] for c in _cases()])
def test_oracle_binner_equals_product_binner(name, X, kw, oracle, mtlib):
    ob, omb, onc, onb = oracle.bin_dense(X, **kw)
    p = {"max_bin": kw["max_bin"]}
    if kw.get("categorical"):
        p["categorical_feature"] = ",".join(str(c) for c in kw["categorical"])
    pb, pmb, pnc, pnb = mtlib.bin_dense(X, p)
    assert onb == pnb
    np.testing.assert_array_equal(omb, pmb)
    np.testing.assert_array_equal(onc, pnc)
    np.testing.assert_array_equal(ob, pb)
