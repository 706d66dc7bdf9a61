"""The reference's cross-feature tie rule (split.mojo:1335-1362; the
constructed ties of tests/test_split_tie_parity.mojo): per-feature bests are
folded in ascending feature order with a strict `>`, so when two features
score exactly the same, the lower feature wins.  Two identical columns tie at
every split."""
import numpy as np
import pytest

from parity_util import oracle_kwargs, params_for


def _duplicated(seed, n=4000):
    rng = np.random.default_rng(seed)
    x = rng.integers(0, 40, size=n)
    other = rng.integers(0, 40, size=n)
    y = np.sin(x / 6.0) + 0.3 * (other > 20) + 0.05 * rng.normal(size=n)
    # columns 1 and 2 are the same feature; column 0 is another
    bins = np.stack([other, x, x]).astype(np.uint8)
    return bins, y


def _split_features(trees):
    return [int(f) for t in trees for f in t if f >= 0]


def test_oracle_keeps_the_lower_of_two_identical_features(oracle):
    bins, y = _duplicated(3)
    for quant in (False, True):
        p = params_for("regression", 4, 15, quant=quant)
        m = oracle.train(bins, 40, y, **oracle_kwargs(p))
        feats = _split_features(m.feature[t, : m.n_nodes[t]] for t in range(m.n_trees))
        assert 1 in feats and 2 not in feats


@pytest.mark.gpu
def test_gpu_keeps_the_lower_of_two_identical_features(mtlib, oracle):
    bins, y = _duplicated(4)
    for quant in (False, True):
        p = params_for("regression", 4, 15, quant=quant)
        m = mtlib.train_binned(bins, 40, y, p)
        feats = _split_features(m.tree(t)["feature"] for t in range(m.num_trees))
        assert 1 in feats and 2 not in feats
