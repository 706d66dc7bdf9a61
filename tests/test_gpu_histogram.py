"""The per-leaf histogram kernel alone, through mojotrees_b200_histogram_u8,
against integer sums computed on the host (the oracle's histogram is exact
integer sums of the quantized pairs; quantized_gradient.mojo:2947-3195)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def host_histogram(bins, n_bins, g, h, rows):
    F = bins.shape[0]
    out = np.zeros((F, 3, n_bins), np.int64)
    for f in range(F):
        b = bins[f, rows]
        np.add.at(out[f, 0], b, g[rows].astype(np.int64))
        np.add.at(out[f, 1], b, h[rows].astype(np.int64))
        np.add.at(out[f, 2], b, 1)
    return out


@pytest.mark.parametrize("n,F,B,frac", [(200_000, 100, 255, 1.0), (100_000, 150, 255, 0.3),
                                        (5_000, 28, 63, 0.01), (70_000, 7, 2, 0.5), (1, 3, 16, 1.0)])
def test_histogram_matches_host(mtlib, n, F, B, frac):
    rng = np.random.default_rng(n + F)
    bins = rng.integers(0, B, size=(F, n), dtype=np.uint8)
    g = rng.integers(-2, 3, size=n).astype(np.int8)
    h = rng.integers(0, 5, size=n).astype(np.uint8)
    rows = np.sort(rng.choice(n, size=max(1, int(n * frac)), replace=False)).astype(np.int32)
    got = mtlib.histogram_u8(bins, B, g, h, rows=rows)
    np.testing.assert_array_equal(got, host_histogram(bins, B, g, h, rows))


def test_histogram_all_rows_and_errors(mtlib):
    rng = np.random.default_rng(1)
    bins = rng.integers(0, 255, size=(20, 40_000), dtype=np.uint8)
    g = rng.integers(-2, 3, size=40_000).astype(np.int8)
    h = rng.integers(0, 5, size=40_000).astype(np.uint8)
    got = mtlib.histogram_u8(bins, 255, g, h)
    np.testing.assert_array_equal(got, host_histogram(bins, 255, g, h, np.arange(40_000)))
    with pytest.raises(mtlib.MojoTreesError):
        mtlib.histogram_u8(bins, 255, (g * 3).astype(np.int8), h)


@pytest.mark.parametrize("qb", [2, 16, 64, 254])
def test_histogram_quantizer_widths(mtlib, qb):
    """Every quantizer width, at the extremes of its range, over more rows
    than one flush of the packed 16-bit cells covers."""
    rng = np.random.default_rng(qb)
    n, F, B = 150_000, 40, 256
    bins = rng.integers(0, B, size=(F, n), dtype=np.uint8)
    lim = qb // 2
    g = rng.choice(np.array([-lim, lim, 0, 1 - lim], np.int64), size=n).astype(np.int8)
    h = rng.choice(np.array([qb, 0, qb - 1], np.int64), size=n).astype(np.uint8)
    # most rows in one bin of every feature: the largest per-cell sums
    bins[:, : n // 2] = 7
    rows = np.arange(n, dtype=np.int32)
    got = mtlib.histogram_u8(bins, B, g, h, rows=rows, num_grad_quant_bins=qb)
    np.testing.assert_array_equal(got, host_histogram(bins, B, g, h, rows))
