"""Known answers for the quantizer primitives the device kernels and the
oracle share (mt_math.h), ported from the procedures of the reference's
tests/test_cpu_quantized_grad.mojo and pinned to the published SplitMix64."""
import numpy as np
import pytest


@pytest.fixture(scope="module")
def q(oracle):
    return oracle.lib()


def test_splitmix64_is_the_published_mixer(q):
    # SplitMix64 (Steele, Lea, Flood; Vigna's reference code): the first
    # output from state 0 is 0xE220A8397B1DCDAF, the next 0x6E789E6AA1B965F4
    assert q.mt_oracle_splitmix64(0) == 0xE220A8397B1DCDAF
    assert q.mt_oracle_splitmix64(0x9E3779B97F4A7C15) == 0x6E789E6AA1B965F4


def test_uniform_is_53_bits_in_unit_interval(q):
    for c in range(2000):
        u = q.mt_oracle_uniform(c)
        assert 0.0 <= u < 1.0
        assert u == (q.mt_oracle_splitmix64(c) >> 11) * 2.0 ** -53


def test_stochastic_rounding_is_magnitude_symmetric(q):
    """test_stochastic_rounding_is_magnitude_symmetric_like_lightgbms:
    |q| = floor(|y| + u) keeps the sign, so y = -1.3 with u >= 0.7 is -2
    (floor(y + u) would give -1), and +1.3 is +2."""
    counter = next(c for c in range(64) if q.mt_oracle_uniform(c) >= 0.7)
    assert q.mt_oracle_quantize_stochastic(-1.3, 1.0, 2.0 ** 30, counter) == -2
    assert q.mt_oracle_quantize_stochastic(1.3, 1.0, 2.0 ** 30, counter) == 2
    low = next(c for c in range(64) if q.mt_oracle_uniform(c) < 0.7)
    assert q.mt_oracle_quantize_stochastic(-1.3, 1.0, 2.0 ** 30, low) == -1


def test_rounding_clamps_and_keeps_lattice_points(q):
    for c in range(50):
        assert q.mt_oracle_quantize_stochastic(10.0, 1.0, 2.0, c) == 2
        assert q.mt_oracle_quantize_stochastic(-10.0, 1.0, 2.0, c) == -2
        assert q.mt_oracle_quantize_stochastic(1.0, 2.0, 4.0, c) == 2  # exactly on the lattice
        assert q.mt_oracle_quantize_stochastic(0.0, 5.0, 4.0, c) == 0


def test_rounding_is_unbiased(q):
    # E[floor(y + u)] = y for u uniform on [0, 1)
    vals = [q.mt_oracle_quantize_stochastic(0.3, 1.0, 2.0, c) for c in range(20000)]
    assert abs(np.mean(vals) - 0.3) < 0.02


def test_the_round_class_and_plane_move_the_dither(q):
    """test_the_round_index_moves_the_dither, and its class and plane twins:
    the stream mixes seed, round, class + 1 and plane (quantized_gradient.mojo
    :475-492), so each gives a different sequence."""
    base = q.mt_oracle_quant_stream(11, 0, 0, 0)
    others = [q.mt_oracle_quant_stream(11, 1, 0, 0), q.mt_oracle_quant_stream(11, 0, 1, 0),
              q.mt_oracle_quant_stream(11, 0, 0, 1), q.mt_oracle_quant_stream(12, 0, 0, 0)]
    assert len({base, *others}) == 5
    g = np.random.default_rng(131).normal(size=2000) * 0.4
    def quantize(stream):
        return [q.mt_oracle_quantize_stochastic(x, 2.0 / 1.2, 2.0, stream + r) for r, x in enumerate(g)]
    a, b_ = quantize(base), quantize(others[0])
    assert sum(x != y for x, y in zip(a, b_)) > 0


def test_fixed_point_scale_is_the_largest_power_of_two(q):
    """quantized_gradient.mojo:856-908: s = 2^k <= 2^30 / max(T, 1e-12)."""
    assert q.mt_oracle_fixed_point_scale(1.0) == 2.0 ** 30
    assert q.mt_oracle_fixed_point_scale(3.0) == 2.0 ** 28
    assert q.mt_oracle_fixed_point_scale(2.0 ** 31) == 0.5
    assert q.mt_oracle_fixed_point_scale(0.0) == 2.0 ** 69  # T floored at 1e-12: 2^30 / 1e-12 ~ 1.07e21
    for t in (0.7, 123.456, 9.9e8):
        s = q.mt_oracle_fixed_point_scale(t)
        assert s <= 2.0 ** 30 / t < 2 * s and np.log2(s) == int(np.log2(s))


def test_fixed_point_scale_shape(q):
    """tests/test_fixed_point_scale_shape.mojo procedures: the scaled total
    stays within 2^30 (half the int32 range), flooring to a power of two costs
    at most one bit, and both the float32 product g * s and its dequantizing
    reciprocal are exact."""
    rng = np.random.default_rng(9)
    for _ in range(200):
        g = rng.normal(size=64) * 10.0 ** rng.uniform(-6, 6)
        total = float(np.sum(np.abs(g)))
        s = q.mt_oracle_fixed_point_scale(total)
        assert total * s <= 2.0 ** 30
        assert total * s > 2.0 ** 29  # at most one bit below the bound
        g32 = g.astype(np.float32)
        prod = g32 * np.float32(s)
        assert np.array_equal(prod.astype(np.float64), g32.astype(np.float64) * s)  # exact product
        inv = 1.0 / s
        assert inv * s == 1.0 and np.log2(inv) == int(np.log2(inv))
