"""The split scan dequantizes integer histogram sums by the quantizer units
without a divide (two FMA residual corrections of a * RN(1/units)).  It must
give the divide's bits for every value the trainer can meet: checked on the
device against the divide over 2^27 random (sum, units) pairs per seed."""
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_divide_free_dequantization_is_exact(mtlib, seed):
    assert mtlib.check_quotients(1 << 27, seed) == 0
