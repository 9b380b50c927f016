"""Tensor-core building blocks (TMEM A operand, SMEM B descriptor, MMA, readback) give
exact results for small-integer operands: D = A . B^T."""
import numpy as np
import pytest

from lowbit_b200 import kernels as K

pytestmark = pytest.mark.gpu


def _expected(kind):
    k = 32 if kind == 0 else 64
    m = np.arange(128)[:, None]
    n = np.arange(16)[:, None]
    kk = np.arange(k)[None, :]
    a = ((m * 3 + kk * 5) % 11) - 5
    b = ((n * 5 + kk * 7) % 13) - 6
    return (a @ b.T).astype(np.int64)


@pytest.mark.parametrize("kind", [0, 1])
def test_tcgen05_selftest_exact(kind):
    d = K.tc_selftest(kind)
    np.testing.assert_array_equal(d, _expected(kind))
    assert K.device_status(reset=True) == 0
