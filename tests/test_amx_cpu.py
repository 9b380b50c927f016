"""The AMX repack layout (lowbit's pack_amx, src/lowbit/formats.py:251-293):
lowbit_b200.pack_amx reproduces the reference's bytes (golden_amx.npz, made
by tests/golden/make_amx_golden.py from lowbit itself), and to_int4() undoes
it exactly, so AMX-packed weights run the GPU's W4A8 kernels unchanged."""
from pathlib import Path

import numpy as np
import pytest

import lowbit_b200 as lb
from lowbit_b200.formats import AMXInt4Weights, pack_amx

G = np.load(Path(__file__).resolve().parent / "golden" / "golden_amx.npz")
SHAPES = [(37, 300, True), (16, 128, False), (50, 1000, True), (3, 256, False)]


@pytest.mark.parametrize("i", range(len(SHAPES)))
def test_pack_amx_matches_reference(i):
    n, k, asym = SHAPES[i]
    W = lb.quantize_int4(G[f"a{i}_w"], asym=asym)
    A = pack_amx(W)
    for f in ("qw", "scales", "sz", "zeros"):
        np.testing.assert_array_equal(getattr(A, f), G[f"a{i}_{f}"], err_msg=f)
    assert (A.n, A.k, A.kp) == (n, k, W.kp)


@pytest.mark.parametrize("i", range(len(SHAPES)))
def test_to_int4_inverts_the_reference_packing(i):
    n, k, asym = SHAPES[i]
    W = lb.quantize_int4(G[f"a{i}_w"], asym=asym)
    A = AMXInt4Weights(G[f"a{i}_qw"], G[f"a{i}_scales"], G[f"a{i}_sz"], G[f"a{i}_zeros"], n, k, W.kp)
    B = A.to_int4()
    np.testing.assert_array_equal(B.qw, W.qw)
    np.testing.assert_array_equal(B.scales, W.scales)
    np.testing.assert_array_equal(B.zeros, W.zeros if W.zeros is not None else np.full_like(B.zeros, 8))
    assert B.k == k
