"""gemm_w4a8_amx / w4a8_group_acc_amx (lowbit's AMX entry points,
src/lowbit/kernels.py:208-225) on the GPU: weights in the reference's AMX
repack layout (bytes made by lowbit's own pack_amx, golden_amx.npz) give the
same results as gemm_w4a8 / w4a8_group_acc on the canonical weights, bit for
bit, and the oracle's within the W4A8 bound."""
from pathlib import Path

import numpy as np
import pytest

import lowbit_b200 as lb
from lowbit_b200 import kernels as K
from lowbit_b200.formats import AMXInt4Weights
from oracle import lbref as R

pytestmark = pytest.mark.gpu
G = np.load(Path(__file__).resolve().parent / "golden" / "golden_amx.npz")
SHAPES = [(37, 300, True), (16, 128, False), (50, 1000, True), (3, 256, False)]


@pytest.mark.parametrize("i", range(len(SHAPES)))
@pytest.mark.parametrize("m", [1, 5, 40])
def test_gemm_w4a8_amx_equals_canonical(rng, i, m):
    n, k, asym = SHAPES[i]
    W = lb.quantize_int4(G[f"a{i}_w"], asym=asym)
    A = AMXInt4Weights(G[f"a{i}_qw"], G[f"a{i}_scales"], G[f"a{i}_sz"], G[f"a{i}_zeros"], n, k, W.kp)
    x = rng.standard_normal((m, k)).astype(np.float32)
    y = lb.gemm_w4a8_amx(x, A)
    np.testing.assert_array_equal(y, K.gemm_w4a8(x, W))
    a = lb.quantize_act_int8(x, W.kp)
    R.assert_close(y, R.gemm_w4a8_ref(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros),
                   R.w4a8_bound(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros), 1e-5)
    np.testing.assert_array_equal(lb.w4a8_group_acc_amx(a, A), K.w4a8_group_acc(a, W))
    assert lb.amx_available()
