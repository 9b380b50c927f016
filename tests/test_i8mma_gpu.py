"""W4A8 on mma.sync.m16n8k32 s8 (the automatic path for 8-63 tokens, or
params isa="mma" for 1-64; passes of 16 tokens): A = q - z as s8 makes each 128-element group's
int32 accumulator exactly the reference's sum(q * xq) - z * asum
(src/lowbit/csrc/kern_scalar.c:49-59); the group scales fold it into fp32 in
group order and the token scale comes last. Checked against the oracle with
the reference's W4A8 bound for 1-64 tokens, ragged N, K from one group to
86, symmetric and asymmetric weights, extreme operands and every warp count
and CTAs-per-SM setting; the int8-only entry point (gemm_w4a8_q) gives the
same bits as the fp32 one."""
import numpy as np
import pytest

import lowbit_b200 as lb
from lowbit_b200 import kernels as K
from oracle import lbref as R

pytestmark = pytest.mark.gpu
W8 = 1e-5


def _check(y, x, W):
    xq, xs, asum = R.quant_act_int8_ref(x, W.kp)
    R.assert_close(y, R.gemm_w4a8_ref(xq, xs, asum, W.qw, W.scales, W.zeros),
                   R.w4a8_bound(xq, xs, asum, W.qw, W.scales, W.zeros), W8)


@pytest.mark.parametrize("m", [1, 2, 3, 8, 9, 16, 17, 33, 64])
@pytest.mark.parametrize("n,k", [(17, 128), (300, 384), (1000, 4096), (129, 11008)])
@pytest.mark.parametrize("asym", [False, True])
def test_i8mma_w4a8(m, n, k, asym):
    rng = np.random.default_rng(m * 7 + n + k + asym)
    W = lb.quantize_int4(rng.standard_normal((n, k)).astype(np.float32), asym=asym)
    x = rng.standard_normal((m, k)).astype(np.float32)
    p = K.Params(isa="mma")
    assert K.describe_plan("w4a8", m, n, W.kp, p)["kernel"] == "i8mma"
    y = K.gemm_w4a8(x, W, p)
    _check(y, x, W)
    y2 = K.gemm_w4a8_q(K.quant_act_int8(x, W.kp), W, p)
    np.testing.assert_array_equal(y, y2)


@pytest.mark.parametrize("nw", [4, 8])
@pytest.mark.parametrize("nb", [1, 2, 3])
def test_i8mma_tilings(nw, nb):
    rng = np.random.default_rng(nw * 10 + nb)
    W = lb.quantize_int4(rng.standard_normal((2900, 4736)).astype(np.float32), asym=True)
    x = rng.standard_normal((12, 4736)).astype(np.float32)
    y = K.gemm_w4a8(x, W, K.Params(isa="mma", nr=nw, nb=nb))
    _check(y, x, W)


def test_i8mma_extreme_operands():
    """Codes 0 and 15 against activations +-127 (the reference's extreme W4A8
    case): every group sum is at its largest magnitude, exact, and the result
    equals the oracle's bit for bit (every partial sum is an fp32 integer)."""
    n, k, m = 64, 1024, 16
    codes = np.where(np.arange(k)[None, :] % 2 == 0, 15, 0).repeat(n, 0)
    W = lb.Int4Weights(lb.formats.pack_nibbles(codes.astype(np.uint8), 128),
                       np.full((n, k // 128), 0.5, np.float32), np.zeros((n, k // 128), np.uint8), k)
    x = np.where(np.arange(k)[None, :] % 2 == 0, 127.0, -127.0).astype(np.float32).repeat(m, 0)
    y = K.gemm_w4a8(x, W, K.Params(isa="mma"))
    _check(y, x, W)
    xq, xs, asum = R.quant_act_int8_ref(x, W.kp)
    np.testing.assert_array_equal(y, R.gemm_w4a8_ref(xq, xs, asum, W.qw, W.scales, W.zeros).astype(np.float32))


@pytest.mark.parametrize("m", [17, 40, 63])
def test_i8mma_automatic_from_17_to_63_tokens(m):
    """The automatic W4A8 path for 17-63 tokens (passes of 16), against the
    oracle; the tcgen05 exact kernel stays reachable with isa="tcgen05"."""
    rng = np.random.default_rng(m)
    W = lb.quantize_int4(rng.standard_normal((700, 2048)).astype(np.float32), asym=True)
    x = rng.standard_normal((m, 2048)).astype(np.float32)
    assert K.describe_plan("w4a8", m, 700, W.kp)["kernel"] == "i8mma"
    _check(K.gemm_w4a8(x, W), x, W)
    assert K.describe_plan("w4a8", m, 700, W.kp, isa="tcgen05")["path"] == "tcgen05"
    _check(K.gemm_w4a8(x, W, isa="tcgen05"), x, W)


def test_i8mma_rejects_more_than_64_tokens():
    W = lb.quantize_int4(np.random.default_rng(2).standard_normal((64, 256)).astype(np.float32))
    with pytest.raises(ValueError):
        K.gemm_w4a8(np.ones((65, 256), np.float32), W, K.Params(isa="mma"))
