"""Register-streamed decode kernel (one or two tokens, default params) vs the
oracle: every row-team shape the planner picks (1..8 warps, 1/2/4 chunks per
thread), ragged row ranges, all three weight formats. Same bounds as the
other SIMT tests: |y - ref| <= 1e-5 * (|X| . |W|^T); W4A8 the reference's
magnitude bound."""
import numpy as np
import pytest

import lowbit_b200 as lb
from lowbit_b200 import kernels as K
from oracle import lbref as R

pytestmark = pytest.mark.gpu
RTOL = 1e-5
# K values covering 1, 4 and 8 warps per row team and 1, 2 and 4 chunks per thread
KS = [96, 128, 1000, 4096, 4096 + 128, 11008, 16384 + 128, 20480]


def _problem(rng, m, n, k):
    return (rng.standard_normal((m, k)).astype(np.float32),
            rng.standard_normal((n, k)).astype(np.float32))


@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("k", KS)
def test_decode_plan_is_rows(m, k):
    """Rows of up to 8 warps x 32 threads x 4 (one token) or 2 (two tokens)
    chunks of 32 elements take the decode kernel; longer rows the staged one."""
    kp = -(-k // 128) * 128
    fits = kp // 32 <= 256 * (4 if m == 1 else 2)
    for kind in ("w4a16", "w4a8"):
        plan = K.describe_plan(kind, m, 300, kp)
        assert plan["kernel"] == ("rows" if fits else "staged"), plan
        if fits:
            assert plan["mt"] == m, plan
        plan = K.describe_plan(kind, m, 300, kp, isa="simt")
        assert plan["kernel"] == ("rows" if fits else "staged"), plan
    # MXFP4 takes the decode kernel for one token only
    plan = K.describe_plan("mxfp4", m, 300, kp)
    assert plan["kernel"] == ("rows" if fits and m == 1 else "staged"), plan


@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("k", KS)
@pytest.mark.parametrize("n", [1, 7, 333])
def test_decode_w4a16(rng, m, k, n):
    x, w = _problem(rng, m, n, k)
    for asym in (False, True):
        W = lb.quantize_int4(w, asym=asym)
        for isa in (None, "simt"):
            y = K.gemm_w4a16(x, W, isa=isa)
            R.assert_close(y, R.gemm_w4a16_ref(x, W.qw, W.scales, W.zeros),
                           R.abs_bound(x, R.dequant_int4(W.qw, W.scales, W.zeros)), RTOL)


@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("k", KS)
@pytest.mark.parametrize("n", [1, 333])
def test_mxfp4_few_tokens(rng, m, k, n):
    x, w = _problem(rng, m, n, k)
    W = lb.quantize_mxfp4(w)
    y = K.gemm_mxfp4(x, W)
    R.assert_close(y, R.gemm_mxfp4_ref(x, W.qw, W.e8m0), R.abs_bound(x, R.dequant_mxfp4(W.qw, W.e8m0)), RTOL)


@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("k", KS)
@pytest.mark.parametrize("n", [1, 333])
def test_decode_w4a8(rng, m, k, n):
    x, w = _problem(rng, m, n, k)
    W = lb.quantize_int4(w, asym=True)
    a = lb.quantize_act_int8(x)
    ref = R.gemm_w4a8_ref(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros)
    bound = R.w4a8_bound(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros)
    R.assert_close(K.gemm_w4a8(x, W), ref, bound, RTOL)
    R.assert_close(K.gemm_w4a8_q(a, W), ref, bound, RTOL)


@pytest.mark.parametrize("nb", [1, 2, 8])
def test_decode_ctas_per_sm(rng, nb):
    x, w = _problem(rng, 1, 1500, 4096)
    W = lb.quantize_int4(w, asym=True)
    p = K.Params(nb=nb)
    assert K.describe_plan("w4a16", 1, 1500, 4096, p)["kernel"] == "rows"
    R.assert_close(K.gemm_w4a16(x, W, p), R.gemm_w4a16_ref(x, W.qw, W.scales, W.zeros),
                   R.abs_bound(x, R.dequant_int4(W.qw, W.scales, W.zeros)), RTOL)


def test_decode_nan_scale_propagates(rng):
    """E8M0 255 is NaN in the OCP MX spec: the row's output is NaN, the others finite."""
    x, w = _problem(rng, 1, 40, 256)
    W = lb.quantize_mxfp4(w)
    e = W.e8m0.copy()
    e[5, 3] = 255
    W2 = lb.MXFP4Weights(W.qw, e, W.k)
    y = K.gemm_mxfp4(x, W2)
    assert np.isnan(y[0, 5]) and np.isfinite(np.delete(y[0], 5)).all()


@pytest.mark.parametrize("m", [3, 4, 5, 8, 13, 16])
@pytest.mark.parametrize("k", [96, 1000, 4096, 8192])
@pytest.mark.parametrize("n", [1, 333])
@pytest.mark.parametrize("asym", [False, True])
def test_decode_w4a8_several_tokens(rng, m, k, n, asym):
    """W4A8 with 3-16 tokens: the automatic path (the decode kernel 4 or 8
    tokens per pass below 8 tokens, the int8 mma kernel from 8) and the
    decode kernel forced by isa="simt" (rows of up to 8192 elements) meet the
    W4A8 bound, exact int32 group sums included."""
    x, w = _problem(rng, m, n, k)
    W = lb.quantize_int4(w, asym=asym)
    plan = K.describe_plan("w4a8", m, n, W.kp)
    assert plan["kernel"] == ("i8mma" if m >= 8 else "rows"), plan
    simt = K.Params(isa="simt")
    plan = K.describe_plan("w4a8", m, n, W.kp, simt)
    assert plan["kernel"] == "rows" and plan["mt"] == (4 if m <= 4 else 8), plan
    a = lb.quantize_act_int8(x)
    ref = R.gemm_w4a8_ref(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros)
    bound = R.w4a8_bound(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros)
    for p in (None, simt):
        R.assert_close(K.gemm_w4a8(x, W, p), ref, bound, RTOL)
        R.assert_close(K.gemm_w4a8_q(a, W, p), ref, bound, RTOL)


@pytest.mark.parametrize("m", [5, 8, 16])
def test_w4a8_fresh_activations_every_call(rng, m):
    """The decode kernel starts while the activation quantizer before it is
    still running and reads the quantized activations only after
    griddepcontrol.wait; with a new X on every call, a read issued before the
    wait would return the previous call's activations."""
    import torch
    w = rng.standard_normal((300, 4096)).astype(np.float32)
    W = lb.quantize_int4(w)
    Wd = W.cuda()
    for _ in range(40):
        x = rng.standard_normal((m, 4096)).astype(np.float32)
        a = lb.quantize_act_int8(x)
        ref = R.gemm_w4a8_ref(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros)
        bound = R.w4a8_bound(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros)
        y = K.gemm_w4a8(torch.from_numpy(x).cuda(), Wd).cpu().numpy()
        R.assert_close(y, ref, bound, RTOL)
