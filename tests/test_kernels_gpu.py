"""CUDA kernels (through the C ABI) vs the oracle, mirroring the reference's
tests/test_kernels.py: odd shapes x tiling parameters, bit-exact W4A8 group
accumulators and activation quantizer, extreme operands, full BASELINE sizes.

Tolerances (SIMT path, fp32 FMA): |y - ref| <= 1e-5 * (|X| . |W|^T), the
reference's own bound (tests/conftest.py:22-27 of lowbit); W4A8 uses the
reference's magnitude bound xs * sum_g |s| (sum q|a| + z|asum|).
"""
import numpy as np
import pytest
from conftest import GOLDEN, SHAPES

import lowbit_b200 as lb
from lowbit_b200 import kernels as K
from oracle import lbref as R

pytestmark = pytest.mark.gpu

RTOL = 1e-5
PARAMS = [
    K.Params(),
    K.Params(mr=1, nr=1),
    K.Params(mr=2, nr=4, kb=256),
    K.Params(mr=4, nr=1, kb=128, order=2),
    K.Params(mr=1, nr=4, nb=1, order=3),
]


def _problem(rng, m, n, k):
    return (rng.standard_normal((m, k)).astype(np.float32),
            rng.standard_normal((n, k)).astype(np.float32))


def _w4a16_check(x, W, y):
    ref = R.gemm_w4a16_ref(x, W.qw, W.scales, W.zeros)
    deq = R.dequant_int4(W.qw, W.scales, W.zeros)
    return R.assert_close(y, ref, R.abs_bound(x, deq), RTOL)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("asym", [False, True])
def test_w4a16(rng, shape, asym):
    x, w = _problem(rng, *shape)
    W = lb.quantize_int4(w, asym=asym)
    for p in PARAMS:
        y = K.gemm_w4a16(x, W, p)
        assert y.shape == (shape[0], shape[1])
        _w4a16_check(x, W, y)


def test_int4_negative_scales(rng):
    x, w = _problem(rng, 5, 37, 300)
    W = lb.quantize_int4(w, scale="signed-max")
    assert (W.scales < 0).any()
    _w4a16_check(x, W, K.gemm_w4a16(x, W))
    a = lb.quantize_act_int8(x)
    np.testing.assert_array_equal(K.w4a8_group_acc(a, W),
                                  R.w4a8_group_acc_ref(a.xq, a.gsum, W.qw, W.zeros))
    ref8 = R.gemm_w4a8_ref(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros)
    b8 = R.w4a8_bound(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros)
    R.assert_close(K.gemm_w4a8(x, W), ref8, b8, RTOL)


@pytest.mark.parametrize("shape", SHAPES)
def test_mxfp4(rng, shape):
    x, w = _problem(rng, *shape)
    W = lb.quantize_mxfp4(w)
    ref = R.gemm_mxfp4_ref(x, W.qw, W.e8m0)
    bound = R.abs_bound(x, R.dequant_mxfp4(W.qw, W.e8m0))
    for p in PARAMS:
        R.assert_close(K.gemm_mxfp4(x, W, p), ref, bound, RTOL)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("asym", [False, True])
def test_w4a8_int32_accumulators_bit_exact(rng, shape, asym):
    x, w = _problem(rng, *shape)
    W = lb.quantize_int4(w, asym=asym)
    a = lb.quantize_act_int8(x)
    np.testing.assert_array_equal(K.w4a8_group_acc(a, W),
                                  R.w4a8_group_acc_ref(a.xq, a.gsum, W.qw, W.zeros))


def test_w4a8_extreme_values_exact(golden):
    W = lb.Int4Weights(golden["ext_qw"], golden["ext_scales"], golden["ext_zeros"], 512)
    a = lb.Int8Acts(golden["ext_xq"], np.ones(3, np.float32), golden["ext_gsum"])
    np.testing.assert_array_equal(K.w4a8_group_acc(a, W), golden["ext_acc_ref"])
    # the GEMM's integer part is exact too: with unit scales y = xs * sum_g acc
    W1 = lb.Int4Weights(golden["ext_qw"], np.ones_like(golden["ext_scales"]), golden["ext_zeros"], 512)
    y = K.gemm_w4a8_q(a, W1)
    np.testing.assert_array_equal(y, golden["ext_acc_ref"].sum(axis=2).astype(np.float32))


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("asym", [False, True])
def test_w4a8_gemm(rng, shape, asym):
    x, w = _problem(rng, *shape)
    W = lb.quantize_int4(w, asym=asym)
    a = lb.quantize_act_int8(x)
    ref = R.gemm_w4a8_ref(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros)
    bound = R.w4a8_bound(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros)
    for p in PARAMS:
        R.assert_close(K.gemm_w4a8(x, W, p), ref, bound, RTOL)
        R.assert_close(K.gemm_w4a8_q(a, W, p), ref, bound, RTOL)


@pytest.mark.parametrize("shape", [(1, 1), (3, 127), (4, 1000), (2, 4096), (17, 300)])
def test_gpu_act_quant_matches_numpy_exactly(rng, shape):
    x = rng.standard_normal(shape).astype(np.float32) * 3
    x[0, 0] = 0.5 * np.abs(x).max() / 127 * 3
    kp = lb.formats.pad_to(shape[1], 128)
    a_gpu = K.quant_act_int8(x, kp)
    xq, xs, gs = R.quant_act_int8_ref(x, kp)
    np.testing.assert_array_equal(a_gpu.xq, xq)
    np.testing.assert_array_equal(a_gpu.scale, xs)
    np.testing.assert_array_equal(a_gpu.gsum, gs)


def test_gpu_act_quant_kat(golden):
    a = K.quant_act_int8(golden["aq_x"], golden["aq_xq"].shape[1])
    np.testing.assert_array_equal(a.xq, golden["aq_xq"])
    np.testing.assert_array_equal(a.scale, golden["aq_xs"])
    np.testing.assert_array_equal(a.gsum, golden["aq_gsum"])


def test_zero_activation_row(rng):
    x = rng.standard_normal((3, 256)).astype(np.float32)
    x[1] = 0
    W = lb.quantize_int4(rng.standard_normal((8, 256)).astype(np.float32))
    y = K.gemm_w4a8(x, W)
    assert np.all(y[1] == 0) and np.all(np.isfinite(y))


def test_bad_tile_rejected(rng):
    W = lb.quantize_int4(rng.standard_normal((8, 128)).astype(np.float32))
    with pytest.raises(ValueError):
        K.gemm_w4a16(np.ones((1, 128), np.float32), W, K.Params(mr=3, nr=3))
    with pytest.raises(ValueError):
        K.gemm_w4a16(np.ones((1, 256), np.float32), W)  # more columns than Kp


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8, 16, 33])
def test_token_counts(rng, m):
    x, w = _problem(rng, m, 96, 640)
    W = lb.quantize_int4(w, asym=True)
    _w4a16_check(x, W, K.gemm_w4a16(x, W))
    M = lb.quantize_mxfp4(w)
    R.assert_close(K.gemm_mxfp4(x, M), R.gemm_mxfp4_ref(x, M.qw, M.e8m0),
                   R.abs_bound(x, R.dequant_mxfp4(M.qw, M.e8m0)), RTOL)


def test_torch_tensors_stay_on_device(rng):
    import torch
    x, w = _problem(rng, 4, 64, 512)
    W = lb.quantize_int4(w).cuda()
    xt = torch.from_numpy(x).cuda()
    yt = K.gemm_w4a16(xt, W)
    assert isinstance(yt, torch.Tensor) and yt.is_cuda and yt.shape == (4, 64)
    np.testing.assert_array_equal(yt.cpu().numpy(), K.gemm_w4a16(x, W))


def test_large_k_split(rng):
    """K beyond one segment (Kp > 32768) and explicit split-K both match."""
    x, w = _problem(rng, 2, 24, 40000)
    W = lb.quantize_int4(w, asym=True)
    _w4a16_check(x, W, K.gemm_w4a16(x, W))
    _w4a16_check(x, W, K.gemm_w4a16(x, W, K.Params(kb=4096)))


def test_baseline_w4a16_decode_full_size(golden):
    """BASELINE config 1 (M=1, N=11008, K=4096, asym) against the reference's own float64 output."""
    x = np.random.default_rng(1).standard_normal((1, 4096)).astype(np.float32)
    w = np.random.default_rng(0).standard_normal((11008, 4096)).astype(np.float32)
    W = lb.quantize_int4(w, asym=True)
    y = K.gemm_w4a16(x, W)
    R.assert_close(y, golden["bl_w4a16_decode_y_ref"], golden["bl_w4a16_decode_bound"], RTOL)


def test_baseline_w4a8_m16_full_size():
    """BASELINE config 2 (M=16, N=4096, K=4096, sym): int32 group sums bit-exact, y within bound."""
    x = np.random.default_rng(1).standard_normal((16, 4096)).astype(np.float32)
    w = np.random.default_rng(0).standard_normal((4096, 4096)).astype(np.float32)
    W = lb.quantize_int4(w)
    a = lb.quantize_act_int8(x)
    np.testing.assert_array_equal(K.w4a8_group_acc(a, W),
                                  R.w4a8_group_acc_ref(a.xq, a.gsum, W.qw, W.zeros))
    ref = R.gemm_w4a8_ref(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros)
    bound = R.w4a8_bound(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros)
    R.assert_close(K.gemm_w4a8(x, W), ref, bound, RTOL)


def test_baseline_mxfp4_m64_full_size():
    """BASELINE config 3 (M=64, N=11008, K=4096) on the SIMT path vs float64."""
    x = np.random.default_rng(1).standard_normal((64, 4096)).astype(np.float32)
    w = np.random.default_rng(0).standard_normal((11008, 4096)).astype(np.float32)
    W = lb.quantize_mxfp4(w)
    y = K.gemm_mxfp4(x, W, isa="simt")
    R.assert_close(y, R.gemm_mxfp4_ref(x, W.qw, W.e8m0),
                   R.abs_bound(x, R.dequant_mxfp4(W.qw, W.e8m0)), RTOL)


def test_no_device_wait_timed_out():
    assert K.device_status(reset=True) == 0
