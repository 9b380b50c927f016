"""Tensor-core path (isa="tcgen05") vs the oracle: dequantized weights in TMEM,
activations in shared memory. fp32-exact mode (X split into three bf16 pieces,
(q - z) exact in bf16, per-group fp32 scaling) is held to the same bound as the
SIMT path, 1e-5 * (|X| . |W|^T); W4A8 group sums are exact int32."""
import numpy as np
import pytest
from conftest import SHAPES

import lowbit_b200 as lb
from lowbit_b200 import kernels as K
from oracle import lbref as R

pytestmark = pytest.mark.gpu
TC = "tcgen05"
RTOL = 1e-5


def _problem(rng, m, n, k):
    return (rng.standard_normal((m, k)).astype(np.float32),
            rng.standard_normal((n, k)).astype(np.float32))


@pytest.mark.parametrize("shape", SHAPES + [(16, 300, 1024), (9, 130, 640), (33, 257, 384)])
@pytest.mark.parametrize("asym", [False, True])
def test_tc_w4a16(rng, shape, asym):
    x, w = _problem(rng, *shape)
    W = lb.quantize_int4(w, asym=asym)
    y = K.gemm_w4a16(x, W, isa=TC)
    R.assert_close(y, R.gemm_w4a16_ref(x, W.qw, W.scales, W.zeros),
                   R.abs_bound(x, R.dequant_int4(W.qw, W.scales, W.zeros)), RTOL)


@pytest.mark.parametrize("shape", SHAPES + [(16, 300, 1024), (5, 64, 96), (33, 257, 384)])
def test_tc_mxfp4(rng, shape):
    x, w = _problem(rng, *shape)
    W = lb.quantize_mxfp4(w)
    y = K.gemm_mxfp4(x, W, isa=TC)
    R.assert_close(y, R.gemm_mxfp4_ref(x, W.qw, W.e8m0),
                   R.abs_bound(x, R.dequant_mxfp4(W.qw, W.e8m0)), RTOL)


@pytest.mark.parametrize("shape", SHAPES + [(16, 300, 1024), (33, 257, 384)])
@pytest.mark.parametrize("asym", [False, True])
def test_tc_w4a8(rng, shape, asym):
    x, w = _problem(rng, *shape)
    W = lb.quantize_int4(w, asym=asym)
    a = lb.quantize_act_int8(x)
    ref = R.gemm_w4a8_ref(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros)
    bound = R.w4a8_bound(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros)
    R.assert_close(K.gemm_w4a8(x, W, isa=TC), ref, bound, RTOL)
    R.assert_close(K.gemm_w4a8_q(a, W, isa=TC), ref, bound, RTOL)


def test_tc_w4a8_extreme_operands_exact(golden):
    """Integer part exact: unit scales make y = xs * sum_g acc exactly representable."""
    W1 = lb.Int4Weights(golden["ext_qw"], np.ones_like(golden["ext_scales"]), golden["ext_zeros"], 512)
    a = lb.Int8Acts(golden["ext_xq"], np.ones(3, np.float32), golden["ext_gsum"])
    y = K.gemm_w4a8_q(a, W1, isa=TC)
    np.testing.assert_array_equal(y, golden["ext_acc_ref"].sum(axis=2).astype(np.float32))


def test_tc_negative_scales(rng):
    x, w = _problem(rng, 5, 37, 300)
    W = lb.quantize_int4(w, scale="signed-max")
    R.assert_close(K.gemm_w4a16(x, W, isa=TC), R.gemm_w4a16_ref(x, W.qw, W.scales, W.zeros),
                   R.abs_bound(x, R.dequant_int4(W.qw, W.scales, W.zeros)), RTOL)


def test_tc_consecutive_calls_and_torch_path(rng):
    import torch
    x, w = _problem(rng, 4, 200, 512)
    W = lb.quantize_int4(w, asym=True).cuda()
    xt = torch.from_numpy(x).cuda()
    ys = [K.gemm_w4a16(xt, W, isa=TC).clone() for _ in range(3)]
    torch.cuda.synchronize()
    ref = R.gemm_w4a16_ref(x, W.qw.cpu().numpy(), W.scales.cpu().numpy(), W.zeros.cpu().numpy())
    for y in ys:
        R.assert_close(y.cpu().numpy(), ref, R.abs_bound(x, R.dequant_int4(
            W.qw.cpu().numpy(), W.scales.cpu().numpy(), W.zeros.cpu().numpy())), RTOL)


def test_tc_baseline_decode_full_size(golden):
    x = np.random.default_rng(1).standard_normal((1, 4096)).astype(np.float32)
    w = np.random.default_rng(0).standard_normal((11008, 4096)).astype(np.float32)
    W = lb.quantize_int4(w, asym=True)
    R.assert_close(K.gemm_w4a16(x, W, isa=TC), golden["bl_w4a16_decode_y_ref"],
                   golden["bl_w4a16_decode_bound"], RTOL)


def test_tc_no_wait_timed_out():
    assert K.device_status(reset=True) == 0
