"""tcgen05 prefill kernel (64 tokens and more, W4A16 and MXFP4) vs the oracle.

The prefill contract casts X to bf16 once: (q - z) and e2m1 * 2^(e-127) are
exact in bf16 and the int4 group scale is applied in fp32 to each group's
accumulator, so every product carries at most the bf16 rounding of x, 2^-8
relative, and |y - ref| <= 4e-3 * (|X| . |W|^T) holds for any input (the
north-star prefill tolerance). The exact kernels stay reachable: params.mr
> 0 keeps the three-piece fp32-exact tensor-core kernel."""
import numpy as np
import pytest

import lowbit_b200 as lb
from lowbit_b200 import kernels as K
from oracle import lbref as R

pytestmark = pytest.mark.gpu
PF_TOL = 4e-3
SHAPES = [(64, 1, 128), (64, 200, 384), (130, 300, 1000), (257, 129, 4096), (128, 256, 256)]


def _problem(rng, m, n, k):
    return (rng.standard_normal((m, k)).astype(np.float32),
            rng.standard_normal((n, k)).astype(np.float32))


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("asym", [False, True])
def test_prefill_w4a16(rng, shape, asym):
    x, w = _problem(rng, *shape)
    W = lb.quantize_int4(w, asym=asym)
    assert K.describe_plan("w4a16", shape[0], shape[1], W.kp)["path"] == "tcgen05"
    y = K.gemm_w4a16(x, W)
    R.assert_close(y, R.gemm_w4a16_ref(x, W.qw, W.scales, W.zeros),
                   R.abs_bound(x, R.dequant_int4(W.qw, W.scales, W.zeros)), PF_TOL)


@pytest.mark.parametrize("shape", SHAPES + [(64, 33, 96)])
def test_prefill_mxfp4(rng, shape):
    x, w = _problem(rng, *shape)
    W = lb.quantize_mxfp4(w)
    y = K.gemm_mxfp4(x, W)
    R.assert_close(y, R.gemm_mxfp4_ref(x, W.qw, W.e8m0), R.abs_bound(x, R.dequant_mxfp4(W.qw, W.e8m0)), PF_TOL)


def test_prefill_worst_case_rounding(rng):
    """Every x at the largest bf16 rounding error (1 + 2^-8 is a tie and rounds
    to 1), all weights of one sign: the errors add up but stay within 2^-8 of
    |X| . |W|^T."""
    m, n, k = 64, 130, 128
    x = np.full((m, k), 1 + 2.0**-8, np.float32) * np.sign(rng.standard_normal((m, 1))).astype(np.float32)
    w = np.abs(rng.standard_normal((n, k))).astype(np.float32) + 0.5
    W = lb.quantize_int4(w, asym=True)
    y = K.gemm_w4a16(x, W)
    R.assert_close(y, R.gemm_w4a16_ref(x, W.qw, W.scales, W.zeros),
                   R.abs_bound(x, R.dequant_int4(W.qw, W.scales, W.zeros)), 2.0**-8 + 1e-6)


def test_exact_kernel_still_reachable(rng):
    """mr > 0 (tokens per pass) keeps the fp32-exact tensor-core kernel at 64+ tokens."""
    x, w = _problem(rng, 70, 150, 512)
    W = lb.quantize_int4(w, asym=True)
    y = K.gemm_w4a16(x, W, K.Params(mr=16), isa="tcgen05")
    R.assert_close(y, R.gemm_w4a16_ref(x, W.qw, W.scales, W.zeros),
                   R.abs_bound(x, R.dequant_int4(W.qw, W.scales, W.zeros)), 1e-5)


def test_prefill_consecutive_calls_reuse_scratch(rng):
    import torch
    x, w = _problem(rng, 200, 260, 768)
    W = lb.quantize_int4(w, asym=True).cuda()
    xt = torch.from_numpy(x).cuda()
    ys = [K.gemm_w4a16(xt, W).clone() for _ in range(3)]
    torch.cuda.synchronize()
    ref = R.gemm_w4a16_ref(x, W.qw.cpu().numpy(), W.scales.cpu().numpy(), W.zeros.cpu().numpy())
    bound = R.abs_bound(x, R.dequant_int4(W.qw.cpu().numpy(), W.scales.cpu().numpy(), W.zeros.cpu().numpy()))
    for y in ys:
        R.assert_close(y.cpu().numpy(), ref, bound, PF_TOL)
