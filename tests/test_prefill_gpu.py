"""tcgen05 prefill kernel (64 tokens and more, W4A16, MXFP4 and W4A8) vs the oracle.

The prefill contract casts X to bf16 once: (q - z) and e2m1 * 2^(e-127) are
exact in bf16 and the int4 group scale is applied in fp32 to each group's
accumulator, so every product carries at most the bf16 rounding of x, 2^-8
relative, and |y - ref| <= 4e-3 * (|X| . |W|^T) holds for any input (the
north-star prefill tolerance). W4A8 needs no relaxation: A = q - z as s8
and int8 activations give the reference's int32 group sums exactly, so its
results meet the W4A8 bound of the exact kernels. The exact kernels stay
reachable: params.mr > 0 keeps the three-piece fp32-exact tensor-core kernel."""
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


W8_TOL = 1e-5  # the W4A8 bound of the exact paths (tests/test_kernels_gpu.py)


@pytest.mark.parametrize("shape", SHAPES + [(200, 513, 4128)])
@pytest.mark.parametrize("asym", [False, True])
def test_prefill_w4a8(rng, shape, asym):
    x, w = _problem(rng, *shape)
    W = lb.quantize_int4(w, asym=asym)
    assert K.describe_plan("w4a8", shape[0], shape[1], W.kp)["kernel"] == "prefill"
    xq, xs, asum = R.quant_act_int8_ref(x, W.kp)
    ref = R.gemm_w4a8_ref(xq, xs, asum, W.qw, W.scales, W.zeros)
    bound = R.w4a8_bound(xq, xs, asum, W.qw, W.scales, W.zeros)
    R.assert_close(K.gemm_w4a8(x, W), ref, bound, W8_TOL)
    a = lb.quantize_act_int8(x, W.kp)
    R.assert_close(K.gemm_w4a8_q(a, W), ref, bound, W8_TOL)


def test_prefill_w4a8_extreme_operands():
    """Codes 0 / 15 against zero points 0 / 15 / 7 / 8 and activations at
    +-127 / -128: the largest int32 group sums the format allows, exact."""
    from lowbit_b200.formats import pack_nibbles
    m, n, k = 128, 4, 512
    W = lb.quantize_int4(np.zeros((n, k), np.float32), asym=True)
    codes = np.zeros((n, k), np.uint8)
    codes[0] = 15
    codes[1, ::2] = 15
    codes[2] = np.arange(k) % 16
    W.qw[:] = pack_nibbles(codes, 128)
    W.zeros[:] = np.array([0, 15, 7, 8], np.uint8)[:, None]
    W.scales[:] = 1.0
    xq = np.full((m, k), 127, np.int8)
    xq[1::3] = -128
    xq[2::3, ::2] = -128
    gs = xq.astype(np.int32).reshape(m, -1, 128).sum(-1).astype(np.int32)
    a = lb.Int8Acts(xq, np.ones(m, np.float32), gs)
    y = K.gemm_w4a8_q(a, W)
    acc = R.w4a8_group_acc_ref(xq, gs, W.qw, W.zeros)
    np.testing.assert_array_equal(y, acc.sum(axis=2).astype(np.float32))


def test_prefill_w4a8_workspace(rng):
    """64+ tokens with a caller workspace give the same result as the
    allocating call; the no-allocation entry declines (its 4 MiB array is
    smaller than lbc_gemm_w4a8_workspace_size, which also covers the exact
    kernel's partial rows) instead of allocating."""
    import ctypes as C
    import torch
    x, w = _problem(rng, 96, 300, 1024)
    W = lb.quantize_int4(w, asym=True).cuda()
    xt = torch.from_numpy(x).cuda()
    y0 = K.gemm_w4a8(xt, W)
    L = K.lib()
    ws = torch.empty(int(L.lbc_gemm_w4a8_workspace_size(96, 1024)), dtype=torch.uint8, device="cuda")
    y1 = torch.empty_like(y0)
    y2 = torch.empty_like(y0)
    P = C.byref(K._Params(-1, 0, 0, 0, 0, 0, 0))
    st = torch.cuda.current_stream().cuda_stream
    args = (W.qw.data_ptr(), W.scales.data_ptr(), W.zeros.data_ptr(), 300)
    assert L.lbc_gemm_w4a8(xt.data_ptr(), 96, 1024, *args, y1.data_ptr(), P, ws.data_ptr(), st) == 1
    assert L.lbc_gemm_w4a8_workspace_size(96, 1024) > (4 << 20)
    assert L.lbc_gemm_w4a8_noalloc(xt.data_ptr(), 96, 1024, *args, y2.data_ptr(), P, st) == -1
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)


@pytest.mark.parametrize("fmt", ["w4a16", "w4a8", "mxfp4"])
def test_prefill_without_split_k(rng, fmt):
    """149 weight-row tiles fill the GPU: no split-K (plain stores); the other
    prefill tests have few tiles and run split-K (adds into a zeroed Y)."""
    x, w = _problem(rng, 128, 149 * 128, 256)
    if fmt == "mxfp4":
        W = lb.quantize_mxfp4(w)
        R.assert_close(K.gemm_mxfp4(x, W), R.gemm_mxfp4_ref(x, W.qw, W.e8m0),
                       R.abs_bound(x, R.dequant_mxfp4(W.qw, W.e8m0)), PF_TOL)
        return
    W = lb.quantize_int4(w, asym=True)
    if fmt == "w4a16":
        R.assert_close(K.gemm_w4a16(x, W), R.gemm_w4a16_ref(x, W.qw, W.scales, W.zeros),
                       R.abs_bound(x, R.dequant_int4(W.qw, W.scales, W.zeros)), PF_TOL)
    else:
        xq, xs, asum = R.quant_act_int8_ref(x, W.kp)
        R.assert_close(K.gemm_w4a8(x, W), R.gemm_w4a8_ref(xq, xs, asum, W.qw, W.scales, W.zeros),
                       R.w4a8_bound(xq, xs, asum, W.qw, W.scales, W.zeros), W8_TOL)
