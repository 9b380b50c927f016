"""Few-token SIMT GEMM (csrc/gemv_tok.cu): W4A16 with 8-16 tokens and MXFP4
with 4-16 tokens on matrices of up to 5M weights (K split into ranges for
rows of 2048+ elements), against the
oracle with the reference's own bound |y - ref| <= 1e-5 * (|X| . |W|^T);
ragged N and K, symmetric and asymmetric int4, repeatability, CUDA-graph
capture on a fresh stream."""
import numpy as np
import pytest
import torch

import lowbit_b200 as lb
from lowbit_b200 import kernels as K
from oracle import lbref as R

pytestmark = pytest.mark.gpu
RTOL = 1e-5
SHAPES = [(1, 128), (33, 300), (1001, 896), (896, 4864), (1152, 896), (1024, 4096), (300, 11008), (64, 2080)]


@pytest.mark.parametrize("m", [8, 9, 12, 16])
@pytest.mark.parametrize("n,k", SHAPES)
def test_tok_w4a16(rng, m, n, k):
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.standard_normal((n, k)).astype(np.float32)
    for asym in (False, True):
        W = lb.quantize_int4(w, asym=asym)
        assert K.describe_plan("w4a16", m, n, W.kp)["kernel"] == "tok"
        y = K.gemm_w4a16(x, W)
        R.assert_close(y, R.gemm_w4a16_ref(x, W.qw, W.scales, W.zeros),
                       R.abs_bound(x, R.dequant_int4(W.qw, W.scales, W.zeros)), RTOL)


@pytest.mark.parametrize("m", [4, 5, 8, 16])
@pytest.mark.parametrize("n,k", SHAPES)
def test_tok_mxfp4(rng, m, n, k):
    x = rng.standard_normal((m, k)).astype(np.float32)
    W = lb.quantize_mxfp4(rng.standard_normal((n, k)).astype(np.float32) * 3)
    assert K.describe_plan("mxfp4", m, n, W.kp)["kernel"] == "tok"
    y = K.gemm_mxfp4(x, W)
    R.assert_close(y, R.gemm_mxfp4_ref(x, W.qw, W.e8m0), R.abs_bound(x, R.dequant_mxfp4(W.qw, W.e8m0)), RTOL)


def test_tok_mxfp4_nan_scale(rng):
    """E8M0 255 decodes to NaN, as in the reference: that block's rows are NaN."""
    x = rng.standard_normal((4, 256)).astype(np.float32)
    W = lb.quantize_mxfp4(rng.standard_normal((40, 256)).astype(np.float32))
    e = W.e8m0.copy()
    e[3, 2] = 255
    W2 = lb.MXFP4Weights(W.qw, e, W.k)
    y = K.gemm_mxfp4(x, W2)
    assert np.isnan(y[:, 3]).all() and not np.isnan(np.delete(y, 3, axis=1)).any()


def test_tok_repeatable_and_graph(rng):
    """Identical results on every call, eager or replayed from a CUDA graph
    captured on a stream whose scratch has not been allocated yet."""
    W = lb.quantize_int4(rng.standard_normal((2048, 1024)).astype(np.float32), asym=True).cuda()
    x = torch.from_numpy(rng.standard_normal((16, 1024)).astype(np.float32)).cuda()
    y0 = K.gemm_w4a16(x, W).clone()
    for _ in range(3):
        assert torch.equal(K.gemm_w4a16(x, W), y0)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        yg = K.gemm_w4a16(x, W)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(yg, y0)


def test_tok_routing():
    assert K.describe_plan("w4a16", 16, 896, 4864)["ksplit"] > 1      # long rows: K ranges
    assert K.describe_plan("w4a16", 16, 896, 896)["ksplit"] == 1
    assert K.describe_plan("w4a16", 16, 4096, 4096)["kernel"] != "tok"  # above 5M weights
    assert K.describe_plan("w4a16", 4, 896, 896)["kernel"] != "tok"    # fewer than 8 tokens
    assert K.describe_plan("mxfp4", 4, 896, 896)["kernel"] == "tok"
    assert K.describe_plan("w4a16", 2, 896, 896)["kernel"] == "rows"
    assert K.describe_plan("w4a16", 17, 896, 896)["kernel"] != "tok"
    assert K.describe_plan("w4a16", 8, 896, 896, lb.Params(mr=4))["kernel"] == "staged"
    assert K.describe_plan("w4a8", 8, 896, 896)["kernel"] != "tok"


def test_tok_k_ranges_alternating_shapes(rng):
    """Calls with K ranges share one partial-sum buffer per stream:
    alternating shapes repeat their first results exactly."""
    cases = []
    for m, n, k in ((16, 896, 4864), (8, 300, 11008), (16, 64, 2080), (9, 1500, 2048)):
        W = lb.quantize_int4(rng.standard_normal((n, k)).astype(np.float32), asym=True).cuda()
        x = torch.from_numpy(rng.standard_normal((m, W.kp)).astype(np.float32)).cuda()
        assert K.describe_plan("w4a16", m, n, W.kp)["ksplit"] > 1
        cases.append((x, W, K.gemm_w4a16(x, W).clone()))
    for _ in range(3):
        for x, W, y0 in cases:
            assert torch.equal(K.gemm_w4a16(x, W), y0)
