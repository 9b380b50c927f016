"""Warp-level tensor-core decode kernel (mma.sync, W4A16, one or two tokens)
vs the oracle, at the reference's own bound |y - ref| <= 1e-5 * (|X| . |W|^T):
every instantiated (warps, depth, CTAs per SM), ragged row counts (partial
16-row blocks, fewer rows than CTAs), rows of 1 to 86 groups, symmetric and
asymmetric weights, extreme codes and zero points, activations spanning a
wide dynamic range, and the full-size BASELINE configs[0] problem."""
import numpy as np
import pytest

import lowbit_b200 as lb
from lowbit_b200 import kernels as K
from oracle import lbref as R

pytestmark = pytest.mark.gpu
RTOL = 1e-5
KS = [96, 128, 1000, 4096, 4096 + 128, 11008]


def _check(x, W, y):
    R.assert_close(y, R.gemm_w4a16_ref(x, W.qw, W.scales, W.zeros),
                   R.abs_bound(x, R.dequant_int4(W.qw, W.scales, W.zeros)), RTOL)


@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("k", KS)
def test_mma_path_on_request(m, k):
    """The automatic choice keeps the register-streamed SIMT kernel for one and
    two tokens; isa="mma" (or the tuner) selects the tensor-core kernel."""
    kp = -(-k // 128) * 128
    assert K.describe_plan("w4a16", m, 4096, kp)["kernel"] == "rows"
    plan = K.describe_plan("w4a16", m, 4096, kp, isa="mma")
    assert plan["kernel"] == "mma" and plan["tokens"] == m, plan


@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("k", KS)
@pytest.mark.parametrize("n", [1, 7, 17, 333, 1500])
def test_mma_w4a16(rng, m, k, n):
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.standard_normal((n, k)).astype(np.float32)
    for asym in (False, True):
        W = lb.quantize_int4(w, asym=asym)
        y = K.gemm_w4a16(x, W, isa="mma")
        _check(x, W, y)


# (tokens, consumer warps, groups per warp per stage) instantiated in gemv_mma.cu
COMBOS = [(1, 4, 2), (1, 4, 4), (1, 8, 1), (1, 8, 2), (1, 8, 4), (1, 16, 1), (1, 16, 2),
          (2, 4, 2), (2, 8, 1), (2, 8, 2), (2, 16, 1)]


@pytest.mark.parametrize("m,nw,jws", COMBOS)
@pytest.mark.parametrize("order", [0, 2, 3])
@pytest.mark.parametrize("nb", [1, 2])
def test_mma_tilings(rng, m, nw, jws, order, nb):
    """Every instantiation, ring depth (0: as many stages as fit in half an SM)
    and CTAs per SM: K = 4096 + 640 gives a last K segment shorter than the
    others (and, with 37 groups, fewer groups than some tilings' warps times
    groups per warp), 2900 rows a partial last block."""
    k = 4096 + 640
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.standard_normal((2900, k)).astype(np.float32)
    for asym in (False, True):
        W = lb.quantize_int4(w, asym=asym)
        p = K.Params(nr=nw, kb=jws * 128 * nw, order=order, nb=nb)
        plan = K.describe_plan("w4a16", m, 2900, W.kp, p, isa="mma")
        assert (plan["warps"], plan["units_per_stage"]) == (nw, jws), plan
        assert plan["stages"] == order or (order == 0 and plan["stages"] >= 2), plan
        _check(x, W, K.gemm_w4a16(x, W, p, isa="mma"))


@pytest.mark.parametrize("k", [128, 640, 896, 1024 + 128])
@pytest.mark.parametrize("nw,jws", [(8, 2), (16, 1), (4, 4)])
def test_mma_fewer_groups_than_tiling(rng, k, nw, jws):
    """Rows of fewer groups than warps x groups per warp (the Qwen2 hidden size
    896 is 7 groups): every stage is a partial segment."""
    x = rng.standard_normal((1, k)).astype(np.float32)
    w = rng.standard_normal((700, k)).astype(np.float32)
    W = lb.quantize_int4(w, asym=True)
    p = K.Params(nr=nw, kb=jws * 128 * nw)
    _check(x, W, K.gemm_w4a16(x, W, p, isa="mma"))


def test_mma_extreme_operands(rng):
    """Codes 0 and 15 against zero points 0 and 15 (|q - z| = 15), activations
    from 1e-30 to 1e30 in one row: the bf16 pieces keep 24 bits of every x."""
    n, k = 64, 1024
    x = (rng.standard_normal((2, k)) * 10.0 ** rng.integers(-30, 30, (2, k))).astype(np.float32)
    qw = rng.choice(np.array([0x00, 0xFF, 0x0F, 0xF0], np.uint8), (n, k // 2))
    scales = (rng.random((n, k // 128)) + 0.5).astype(np.float32)
    zeros = rng.choice(np.array([0, 15], np.uint8), (n, k // 128))
    W = lb.Int4Weights(qw, scales, zeros, k)
    for m in (1, 2):
        _check(x[:m], W, K.gemm_w4a16(x[:m], W, isa="mma"))


def test_mma_zero_and_sparse_activations(rng):
    n, k = 100, 2048
    w = rng.standard_normal((n, k)).astype(np.float32)
    W = lb.quantize_int4(w, asym=True)
    x = np.zeros((2, k), np.float32)
    assert not np.any(K.gemm_w4a16(x, W, isa="mma"))
    x[0, ::97] = 3.0
    x[1, 5] = -1e-20
    _check(x, W, K.gemm_w4a16(x, W, isa="mma"))


def test_mma_baseline_config0():
    """BASELINE configs[0] at full size: M=1, N=11008, K=4096, asym, numpy
    seeds 0 (W) and 1 (X), on the automatic path."""
    w = np.random.default_rng(0).standard_normal((11008, 4096)).astype(np.float32)
    x = np.random.default_rng(1).standard_normal((1, 4096)).astype(np.float32)
    W = lb.quantize_int4(w, asym=True)
    _check(x, W, K.gemm_w4a16(x, W, isa="mma"))
    _check(x, W, K.gemm_w4a16(x, W, K.Params(nr=8, kb=4096, order=2), isa="mma"))


def test_mma_repeat_calls_fresh_activations(rng):
    """The kernel starts under programmatic dependent launch and builds its
    activation fragments after griddepcontrol.wait: a new X on every call
    (produced by the copy before it on the stream) is always the one used."""
    import torch
    w = rng.standard_normal((3000, 4096)).astype(np.float32)
    W = lb.quantize_int4(w, asym=True)
    Wd = W.cuda()
    for _ in range(30):
        x = rng.standard_normal((2, 4096)).astype(np.float32)
        y = K.gemm_w4a16(torch.from_numpy(x).cuda(), Wd, isa="mma").cpu().numpy()
        _check(x, W, y)
