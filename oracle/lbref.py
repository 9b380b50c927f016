"""Oracle: numpy restatement of lowbit's reference arithmetic (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this module, and only as the checker. The product (lowbit_b200) never calls it.

Pinned against the reference: tests/test_oracle.py checks every function here
against the golden vectors in tests/golden/ (generated from the reference
itself by tests/golden/make_golden.py) and against the reference's own
known-answer tests (E2M1 ties, E8M0 decode, extreme W4A8 operands).

Every function decodes the packed arrays itself (no lowbit_b200 import), so it
is independent of the product's format code. Citations are to the reference
project (azrabano23/lowbit).
"""
from __future__ import annotations

import numpy as np

GROUP = 128   # src/lowbit/csrc/lowbit.h:31
MXBLOCK = 32  # src/lowbit/csrc/lowbit.h:32


def unpack(qw: np.ndarray, block: int) -> np.ndarray:
    """Codes [N, Kp] from packed bytes [N, Kp/2]: per block, byte j = elem j (low
    nibble) | elem j + block/2 (high nibble) (src/lowbit/csrc/lowbit.h:11-19)."""
    qw = np.asarray(qw, np.uint8)
    n, nb = qw.shape
    kp = 2 * nb
    out = np.empty((n, kp // block, block), np.uint8)
    p = qw.reshape(n, kp // block, block // 2)
    out[:, :, : block // 2] = p & 0x0F
    out[:, :, block // 2:] = p >> 4
    return out.reshape(n, kp)


def e8m0_value(e: np.ndarray) -> np.ndarray:
    """2^(e-127) in float64; 255 -> NaN (src/lowbit/csrc/lowbit.h:84-88)."""
    e = np.asarray(e).astype(np.int64)
    v = np.power(2.0, (e - 127).astype(np.float64))
    return np.where(e == 255, np.nan, v)


def e2m1_value(code: np.ndarray) -> np.ndarray:
    """OCP E2M1 code -> float64: sign bit 3, exponent bits 2..1 (bias 1), mantissa bit 0."""
    c = np.asarray(code).astype(np.int64)
    sign = np.where(c & 8, -1.0, 1.0)
    ex = (c >> 1) & 3
    man = c & 1
    mag = np.where(ex == 0, 0.5 * man, np.power(2.0, ex - 1) * (1.0 + 0.5 * man))
    return sign * mag


def dequant_int4(qw, scales, zeros, k: int | None = None) -> np.ndarray:
    """[N, K] of (q - z) * s, the product rounded to fp32 as the reference's
    dequantize() does (src/lowbit/formats.py:82-87), returned as float64."""
    q = unpack(qw, GROUP).astype(np.float32)
    n, kp = q.shape
    g = kp // GROUP
    z = np.full((n, g), 8.0, np.float32) if zeros is None else np.asarray(zeros).astype(np.float32)
    s = np.asarray(scales, np.float32)
    w = ((q.reshape(n, g, GROUP) - z[:, :, None]) * s[:, :, None]).reshape(n, kp)
    w = w.astype(np.float64)
    return w if k is None else w[:, :k]


def dequant_mxfp4(qw, e8m0, k: int | None = None) -> np.ndarray:
    """[N, K] float64 of e2m1(q) * 2^(e-127) (src/lowbit/formats.py:169-172)."""
    v = e2m1_value(unpack(qw, MXBLOCK))
    n, kp = v.shape
    w = (v.reshape(n, kp // MXBLOCK, MXBLOCK) * e8m0_value(e8m0)[:, :, None]).reshape(n, kp)
    return w if k is None else w[:, :k]


def _pad(x, kp):
    x = np.atleast_2d(np.asarray(x, np.float64))
    out = np.zeros((x.shape[0], kp))
    out[:, : x.shape[1]] = x
    return out


def gemm_w4a16_ref(x, qw, scales, zeros) -> np.ndarray:
    """Y = X . deq(W)^T in float64 (src/lowbit/reference.py:9-11)."""
    w = dequant_int4(qw, scales, zeros)
    return _pad(x, w.shape[1]) @ w.T


def gemm_mxfp4_ref(x, qw, e8m0) -> np.ndarray:
    """Y = X . deq(W)^T in float64 (src/lowbit/reference.py:14-15)."""
    w = dequant_mxfp4(qw, e8m0)
    return _pad(x, w.shape[1]) @ w.T


def abs_bound(x, w_deq: np.ndarray) -> np.ndarray:
    """|X| . |W|^T, the scale of fp32 dot-product error (tests/conftest.py:22-27)."""
    return np.abs(_pad(x, w_deq.shape[1])) @ np.abs(w_deq).T


def quant_act_int8_ref(x, kp: int | None = None):
    """Per-token int8 (src/lowbit/csrc/dispatch.c:231-257, src/lowbit/formats.py:236-248):
    sc = amax/127 in fp32 (1 if amax == 0), q = clamp(rint(x/sc) [fp32 division,
    ties to even], -127, 127), asum[m,g] = sum of group codes. Returns (xq, xs, asum)."""
    x = np.atleast_2d(np.asarray(x, np.float32))
    kp = ((x.shape[1] + GROUP - 1) // GROUP) * GROUP if kp is None else kp
    xp = np.zeros((x.shape[0], kp), np.float32)
    xp[:, : x.shape[1]] = x
    amax = np.max(np.abs(xp), axis=1)
    sc = np.where(amax > 0, np.float32(amax) / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    v = (xp / sc[:, None]).astype(np.float32)
    q = np.clip(np.rint(v), -127, 127).astype(np.int8)
    asum = q.astype(np.int64).reshape(q.shape[0], -1, GROUP).sum(axis=2).astype(np.int32)
    return q, sc, asum


def w4a8_group_acc_ref(xq, asum, qw, zeros) -> np.ndarray:
    """Exact acc[m,n,g] = sum_{k in g} q*xq - z*asum[m,g] in int64 (src/lowbit/csrc/
    kern_scalar.c:49-59,86-99); equals sum (q - z)*xq when asum is the code sum
    (src/lowbit/reference.py:18-26)."""
    q = unpack(qw, GROUP).astype(np.int64)
    n, kp = q.shape
    g = kp // GROUP
    xa = np.asarray(xq, np.int64).reshape(-1, g, GROUP)
    z = np.full((n, g), 8, np.int64) if zeros is None else np.asarray(zeros, np.int64)
    dot = np.einsum("mgk,ngk->mng", xa, q.reshape(n, g, GROUP))
    return dot - z[None, :, :] * np.asarray(asum, np.int64)[:, None, :]


def gemm_w4a8_ref(xq, xs, asum, qw, scales, zeros) -> np.ndarray:
    """Y[m,n] = xs[m] * sum_g s[n,g] * acc[m,n,g] in float64 (src/lowbit/reference.py:29-34)."""
    acc = w4a8_group_acc_ref(xq, asum, qw, zeros).astype(np.float64)
    y = np.einsum("mng,ng->mn", acc, np.asarray(scales, np.float64))
    return y * np.asarray(xs, np.float64)[:, None]


def w4a8_bound(xq, xs, asum, qw, scales, zeros) -> np.ndarray:
    """Magnitude bound of the W4A8 fp part: xs * sum_g |s| (sum q|a| + z|asum|)
    (tests/test_kernels.py:135-143 of the reference)."""
    q = unpack(qw, GROUP).astype(np.float64)
    n, kp = q.shape
    g = kp // GROUP
    z = np.full((n, g), 8.0) if zeros is None else np.asarray(zeros, np.float64)
    aa = np.abs(np.asarray(xq, np.float64)).reshape(-1, g, GROUP)
    mag = np.einsum("mgk,ngk->mng", aa, q.reshape(n, g, GROUP)) + z[None] * np.abs(
        np.asarray(asum, np.float64))[:, None, :]
    return np.einsum("mng,ng->mn", mag, np.abs(np.asarray(scales, np.float64))) * np.abs(
        np.asarray(xs, np.float64))[:, None]


def assert_close(y, ref, bound, rtol: float) -> float:
    """|y - ref| <= rtol * bound elementwise (tests/conftest.py:22-27); returns max err/limit."""
    y = np.asarray(y, np.float64)
    err = np.abs(y - ref)
    lim = rtol * bound + 1e-30
    worst = float(np.max(err / lim)) if err.size else 0.0
    assert worst <= 1.0, f"max err/limit = {worst:.3g} (max abs err {float(err.max()):.3g})"
    return worst
