"""Pins the oracle (oracle/lbref.py, oracle/lbref.c) to the reference: golden
vectors generated from lowbit itself plus the reference's known-answer tests."""
import ctypes as C
import subprocess

import numpy as np
import pytest
from conftest import ROOT, SHAPES, case

from oracle import lbref as R

TAGS = ("sym", "asym", "smax")


@pytest.mark.parametrize("i", range(len(SHAPES)))
@pytest.mark.parametrize("tag", TAGS)
def test_int4_refs_match_reference(golden, i, tag):
    c = case(golden, i, tag)
    y = R.gemm_w4a16_ref(c["x"], c["qw"], c["scales"], c["zeros"])
    np.testing.assert_allclose(y, golden[f"s{i}_{tag}_y_ref"], rtol=1e-12, atol=1e-12)
    acc = R.w4a8_group_acc_ref(golden[f"s{i}_xq"], golden[f"s{i}_gsum"], c["qw"], c["zeros"])
    np.testing.assert_array_equal(acc, golden[f"s{i}_{tag}_acc_ref"])
    np.testing.assert_array_equal(acc, golden[f"s{i}_{tag}_acc_c"])  # reference C kernel
    y8 = R.gemm_w4a8_ref(golden[f"s{i}_xq"], golden[f"s{i}_xs"], golden[f"s{i}_gsum"],
                         c["qw"], c["scales"], c["zeros"])
    np.testing.assert_allclose(y8, golden[f"s{i}_{tag}_y8_ref"], rtol=1e-12, atol=1e-12)
    # the reference's own C kernels sit inside the oracle's fp32 error bound
    deq = R.dequant_int4(c["qw"], c["scales"], c["zeros"])
    R.assert_close(golden[f"s{i}_{tag}_y_c"], y, R.abs_bound(c["x"], deq), 1e-5)
    b8 = R.w4a8_bound(golden[f"s{i}_xq"], golden[f"s{i}_xs"], golden[f"s{i}_gsum"],
                      c["qw"], c["scales"], c["zeros"])
    R.assert_close(golden[f"s{i}_{tag}_y8_c"], y8, b8, 1e-5)


@pytest.mark.parametrize("i", range(len(SHAPES)))
def test_mxfp4_ref_matches_reference(golden, i):
    x = golden[f"s{i}_x"]
    y = R.gemm_mxfp4_ref(x, golden[f"s{i}_mx_qw"], golden[f"s{i}_mx_e8m0"])
    np.testing.assert_allclose(y, golden[f"s{i}_mx_y_ref"], rtol=1e-12, atol=1e-12)
    deq = R.dequant_mxfp4(golden[f"s{i}_mx_qw"], golden[f"s{i}_mx_e8m0"])
    R.assert_close(golden[f"s{i}_mx_y_c"], y, R.abs_bound(x, deq), 1e-5)


@pytest.mark.parametrize("i", range(len(SHAPES)))
def test_act_quant_ref_bit_exact(golden, i):
    xq, xs, gs = R.quant_act_int8_ref(golden[f"s{i}_x"])
    np.testing.assert_array_equal(xq, golden[f"s{i}_xq"])
    np.testing.assert_array_equal(xs, golden[f"s{i}_xs"])
    np.testing.assert_array_equal(gs, golden[f"s{i}_gsum"])


def test_act_quant_kat(golden):
    """.5 tie, zero row and large dynamic range: numpy oracle == reference numpy == reference C."""
    xq, xs, gs = R.quant_act_int8_ref(golden["aq_x"])
    for suffix in ("", "_c"):
        np.testing.assert_array_equal(xq, golden["aq_xq" + suffix])
        np.testing.assert_array_equal(xs, golden["aq_xs" + suffix])
        np.testing.assert_array_equal(gs, golden["aq_gsum" + suffix])


def test_e2m1_e8m0_known_answers(golden):
    codes = np.arange(16)
    table = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6])
    np.testing.assert_array_equal(R.e2m1_value(codes), table)
    # the reference's rounding of the table maps every value to itself
    np.testing.assert_array_equal(R.e2m1_value(golden["kat_e2m1_roundtrip"]), table + 0.0)
    e = golden["kat_e8m0_in"]
    ref = golden["kat_e8m0_out"].astype(np.float64)
    v = R.e8m0_value(e)
    np.testing.assert_array_equal(v[:255], ref[:255])
    assert np.isnan(v[255]) and np.isnan(ref[255])
    assert v[0] == 2.0 ** -127


def test_extreme_w4a8_operands(golden):
    acc = R.w4a8_group_acc_ref(golden["ext_xq"], golden["ext_gsum"], golden["ext_qw"], golden["ext_zeros"])
    np.testing.assert_array_equal(acc, golden["ext_acc_ref"])
    np.testing.assert_array_equal(acc, golden["ext_acc_c"])


# ------------------------------------------------------------------ C restatement
def _liblbref():
    so = ROOT / "oracle" / "_build" / "liblbref.so"
    if not so.exists():
        subprocess.run(["make", "-C", str(ROOT / "oracle"), "all"], check=True, capture_output=True)
    return C.CDLL(str(so))


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


@pytest.mark.parametrize("i", [1, 3, 4, 5])
def test_c_oracle_matches_numpy_oracle(golden, i):
    L = _liblbref()
    c = case(golden, i, "asym")
    x = np.ascontiguousarray(golden[f"s{i}_x"])
    m, k = x.shape
    n = c["qw"].shape[0]
    kp = c["qw"].shape[1] * 2
    xp = np.zeros((m, kp), np.float32)
    xp[:, :k] = x
    y = np.zeros((m, n), np.float64)
    L.lbref_gemm_w4a16(_p(xp), m, kp, _p(c["qw"]), _p(c["scales"]), _p(c["zeros"]), n, _p(y))
    np.testing.assert_allclose(y, golden[f"s{i}_asym_y_ref"], rtol=1e-10, atol=1e-10)
    mq, me = golden[f"s{i}_mx_qw"], golden[f"s{i}_mx_e8m0"]
    kpm = mq.shape[1] * 2
    xm = np.zeros((m, kpm), np.float32)
    xm[:, :k] = x
    ym = np.zeros((m, n), np.float64)
    L.lbref_gemm_mxfp4(_p(xm), m, kpm, _p(mq), _p(me), n, _p(ym))
    np.testing.assert_allclose(ym, golden[f"s{i}_mx_y_ref"], rtol=1e-10, atol=1e-10)
    xq = np.zeros((m, kp), np.int8)
    xs = np.zeros(m, np.float32)
    gs = np.zeros((m, kp // 128), np.int32)
    L.lbref_quant_act_int8(_p(xp), m, kp, _p(xq), _p(xs), _p(gs))
    np.testing.assert_array_equal(xq, golden[f"s{i}_xq"])
    np.testing.assert_array_equal(xs, golden[f"s{i}_xs"])
    acc = np.zeros((m, n, kp // 128), np.int32)
    L.lbref_w4a8_group_acc(_p(xq), _p(gs), m, kp, _p(c["qw"]), _p(c["zeros"]), n, _p(acc))
    np.testing.assert_array_equal(acc, golden[f"s{i}_asym_acc_ref"])
