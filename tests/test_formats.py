"""lowbit_b200's quantizers and packed layouts are bit-identical to the reference's
(golden vectors from lowbit, tests/golden/make_golden.py) and pass the
reference's format tests (tests/test_formats.py of lowbit)."""
import hashlib
import json

import numpy as np
import pytest
from conftest import GOLDEN, SHAPES

import lowbit_b200 as lb
from lowbit_b200 import formats as F


@pytest.mark.parametrize("i", range(len(SHAPES)))
def test_int4_quantizers_bit_identical(golden, i):
    w = golden[f"s{i}_w"]
    for tag, kw in (("sym", {}), ("asym", {"asym": True}), ("smax", {"scale": "signed-max"})):
        W = lb.quantize_int4(w, **kw)
        np.testing.assert_array_equal(W.qw, golden[f"s{i}_{tag}_qw"])
        np.testing.assert_array_equal(W.scales, golden[f"s{i}_{tag}_scales"])
        if tag == "asym":
            np.testing.assert_array_equal(W.zeros, golden[f"s{i}_{tag}_zeros"])
        else:
            assert W.zeros is None


@pytest.mark.parametrize("i", range(len(SHAPES)))
def test_mxfp4_quantizer_bit_identical(golden, i):
    M = lb.quantize_mxfp4(golden[f"s{i}_w"])
    np.testing.assert_array_equal(M.qw, golden[f"s{i}_mx_qw"])
    np.testing.assert_array_equal(M.e8m0, golden[f"s{i}_mx_e8m0"])


@pytest.mark.parametrize("i", range(len(SHAPES)))
def test_act_quantizer_bit_identical(golden, i):
    a = lb.quantize_act_int8(golden[f"s{i}_x"])
    np.testing.assert_array_equal(a.xq, golden[f"s{i}_xq"])
    np.testing.assert_array_equal(a.scale, golden[f"s{i}_xs"])
    np.testing.assert_array_equal(a.gsum, golden[f"s{i}_gsum"])


def test_act_quantizer_kat(golden):
    a = lb.quantize_act_int8(golden["aq_x"])
    np.testing.assert_array_equal(a.xq, golden["aq_xq"])
    np.testing.assert_array_equal(a.scale, golden["aq_xs"])
    np.testing.assert_array_equal(a.gsum, golden["aq_gsum"])


def test_e2m1_e8m0_kat(golden):
    np.testing.assert_array_equal(F.fp32_to_e2m1(F.E2M1_VALUES), golden["kat_e2m1_roundtrip"])
    np.testing.assert_array_equal(F.fp32_to_e2m1(golden["kat_e2m1_ties_in"]), golden["kat_e2m1_ties_out"])
    f = F.e8m0_to_float(golden["kat_e8m0_in"])
    np.testing.assert_array_equal(f[:255], golden["kat_e8m0_out"][:255])
    assert np.isnan(f[255])


@pytest.mark.parametrize("block", [32, 128])
def test_nibble_layout(rng, block):
    codes = rng.integers(0, 16, size=(5, 3 * block), dtype=np.uint8)
    packed = F.pack_nibbles(codes, block)
    assert packed.shape == (5, 3 * block // 2)
    np.testing.assert_array_equal(F.unpack_nibbles(packed, block), codes)
    assert packed[0, 0] == codes[0, 0] | (codes[0, block // 2] << 4)


@pytest.mark.parametrize("asym", [False, True])
@pytest.mark.parametrize("k", [128, 300, 1, 257])
def test_int4_roundtrip_and_padding(rng, asym, k):
    w = rng.standard_normal((7, k)).astype(np.float32) * 3
    q = lb.quantize_int4(w, asym=asym)
    assert q.kp % 128 == 0 and q.kp >= k
    s = np.repeat(q.scales, 128, axis=1)[:, :k]
    assert np.all(np.abs(q.dequantize() - w) <= 0.5 * s * (1 + 1e-5) + 1e-7)
    codes = q.codes()
    z = 8 if q.zeros is None else q.zeros[:, -1:]
    np.testing.assert_array_equal(codes[:, k:], np.broadcast_to(z, codes[:, k:].shape))


def test_signed_max_rejects_asym(rng):
    with pytest.raises(ValueError):
        lb.quantize_int4(rng.standard_normal((2, 128)).astype(np.float32), asym=True, scale="signed-max")


def test_shard_bounds_cover_rows():
    for n in (1, 7, 11008, 151936):
        for world in (1, 2, 4, 8):
            spans = [F.shard_bounds(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[r][1] == spans[r + 1][0] for r in range(world - 1))


def _sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        if a is None:
            h.update(b"none")
        else:
            a = np.ascontiguousarray(a)
            h.update(str(a.dtype).encode() + str(a.shape).encode())
            h.update(a.tobytes())
    return h.hexdigest()


def test_baseline_config_packing_matches_reference():
    """Full-size BASELINE inputs: quantized weights and activations hash to the
    reference's (digests recorded by make_golden.py from lowbit itself)."""
    dig = json.loads((GOLDEN / "golden_meta.json").read_text())["digests"]
    x = np.random.default_rng(1).standard_normal((1, 4096)).astype(np.float32)
    w = np.random.default_rng(0).standard_normal((11008, 4096)).astype(np.float32)
    assert _sha(x, w) == dig["w4a16_decode_inputs"]
    W = lb.quantize_int4(w, asym=True)
    assert _sha(W.qw, W.scales, W.zeros) == dig["w4a16_decode_packed"]
    M = lb.quantize_mxfp4(w)
    assert _sha(M.qw, M.e8m0) == dig["mxfp4_m64_packed"]
    x16 = np.random.default_rng(1).standard_normal((16, 4096)).astype(np.float32)
    a = lb.quantize_act_int8(x16)
    assert _sha(a.xq, a.scale, a.gsum) == dig["w4a8_m16_acts"]
