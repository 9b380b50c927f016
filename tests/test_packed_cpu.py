"""Packed-weight files (lowbit_b200.packed): the safetensors container, the
packed containers' round trip (bit-identical bytes, same K), and the checks
that reject malformed files. No GPU."""
import json

import numpy as np
import pytest

import lowbit_b200 as lb
from lowbit_b200 import packed as PK


def _raw_parse(path):
    """An independent reading of the container: 8-byte length, JSON header, data."""
    b = open(path, "rb").read()
    hlen = int.from_bytes(b[:8], "little")
    header = json.loads(b[8:8 + hlen])
    return header, b[8 + hlen:]


def test_tensors_round_trip(tmp_path, rng):
    arrs = {"a": rng.standard_normal((3, 5)).astype(np.float32), "b": rng.integers(0, 256, (7,), dtype=np.uint8),
            "c": rng.integers(-128, 128, (2, 2, 3), dtype=np.int8), "d": rng.integers(-9, 9, (4,), dtype=np.int32),
            "e": np.zeros((0, 4), np.float32), "f": rng.standard_normal(6).astype(np.float16)}
    p = tmp_path / "t.safetensors"
    PK.write_tensors(p, arrs, {"k": 3, "s": "x"})
    got, meta = PK.read_tensors(p)
    assert meta == {"k": "3", "s": "x"}
    assert set(got) == set(arrs)
    for k, v in arrs.items():
        assert got[k].dtype == v.dtype and got[k].shape == v.shape
        np.testing.assert_array_equal(got[k], v)
    header, data = _raw_parse(p)
    assert (8 + len(json.dumps(header, separators=(",", ":"))) <= 8 + int.from_bytes(open(p, "rb").read(8), "little"))
    for k, v in arrs.items():
        lo, hi = header[k]["data_offsets"]
        assert lo % 64 == 0 and hi - lo == v.nbytes
        assert data[lo:hi] == v.tobytes()


@pytest.mark.parametrize("kind", ["int4_sym", "int4_asym", "int4_signed", "mxfp4"])
def test_weights_round_trip(tmp_path, rng, kind):
    w = rng.standard_normal((37, 300)).astype(np.float32)
    W = (lb.quantize_mxfp4(w) if kind == "mxfp4" else
         lb.quantize_int4(w, asym=(kind == "int4_asym"), scale="signed-max" if kind == "int4_signed" else "absmax"))
    p = tmp_path / "w.safetensors"
    bias = rng.standard_normal(37).astype(np.float32)
    PK.save_weights(p, {"layer.0": W}, {"layer.0.bias": bias}, {"note": "x"})
    weights, extra, meta = PK.load_weights(p)
    V = weights["layer.0"]
    assert type(V) is type(W) and V.k == W.k == 300
    for f in ("qw", "scales", "zeros", "e8m0"):
        a, b = getattr(W, f, None), getattr(V, f, None)
        assert (a is None) == (b is None)
        if a is not None:
            assert a.dtype == b.dtype
            np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(extra["layer.0.bias"], bias)
    assert meta["note"] == "x" and meta["layer.0.format"] in (PK.FORMAT_INT4, PK.FORMAT_MXFP4)
    np.testing.assert_array_equal(V.dequantize(), W.dequantize())


def test_rejects_malformed(tmp_path, rng):
    W = lb.quantize_int4(rng.standard_normal((8, 256)).astype(np.float32), asym=True)
    p = tmp_path / "w.safetensors"
    t, m = PK.weights_tensors("x", W)
    PK.write_tensors(p, t, dict(m, **{"x.format": "int3"}))
    with pytest.raises(ValueError, match="unknown packed format"):
        PK.load_weights(p)
    PK.write_tensors(p, dict(t, **{"x.scales": np.ones((8, 3), np.float32)}), m)
    with pytest.raises(ValueError, match="inconsistent"):
        PK.load_weights(p)
    PK.write_tensors(p, t, dict(m, **{"x.k": 999}))
    with pytest.raises(ValueError, match="outside"):
        PK.load_weights(p)
    PK.write_tensors(p, dict(t, **{"x.qw": W.qw.astype(np.int32)}), m)
    with pytest.raises(ValueError, match="wants U8"):
        PK.load_weights(p)
    # a header whose offsets run past the data
    PK.write_tensors(p, {"a": np.ones(4, np.float32)})
    b = bytearray(open(p, "rb").read())
    hlen = int.from_bytes(b[:8], "little")
    h = json.loads(b[8:8 + hlen])
    h["a"]["data_offsets"] = [0, 4096]
    hb = json.dumps(h).encode()
    open(p, "wb").write(len(hb).to_bytes(8, "little") + hb + bytes(b[8 + hlen:]))
    with pytest.raises(ValueError, match="outside the file"):
        PK.read_tensors(p)
    with pytest.raises(TypeError):
        PK.weights_tensors("y", np.ones(3))
