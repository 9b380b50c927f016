"""Generate the golden fixtures in tests/golden/ from the reference implementation.

Run in a container that has the reference checkout (it is not needed at test
time; the fixtures are committed):

    CC=/usr/bin/gcc LOWBIT_BUILD_DIR=/tmp/lbbuild \\
        python tests/golden/make_golden.py /path/to/lowbit/src

It imports the reference package (`lowbit`) and records, for the reference's
own kernel-test shapes (tests/test_kernels.py:12-20 of the reference) and
seeded inputs:
  * its quantizers' packed outputs (int4 sym / asym / signed-max, MXFP4,
    per-token int8 activations),
  * its float64 / int64 oracle outputs (src/lowbit/reference.py),
  * its C kernels' outputs (lowbit.kernels, AVX-512 / VNNI paths),
  * its known-answer tests (E2M1 ties, E8M0 decode, extreme W4A8 operands),
  * SHA-256 digests of the packed weights of the BASELINE configurations
    (too large to store), so the GPU box can check that lowbit_b200's
    quantizers reproduce them bit for bit.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

SHAPES = [(1, 1, 1), (1, 64, 128), (3, 5, 127), (7, 33, 129), (5, 37, 300),
          (17, 70, 1000), (2, 16, 4096 + 32)]

# BASELINE.json configurations (W and X ~ N(0,1), W from seed 0, X from seed 1)
BASELINE = {
    "w4a16_decode": dict(fmt="w4a16", m=1, n=11008, k=4096, asym=True),
    "w4a8_m16": dict(fmt="w4a8", m=16, n=4096, k=4096, asym=False),
    "mxfp4_m64": dict(fmt="mxfp4", m=64, n=11008, k=4096),
}


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        if a is None:
            h.update(b"none")
        else:
            a = np.ascontiguousarray(a)
            h.update(str(a.dtype).encode() + str(a.shape).encode())
            h.update(a.tobytes())
    return h.hexdigest()


def baseline_inputs(m, n, k):
    w = np.random.default_rng(0).standard_normal((n, k)).astype(np.float32)
    x = np.random.default_rng(1).standard_normal((m, k)).astype(np.float32)
    return x, w


def main(ref_src: str) -> None:
    sys.path.insert(0, ref_src)
    import lowbit as lb
    from lowbit import formats as F
    from lowbit import kernels as K
    from lowbit import reference as R

    out: dict[str, np.ndarray] = {}
    meta = {"shapes": SHAPES, "reference": "azrabano23/lowbit", "cpu": K.cpu_info()}

    for i, (m, n, k) in enumerate(SHAPES):
        rng = np.random.default_rng(1000 + i)
        x = rng.standard_normal((m, k)).astype(np.float32)
        w = rng.standard_normal((n, k)).astype(np.float32)
        p = f"s{i}_"
        out[p + "x"] = x
        out[p + "w"] = w
        for tag, kw in (("sym", {}), ("asym", {"asym": True}), ("smax", {"scale": "signed-max"})):
            W = lb.quantize_int4(w, **kw)
            out[p + f"{tag}_qw"] = W.qw
            out[p + f"{tag}_scales"] = W.scales
            if W.zeros is not None:
                out[p + f"{tag}_zeros"] = W.zeros
            out[p + f"{tag}_y_ref"] = R.gemm_w4a16_ref(x, W)
            out[p + f"{tag}_y_c"] = K.gemm_w4a16(x, W).copy()
            a = lb.quantize_act_int8(x)
            out[p + f"{tag}_acc_ref"] = R.w4a8_group_acc_ref(a, W).astype(np.int32)
            out[p + f"{tag}_acc_c"] = K.w4a8_group_acc(a, W).copy()
            out[p + f"{tag}_y8_ref"] = R.gemm_w4a8_ref(x, W, a)
            out[p + f"{tag}_y8_c"] = K.gemm_w4a8(x, W).copy()
        M4 = lb.quantize_mxfp4(w)
        out[p + "mx_qw"] = M4.qw
        out[p + "mx_e8m0"] = M4.e8m0
        out[p + "mx_y_ref"] = R.gemm_mxfp4_ref(x, M4)
        out[p + "mx_y_c"] = K.gemm_mxfp4(x, M4).copy()
        a = lb.quantize_act_int8(x)
        out[p + "xq"] = a.xq
        out[p + "xs"] = a.scale
        out[p + "gsum"] = a.gsum
        ac = K.quant_act_int8(x, a.xq.shape[1])
        assert np.array_equal(ac.xq, a.xq) and np.array_equal(ac.scale, a.scale)

    # activation quantizer KATs: an exact .5 tie after scaling, a zero row,
    # large dynamic range (reference tests/test_kernels.py:123-140)
    rng = np.random.default_rng(77)
    xa = rng.standard_normal((4, 1000)).astype(np.float32) * 3
    xa[0, 0] = 0.5 * np.abs(xa[0]).max() / 127 * 3
    xa[1] = 0.0
    xa[2, ::7] *= 1e4
    ac = lb.quantize_act_int8(xa)
    out["aq_x"], out["aq_xq"], out["aq_xs"], out["aq_gsum"] = xa, ac.xq, ac.scale, ac.gsum
    cc = K.quant_act_int8(xa, ac.xq.shape[1])
    out["aq_xq_c"], out["aq_xs_c"], out["aq_gsum_c"] = cc.xq, cc.scale, cc.gsum

    # E2M1 / E8M0 known answers (reference tests/test_formats.py:75-97)
    vals = F.E2M1_VALUES
    out["kat_e2m1_roundtrip"] = F.fp32_to_e2m1(vals)
    ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.9, 100.0], np.float32)
    out["kat_e2m1_ties_in"] = np.concatenate([ties, -ties])
    out["kat_e2m1_ties_out"] = F.fp32_to_e2m1(out["kat_e2m1_ties_in"])
    e = np.arange(256, dtype=np.uint8)
    out["kat_e8m0_in"] = e
    out["kat_e8m0_out"] = F.e8m0_to_float(e)

    # extreme W4A8 operands (reference tests/test_kernels.py:81-97)
    m, n, k = 3, 4, 512
    W = lb.quantize_int4(np.zeros((n, k), np.float32), asym=True)
    codes = np.zeros((n, k), np.uint8)
    codes[0] = 15
    codes[1, ::2] = 15
    codes[2] = np.arange(k) % 16
    W.qw[:] = F.pack_nibbles(codes, 128)
    W.zeros[:] = np.array([0, 15, 7, 8], np.uint8)[:, None]
    xq = np.full((m, k), 127, np.int8)
    xq[1] = -128
    xq[2, ::2] = -128
    gs = xq.astype(np.int32).reshape(m, -1, 128).sum(-1).astype(np.int32)
    a = lb.Int8Acts(xq, np.ones(m, np.float32), gs)
    out["ext_qw"], out["ext_zeros"], out["ext_scales"] = W.qw, W.zeros, W.scales
    out["ext_xq"], out["ext_gsum"] = xq, gs
    out["ext_acc_ref"] = R.w4a8_group_acc_ref(a, W).astype(np.int32)
    out["ext_acc_c"] = K.w4a8_group_acc(a, W).copy()

    # BASELINE configurations: digests of the packed weights / activations
    digests = {}
    for name, c in BASELINE.items():
        x, w = baseline_inputs(c["m"], c["n"], c["k"])
        digests[name + "_inputs"] = sha(x, w)
        if c["fmt"] == "mxfp4":
            Wq = lb.quantize_mxfp4(w)
            digests[name + "_packed"] = sha(Wq.qw, Wq.e8m0)
        else:
            Wq = lb.quantize_int4(w, asym=c["asym"])
            digests[name + "_packed"] = sha(Wq.qw, Wq.scales, Wq.zeros)
        a = lb.quantize_act_int8(x)
        digests[name + "_acts"] = sha(a.xq, a.scale, a.gsum)
        if name == "w4a16_decode":
            y = R.gemm_w4a16_ref(x, Wq)
            out["bl_w4a16_decode_y_ref"] = y.astype(np.float64)
            out["bl_w4a16_decode_bound"] = (np.abs(x).astype(np.float64)
                                            @ np.abs(Wq.dequantize()).T.astype(np.float64))
    meta["digests"] = digests
    np.savez_compressed(HERE / "golden.npz", **out)
    (HERE / "golden_meta.json").write_text(json.dumps(meta, indent=1, default=str))
    print(f"wrote {len(out)} arrays, {(HERE / 'golden.npz').stat().st_size / 1e6:.2f} MB")


if __name__ == "__main__":
    # the reference's `src` directory: argument, LOWBIT_REF_SRC, or a
    # `reference` checkout beside this repository
    import os
    default = os.environ.get("LOWBIT_REF_SRC", str(HERE.parents[2] / "reference" / "src"))
    main(sys.argv[1] if len(sys.argv) > 1 else default)
