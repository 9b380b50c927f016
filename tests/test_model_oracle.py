"""The decoder oracle (oracle/model_ref.py) against the reference's own model
forward (tests/golden/golden_model.npz, made by tests/golden/make_model_golden.py).
CPU only: pins the checker the GPU model tests compare against."""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from lowbit_b200 import model as PM
from lowbit_b200.formats import quantize_int4, quantize_mxfp4
from oracle import model_ref as O

GOLD = Path(__file__).parent / "golden"
Z = np.load(GOLD / "golden_model.npz")
META = json.loads((GOLD / "golden_model_meta.json").read_text())

BACKEND_KW = {
    "fp32": ("fp32", {}), "w4a16": ("w4a16", {}), "w4a16_asym": ("w4a16", dict(asym=True)),
    "w4a16_smax": ("w4a16", dict(int4_scale="signed-max")), "w4a8": ("w4a8", {}),
    "w4a8_asym": ("w4a8", dict(asym=True)), "mxfp4": ("mxfp4", {}),
    "w4a16_fp32head": ("w4a16", dict(quantize_lm_head=False)),
}


def _digest(W):
    h = hashlib.sha256()
    for name in sorted(W):
        a = np.ascontiguousarray(W[name], np.float32)
        h.update(name.encode() + str(a.shape).encode() + a.tobytes())
    return h.hexdigest()


def oracle_linears(cfg, W, backend, asym=False, int4_scale="absmax", quantize_lm_head=True):
    """Oracle linears on weights packed by lowbit_b200's quantizers (pinned bit
    for bit to the reference's by tests/test_formats.py)."""
    lin = {}
    for key, (w, b) in O.concat_weights(cfg, W).items():
        kind = backend if (key != "lm_head" or quantize_lm_head) else "fp32"
        if kind == "fp32":
            lin[key] = O.lin_fp32(w, b)
        elif kind == "mxfp4":
            q = quantize_mxfp4(w)
            lin[key] = O.lin_mxfp4(q.qw, q.e8m0, q.k, b)
        else:
            q = quantize_int4(w, asym=asym, scale=int4_scale)
            lin[key] = (O.lin_w4a16(q.qw, q.scales, q.zeros, q.k, b) if kind == "w4a16"
                        else O.lin_w4a8(q.qw, q.scales, q.zeros, b))
    return lin


def case(tag):
    c = META["cases"][tag]
    cfg = O.tiny_cfg(**c["config"])
    return cfg, O.random_weights(cfg, seed=c["seed"]), c["tokens"]


def rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


@pytest.mark.parametrize("tag", sorted(META["cases"]))
def test_random_weights_bit_identical(tag):
    cfg, W, _ = case(tag)
    assert _digest(W) == META["cases"][tag]["weights_sha256"]
    # the product's generator draws the same numbers
    pc = PM.tiny_config(**META["cases"][tag]["config"])
    assert _digest(PM.random_weights(pc, seed=META["cases"][tag]["seed"])) == META["cases"][tag]["weights_sha256"]


GOLD_KEYS = sorted({k[: -len("_all")] for k in Z.files if k.endswith("_all")})


@pytest.mark.parametrize("key", GOLD_KEYS)
def test_oracle_matches_reference_forward(key):
    tag, btag = key.split("_", 1)
    cfg, W, toks = case(tag)
    backend, kw = BACKEND_KW[btag]
    m = O.Model(cfg, W, oracle_linears(cfg, W, backend, **kw))
    # int8 activations: a last-bit difference upstream can move a value across a
    # rounding boundary of the per-token quantizer, so w4a8 agrees to ~1e-3
    tol = 1e-2 if backend == "w4a8" else 1e-5
    assert rel(m.forward(toks, logits="all"), Z[key + "_all"]) < tol
    c = O.new_cache(cfg, len(toks) + 8)
    a, b = (10, 17) if len(toks) >= 17 else (4, 6)
    parts = [m.forward(toks[:a], c, logits="all"), m.forward(toks[a:b], c, logits="all")]
    parts += [m.forward([t], c)[None] for t in toks[b:]]
    assert rel(np.concatenate(parts), Z[key + "_cached"]) < tol
    assert m.generate(toks[:5], 6) == list(Z[key + "_gen"])
