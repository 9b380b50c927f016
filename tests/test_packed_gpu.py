"""A model written with save_packed and read back with load_packed is the same
model: identical packed bytes, identical logits (bit for bit), identical greedy
tokens, for every backend, and a loaded model matches the reference's golden
logits like a freshly quantized one."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from lowbit_b200 import model as PM

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).parent / "golden"
META = json.loads((GOLD / "golden_model_meta.json").read_text())
Z = np.load(GOLD / "golden_model.npz")
VARIANTS = {"fp32": ("fp32", {}), "w4a16": ("w4a16", {}), "w4a16_asym": ("w4a16", dict(asym=True)),
            "w4a16_smax": ("w4a16", dict(int4_scale="signed-max")), "w4a8_asym": ("w4a8", dict(asym=True)),
            "mxfp4": ("mxfp4", {}), "w4a16_fp32head": ("w4a16", dict(quantize_lm_head=False))}


def _tiny(variant, tag="tiny"):
    c = META["cases"][tag]
    cfg = PM.tiny_config(**c["config"])
    backend, kw = VARIANTS[variant]
    return PM.Model(cfg, PM.random_weights(cfg, seed=c["seed"]), backend=backend, **kw), c["tokens"]


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_packed_model_round_trip(tmp_path, variant):
    m, toks = _tiny(variant)
    p = tmp_path / "m.safetensors"
    PM.save_packed(m, p)
    m2 = PM.load_packed(p)
    assert (m2.backend, m2.asym, m2.quantize_lm_head, m2.int4_scale) == \
        (m.backend, m.asym, m.quantize_lm_head, m.int4_scale)
    for a, b in zip(m.linears(), m2.linears()):
        assert type(a) is type(b) and (a.n, a.k) == (b.n, b.k)
        if hasattr(a, "wq"):
            for f in ("qw", "scales", "zeros", "e8m0"):
                x, y = getattr(a.wq, f, None), getattr(b.wq, f, None)
                assert (x is None) == (y is None)
                if x is not None:
                    np.testing.assert_array_equal(x, y)
                    assert torch.equal(getattr(a.d, f), getattr(b.d, f))
    np.testing.assert_array_equal(m.forward(toks, logits="all"), m2.forward(toks, logits="all"))
    assert m.generate(toks[:5], 6) == m2.generate(toks[:5], 6)


def test_packed_model_matches_reference_golden(tmp_path):
    """The loaded model against the reference's own logits (same bound as a
    freshly quantized one)."""
    m, toks = _tiny("w4a16_asym")
    p = tmp_path / "m.safetensors"
    PM.save_packed(m, p)
    got = PM.load_packed(p).forward(toks, logits="all")
    ref = Z["tiny_w4a16_asym_all"]
    assert float(np.abs(got - ref).max() / np.abs(ref).max()) < 1e-4


def test_load_packed_rejects_other_files(tmp_path):
    from lowbit_b200 import packed as PK
    p = tmp_path / "x.safetensors"
    PK.write_tensors(p, {"a": np.ones(2, np.float32)})
    with pytest.raises(ValueError, match="not a lowbit_b200 packed model"):
        PM.load_packed(p)
