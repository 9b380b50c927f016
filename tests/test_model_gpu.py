"""The GPU decoder (lowbit_b200.model) against the reference's own model
forward (tests/golden/golden_model.npz) and the pinned numpy oracle
(oracle/model_ref.py): logits, the KV-cache path, greedy generation, CUDA-graph
decode and batched decode."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from lowbit_b200 import model as PM
from oracle import model_ref as O

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).parent / "golden"
Z = np.load(GOLD / "golden_model.npz")
META = json.loads((GOLD / "golden_model_meta.json").read_text())
KW = {
    "fp32": ("fp32", {}), "w4a16": ("w4a16", {}), "w4a16_asym": ("w4a16", dict(asym=True)),
    "w4a16_smax": ("w4a16", dict(int4_scale="signed-max")), "w4a8": ("w4a8", {}),
    "w4a8_asym": ("w4a8", dict(asym=True)), "mxfp4": ("mxfp4", {}),
    "w4a16_fp32head": ("w4a16", dict(quantize_lm_head=False)),
}
KEYS = sorted({k[: -len("_all")] for k in Z.files if k.endswith("_all")})


def rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


def build(key):
    tag, btag = key.split("_", 1)
    c = META["cases"][tag]
    cfg = PM.tiny_config(**c["config"])
    W = PM.random_weights(cfg, seed=c["seed"])
    backend, kw = KW[btag]
    return PM.Model(cfg, W, backend=backend, **kw), c["tokens"], backend


def tol(backend):
    # fp32 paths differ from the reference only by summation order; int8
    # activations can cross a rounding boundary of the per-token quantizer
    return 1e-2 if backend == "w4a8" else 1e-4


@pytest.mark.parametrize("key", KEYS)
def test_forward_matches_reference(key):
    m, toks, backend = build(key)
    assert rel(m.forward(toks, logits="all"), Z[key + "_all"]) < tol(backend)
    last = m.forward(toks)
    assert last.shape == (m.cfg.vocab_size,)
    assert rel(last, Z[key + "_all"][-1]) < tol(backend)
    assert m.forward(toks, logits="none").shape == (len(toks), m.cfg.hidden_size)


@pytest.mark.parametrize("key", KEYS)
def test_kv_cache_pieces_match_reference(key):
    m, toks, backend = build(key)
    c = m.new_cache(len(toks) + 8)
    a, b = (10, 17) if len(toks) >= 17 else (4, 6)
    parts = [m.forward(toks[:a], c, logits="all"), m.forward(toks[a:b], c, logits="all")]
    parts += [m.forward([t], c)[None] for t in toks[b:]]
    assert c.length == len(toks)
    assert rel(np.concatenate(parts), Z[key + "_cached"]) < tol(backend)
    with pytest.raises(ValueError):
        m.forward(list(range(9)), c)  # len + 9 > capacity


@pytest.mark.parametrize("key", KEYS)
def test_generate_matches_reference(key):
    m, toks, _ = build(key)
    t = {}
    assert m.generate(toks[:5], 6, timings=t) == list(Z[key + "_gen"])
    assert t["decode_forwards"] == 5
    assert m.generate(toks[:5], 6, graph=False) == list(Z[key + "_gen"])


@pytest.mark.parametrize("backend", ["w4a16", "w4a8", "mxfp4", "fp32"])
def test_batched_decode_equals_single(backend):
    cfg = PM.tiny_config()
    W = PM.random_weights(cfg, seed=3)
    m = PM.Model(cfg, W, backend=backend, asym=True)
    prompts = (np.arange(4 * 9).reshape(4, 9) * 11) % cfg.vocab_size
    got = m.generate_batch(prompts, 7)
    for b in range(4):
        assert list(got[b]) == m.generate(prompts[b], 7), b


def test_graph_replay_logits_equal_eager():
    cfg = PM.tiny_config()
    W = PM.random_weights(cfg, seed=5)
    m = PM.Model(cfg, W, backend="w4a16", asym=True)
    toks = [(i * 13) % 97 for i in range(12)]
    c1, c2 = m.new_cache(40), m.new_cache(40)
    m.forward(toks, c1)
    m.forward(toks, c2)
    g, tok = m._decode_graph(c1)
    for step in range(6):
        tok.fill_(step * 7 % 97)
        g.replay()
        c1._length += 1
        ref = m.forward([step * 7 % 97], c2)
        assert int(tok.item()) == int(np.argmax(ref))
        assert int(c1.pos.item()) == c2.length


def test_prefill_path_against_oracle():
    """64+ token prefill runs the bf16 prefill GEMMs (4e-3 per-GEMM contract):
    logits stay within 2e-2 of the fp32 oracle."""
    from lowbit_b200.formats import quantize_int4
    cfg = PM.tiny_config()
    W = PM.random_weights(cfg, seed=11)
    m = PM.Model(cfg, W, backend="w4a16", asym=True)
    toks = [(i * 17 + 3) % 97 for i in range(96)]
    ocfg = O.tiny_cfg()
    lin = {}
    for key, (w, b) in O.concat_weights(ocfg, W).items():
        q = quantize_int4(w, asym=True)
        lin[key] = O.lin_w4a16(q.qw, q.scales, q.zeros, q.k, b)
    ref = O.Model(ocfg, W, lin).forward(toks, logits="all")
    assert rel(m.forward(toks, logits="all"), ref) < 2e-2


def test_operator_errors():
    from lowbit_b200.kernels import lib
    assert lib().lbc_attention(None, None, None, None, None, 1, 1, 4, 2, 48, 16, None) < 0  # head_dim 48
    assert lib().lbc_qkv_rope(None, None, None, None, None, None, None, None, 1, 1, 3, 2, 64, 16, None) < 0
    assert lib().lbc_rmsnorm(None, None, None, None, None, 1, 0, 1e-6, None) < 0
    torch.cuda.synchronize()
