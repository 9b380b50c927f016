"""Generate tests/golden/golden_model.npz from the reference's numpy model forward.

Run in a container that has the reference checkout (the fixture is committed;
the GPU box never needs the reference):

    CC=/usr/bin/gcc LOWBIT_BUILD_DIR=/tmp/lbbuild \\
        python tests/golden/make_model_golden.py /path/to/lowbit/src

It imports the reference package (`lowbit`) and records, for its tiny random
test models (src/lowbit/model.py:481-513, seeds as in the reference's
tests/test_model.py), with every linear backend it has:
  * the logits of a full forward pass over a token sequence (logits="all"),
  * the logits of the same sequence run through the KV cache in pieces
    (10 tokens, 7 tokens, then one token at a time; 4, 2, then single tokens
    for sequences shorter than 17),
  * the greedy continuation generate() produces,
  * a SHA-256 digest of random_weights(), so lowbit_b200's restatement of the
    weight generator is pinned bit for bit.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# (tag, tiny_config overrides, random_weights seed, token sequence)
CASES = [
    ("tiny", {}, 3, [(i * 5) % 97 for i in range(24)]),
    ("gqa1", dict(num_kv_heads=1, tie_word_embeddings=False, qkv_bias=False, head_dim=32,
                  num_heads=8), 7, [3, 1, 4, 1, 5, 9, 2, 6]),
    ("mha", dict(num_kv_heads=4), 7, [(i * 7) % 97 for i in range(20)]),
]
# (tag, Model keyword arguments)
BACKENDS = [
    ("fp32", dict(backend="fp32")),
    ("w4a16", dict(backend="w4a16")),
    ("w4a16_asym", dict(backend="w4a16", asym=True)),
    ("w4a16_smax", dict(backend="w4a16", int4_scale="signed-max")),
    ("w4a8", dict(backend="w4a8")),
    ("w4a8_asym", dict(backend="w4a8", asym=True)),
    ("mxfp4", dict(backend="mxfp4")),
    ("w4a16_fp32head", dict(backend="w4a16", quantize_lm_head=False)),
]


def weights_digest(W: dict) -> str:
    h = hashlib.sha256()
    for name in sorted(W):
        a = np.ascontiguousarray(W[name], np.float32)
        h.update(name.encode() + str(a.shape).encode() + a.tobytes())
    return h.hexdigest()


def main(ref_src: str) -> None:
    sys.path.insert(0, ref_src)
    from lowbit import model as M

    out: dict[str, np.ndarray] = {}
    meta = {"reference": "azrabano23/lowbit", "cases": {}}
    for tag, over, seed, toks in CASES:
        cfg = M.tiny_config(**over)
        W = M.random_weights(cfg, seed=seed)
        meta["cases"][tag] = {"config": over, "seed": seed, "tokens": toks,
                              "weights_sha256": weights_digest(W)}
        out[f"{tag}_tokens"] = np.asarray(toks, np.int64)
        for btag, kw in BACKENDS:
            if tag != "tiny" and btag not in ("fp32", "w4a16_asym"):
                continue
            m = M.Model(cfg, W, **kw)
            p = f"{tag}_{btag}_"
            out[p + "all"] = m.forward(toks, logits="all").astype(np.float32)
            c = m.new_cache(len(toks) + 8)
            a, b = (10, 17) if len(toks) >= 17 else (4, 6)
            parts = [m.forward(toks[:a], c, logits="all"), m.forward(toks[a:b], c, logits="all")]
            parts += [m.forward([t], c)[None] for t in toks[b:]]
            out[p + "cached"] = np.concatenate(parts).astype(np.float32)
            out[p + "gen"] = np.asarray(m.generate(toks[:5], 6), np.int64)
    np.savez_compressed(HERE / "golden_model.npz", **out)
    (HERE / "golden_model_meta.json").write_text(json.dumps(meta, indent=1) + "\n")
    print(f"wrote {len(out)} arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "src")
