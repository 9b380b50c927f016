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


@pytest.mark.parametrize("H,KV,D", [(14, 2, 64), (4, 4, 32), (8, 1, 128)])
def test_fused_rope_attention_equals_separate_kernels(H, KV, D):
    """lbc_rope_attention (decode steps) = lbc_qkv_rope then lbc_attention, bit for bit."""
    from lowbit_b200.kernels import lib
    B, S, pos = 3, 40, 13
    g = torch.Generator().manual_seed(0)
    W = (H + 2 * KV) * D
    qkv = torch.randn(B, W, generator=g).cuda()
    bias = torch.randn(W, generator=g).cuda()
    cos, sin = (torch.from_numpy(a).cuda() for a in PM.rope_tables(D, 64, 1e4))
    kc = torch.randn(B, KV, S, D, generator=g).cuda()
    vc = torch.randn(B, KV, S, D, generator=g).cuda()
    k2, v2 = kc.clone(), vc.clone()
    p = torch.tensor([pos], dtype=torch.int32, device="cuda")
    q = torch.empty(B, H * D, device="cuda")
    o1, o2 = torch.empty(B, H * D, device="cuda"), torch.empty(B, H * D, device="cuda")
    L, st = lib(), torch.cuda.current_stream().cuda_stream
    assert L.lbc_qkv_rope(qkv.data_ptr(), bias.data_ptr(), cos.data_ptr(), sin.data_ptr(), p.data_ptr(), q.data_ptr(),
                          kc.data_ptr(), vc.data_ptr(), B, 1, H, KV, D, S, st) == 0
    assert L.lbc_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), p.data_ptr(), o1.data_ptr(), B, 1, H, KV, D,
                           S, st) == 0
    assert L.lbc_rope_attention(qkv.data_ptr(), bias.data_ptr(), cos.data_ptr(), sin.data_ptr(), p.data_ptr(),
                                k2.data_ptr(), v2.data_ptr(), o2.data_ptr(), B, H, KV, D, S, st) == 0
    torch.cuda.synchronize()
    assert torch.equal(kc, k2) and torch.equal(vc, v2)
    assert torch.equal(o1, o2)
    # against a float64 evaluation of the same attention
    qd = q.double().view(B, H, D)
    kd, vd = kc.double()[:, :, :pos + 1], vc.double()[:, :, :pos + 1]
    G = H // KV
    ref = torch.empty(B, H, D, dtype=torch.float64)
    for b in range(B):
        for h in range(H):
            s = (kd[b, h // G] @ qd[b, h]) / np.sqrt(D)
            ref[b, h] = torch.softmax(s, 0) @ vd[b, h // G]
    assert float((o1.double().cpu().view(B, H, D) - ref.cpu()).abs().max()) < 1e-4


@pytest.mark.parametrize("m,n,k", [(1, 1152, 896), (2, 300, 256), (1, 96, 4864), (2, 513, 1024)])
def test_fused_decode_gemvs_equal_two_kernel_path(m, n, k):
    """lbc_gemm_w4a16_glu equals lbc_silu_mul + lbc_gemm_w4a16 bit for bit;
    lbc_gemm_w4a16_rmsnorm equals lbc_rmsnorm + lbc_gemm_w4a16 up to the order
    of the norm's sum of squares, and stores x + residual."""
    import ctypes as C
    from lowbit_b200.kernels import _Params, lib
    from lowbit_b200.kernels import quantize_int4_cuda
    L, st = lib(), torch.cuda.current_stream().cuda_stream
    g = torch.Generator().manual_seed(m * 7 + n)
    W = quantize_int4_cuda(torch.randn(n, k, generator=g), asym=True)
    args = (W.qw.data_ptr(), W.scales.data_ptr(), W.zeros.data_ptr(), n)
    P = C.byref(_Params(-1, 0, 0, 0, 0, 0, 0))
    # GLU
    gu = torch.randn(m, 2 * k, generator=g).cuda()
    mid = torch.empty(m, k, device="cuda")
    y1, y2 = torch.empty(m, n, device="cuda"), torch.empty(m, n, device="cuda")
    assert L.lbc_silu_mul(gu.data_ptr(), mid.data_ptr(), m, k, st) == 0
    assert L.lbc_gemm_w4a16(mid.data_ptr(), m, k, *args, y1.data_ptr(), P, st) >= 0
    assert L.lbc_gemm_w4a16_glu(gu.data_ptr(), m, k, *args, y2.data_ptr(), P, st) >= 0
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    # RMSNorm with a residual
    x = torch.randn(m, k, generator=g).cuda()
    r = torch.randn(m, k, generator=g).cuda()
    w = (1 + 0.1 * torch.randn(k, generator=g)).cuda()
    xs, h = x.clone(), torch.empty(m, k, device="cuda")
    xo = torch.empty(m, k, device="cuda")
    assert L.lbc_rmsnorm(xs.data_ptr(), r.data_ptr(), xs.data_ptr(), w.data_ptr(), h.data_ptr(), m, k, 1e-6, st) == 0
    assert L.lbc_gemm_w4a16(h.data_ptr(), m, k, *args, y1.data_ptr(), P, st) >= 0
    assert L.lbc_gemm_w4a16_rmsnorm(x.data_ptr(), r.data_ptr(), xo.data_ptr(), w.data_ptr(), 1e-6, m, k, *args,
                                    y2.data_ptr(), P, st) >= 0
    torch.cuda.synchronize()
    assert torch.equal(xo, xs)
    scale = float(y1.abs().max())
    assert float((y1 - y2).abs().max()) <= 1e-5 * scale
    # no residual: x as given, x_out untouched
    assert L.lbc_gemm_w4a16_rmsnorm(x.data_ptr(), None, None, w.data_ptr(), 1e-6, m, k, *args, y2.data_ptr(), P,
                                    st) >= 0
    assert L.lbc_rmsnorm(x.data_ptr(), None, None, w.data_ptr(), h.data_ptr(), m, k, 1e-6, st) == 0
    assert L.lbc_gemm_w4a16(h.data_ptr(), m, k, *args, y1.data_ptr(), P, st) >= 0
    torch.cuda.synchronize()
    assert float((y1 - y2).abs().max()) <= 1e-5 * float(y1.abs().max())


def test_fused_decode_gemv_rejects_ineligible_calls():
    import ctypes as C
    from lowbit_b200.kernels import _Params, lib
    L = lib()
    P = C.byref(_Params(-1, 0, 0, 0, 0, 0, 0))
    x = torch.zeros(3, 256, device="cuda")
    q = torch.zeros(8, 128, dtype=torch.uint8, device="cuda")
    s = torch.ones(8, 2, device="cuda")
    y = torch.empty(3, 8, device="cuda")
    # three tokens: not a decode shape
    assert L.lbc_gemm_w4a16_glu(x.data_ptr(), 3, 128, q.data_ptr(), s.data_ptr(), None, 8, y.data_ptr(), P, None) == -2
    # x_out aliasing x
    assert L.lbc_gemm_w4a16_rmsnorm(x.data_ptr(), x.data_ptr(), x.data_ptr(), s.data_ptr(), 1e-6, 1, 256,
                                    q.data_ptr(), s.data_ptr(), None, 8, y.data_ptr(), P, None) == -1


@pytest.mark.parametrize("B,S,pos", [(1, 1100, 0), (1, 1100, 130), (2, 4100, 4000), (3, 20000, 17000), (1, 300, 200)])
def test_key_split_attention(B, S, pos):
    """Long caches with few (sequence, KV head) pairs take the key-split path
    (blocks of 64 keys merged by a second kernel; 20000 positions would not
    fit the single-pass kernel's shared memory), short ones the single-pass
    kernel: both equal a float64 softmax attention, and the fused RoPE variant
    equals the separate kernels bit for bit."""
    from lowbit_b200.kernels import lib
    H, KV, D = 14, 2, 64
    g = torch.Generator().manual_seed(B * 1000 + pos)
    W = (H + 2 * KV) * D
    qkv = torch.randn(B, W, generator=g).cuda()
    bias = torch.randn(W, generator=g).cuda()
    cos, sin = (torch.from_numpy(a).cuda() for a in PM.rope_tables(D, S, 1e6))
    kc = torch.randn(B, KV, S, D, generator=g).cuda()
    vc = torch.randn(B, KV, S, D, generator=g).cuda()
    k2, v2 = kc.clone(), vc.clone()
    p = torch.tensor([pos], dtype=torch.int32, device="cuda")
    q = torch.empty(B, H * D, device="cuda")
    o1, o2 = torch.empty(B, H * D, device="cuda"), torch.empty(B, H * D, device="cuda")
    L, st = lib(), torch.cuda.current_stream().cuda_stream
    assert L.lbc_qkv_rope(qkv.data_ptr(), bias.data_ptr(), cos.data_ptr(), sin.data_ptr(), p.data_ptr(), q.data_ptr(),
                          kc.data_ptr(), vc.data_ptr(), B, 1, H, KV, D, S, st) == 0
    assert L.lbc_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), p.data_ptr(), o1.data_ptr(), B, 1, H, KV, D,
                           S, st) == 0
    assert L.lbc_rope_attention(qkv.data_ptr(), bias.data_ptr(), cos.data_ptr(), sin.data_ptr(), p.data_ptr(),
                                k2.data_ptr(), v2.data_ptr(), o2.data_ptr(), B, H, KV, D, S, st) == 0
    torch.cuda.synchronize()
    assert torch.equal(kc, k2) and torch.equal(vc, v2)
    assert torch.equal(o1, o2)
    qd = q.double().view(B, H, D).cpu()
    kd, vd = kc.double()[:, :, :pos + 1].cpu(), vc.double()[:, :, :pos + 1].cpu()
    G = H // KV
    ref = torch.empty(B, H, D, dtype=torch.float64)
    for b in range(B):
        for h in range(H):
            s = (kd[b, h // G] @ qd[b, h]) / np.sqrt(D)
            ref[b, h] = torch.softmax(s, 0) @ vd[b, h // G]
    assert float((o1.double().cpu().view(B, H, D) - ref).abs().max()) < 1e-4


@pytest.mark.parametrize("backend", ["w4a16", "w4a8"])
def test_profile_sections(backend):
    """Model.prof (the reference's Profile, src/lowbit/model.py:243-261): with
    profiling on, prefill and graph-replayed decode record device time in the
    reference's four sections; results are identical with it off; the
    sections of a decode step sum to no more than the step's wall time."""
    key = next(k for k in KEYS if k.endswith("_" + backend))
    m, toks, _ = build(key)
    c = m.new_cache(len(toks) + 12)
    ref = m.generate(toks, 10, cache=c)
    m.prof.enabled = True
    m.prof.reset()
    c.reset()
    t = {}
    got = m.generate(toks, 10, cache=c, timings=t)
    assert got == ref
    prof = dict(m.prof.t)
    assert set(prof) == {"linear", "attention", "lm_head", "other"}, prof
    assert all(v > 0 for v in prof.values()), prof
    assert sum(prof.values()) <= t["prefill_s"] + t["decode_s"], (prof, t)
    m.prof.enabled = False
    m.prof.reset()
    c.reset()
    assert m.generate(toks, 10, cache=c) == ref
    assert dict(m.prof.t) == {}
