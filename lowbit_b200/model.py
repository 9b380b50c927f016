"""Decoder-only LLM forward (Qwen2 / Llama architecture) on the GPU.

The model-side caller of the quantized GEMMs, with the interface of the
reference's numpy model (src/lowbit/model.py of azrabano23/lowbit): the same
ModelConfig, Linear backends (fp32 / w4a16 / w4a8 / mxfp4), Model(cfg,
weights, backend, ...) with forward(tokens, cache, logits) and greedy
generate(), KV caches, tiny_config() and random_weights(). q/k/v and
gate/up are concatenated along N into one GEMM each (src/lowbit/model.py:
297-306), so a layer runs four quantized GEMMs.

Everything between the GEMMs runs as this library's CUDA kernels
(lbc_rmsnorm with the residual add fused in, lbc_qkv_rope with the qkv bias
fused in and the KV-cache append, lbc_attention, lbc_silu_mul). Positions
live in device memory, so a whole decode step (embedding, 24 layers, head,
argmax) is captured once as a CUDA graph and replayed for every token.
Activations, norms, biases and the KV cache are fp32, as in the reference.
Weights are quantized on the GPU (lbc_quantize_int4 / lbc_quantize_mxfp4,
bit-identical to the numpy quantizers), so loading never round-trips W
through the host quantizer.

Beyond the reference: several sequences of equal length decode together
(generate_batch): their rows share every GEMM, so the weights stream once
per step for the whole batch.
"""
from __future__ import annotations

import json
import time
from collections import defaultdict
from contextlib import contextmanager
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .kernels import quantize_int4_cuda, quantize_mxfp4_cuda

BACKENDS = ("fp32", "w4a16", "w4a8", "mxfp4")


def _torch():
    import torch
    return torch


def _lib():
    from .kernels import lib
    return lib()


def _check(rc: int, what: str) -> None:
    from .kernels import _check as chk
    chk(rc, what)


def _stream() -> int:
    from ._torch import stream_handle
    return stream_handle()


# ---------------------------------------------------------------- config

@dataclass
class ModelConfig:
    """Architecture hyper-parameters (src/lowbit/model.py:40-76)."""
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    tie_word_embeddings: bool = False
    qkv_bias: bool = False
    max_position: int = 4096
    name: str = "custom"

    @classmethod
    def from_hf(cls, cfg: dict, name: str = "custom") -> "ModelConfig":
        """From a Hugging Face config.json (qwen2 / llama / mistral)."""
        mt = cfg.get("model_type", "llama")
        if mt not in ("qwen2", "llama", "mistral"):
            raise ValueError(f"unsupported model_type {mt!r} (qwen2/llama/mistral only)")
        if cfg.get("rope_scaling"):
            raise ValueError("rope_scaling is not implemented")
        h, nh = cfg["hidden_size"], cfg["num_attention_heads"]
        return cls(vocab_size=cfg["vocab_size"], hidden_size=h, intermediate_size=cfg["intermediate_size"],
                   num_layers=cfg["num_hidden_layers"], num_heads=nh,
                   num_kv_heads=cfg.get("num_key_value_heads", nh), head_dim=cfg.get("head_dim") or h // nh,
                   rms_norm_eps=cfg.get("rms_norm_eps", 1e-6), rope_theta=cfg.get("rope_theta", 10000.0),
                   tie_word_embeddings=cfg.get("tie_word_embeddings", False),
                   qkv_bias=(mt == "qwen2") or cfg.get("attention_bias", False),
                   max_position=cfg.get("max_position_embeddings", 4096), name=name)


def tiny_config(**over) -> ModelConfig:
    """The reference's tiny test model (src/lowbit/model.py:481-488)."""
    base = dict(vocab_size=97, hidden_size=256, intermediate_size=384, num_layers=2, num_heads=4,
                num_kv_heads=2, head_dim=64, rms_norm_eps=1e-6, rope_theta=10000.0, tie_word_embeddings=True,
                qkv_bias=True, max_position=256, name="tiny")
    base.update(over)
    return ModelConfig(**base)


def qwen2_0_5b_config() -> ModelConfig:
    """Qwen2-0.5B's shape (24 layers, hidden 896, 14/2 heads of 64, SwiGLU 4864,
    vocabulary 151936, tied embeddings, qkv bias, RoPE theta 1e6)."""
    return ModelConfig(vocab_size=151936, hidden_size=896, intermediate_size=4864, num_layers=24, num_heads=14,
                       num_kv_heads=2, head_dim=64, rms_norm_eps=1e-6, rope_theta=1e6, tie_word_embeddings=True,
                       qkv_bias=True, max_position=4096, name="qwen2-0.5b-shape")


def random_weights(cfg: ModelConfig, seed: int = 0, scale: float = 0.05) -> dict:
    """Seeded random weights with the reference's draw order, so the same seed
    gives bit-identical arrays (src/lowbit/model.py:491-513): embedding
    (scaled x20), final norm (1 + r), then per layer the two norms, q/k/v
    weights (+ biases), o, gate, up, down; an untied head last."""
    rng = np.random.default_rng(seed)

    def r(*shape):
        return (rng.standard_normal(shape) * scale).astype(np.float32)

    h, i, d = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    W = {"model.embed_tokens.weight": r(cfg.vocab_size, h) * 20, "model.norm.weight": 1 + r(h)}
    for li in range(cfg.num_layers):
        p = f"model.layers.{li}."
        W[p + "input_layernorm.weight"] = 1 + r(h)
        W[p + "post_attention_layernorm.weight"] = 1 + r(h)
        for nm, n in (("q", cfg.num_heads * d), ("k", cfg.num_kv_heads * d), ("v", cfg.num_kv_heads * d)):
            W[p + f"self_attn.{nm}_proj.weight"] = r(n, h)
            if cfg.qkv_bias:
                W[p + f"self_attn.{nm}_proj.bias"] = r(n)
        W[p + "self_attn.o_proj.weight"] = r(h, cfg.num_heads * d)
        W[p + "mlp.gate_proj.weight"] = r(i, h)
        W[p + "mlp.up_proj.weight"] = r(i, h)
        W[p + "mlp.down_proj.weight"] = r(h, i)
    if not cfg.tie_word_embeddings:
        W["lm_head.weight"] = r(cfg.vocab_size, h)
    return W


# ---------------------------------------------------------------- safetensors

_ST_DTYPES = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16}


def load_safetensors(path: Path | str) -> dict[str, np.ndarray]:
    """A .safetensors file as fp32 numpy arrays (bf16 widened exactly); the
    format is an 8-byte little-endian header length, a JSON header of
    {name: {dtype, shape, data_offsets}}, then the raw tensor bytes."""
    path = Path(path)
    with open(path, "rb") as f:
        hlen = int.from_bytes(f.read(8), "little")
        header = json.loads(f.read(hlen))
    data = np.memmap(path, dtype=np.uint8, mode="r", offset=8 + hlen)
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        dt = info["dtype"]
        if dt not in _ST_DTYPES:
            raise ValueError(f"{name}: unsupported dtype {dt}")
        lo, hi = info["data_offsets"]
        raw = np.frombuffer(data[lo:hi], dtype=_ST_DTYPES[dt])
        arr = (raw.astype(np.uint32) << 16).view(np.float32) if dt == "BF16" else raw.astype(np.float32)
        out[name] = arr.reshape(info["shape"])
    return out


# ---------------------------------------------------------------- profile

class Profile:
    """Device time per section, accumulated across forward calls: the GPU
    counterpart of the reference's Profile (src/lowbit/model.py:243-261), with
    the same `t`, `enabled`, `section(name)` and `reset()` and the sections it
    uses (linear, attention, lm_head, other). One CUDA timing event is
    recorded on the current stream where a section begins; the time from it
    to the next boundary (the next section, or the end of the forward) is the
    section's device time. Reading `t` synchronises and folds pending events
    in. Inside a CUDA-graph capture the events become event-record nodes of
    the graph, kept with it and read after each replay, so graph-replayed
    decode steps are split on the device's own clock. Event nodes sit between
    the kernels and cost each boundary the overlap of consecutive launches:
    a profiled step runs slower than an unprofiled one. The fused decode
    kernels count as "linear" (the input norms and SiLU*up run inside the
    GEMVs there). Off by default."""

    def __init__(self, enabled: bool = False):
        self.enabled = enabled
        self._t: dict = defaultdict(float)
        self._pending: list = []
        self._sink: list | None = None
        self._open = None  # (name, start event) of the section in progress

    def _mark(self):
        e = _torch().cuda.Event(enable_timing=True, external=True)
        e.record()
        if self._open is not None:
            name, e0 = self._open
            (self._sink if self._sink is not None else self._pending).append((name, e0, e))
        return e

    @contextmanager
    def section(self, name: str):
        if not self.enabled:
            yield
            return
        if self._open is None or self._open[0] != name:
            self._open = (name, self._mark())
        yield

    def close(self) -> None:
        """End the section in progress (at the end of a forward)."""
        if self.enabled and self._open is not None:
            self._mark()
            self._open = None

    @contextmanager
    def capturing(self):
        """Collect the sections recorded inside a graph capture (returned list)
        instead of treating them as pending."""
        marks: list = []
        self.close()
        prev, self._sink = self._sink, marks
        try:
            yield marks
        finally:
            self.close()
            self._sink = prev

    def add(self, marks) -> None:
        """Fold the (synchronised) events of one graph replay into the totals."""
        for name, e0, e1 in marks:
            self._t[name] += e0.elapsed_time(e1) * 1e-3

    def collect(self) -> None:
        self.close()
        if self._pending:
            _torch().cuda.synchronize()
            self.add(self._pending)
            self._pending = []

    @property
    def t(self) -> dict:
        self.collect()
        return self._t

    def reset(self) -> None:
        self._t = defaultdict(float)
        self._pending = []
        self._open = None


# ---------------------------------------------------------------- linear backends

class Linear:
    """y = x @ W.T (+ b) on the GPU: x a CUDA fp32 tensor [T, K]. Subclasses
    hold W in one format (src/lowbit/model.py:109-177)."""
    kind = "?"

    def __init__(self, w: np.ndarray, b: np.ndarray | None, threads: int | None):
        from ._torch import to_cuda
        self.n, self.k = w.shape
        self.b = None if b is None else to_cuda(np.asarray(b, np.float32))
        self.threads = threads

    def mm(self, x):  # pragma: no cover - abstract
        raise NotImplementedError

    def __call__(self, x):
        y = self.mm(x)
        if self.b is not None:
            y += self.b
        return y


class FP32Linear(Linear):
    """fp32 weights through torch.matmul (cuBLAS SGEMM, TF32 off): the
    unquantized baseline backend, not the product's hot path."""
    kind = "fp32"

    def __init__(self, w, b=None, threads=None, **_):
        from ._torch import to_cuda
        super().__init__(w, b, threads)
        self.w = to_cuda(np.ascontiguousarray(w, np.float32))
        self.nbytes = self.w.numel() * 4

    def mm(self, x):
        torch = _torch()
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            return x @ self.w.T
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev


class _LowbitLinear(Linear):
    """A quantized linear: the library GEMM on device-resident packed weights."""
    fn = ""

    def _setup(self, d, params):
        """d: the packed weights on the GPU (quantized there); `wq` keeps a host
        copy, as the reference's linears hold their packed arrays."""
        from dataclasses import replace
        self.d = d
        host = {f: (None if getattr(d, f) is None else getattr(d, f).cpu().numpy())
                for f in ("qw", "scales", "zeros", "e8m0") if hasattr(d, f)}
        self.wq = replace(d, **host)
        self.params = params
        self.nbytes = self.wq.nbytes

    def _setup_packed(self, d, host, params):
        """Packed weights read from a file: `d` on the GPU, `host` the same
        arrays on the host (no quantization, no device-to-host copy)."""
        self.d, self.wq, self.params = d, host, params
        self.nbytes = host.nbytes

    @classmethod
    def from_packed(cls, host, b=None, threads=None, params=None, device=None):
        """A linear on already packed weights (`host`: numpy arrays)."""
        from ._torch import to_cuda
        self = cls.__new__(cls)
        self.n, self.k = host.n, host.k
        self.b = None if b is None else to_cuda(np.asarray(b, np.float32), device)
        self.threads = threads
        self._setup_packed(host.cuda(device), host, params)
        return self

    def _x(self, x):
        torch = _torch()
        if x.shape[1] != self.wq.kp:
            x = torch.nn.functional.pad(x, (0, self.wq.kp - x.shape[1]))
        return x.contiguous()

    def _pparams(self, m: int):
        import ctypes as C
        from .kernels import _params
        return C.byref(_params(self.params, None, self.kind, (m, self.wq.n, self.wq.k)))


class ColumnParallelLinear(Linear):
    """Tensor parallelism for one linear (column parallel, as the north star and
    the survey fix it): this rank's rows shard_bounds(N, rank, world) of W in
    `inner` (any backend), Y [M, N] assembled on every rank, then the full
    bias. W4A16 decode (one or two tokens, default tiling) runs the GEMV with
    the all-gather fused in (lowbit_b200.sharding.FusedColumnParallel, one per
    (tokens, N) shared by the model's linears of that width); everything else
    runs the slice's GEMM and an NCCL all-gather (sharding.ColumnParallel).
    The model replicates the rest (norms, RoPE, attention: 14 query / 2 KV
    heads do not divide by 4 or 8)."""

    def __init__(self, inner: Linear, n: int, b, group, fused_pool: dict | None = None):
        from ._torch import to_cuda
        from .formats import shard_bounds
        import torch.distributed as dist
        self.inner, self.n, self.k, self.group = inner, n, inner.k, group
        self.kind = inner.kind
        self.b = None if b is None else to_cuda(np.asarray(b, np.float32))
        self.threads = inner.threads
        self.nbytes = inner.nbytes
        self._world = dist.get_world_size(group)
        self.lo, self.hi = shard_bounds(n, dist.get_rank(group), self._world)
        self._cps: dict = {}
        self._fused = fused_pool

    @property
    def wq(self):
        return self.inner.wq

    @property
    def params(self):
        return getattr(self.inner, "params", None)

    @params.setter
    def params(self, p):
        self.inner.params = p

    def mm(self, x):
        from .sharding import ColumnParallel, FusedColumnParallel
        m = int(x.shape[0])
        if (self._fused is not None and m <= 2 and self.kind == "w4a16" and self.params is None
                and self.inner.wq.kp % 128 == 0 and self._world <= 8):
            fc = self._fused.get((m, self.n))
            if fc is None:
                fc = self._fused[(m, self.n)] = FusedColumnParallel(m, self.n, self.group)
            return fc(self.inner._x(x), self.inner.d)
        y = self.inner.mm(x)
        cp = self._cps.get(m)
        if cp is None:
            cp = self._cps[m] = ColumnParallel(m, self.n, self.group)
        return cp.gather(y)


def tp_shard(w: np.ndarray, rank: int, world: int) -> np.ndarray:
    """Rows shard_bounds(N, rank, world) of a weight [N, K]: this rank's part of
    a column-parallel linear."""
    from .formats import shard_bounds
    lo, hi = shard_bounds(w.shape[0], rank, world)
    return np.ascontiguousarray(w[lo:hi])


class W4A16Linear(_LowbitLinear):
    kind = "w4a16"

    def __init__(self, w, b=None, threads=None, asym=False, params=None, int4_scale="absmax", **_):
        super().__init__(w, b, threads)
        self._setup(quantize_int4_cuda(np.asarray(w, np.float32), asym=asym, scale=int4_scale), params)

    def mm(self, x):
        torch = _torch()
        x = self._x(x)
        m = int(x.shape[0])
        y = torch.empty((m, self.n), dtype=torch.float32, device=x.device)
        d = self.d
        _check(_lib().lbc_gemm_w4a16(x.data_ptr(), m, self.wq.kp, d.qw.data_ptr(), d.scales.data_ptr(),
                                     None if d.zeros is None else d.zeros.data_ptr(), self.n, y.data_ptr(),
                                     self._pparams(m), _stream()), "lbc_gemm_w4a16")
        return y


    def mm_rmsnorm(self, x, res, x_out, norm_w, eps: float):
        """rmsnorm(x + res) @ W.T in one decode kernel (M <= 2); x + res -> x_out."""
        torch = _torch()
        m = int(x.shape[0])
        y = torch.empty((m, self.n), dtype=torch.float32, device=x.device)
        d = self.d
        _check(_lib().lbc_gemm_w4a16_rmsnorm(x.data_ptr(), None if res is None else res.data_ptr(),
                                             None if res is None else x_out.data_ptr(), norm_w.data_ptr(), eps, m,
                                             self.wq.kp, d.qw.data_ptr(), d.scales.data_ptr(),
                                             None if d.zeros is None else d.zeros.data_ptr(), self.n, y.data_ptr(),
                                             self._pparams(m), _stream()), "lbc_gemm_w4a16_rmsnorm")
        return y

    def mm_glu(self, gu):
        """(silu(gu[:, :K]) * gu[:, K:]) @ W.T in one decode kernel (M <= 2)."""
        torch = _torch()
        m = int(gu.shape[0])
        y = torch.empty((m, self.n), dtype=torch.float32, device=gu.device)
        d = self.d
        _check(_lib().lbc_gemm_w4a16_glu(gu.data_ptr(), m, self.wq.kp, d.qw.data_ptr(), d.scales.data_ptr(),
                                         None if d.zeros is None else d.zeros.data_ptr(), self.n, y.data_ptr(),
                                         self._pparams(m), _stream()), "lbc_gemm_w4a16_glu")
        return y


class W4A8Linear(_LowbitLinear):
    kind = "w4a8"

    def __init__(self, w, b=None, threads=None, asym=False, params=None, int4_scale="absmax", **_):
        super().__init__(w, b, threads)
        self._setup(quantize_int4_cuda(np.asarray(w, np.float32), asym=asym, scale=int4_scale), params)

    def mm(self, x):
        from .kernels import _workspace
        torch = _torch()
        x = self._x(x)
        m = int(x.shape[0])
        y = torch.empty((m, self.n), dtype=torch.float32, device=x.device)
        ws = _workspace(int(_lib().lbc_gemm_w4a8_workspace_size(m, self.wq.kp)))
        d = self.d
        _check(_lib().lbc_gemm_w4a8(x.data_ptr(), m, self.wq.kp, d.qw.data_ptr(), d.scales.data_ptr(),
                                    None if d.zeros is None else d.zeros.data_ptr(), self.n, y.data_ptr(),
                                    self._pparams(m), ws.data_ptr(), _stream()), "lbc_gemm_w4a8")
        return y


class MXFP4Linear(_LowbitLinear):
    kind = "mxfp4"

    def __init__(self, w, b=None, threads=None, params=None, **_):
        super().__init__(w, b, threads)
        self._setup(quantize_mxfp4_cuda(np.asarray(w, np.float32)), params)

    def mm(self, x):
        torch = _torch()
        x = self._x(x)
        m = int(x.shape[0])
        y = torch.empty((m, self.n), dtype=torch.float32, device=x.device)
        d = self.d
        _check(_lib().lbc_gemm_mxfp4(x.data_ptr(), m, self.wq.kp, d.qw.data_ptr(), d.e8m0.data_ptr(), self.n,
                                     y.data_ptr(), self._pparams(m), _stream()), "lbc_gemm_mxfp4")
        return y


LINEARS = {"fp32": FP32Linear, "w4a16": W4A16Linear, "w4a8": W4A8Linear, "mxfp4": MXFP4Linear}


# ---------------------------------------------------------------- KV cache

class KVCache:
    """Per layer K and V [B, KV, max_len, D] fp32 on the GPU; `length` tokens
    are filled (the same count for every sequence), mirrored on the device in
    `pos` (int32) for the kernels and CUDA graphs."""

    def __init__(self, cfg: ModelConfig, max_len: int, batch: int = 1):
        torch = _torch()
        shape = (batch, cfg.num_kv_heads, max_len, cfg.head_dim)
        self.k = [torch.zeros(shape, dtype=torch.float32, device="cuda") for _ in range(cfg.num_layers)]
        self.v = [torch.zeros(shape, dtype=torch.float32, device="cuda") for _ in range(cfg.num_layers)]
        self.batch = batch
        self.pos = torch.zeros(1, dtype=torch.int32, device="cuda")
        self._length = 0

    @classmethod
    def empty(cls, cfg: ModelConfig, max_len: int, batch: int = 1) -> "KVCache":
        return cls(cfg, max_len, batch)

    @property
    def capacity(self) -> int:
        return int(self.k[0].shape[2])

    @property
    def length(self) -> int:
        return self._length

    @length.setter
    def length(self, n: int) -> None:
        self._length = int(n)
        self.pos.fill_(int(n))

    def reset(self) -> None:
        """Empty the cache (keeps its buffers, so a captured decode graph stays valid)."""
        self.length = 0


@dataclass
class Layer:
    ln1: object
    qkv: Linear
    o: Linear
    ln2: object
    gate_up: Linear
    down: Linear


# ---------------------------------------------------------------- model

class Model:
    """Decoder forward with quantized linears (src/lowbit/model.py:276-457)."""

    def __init__(self, cfg: ModelConfig, weights: dict, backend: str = "fp32", threads: int | None = None,
                 asym: bool = False, quantize_lm_head: bool = True, params=None, int4_scale: str = "absmax",
                 _packed: tuple | None = None, group=None):
        from ._torch import require_cuda, to_cuda
        require_cuda()
        if backend not in LINEARS:
            raise ValueError(f"backend must be one of {BACKENDS}")
        self.cfg, self.backend, self.threads = cfg, backend, threads
        self.asym, self.quantize_lm_head, self.int4_scale = asym, quantize_lm_head, int4_scale
        lin = LINEARS[backend]
        kw = dict(threads=threads, asym=asym, params=params, int4_scale=int4_scale)
        W = weights

        def g(n):
            return np.asarray(W[n], np.float32)

        # tensor parallelism over `group` (a torch.distributed process group,
        # one rank per GPU): every linear column parallel, the rest replicated
        tp_world, tp_rank = 1, 0
        if group is not None:
            import torch.distributed as dist
            tp_world, tp_rank = dist.get_world_size(group), dist.get_rank(group)
        self.group, self.tp_world, self.tp_rank = group, tp_world, tp_rank
        self._tp_fused: dict = {}   # fused all-gather decode state per (tokens, N)

        def linear(name, cls, w, b):
            """The linear `name`: quantized from fp32 (w(), b() give the
            arrays), or built from a packed file's arrays (load_packed); with
            tensor parallelism this rank's row shard plus the all-gather."""
            if _packed is None:
                if tp_world > 1:
                    wf = w()
                    inner = cls(tp_shard(wf, tp_rank, tp_world), None, **kw)
                    return ColumnParallelLinear(inner, wf.shape[0], b(), group, self._tp_fused)
                return cls(w(), b(), **kw)
            if tp_world > 1:
                raise ValueError("tensor parallelism builds from fp32 weights, not packed files")
            return _packed_linear(name, cls, _packed, kw)

        self.embed = to_cuda(np.ascontiguousarray(g("model.embed_tokens.weight")))
        self.layers: list[Layer] = []
        for i in range(cfg.num_layers):
            p, a = f"model.layers.{i}.", f"model.layers.{i}.self_attn."

            def wqkv(a=a):
                return np.concatenate([g(a + "q_proj.weight"), g(a + "k_proj.weight"), g(a + "v_proj.weight")], 0)

            def bqkv(a=a):
                return (np.concatenate([g(a + "q_proj.bias"), g(a + "k_proj.bias"), g(a + "v_proj.bias")])
                        if cfg.qkv_bias else None)

            def wgu(p=p):
                return np.concatenate([g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight")], 0)

            def none():
                return None

            self.layers.append(Layer(
                ln1=to_cuda(g(p + "input_layernorm.weight")),
                qkv=linear(p + "qkv", lin, wqkv, bqkv),
                o=linear(p + "o", lin, lambda a=a: g(a + "o_proj.weight"), none),
                ln2=to_cuda(g(p + "post_attention_layernorm.weight")),
                gate_up=linear(p + "gate_up", lin, wgu, none),
                down=linear(p + "down", lin, lambda p=p: g(p + "mlp.down_proj.weight"), none)))
        self.norm = to_cuda(g("model.norm.weight"))

        def head():
            return g("model.embed_tokens.weight") if cfg.tie_word_embeddings or "lm_head.weight" not in W \
                else g("lm_head.weight")

        self.lm_head = linear("lm_head", lin if quantize_lm_head else FP32Linear, head, lambda: None)
        cos, sin = rope_tables(cfg.head_dim, cfg.max_position, cfg.rope_theta)
        self.cos, self.sin = to_cuda(cos), to_cuda(sin)
        # decode steps fuse the norms and the SiLU*up into the w4a16 GEMVs
        # (default tiling, unpadded hidden and intermediate sizes)
        self._fusable = (backend == "w4a16" and params is None and tp_world == 1 and cfg.hidden_size % 128 == 0
                         and cfg.intermediate_size % 128 == 0)
        self._graphs: dict = {}
        self.prof = Profile()

    # ------------------------------------------------------------ bookkeeping

    @property
    def linear_weight_bytes(self) -> int:
        return sum(x.nbytes for x in self.linears())

    def linears(self) -> list[Linear]:
        return [x for L in self.layers for x in (L.qkv, L.o, L.gate_up, L.down)] + [self.lm_head]

    def set_threads(self, threads: int | None) -> None:
        """Accepted for interface parity; the GPU kernels size their own grids."""
        self.threads = threads
        for x in self.linears():
            x.threads = threads

    def new_cache(self, max_len: int, batch: int = 1) -> KVCache:
        return KVCache(self.cfg, max_len, batch)

    # ------------------------------------------------------------ forward

    def _run(self, tok, B: int, T: int, cache: KVCache, logits: str, head_chunk: int = 256):
        """Device forward of B sequences x T tokens (rows b*T + t) at positions
        cache.pos..; returns device logits ([B, V] last, [B*T, V] all) or the
        final hidden states [B*T, hidden] for logits="none"."""
        torch = _torch()
        cfg = self.cfg
        lib, st = _lib(), _stream()
        H, KV, D, hid, I = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.hidden_size, cfg.intermediate_size
        n = B * T
        eps = float(cfg.rms_norm_eps)
        S = cache.capacity
        P = self.prof
        with P.section("other"):
            x = self.embed.index_select(0, tok)
        h = torch.empty((n, hid), dtype=torch.float32, device=x.device)
        q = torch.empty((n, H * D), dtype=torch.float32, device=x.device)
        att = torch.empty((n, H * D), dtype=torch.float32, device=x.device)
        m = torch.empty((n, I), dtype=torch.float32, device=x.device)
        # decode (one or two token rows) with w4a16 linears: the norms and the
        # SiLU*up run inside the GEMV kernels; the residual stream ping-pongs
        # between two buffers because the fused kernels read x while writing x + res
        fuse = self._fusable and n <= 2
        xb = torch.empty_like(x) if fuse else None
        res = None
        for li, L in enumerate(self.layers):
            if fuse:
                with P.section("linear"):
                    qkv = L.qkv.mm_rmsnorm(x, res, xb, L.ln1, eps)
                if res is not None:
                    x, xb = xb, x
            else:
                with P.section("other"):
                    _check(lib.lbc_rmsnorm(x.data_ptr(), None if res is None else res.data_ptr(), x.data_ptr(),
                                           L.ln1.data_ptr(), h.data_ptr(), n, hid, eps, st), "lbc_rmsnorm")
                with P.section("linear"):
                    qkv = L.qkv.mm(h)
            bias = None if L.qkv.b is None else L.qkv.b.data_ptr()
            with P.section("attention"):
                if T == 1:  # one launch: RoPE, cache append and attention
                    _check(lib.lbc_rope_attention(qkv.data_ptr(), bias, self.cos.data_ptr(), self.sin.data_ptr(),
                                                  cache.pos.data_ptr(), cache.k[li].data_ptr(),
                                                  cache.v[li].data_ptr(), att.data_ptr(), B, H, KV, D, S, st),
                           "lbc_rope_attention")
                else:
                    _check(lib.lbc_qkv_rope(qkv.data_ptr(), bias, self.cos.data_ptr(), self.sin.data_ptr(),
                                            cache.pos.data_ptr(), q.data_ptr(), cache.k[li].data_ptr(),
                                            cache.v[li].data_ptr(), B, T, H, KV, D, S, st), "lbc_qkv_rope")
                    _check(lib.lbc_attention(q.data_ptr(), cache.k[li].data_ptr(), cache.v[li].data_ptr(),
                                             cache.pos.data_ptr(), att.data_ptr(), B, T, H, KV, D, S, st),
                           "lbc_attention")
            with P.section("linear"):
                y = L.o.mm(att)
            if fuse:
                with P.section("linear"):
                    gu = L.gate_up.mm_rmsnorm(x, y, xb, L.ln2, eps)
                x, xb = xb, x
                with P.section("linear"):
                    res = L.down.mm_glu(gu)
            else:
                with P.section("other"):
                    _check(lib.lbc_rmsnorm(x.data_ptr(), y.data_ptr(), x.data_ptr(), L.ln2.data_ptr(),
                                           h.data_ptr(), n, hid, eps, st), "lbc_rmsnorm")
                with P.section("linear"):
                    gu = L.gate_up.mm(h)
                with P.section("other"):
                    _check(lib.lbc_silu_mul(gu.data_ptr(), m.data_ptr(), n, I, st), "lbc_silu_mul")
                with P.section("linear"):
                    res = L.down.mm(m)
        with P.section("other"):
            xn = torch.empty_like(h)
            _check(lib.lbc_rmsnorm(x.data_ptr(), res.data_ptr(), x.data_ptr(), self.norm.data_ptr(), xn.data_ptr(),
                                   n, hid, eps, st), "lbc_rmsnorm")
        if logits == "none":
            return xn
        with P.section("lm_head"):
            if logits == "last":
                return self.lm_head(xn.view(B, T, hid)[:, T - 1].contiguous())
            return torch.cat([self.lm_head(xn[i:i + head_chunk]) for i in range(0, n, head_chunk)])

    def forward(self, tokens, cache: KVCache | None = None, logits: str = "last",
                head_chunk: int = 256) -> np.ndarray:
        """Run tokens [T] at positions cache.length.. (0 without a cache), like
        the reference (src/lowbit/model.py:380-434): logits="last" -> [V],
        "all" -> [T, V], "none" -> final hidden states [T, hidden]. numpy out."""
        torch = _torch()
        tokens = np.asarray(tokens, np.int64).reshape(-1)
        T = int(tokens.shape[0])
        if cache is None:
            cache = self.new_cache(T)
        elif cache.batch != 1:
            raise ValueError("forward() runs one sequence; use generate_batch for several")
        if cache.length + T > cache.capacity:
            raise ValueError(f"KV cache full ({cache.length}+{T} > {cache.capacity})")
        tok = torch.from_numpy(tokens).to("cuda")
        out = self._run(tok, 1, T, cache, logits, head_chunk)
        self.prof.close()
        cache.length = cache.length + T
        out = out.cpu().numpy()
        return out[0] if logits == "last" else out

    # ------------------------------------------------------------ decoding

    def _decode_graph(self, cache: KVCache):
        """A CUDA graph of one greedy decode step for `cache`: embed the token
        in `tok`, run every layer at cache.pos, argmax into `tok`, pos += 1."""
        torch = _torch()
        live = self._graphs.get("decode")
        if live is not None and live[0] is cache and live[3] == self.prof.enabled:
            return live[1], live[2]
        B = cache.batch
        tok = torch.zeros(B, dtype=torch.int64, device="cuda")
        # warm-up and capture on one persistent side stream: the library's
        # per-(device, stream) scratch buffers are sized by the warm-up and
        # cannot first grow inside the capture
        if getattr(self, "_gstream", None) is None:
            self._gstream = torch.cuda.Stream()
        s = self._gstream
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):  # warm-up outside capture: workspaces, plans, cuBLAS handles
            saved = int(cache.pos.item())
            self._step(tok, cache)
            cache.pos.fill_(saved)
        g = torch.cuda.CUDAGraph()
        self.prof.collect()  # the warm-up step's sections, before the capture
        with self.prof.capturing() as marks:
            with torch.cuda.graph(g, stream=s):
                self._step(tok, cache)
        torch.cuda.current_stream().wait_stream(s)
        # one live decode graph per model; with profiling on it records the
        # sections of every replay (marks)
        self._graphs = {"decode": (cache, g, tok, self.prof.enabled, marks)}
        return g, tok

    def release_graphs(self) -> None:
        """Drop the cached decode graph (with tensor parallelism it holds NCCL
        calls: release it before destroying the process group) and close the
        fused all-gather buffers (collective: every rank calls it)."""
        self._graphs = {}
        for fc in self._tp_fused.values():
            fc.close()
        self._tp_fused.clear()

    def _step(self, tok, cache: KVCache):
        torch = _torch()
        logit = self._run(tok, cache.batch, 1, cache, "last")
        with self.prof.section("other"):
            tok.copy_(torch.argmax(logit, dim=-1))
            _check(_lib().lbc_advance_pos(cache.pos.data_ptr(), 1, _stream()), "lbc_advance_pos")
        self.prof.close()

    def generate(self, prompt, n_new: int, cache: KVCache | None = None, timings: dict | None = None,
                 graph: bool = True) -> list[int]:
        """Greedy decoding: prefill the prompt, then n_new tokens one at a time
        (src/lowbit/model.py:436-457). Decode steps replay one CUDA graph."""
        out = self.generate_batch([list(prompt)], n_new, cache=cache, timings=timings, graph=graph)
        return [int(t) for t in out[0]]

    def generate_batch(self, prompts, n_new: int, cache: KVCache | None = None, timings: dict | None = None,
                       graph: bool = True) -> np.ndarray:
        """Greedy decoding of B equal-length prompts together: [B, n_new] tokens.
        Each sequence's logits equal those of decoding it alone."""
        torch = _torch()
        prompts = np.asarray(prompts, np.int64)
        if prompts.ndim != 2:
            raise ValueError("prompts must be [B, T] (equal lengths)")
        B, T0 = prompts.shape
        cache = cache or self.new_cache(T0 + n_new, batch=B)
        if cache.batch != B:
            raise ValueError(f"cache holds {cache.batch} sequences, prompts {B}")
        if cache.length + T0 + max(0, n_new - 1) > cache.capacity:
            raise ValueError("KV cache too short for prompt + n_new")
        hist = torch.empty((max(n_new, 1), B), dtype=torch.int64, device="cuda")
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        logit = self._run(torch.from_numpy(prompts.reshape(-1)).to("cuda"), B, T0, cache, "last")
        cache.length = cache.length + T0
        if n_new > 0:
            with self.prof.section("other"):
                hist[0].copy_(torch.argmax(logit, dim=-1))
        self.prof.close()
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        prof0 = dict(self.prof.t) if self.prof.enabled else None
        if n_new > 1:
            if graph:
                g, tok = self._decode_graph(cache)
                marks = self._graphs["decode"][4] if self.prof.enabled else None
                tok.copy_(hist[0])
                for i in range(1, n_new):
                    g.replay()
                    hist[i].copy_(tok)
                    if marks:  # read this replay's section events
                        torch.cuda.synchronize()
                        self.prof.add(marks)
            else:
                tok = hist[0].clone()
                for i in range(1, n_new):
                    self._step(tok, cache)
                    hist[i].copy_(tok)
            cache._length += n_new - 1  # the device position advanced inside the steps
        out = hist[:n_new].T.cpu().numpy()
        t2 = time.perf_counter()
        if timings is not None:
            timings["prefill_s"] = t1 - t0
            timings["decode_s"] = t2 - t1
            timings["decode_forwards"] = max(0, n_new - 1)
            if prof0 is not None:  # the section split of this call (reference e2e.py:_one_run)
                now = self.prof.t
                timings["prof_prefill"] = {k: v for k, v in prof0.items()}
                timings["prof_decode"] = {k: now[k] - prof0.get(k, 0.0) for k in now}
        return out


def rope_tables(head_dim: int, n_pos: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    """cos / sin [n_pos, head_dim/2] of position * theta^(-2i/D), float64 angles
    rounded to fp32 (src/lowbit/model.py:193-196)."""
    inv = 1.0 / theta ** (np.arange(0, head_dim, 2, dtype=np.float64) / head_dim)
    ang = np.arange(n_pos, dtype=np.float64)[:, None] * inv[None]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


# ---------------------------------------------------------------- packed files

PACKED_VERSION = "1"


def _packed_linear(name: str, cls, packed: tuple, kw: dict):
    """Linear `name` of a packed file: its packed container (or, for an fp32
    linear, `<name>.weight`) and optional `<name>.bias`."""
    weights, extra = packed
    b = extra.get(name + ".bias")
    if cls is FP32Linear:
        if name + ".weight" not in extra:
            raise ValueError(f"{name}: the file holds no fp32 weight for an fp32 linear")
        return FP32Linear(extra[name + ".weight"], b, **kw)
    if name not in weights:
        raise ValueError(f"{name}: the file holds no packed weights")
    host = weights[name]
    from .formats import Int4Weights, MXFP4Weights
    want = MXFP4Weights if cls is MXFP4Linear else Int4Weights
    if not isinstance(host, want):
        raise ValueError(f"{name}: packed as {type(host).__name__}, backend {cls.kind} needs {want.__name__}")
    return cls.from_packed(host, b, kw.get("threads"), kw.get("params"))


def save_packed(model: Model, path: Path | str) -> None:
    """Write `model` as a packed-weight file (lowbit_b200.packed): every
    quantized linear's packed arrays as consumed by the kernels, fp32 linears,
    biases, norms and the embedding, and the configuration in the metadata,
    so that load_packed rebuilds the same model without quantizing."""
    from dataclasses import asdict

    from . import packed as PK
    weights, extra = {}, {"model.embed_tokens.weight": model.embed, "model.norm.weight": model.norm}
    named = [("lm_head", model.lm_head)]
    for i, L in enumerate(model.layers):
        p = f"model.layers.{i}."
        extra[p + "input_layernorm.weight"] = L.ln1
        extra[p + "post_attention_layernorm.weight"] = L.ln2
        named += [(p + "qkv", L.qkv), (p + "o", L.o), (p + "gate_up", L.gate_up), (p + "down", L.down)]
    for name, lin in named:
        if isinstance(lin, FP32Linear):
            extra[name + ".weight"] = lin.w
        else:
            weights[name] = lin.wq
        if lin.b is not None:
            extra[name + ".bias"] = lin.b
    meta = {"lowbit_b200.packed": PACKED_VERSION, "config": json.dumps(asdict(model.cfg)),
            "backend": model.backend, "asym": int(model.asym), "quantize_lm_head": int(model.quantize_lm_head),
            "int4_scale": model.int4_scale}
    PK.save_weights(path, weights, extra, meta)


def load_packed(path: Path | str, threads: int | None = None, params=None) -> Model:
    """A model written by save_packed, with its weights uploaded as stored."""
    from . import packed as PK
    weights, extra, meta = PK.load_weights(path)
    if meta.get("lowbit_b200.packed") != PACKED_VERSION:
        raise ValueError(f"{path}: not a lowbit_b200 packed model (version {meta.get('lowbit_b200.packed')!r})")
    cfg = ModelConfig(**json.loads(meta["config"]))
    return Model(cfg, extra, backend=meta["backend"], threads=threads, asym=bool(int(meta["asym"])),
                 quantize_lm_head=bool(int(meta["quantize_lm_head"])), params=params,
                 int4_scale=meta["int4_scale"], _packed=(weights, extra))


# ---------------------------------------------------------------- loading

def load(model_dir: Path | str, backend: str = "fp32", threads: int | None = None, **kw) -> Model:
    """A Hugging Face checkpoint directory (config.json + *.safetensors)."""
    d = Path(model_dir)
    cfg = ModelConfig.from_hf(json.loads((d / "config.json").read_text()), name=d.name)
    files = sorted(d.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no .safetensors in {d}")
    W: dict[str, np.ndarray] = {}
    for f in files:
        W.update(load_safetensors(f))
    return Model(cfg, W, backend=backend, threads=threads, **kw)
