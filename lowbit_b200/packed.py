"""Packed-weight files: quantized weights stored as they are consumed, so a
model loads without re-quantizing.

The container is safetensors (an 8-byte little-endian header length, a JSON
header {name: {dtype, shape, data_offsets}} plus an optional
"__metadata__" map of strings, then the raw bytes; offsets are relative to
the end of the header). The reference's own loader (src/lowbit/model.py:81-103)
reads fp32/bf16 checkpoints of this container and quantizes at load time; its
packed arrays (src/lowbit/formats.py:57-87, 148-172) are stored here unchanged:

    <name>.qw      U8  [N, Kp/2]   both formats
    <name>.scales  F32 [N, Kp/128] int4 g128
    <name>.zeros   U8  [N, Kp/128] int4 g128, asymmetric only
    <name>.e8m0    U8  [N, Kp/32]  MXFP4
    metadata "<name>.format" = "int4_g128" | "mxfp4_b32", "<name>.k" = logical K

Other tensors (biases, norms, embeddings) are stored as plain arrays. Reading
maps the file (numpy memmap) and copies each tensor once, to the host or
straight to a CUDA device.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from .formats import Int4Weights, MXFP4Weights

_DT = {"U8": np.uint8, "I8": np.int8, "I32": np.int32, "I64": np.int64, "F32": np.float32, "F16": np.float16,
       "F64": np.float64}
_NAME = {np.dtype(v): k for k, v in _DT.items()}
FORMAT_INT4 = "int4_g128"
FORMAT_MXFP4 = "mxfp4_b32"
_ALIGN = 64   # tensor data offsets are multiples of this (aligned device copies, memmap views)


def _host(a) -> np.ndarray:
    if isinstance(a, np.ndarray):
        return a
    import torch
    if isinstance(a, torch.Tensor):
        return a.detach().cpu().numpy()
    return np.asarray(a)


def write_tensors(path: Path | str, tensors: dict, metadata: dict | None = None) -> None:
    """Write named arrays (numpy or torch, any device) and string metadata."""
    arrays = {k: np.ascontiguousarray(_host(v)) for k, v in tensors.items()}
    header: dict = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    off = 0
    for k, a in arrays.items():
        if a.dtype not in _NAME:
            raise ValueError(f"{k}: unsupported dtype {a.dtype}")
        off = -(-off // _ALIGN) * _ALIGN
        header[k] = {"dtype": _NAME[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes
    hdr = json.dumps(header, separators=(",", ":")).encode()
    hdr += b" " * ((-(8 + len(hdr))) % _ALIGN)   # data starts aligned
    with open(path, "wb") as f:
        f.write(len(hdr).to_bytes(8, "little"))
        f.write(hdr)
        pos = 0
        for k, a in arrays.items():
            lo = header[k]["data_offsets"][0]
            f.write(b"\0" * (lo - pos))
            f.write(a.tobytes())
            pos = lo + a.nbytes


def read_tensors(path: Path | str) -> tuple[dict[str, np.ndarray], dict[str, str]]:
    """Named arrays (read-only views of a memory map, dtypes kept) and metadata."""
    path = Path(path)
    with open(path, "rb") as f:
        hlen = int.from_bytes(f.read(8), "little")
        header = json.loads(f.read(hlen))
    meta = header.pop("__metadata__", {}) or {}
    size = path.stat().st_size - 8 - hlen
    data = np.memmap(path, dtype=np.uint8, mode="r", offset=8 + hlen) if size > 0 else np.zeros(0, np.uint8)
    out = {}
    for name, info in header.items():
        if info["dtype"] not in _DT:
            raise ValueError(f"{name}: unsupported dtype {info['dtype']}")
        lo, hi = info["data_offsets"]
        if not 0 <= lo <= hi <= size:
            raise ValueError(f"{name}: data offsets {lo}..{hi} outside the file's {size} data bytes")
        dt = np.dtype(_DT[info["dtype"]])
        shape = tuple(int(s) for s in info["shape"])
        if (hi - lo) != int(np.prod(shape, dtype=np.int64)) * dt.itemsize:
            raise ValueError(f"{name}: {hi - lo} bytes do not hold {shape} x {dt}")
        out[name] = np.frombuffer(data, dtype=dt, count=(hi - lo) // dt.itemsize, offset=lo).reshape(shape)
    return out, meta


# ---------------------------------------------------------------- weight containers

def weights_tensors(name: str, w) -> tuple[dict, dict]:
    """(tensors, metadata) of one Int4Weights / MXFP4Weights under `name`."""
    if isinstance(w, Int4Weights):
        t = {f"{name}.qw": w.qw, f"{name}.scales": w.scales}
        if w.zeros is not None:
            t[f"{name}.zeros"] = w.zeros
        return t, {f"{name}.format": FORMAT_INT4, f"{name}.k": w.k}
    if isinstance(w, MXFP4Weights):
        return ({f"{name}.qw": w.qw, f"{name}.e8m0": w.e8m0},
                {f"{name}.format": FORMAT_MXFP4, f"{name}.k": w.k})
    raise TypeError(f"{name}: not a packed weight container ({type(w).__name__})")


def _check_int4(name, qw, scales, zeros, k):
    n, half = qw.shape
    kp = 2 * half
    if kp % 128 or scales.shape != (n, kp // 128) or (zeros is not None and zeros.shape != (n, kp // 128)):
        raise ValueError(f"{name}: inconsistent int4 g128 shapes qw {qw.shape} scales {scales.shape}"
                         + ("" if zeros is None else f" zeros {zeros.shape}"))
    if not 0 < k <= kp:
        raise ValueError(f"{name}: k={k} outside (0, Kp={kp}]")


def weights_from_tensors(name: str, tensors: dict, meta: dict, device=None):
    """The container stored under `name` (arrays on `device` when given)."""
    fmt = meta.get(f"{name}.format")
    k = int(meta[f"{name}.k"])
    if device is not None:
        from ._torch import to_cuda

        def put(a):
            return None if a is None else to_cuda(np.ascontiguousarray(a), device)
    else:
        def put(a):
            return None if a is None else np.array(a)
    if fmt == FORMAT_INT4:
        qw, sc, z = tensors[f"{name}.qw"], tensors[f"{name}.scales"], tensors.get(f"{name}.zeros")
        if qw.dtype != np.uint8 or sc.dtype != np.float32 or (z is not None and z.dtype != np.uint8):
            raise ValueError(f"{name}: int4 g128 wants U8 qw, F32 scales, U8 zeros")
        _check_int4(name, qw, sc, z, k)
        return Int4Weights(put(qw), put(sc), put(z), k)
    if fmt == FORMAT_MXFP4:
        qw, e = tensors[f"{name}.qw"], tensors[f"{name}.e8m0"]
        if qw.dtype != np.uint8 or e.dtype != np.uint8:
            raise ValueError(f"{name}: MXFP4 wants U8 qw and e8m0")
        kp = 2 * qw.shape[1]
        if kp % 32 or e.shape != (qw.shape[0], kp // 32) or not 0 < k <= kp:
            raise ValueError(f"{name}: inconsistent MXFP4 shapes qw {qw.shape} e8m0 {e.shape} k={k}")
        return MXFP4Weights(put(qw), put(e), k)
    raise ValueError(f"{name}: unknown packed format {fmt!r}")


def save_weights(path: Path | str, weights: dict, extra: dict | None = None, metadata: dict | None = None) -> None:
    """Save {name: Int4Weights | MXFP4Weights} (+ plain arrays in `extra`)."""
    tensors, meta = {}, dict(metadata or {})
    for name, w in weights.items():
        t, m = weights_tensors(name, w)
        tensors.update(t)
        meta.update(m)
    for k, v in (extra or {}).items():
        if k in tensors:
            raise ValueError(f"{k}: name used twice")
        tensors[k] = v
    write_tensors(path, tensors, meta)


def load_weights(path: Path | str, device=None) -> tuple[dict, dict, dict]:
    """(packed containers by name, the other arrays by name, metadata)."""
    tensors, meta = read_tensors(path)
    names = sorted(k[: -len(".format")] for k in meta if k.endswith(".format"))
    weights = {n: weights_from_tensors(n, tensors, meta, device) for n in names}
    used = {f"{n}.{f}" for n in names for f in ("qw", "scales", "zeros", "e8m0")}
    extra = {k: v for k, v in tensors.items() if k not in used}
    return weights, extra, meta
