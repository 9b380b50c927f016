"""Autotuner for the GPU kernels with a JSON cache (GPU counterpart of src/lowbit/tune.py).

Search space per (kernel, M, N, K, path): tokens per pass (mr), rows per team
per tile (nr), resident CTAs per SM (nb), split-K length (kb) and pipeline
stages (order). Candidates are timed with CUDA events on the current stream
(median of `reps` launches after a warm-up). The cache is keyed by GPU name,
SM count and driver version, so a cache from another GPU is ignored
(as src/lowbit/tune.py:43-50 ignores a cache from another CPU).
"""
from __future__ import annotations

import json
import os
from pathlib import Path

from . import kernels as K

DEFAULT_CACHE = Path(os.environ.get("LOWBIT_B200_TUNE_CACHE",
                                    Path.home() / ".cache" / "lowbit_b200" / "tune.json"))


def gpu_key() -> str:
    import torch
    d = torch.cuda.current_device()
    p = torch.cuda.get_device_properties(d)
    drv = torch.version.cuda or "?"
    return f"{p.name}|{p.multi_processor_count}sm|cuda{drv}"


def key(kind: str, m: int, n: int, k: int, path: str) -> str:
    return f"{kind}|{path}|{m}x{n}x{k}"


def load_cache(path: Path | str = DEFAULT_CACHE) -> dict:
    p = Path(path)
    if not p.exists():
        return {"gpu": gpu_key(), "entries": {}}
    data = json.loads(p.read_text())
    if data.get("gpu") != gpu_key():
        return {"gpu": gpu_key(), "entries": {}}
    return data


def save_cache(data: dict, path: Path | str = DEFAULT_CACHE) -> None:
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    tmp = p.with_suffix(".tmp")
    tmp.write_text(json.dumps(data, indent=1, sort_keys=True))
    os.replace(tmp, p)


def lookup(kind: str, m: int, n: int, k: int, isa=None,
           path: Path | str = DEFAULT_CACHE) -> K.Params | None:
    try:
        e = load_cache(path)["entries"].get(key(kind, m, n, k, K.effective_isa(kind, isa, m, n, k)))
    except (OSError, ValueError):
        return None
    return K.Params(**e["params"]) if e else None
