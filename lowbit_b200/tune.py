"""Autotuner for the GPU kernels with a JSON cache (GPU counterpart of
src/lowbit/tune.py: the same entry points tune / lookup / load_cache /
save_cache, the same two-stage search and cache-entry fields).

Stage 1 picks the kernel path and the shape of the work: the automatic
choice, then every alternative the planner accepts for the problem (for one
or two tokens the register-streamed decode kernel at 2-8 CTAs per SM and the
warp-level tensor-core kernel at several tilings (W4A16); for W4A8 with up
to 64 tokens the int8 mma.sync kernel at 4 and 8 warps; for 3-63 tokens the
tcgen05 exact kernel; from 64 tokens the exact kernel beside the bf16
prefill kernel; below 64 tokens the staged SIMT kernel at every compiled
tokens-per-pass x rows-per-team). Stage 2 refines the three fastest: pipeline
stages (`order`), CTAs per SM (`nb`) and split-K length (`kb`) for the
staged kernel, CTAs per SM for the decode kernel, warps / K per stage / ring
depth for the tensor-core decode kernel, warps and CTAs per SM for the int8
mma kernel.

Every candidate is timed as the library is used: a CUDA graph of `steps`
calls over a pool of weight copies larger than twice the L2 cache (each call
streams its weights from HBM), replayed `reps` times, CUDA events, median
per call. Candidates the planner rejects are skipped. The winner (its path
included: `Params.isa`) goes into the cache, written atomically, keyed by
GPU name, SM count and CUDA version (a cache from another GPU is ignored, as
src/lowbit/tune.py:43-50 ignores one from another CPU); `params="auto"`
reads it back through `lookup`.
"""
from __future__ import annotations

import json
import os
import statistics
from pathlib import Path

import numpy as np

from . import kernels as K

DEFAULT_CACHE = Path(os.environ.get("LOWBIT_B200_TUNE_CACHE",
                                    Path.home() / ".cache" / "lowbit_b200" / "tune.json"))
L2_BYTES = 126 << 20


def gpu_key() -> str:
    import torch
    d = torch.cuda.current_device()
    p = torch.cuda.get_device_properties(d)
    drv = torch.version.cuda or "?"
    return f"{p.name}|{p.multi_processor_count}sm|cuda{drv}"


def key(kind: str, m: int, n: int, k: int, isa=None) -> str:
    return f"{kind}|{isa or 'auto'}|{m}x{n}x{k}"


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
    tmp = p.with_suffix(f".tmp{os.getpid()}")
    tmp.write_text(json.dumps(data, indent=1, sort_keys=True))
    os.replace(tmp, p)


def lookup(kind: str, m: int, n: int, k: int, isa=None, threads: int | None = None,
           path: Path | str = DEFAULT_CACHE) -> K.Params | None:
    """The tuned Params for this problem (its `isa` is the tuned path), or None."""
    try:
        e = load_cache(path)["entries"].get(key(kind, m, n, k, isa))
    except (OSError, ValueError):
        return None
    return K.Params(**e["params"]) if e else None


# ---------------------------------------------------------------- candidates

def _stage1(kind: str, m: int) -> list[K.Params]:
    P = K.Params
    c = [P()]
    if m <= 2:
        c += [P(nb=b) for b in (2, 4, 8)]                      # decode kernel, CTAs per SM
        if kind == "w4a16":                                      # warp-level tensor-core kernel
            c += [P(isa="mma", nr=nw, kb=kb, order=ns) for nw, kb, ns in
                  ((8, 4096, 2), (8, 2048, 4), (16, 4096, 3), (4, 2048, 4), (16, 2048, 4))]
    if kind == "w4a8" and m <= 64:                               # int8 mma.sync kernel
        c += [P(isa="mma", nr=8), P(isa="mma", nr=4)]
    if m > 2:
        c.append(P(isa="tcgen05", mr=16))                        # tcgen05 exact kernel
    if m < 64:
        for mt in (1, 2, 4, 8):                                  # staged SIMT kernel
            if mt > 2 * max(1, m):
                continue
            for nr in (1, 4):
                c.append(P(mr=mt, nr=nr))
    return c


def _stage2(kind: str, m: int, kp: int, base: K.Params) -> list[K.Params]:
    P = K.Params
    out = []
    if base.isa == "mma" and kind == "w4a8":
        out += [P(isa="mma", nr=nw, nb=nb) for nw in (4, 8) for nb in (1, 2, 3, 4)]
    elif base.isa == "mma":
        for nw, kb in ((8, 4096), (8, 2048), (16, 4096), (16, 2048), (4, 2048)):
            for ns in (2, 3, 4):
                for nb in (1, 2):
                    out.append(P(isa="mma", nr=nw, kb=kb, order=ns, nb=nb))
    elif base.isa is None and base.mr == 0 and base.nr == 0 and m <= 2:
        out += [P(nb=b) for b in (1, 2, 3, 4, 6, 8)]
    elif base.mr > 0 and base.isa is None:
        kbs = [0] + [b for b in (1024, 2048, 4096) if b < kp]
        for order in (2, 4, 8):
            for nb in (1, 2, 3):
                for kb in kbs:
                    out.append(P(mr=base.mr, nr=base.nr, nb=nb, kb=kb, order=order))
    return out


# ---------------------------------------------------------------- timing

def _problem(kind: str, m: int, n: int, k: int, seed: int = 0):
    """The reference's tuning problem (src/lowbit/tune.py:81-86): W ~ 0.02 N(0, 1),
    X ~ N(0, 1), symmetric int4 (or MXFP4); quantized on the GPU."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    x = rng.standard_normal((m, k)).astype(np.float32)
    wq = K.quantize_mxfp4_cuda(w) if kind == "mxfp4" else K.quantize_int4_cuda(w)
    return x, wq


class _Timer:
    """Times candidates as CUDA graphs of `steps` calls over rotating weight copies."""

    def __init__(self, kind: str, x, wq, steps: int, reps: int):
        import torch
        from dataclasses import replace
        self.torch = torch
        self.gemm = K.GEMMS[kind]
        self.kind, self.steps, self.reps = kind, steps, reps
        fields = ("qw", "scales", "zeros", "e8m0")
        wbytes = sum(getattr(wq, f).numel() * getattr(wq, f).element_size() for f in fields
                     if getattr(wq, f, None) is not None)
        copies = int(max(1, min(16, np.ceil(2 * L2_BYTES / max(1, wbytes)))))
        self.pool = [wq] + [replace(wq, **{f: getattr(wq, f).clone() for f in fields
                                           if getattr(wq, f, None) is not None}) for _ in range(copies - 1)]
        xd = x if isinstance(x, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(x, np.float32))
        self.prep = K._Prepared(xd.cuda(), wq.kp, wq.n)   # device X: calls return device Y (capturable)
        self.x = self.prep.x

    def __call__(self, p: K.Params) -> float:
        torch = self.torch
        fn = self.gemm
        # eager first call: the planner's verdict (ValueError when it rejects p)
        fn(self.x, self.pool[0], p, _prep=self.prep)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                for i in range(self.steps):
                    fn(self.x, self.pool[i % len(self.pool)], p, _prep=self.prep)
        torch.cuda.current_stream().wait_stream(s)
        g.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(self.reps):
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e-3 / self.steps)
        del g
        return statistics.median(ts)


def tune(kind: str, m: int, n: int, k: int, isa=None, threads: int | None = None, reps: int = 5,
         problem=None, top: int = 3, path: Path | str | None = DEFAULT_CACHE, verbose: bool = False,
         steps: int = 20) -> dict:
    """Search kernel path and tile parameters for GEMM `kind` with m tokens on an
    n x k weight; returns the cache entry and stores it if path is set.

    `isa` restricts the search to one path ("simt", "tcgen05", "mma"); the
    default searches them all and records the winner's path in its Params.
    `threads` is accepted for interface parity (the CPU thread count)."""
    x, wq = problem if problem is not None else _problem(kind, m, n, k)
    timer = _Timer(kind, x, wq, steps, reps)
    tried: dict[K.Params, float] = {}

    def run(p: K.Params) -> float | None:
        if isa is not None and p.isa is None:
            p = K.Params(p.mr, p.nr, p.nb, p.kb, p.order, isa=isa)
        if p not in tried:
            try:
                tried[p] = timer(p)
            except ValueError:      # the planner rejects this tiling for this problem
                tried[p] = None
            if verbose and tried[p] is not None:
                print(f"  {p}  {tried[p] * 1e6:.2f} us")
        return tried[p]

    for p in _stage1(kind, m):
        if isa is None or p.isa in (None, isa):
            run(p)
    ok = {p: t for p, t in tried.items() if t is not None}
    for base in sorted(ok, key=ok.get)[:top]:
        for p in _stage2(kind, m, wq.kp, base):
            run(p)
    ok = {p: t for p, t in tried.items() if t is not None}
    if not ok:
        raise ValueError(f"no kernel configuration runs {kind} M={m} N={n} K={k}"
                         + (f" on path {isa!r}" if isa else ""))
    best = min(ok, key=ok.get)
    default_t = run(K.Params())
    entry = {
        "params": best.as_dict(),
        "time_s": ok[best],
        "default_time_s": default_t,
        "n_configs": len(ok),
        "gflops": 2.0 * m * n * k / ok[best] / 1e9,
    }
    if path is not None:
        data = load_cache(path)
        data["entries"][key(kind, m, n, k, isa)] = entry
        save_cache(data, path)
    return entry
