"""ctypes access to the reference's own C kernels, compiled from the reference's
sources by `make -C oracle ref` into oracle/_ref/liblowbit_ref.so.

TEST / BASELINE INFRASTRUCTURE ONLY: used by tests and by bench.py's CPU
baseline ("kind": "reference") to time lowbit's CPU path on the host cores.
The entry points and the lb_params struct follow the reference's C ABI
(src/lowbit/csrc/lowbit.h:37-45,95-123).
"""
from __future__ import annotations

import ctypes as C
import os
import time
from pathlib import Path

import numpy as np

SO = Path(__file__).resolve().parent / "_ref" / "liblowbit_ref.so"


class LbParams(C.Structure):
    _fields_ = [(f, C.c_int) for f in ("isa", "mr", "nr", "nb", "kb", "order", "nthreads")]


# the reference's compiled micro-tiles (src/lowbit/kernels.py:35)
TILES = [(1, 1), (1, 2), (1, 4), (2, 1), (2, 2), (2, 4), (4, 1), (4, 2), (4, 4), (8, 1), (8, 2)]
ISA = {0: "scalar", 1: "avx2", 2: "avx512"}


def available() -> bool:
    return SO.exists()


def load() -> C.CDLL:
    L = C.CDLL(str(SO))
    vp, i = C.c_void_p, C.c_int
    pp = C.POINTER(LbParams)
    L.lb_gemm_w4a16.argtypes = [vp, i, i, vp, vp, vp, i, vp, pp]
    L.lb_gemm_mxfp4.argtypes = [vp, i, i, vp, vp, i, vp, pp]
    L.lb_gemm_w4a8.argtypes = [vp, i, i, vp, vp, vp, i, vp, pp]
    L.lb_gemm_w4a8_amx.argtypes = [vp, i, i, vp, vp, vp, i, vp, i]
    for f in ("lb_gemm_w4a16", "lb_gemm_mxfp4", "lb_gemm_w4a8", "lb_gemm_w4a8_amx", "lb_active_isa",
              "lb_has_openmp", "lb_max_threads", "lb_has_vnni", "lb_amx_available"):
        getattr(L, f).restype = C.c_int
    return L


def amx_available() -> bool:
    """The reference's own check (src/lowbit/kernels.py:89-94): AVX-512 active
    and AMX-INT8 usable by this process."""
    L = load()
    return L.lb_active_isa() >= 2 and bool(L.lb_amx_available())


class RefGemmAMX:
    """One reference lb_gemm_w4a8_amx call (src/lowbit/csrc/kern_amx.c:121-164) on
    host buffers, weights in the AMX repack layout (AMXInt4Weights: qw, scales,
    sz = s * z)."""

    def __init__(self, x: np.ndarray, wa, threads: int | None = None):
        self.L = load()
        self.x = np.ascontiguousarray(x, np.float32)
        self.w = wa
        self.m = self.x.shape[0]
        self.y = np.empty((self.m, wa.n), np.float32)
        self.threads = threads or os.cpu_count() or 1

    def __call__(self) -> int:
        w = self.w
        rc = self.L.lb_gemm_w4a8_amx(_p(self.x), self.m, w.kp, _p(w.qw), _p(w.scales), _p(w.sz), w.n,
                                     _p(self.y), self.threads)
        if rc < 0:
            raise ValueError(f"reference lb_gemm_w4a8_amx failed rc={rc}")
        return rc


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class RefGemm:
    """One reference GEMM call (fmt in w4a16 / w4a8 / mxfp4) on host buffers."""

    def __init__(self, fmt: str, x: np.ndarray, w, threads: int | None = None):
        self.L = load()
        self.fmt = fmt
        self.x = np.ascontiguousarray(x, np.float32)
        self.w = w
        self.m = self.x.shape[0]
        self.y = np.empty((self.m, w.n), np.float32)
        self.threads = threads or os.cpu_count() or 1
        self.params = LbParams(-1, 0, 0, 0, 0, 0, self.threads)

    def __call__(self, params: LbParams | None = None) -> int:
        p = C.byref(params or self.params)
        w = self.w
        if self.fmt == "mxfp4":
            rc = self.L.lb_gemm_mxfp4(_p(self.x), self.m, w.kp, _p(w.qw), _p(w.e8m0), w.n, _p(self.y), p)
        else:
            fn = self.L.lb_gemm_w4a16 if self.fmt == "w4a16" else self.L.lb_gemm_w4a8
            rc = fn(_p(self.x), self.m, w.kp, _p(w.qw), _p(w.scales), _p(w.zeros), w.n, _p(self.y), p)
        if rc < 0:
            raise ValueError(f"reference lb_gemm_{self.fmt} failed rc={rc}")
        return rc

    def info(self) -> dict:
        return {"isa": ISA.get(self.L.lb_active_isa(), "?"), "openmp": bool(self.L.lb_has_openmp()),
                "max_threads": self.L.lb_max_threads(), "vnni": bool(self.L.lb_has_vnni())}

    def tune(self, budget_s: float = 4.0) -> LbParams:
        """Short version of the reference's two-stage tile search (src/lowbit/tune.py:99-145):
        every micro-tile at a shape-derived N-tile, then N-tile / K-block for the best."""
        n = self.w.n
        nb0 = max(8, min(256, n // max(1, 4 * self.threads)))
        nb0 = 1 << (nb0.bit_length() - 1)
        t_end = time.perf_counter() + budget_s

        def t(p):
            self(p)
            best = float("inf")
            for _ in range(3):
                t0 = time.perf_counter()
                self(p)
                best = min(best, time.perf_counter() - t0)
            return best

        tried = {}
        for mr, nr in TILES:
            if mr > max(1, self.m) or time.perf_counter() > t_end:
                continue
            p = LbParams(-1, mr, nr, max(nb0, nr), 0, 0, self.threads)
            tried[(mr, nr, p.nb, 0)] = t(p)
        mr, nr, _, _ = min(tried, key=tried.get)
        for nb in (16, 32, 64, 128, 256):
            for kb in (0, 1024, 2048):
                if time.perf_counter() > t_end or nb < nr or (kb and kb >= self.w.kp):
                    continue
                p = LbParams(-1, mr, nr, nb, kb, 0, self.threads)
                tried[(mr, nr, nb, kb)] = t(p)
        mr, nr, nb, kb = min(tried, key=tried.get)
        self.params = LbParams(-1, mr, nr, nb, kb, 0, self.threads)
        return self.params
