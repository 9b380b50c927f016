"""ctypes binding of liblowbit_b200.so: lowbit's kernel API on B200 GPUs.

Mirrors src/lowbit/kernels.py (same function names, argument meaning and
error behaviour) with the computation on the GPU:

* ``x`` may be a numpy array (uploaded per call; the result comes back as a
  numpy array, synchronously) or a torch CUDA tensor (no copies; the result is
  a torch CUDA tensor produced on the current stream, no synchronisation);
* weights may hold numpy arrays (uploaded once and cached on the object) or
  torch CUDA tensors;
* ``params`` is a :class:`Params` (fields reinterpreted for the GPU, see
  include/lowbit_b200.h), ``None`` or ``"auto"`` (tuned cache, lowbit_b200.tune);
* ``isa`` selects the kernel path: None/"auto" (one or two tokens: the SIMT
  decode kernels; more: the tcgen05 tensor-core kernel, for W4A8 from 32
  tokens), "simt", "tcgen05", "mma" (the warp-level tensor-core decode
  kernel, W4A16 with one or two tokens); the reference's CPU ISA names
  ("scalar", "avx2", "avx512") are accepted and mean "auto". Explicit tiling
  fields in ``params`` (mr, nr, nb, kb, order) keep "auto" on the SIMT kernels;
* ``threads`` is accepted and ignored (CPU thread count).

A negative return code raises ValueError for shape/parameter errors (as the
reference, src/lowbit/kernels.py:132-135) and RuntimeError for CUDA errors.
There is no CPU fallback: without a CUDA device every call raises.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import asdict, dataclass
from functools import lru_cache

import numpy as np

from ._build import build
from .formats import GROUP, MXBLOCK, Int4Weights, Int8Acts, MXFP4Weights, pad_to

PATHS = {-1: "auto", 0: "simt", 1: "tcgen05", 3: "mma"}
PATH_IDS = {"auto": -1, "simt": 0, "tcgen05": 1, "mma": 3}
REFERENCE_ISAS = ("scalar", "avx2", "avx512")
KIND_IDS = {"w4a16": 0, "mxfp4": 1, "w4a8": 2}
ERR_NAMES = {-1: "bad shape or pointer", -2: "tile parameters not supported", -3: "allocation failed",
             -5: "CUDA error", -6: "device is not sm_100", -7: "device-side wait timed out"}


class _Params(C.Structure):
    _fields_ = [(f, C.c_int) for f in ("isa", "mr", "nr", "nb", "kb", "order", "nthreads")]


@dataclass(frozen=True)
class Params:
    """Kernel tiling parameters (0 = library default), reinterpreted for the GPU:

    mr    tokens per pass of the SIMT kernels (1, 2, 4, 8)
    nr    rows per team per pipeline tile (1 or 4); warps per CTA on the mma path
    nb    resident CTAs per SM
    kb    split-K length in elements (multiple of 128), 0 = whole K; K elements
          per ring stage on the mma path
    order TMA pipeline stages
    isa   kernel path these parameters were tuned for ("simt", "tcgen05",
          "mma"), used when the call gives no `isa`; None = automatic. The
          reference's Params has no such field (its tuner searches one ISA);
          the GPU tuner records the path it chose here.
    """
    mr: int = 0
    nr: int = 0
    nb: int = 0
    kb: int = 0
    order: int = 0
    isa: str | None = None

    def as_dict(self) -> dict:
        d = asdict(self)
        if d["isa"] is None:
            del d["isa"]
        return d


_vp = C.c_void_p
_int = C.c_int
_pp = C.POINTER(_Params)


@lru_cache(maxsize=1)
def lib() -> C.CDLL:
    """Load (building first if needed) the CUDA library."""
    import torch  # noqa: F401  (initialises the CUDA runtime torch uses)
    so = C.CDLL(str(build()))
    sig = {
        "lbc_version": ([], _int),
        "lbc_device_ok": ([], _int),
        "lbc_sm_count": ([], _int),
        "lbc_last_error": ([], C.c_char_p),
        "lbc_device_status": ([_int], _int),
        "lbc_set_wait_cycles": ([C.c_longlong], _int),
        "lbc_wait_cycles": ([], C.c_longlong),
        "lbc_describe_plan": ([_int, _int, _int, _int, _pp, C.c_char_p, _int], _int),
        "lbc_tc_selftest": ([_int, _vp, _vp], _int),
        "lbc_gemm_w4a16": ([_vp, _int, _int, _vp, _vp, _vp, _int, _vp, _pp, _vp], _int),
        "lbc_gemm_mxfp4": ([_vp, _int, _int, _vp, _vp, _int, _vp, _pp, _vp], _int),
        "lbc_gemm_w4a8_workspace_size": ([_int, _int], C.c_size_t),
        "lbc_gemm_w4a8": ([_vp, _int, _int, _vp, _vp, _vp, _int, _vp, _pp, _vp, _vp], _int),
        "lbc_gemm_w4a16_host": ([_vp, _int, _int, _vp, _vp, _vp, _int, _vp, _pp, _vp], _int),
        "lbc_gemm_mxfp4_host": ([_vp, _int, _int, _vp, _vp, _int, _vp, _pp, _vp], _int),
        "lbc_gemm_w4a8_host": ([_vp, _int, _int, _vp, _vp, _vp, _int, _vp, _pp, _vp], _int),
        "lbc_gemm_w4a8_q": ([_vp, _vp, _vp, _int, _int, _vp, _vp, _vp, _int, _vp, _pp, _vp], _int),
        "lbc_quant_act_int8": ([_vp, _int, _int, _vp, _vp, _vp, _vp], _int),
        "lbc_w4a8_group_acc": ([_vp, _vp, _int, _int, _vp, _vp, _int, _vp, _int, _vp], _int),
        "lbc_device_alloc": ([C.c_size_t, C.POINTER(_vp)], _int),
        "lbc_device_free": ([_vp], _int),
        "lbc_ipc_get_handle": ([_vp, _vp], _int),
        "lbc_ipc_open_handle": ([_vp, C.POINTER(_vp)], _int),
        "lbc_ipc_close_handle": ([_vp], _int),
        "lbc_gemm_w4a16_allgather": ([_vp, _int, _int, _vp, _vp, _vp, _int, _int, _int, _vp, _vp, _vp, _vp,
                                      _int, _int, _pp, _vp], _int),
        "lbc_gemm_allgather": ([_int, _vp, _int, _int, _vp, _vp, _vp, _vp, _int, _int, _int, _vp, _vp, _vp, _vp,
                                _int, _int, _pp, _vp], _int),
        "lbc_rmsnorm": ([_vp, _vp, _vp, _vp, _vp, _int, _int, C.c_float, _vp], _int),
        "lbc_qkv_rope": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _int, _int, _int, _int, _int, _int, _vp], _int),
        "lbc_attention": ([_vp, _vp, _vp, _vp, _vp, _int, _int, _int, _int, _int, _int, _vp], _int),
        "lbc_silu_mul": ([_vp, _vp, _int, _int, _vp], _int),
        "lbc_gemm_w4a16_rmsnorm": ([_vp, _vp, _vp, _vp, C.c_float, _int, _int, _vp, _vp, _vp, _int, _vp, _pp, _vp],
                                   _int),
        "lbc_gemm_w4a16_glu": ([_vp, _int, _int, _vp, _vp, _vp, _int, _vp, _pp, _vp], _int),
        "lbc_rope_attention": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _int, _int, _int, _int, _int, _vp], _int),
        "lbc_advance_pos": ([_vp, _int, _vp], _int),
        "lbc_quantize_int4": ([_vp, _int, _int, _int, _vp, _vp, _vp, _vp], _int),
        "lbc_quantize_mxfp4": ([_vp, _int, _int, _vp, _vp, _vp], _int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(so, name)
        fn.argtypes = args
        fn.restype = res
    return so


def _torch():
    import torch
    return torch


def gpu_info() -> dict:
    torch = _torch()
    from ._torch import require_cuda
    require_cuda()
    d = torch.cuda.current_device()
    props = torch.cuda.get_device_properties(d)
    L = lib()
    return {"device": props.name, "index": d, "cc": f"{props.major}.{props.minor}",
            "sm_count": L.lbc_sm_count(), "sm100": bool(L.lbc_device_ok()),
            "lib_version": L.lbc_version(), "mem_gb": round(props.total_memory / 2**30, 1)}


def cpu_info() -> dict:
    """lowbit.cpu_info() compatibility: the keys callers read, describing the GPU backend."""
    g = gpu_info()
    return {"cpu_isa": "sm_100a", "active_isa": "sm_100a", "vnni": False, "openmp": False,
            "max_threads": 1, "amx": True, "gpu": g}


def _path_id(isa) -> int:
    if isa is None or isa == "auto" or isa in REFERENCE_ISAS:
        return -1
    if isinstance(isa, int):
        return isa if isa in PATHS else -1
    if isa not in PATH_IDS:
        raise ValueError(f"isa must be one of {sorted(PATH_IDS)} or a lowbit ISA name, not {isa!r}")
    return PATH_IDS[isa]


def effective_isa(kind: str, isa=None, m: int = 1, n: int | None = None, k: int | None = None) -> str:
    """Kernel path a GEMM of `kind` with `m` tokens (and an n x k weight, when
    given) runs on with default params; the library's rule (capi.cu want_tc)."""
    pid = _path_id(isa)
    if pid == -1:
        if (kind != "w4a8" and n is not None and k is not None and (4 if kind == "mxfp4" else 8) <= m <= 16
                and n * pad_to(k, MXBLOCK if kind == "mxfp4" else GROUP) <= 5e6):
            pid = 0     # the few-token SIMT kernel (capi.cu want_tok)
        elif kind == "w4a8":
            kp = pad_to(k, GROUP) if k is not None else 0
            big = n is not None and k is not None and n * kp >= 32e6
            pid = 1 if m >= 32 or (big and (m > 16 or (m >= 12 and kp > 8192))) else 0
        elif m < 3:
            pid = 0
        elif n is not None and k is not None and m < 32 and n * pad_to(k, GROUP) < (10e6 if m <= 4 else 6e6):
            pid = 0
        else:
            pid = 1
    return PATHS[pid]


_AUTO_MEMO: dict = {}


def auto_params(kind: str, m: int, n: int, k: int, isa=None, threads=None) -> Params:
    """Tuned parameters from the tune cache (lowbit_b200.tune), else defaults."""
    key = (kind, m, n, k, isa)
    if key not in _AUTO_MEMO:
        from .tune import lookup
        _AUTO_MEMO[key] = lookup(kind, m, n, k, isa) or Params()
    return _AUTO_MEMO[key]


_P_AUTO = _Params(-1, 0, 0, 0, 0, 0, 0)


def _params(p, isa, kind=None, shape=None) -> _Params:
    if p is None and isa is None:
        return _P_AUTO
    if isinstance(p, str):
        if p != "auto":
            raise ValueError(f"params must be a Params, None or 'auto', not {p!r}")
        p = auto_params(kind, *shape, isa=isa)
    p = p or Params()
    return _Params(_path_id(isa if isa is not None else p.isa), p.mr, p.nr, p.nb, p.kb, p.order, 0)


def _pref(params, isa, kind: str, m: int, n: int, k: int):
    """byref(_Params) for a GEMM of m tokens on an n x k weight."""
    return C.byref(_P_AUTO if params is None and isa is None else _params(params, isa, kind, (m, n, k)))


def _check(rc: int, what: str) -> int:
    if rc < 0:
        detail = lib().lbc_last_error().decode(errors="replace")
        msg = f"{what} failed (rc={rc}, {ERR_NAMES.get(rc, 'error')}): {detail}"
        if rc in (-1, -2):
            raise ValueError(msg)
        raise RuntimeError(msg)
    return rc


# ---------------------------------------------------------------- operands

def _dev_weights(w):
    """The weight container with its arrays on the current CUDA device (cached)."""
    torch = _torch()
    if isinstance(w.qw, torch.Tensor) and w.qw.is_cuda:
        return w
    cache = getattr(w, "_lbc_dev", None)
    dev = torch.cuda.current_device()
    if cache is None or cache[0] != dev:
        cache = (dev, w.cuda())
        object.__setattr__(w, "_lbc_dev", cache)
    return cache[1]


class _Prepared:
    """Padded device X plus an output buffer, reusable across calls (timing reps)."""

    def __init__(self, x, kp: int, n: int):
        torch = _torch()
        from ._torch import to_cuda
        self.host = not isinstance(x, torch.Tensor)
        if (not self.host and x.is_cuda and x.dtype == torch.float32 and x.dim() == 2
                and x.shape[1] == kp and x.is_contiguous()):
            xt = x          # already in the kernel's layout: no copies
        elif self.host:
            x = np.asarray(x, np.float32)
            if x.ndim == 1:
                x = x[None]
            xt = to_cuda(x)
        else:
            xt = x if x.dim() == 2 else x.reshape(1, -1)
            if not xt.is_cuda:
                xt = to_cuda(xt)
            xt = xt.to(torch.float32)
        if xt.shape[1] != kp:
            if xt.shape[1] > kp:
                raise ValueError(f"x has {xt.shape[1]} columns, more than Kp={kp}")
            xt = torch.nn.functional.pad(xt, (0, kp - xt.shape[1]))
        self.x = xt.contiguous()
        self.m = int(self.x.shape[0])
        self.y = torch.empty((self.m, n), dtype=torch.float32, device=self.x.device)

    def result(self):
        return self.y.cpu().numpy() if self.host else self.y


def _host_x(x, kp: int) -> np.ndarray:
    """Host X as a C-contiguous float32 (M, kp) array, zero-padded to kp columns."""
    a = np.asarray(x, np.float32)
    if a.ndim == 1:
        a = a[None]
    if a.shape[1] != kp:
        if a.shape[1] > kp:
            raise ValueError(f"x has {a.shape[1]} columns, more than Kp={kp}")
        a = np.pad(a, ((0, 0), (0, kp - a.shape[1])))
    return np.ascontiguousarray(a)


def _is_host(x) -> bool:
    return not isinstance(x, _torch().Tensor)


def _hptr(a: np.ndarray) -> int:
    """Address of a C-contiguous host array's data."""
    try:
        return C.addressof(C.c_char.from_buffer(a))
    except (TypeError, ValueError):   # read-only or zero-size buffers
        return a.ctypes.data


def _call(fn_name, *args):
    return getattr(lib(), fn_name)(*args)


def _raw_stream(device_index: int) -> int:
    """The current stream of a CUDA device as a raw handle (torch's own accessor)."""
    return _torch()._C._cuda_getCurrentRawStream(device_index)


def _stream():
    torch = _torch()
    return torch._C._cuda_getCurrentRawStream(torch.cuda.current_device())


def _zp(d):
    return None if d.zeros is None else d.zeros.data_ptr()


# ---------------------------------------------------------------- GEMMs

def gemm_w4a16(x, w: Int4Weights, params: Params | None = None, isa=None,
               threads: int | None = None, _prep: _Prepared | None = None):
    """Y = X @ dequant(W).T for int4 g128 weights (fp32 activations)."""
    d = _dev_weights(w)
    n, kp = w.n, w.kp
    if _prep is None and _is_host(x):
        xh = _host_x(x, kp)
        m = xh.shape[0]
        y = np.empty((m, n), np.float32)
        _check(lib().lbc_gemm_w4a16_host(_hptr(xh), m, kp, d.qw.data_ptr(), d.scales.data_ptr(), _zp(d), n,
                                          _hptr(y), _pref(params, isa, "w4a16", m, n, w.k), _stream()),
               "lbc_gemm_w4a16")
        return y
    pr = _prep or _Prepared(x, kp, n)
    _check(lib().lbc_gemm_w4a16(pr.x.data_ptr(), pr.m, kp, d.qw.data_ptr(), d.scales.data_ptr(), _zp(d), n,
                                pr.y.data_ptr(), _pref(params, isa, "w4a16", pr.m, n, w.k),
                                _raw_stream(pr.x.device.index)), "lbc_gemm_w4a16")
    return pr.result()


def gemm_mxfp4(x, w: MXFP4Weights, params: Params | None = None, isa=None,
               threads: int | None = None, _prep: _Prepared | None = None):
    """Y = X @ dequant(W).T for OCP MXFP4 weights."""
    d = _dev_weights(w)
    n, kp = w.n, w.kp
    if _prep is None and _is_host(x):
        xh = _host_x(x, kp)
        m = xh.shape[0]
        y = np.empty((m, n), np.float32)
        _check(lib().lbc_gemm_mxfp4_host(_hptr(xh), m, kp, d.qw.data_ptr(), d.e8m0.data_ptr(), n, _hptr(y),
                                          _pref(params, isa, "mxfp4", m, n, w.k), _stream()), "lbc_gemm_mxfp4")
        return y
    pr = _prep or _Prepared(x, kp, n)
    _check(lib().lbc_gemm_mxfp4(pr.x.data_ptr(), pr.m, kp, d.qw.data_ptr(), d.e8m0.data_ptr(), n,
                                pr.y.data_ptr(), _pref(params, isa, "mxfp4", pr.m, n, w.k),
                                _raw_stream(pr.x.device.index)), "lbc_gemm_mxfp4")
    return pr.result()


_WS: dict = {}


def _workspace(nbytes: int):
    """Cached device scratch per (device, size class); stream-ordered reuse."""
    torch = _torch()
    dev = torch.cuda.current_device()
    cur = _WS.get(dev)
    if cur is None or cur.numel() < nbytes:
        cur = torch.empty(max(nbytes, 1 << 16), dtype=torch.uint8, device=dev)
        _WS[dev] = cur
    return cur


def gemm_w4a8(x, w: Int4Weights, params: Params | None = None, isa=None,
              threads: int | None = None, _prep: _Prepared | None = None):
    """fp32 X in; X is quantized per token to int8 inside the call (counted in timings)."""
    d = _dev_weights(w)
    n, kp = w.n, w.kp
    if _prep is None and _is_host(x):
        xh = _host_x(x, kp)
        m = xh.shape[0]
        y = np.empty((m, n), np.float32)
        _check(lib().lbc_gemm_w4a8_host(_hptr(xh), m, kp, d.qw.data_ptr(), d.scales.data_ptr(), _zp(d), n,
                                         _hptr(y), _pref(params, isa, "w4a8", m, n, w.k), _stream()),
               "lbc_gemm_w4a8")
        return y
    pr = _prep or _Prepared(x, kp, n)
    ws = _workspace(int(lib().lbc_gemm_w4a8_workspace_size(pr.m, kp)))
    _check(lib().lbc_gemm_w4a8(pr.x.data_ptr(), pr.m, kp, d.qw.data_ptr(), d.scales.data_ptr(), _zp(d), n,
                               pr.y.data_ptr(), _pref(params, isa, "w4a8", pr.m, n, w.k), ws.data_ptr(),
                               _raw_stream(pr.x.device.index)), "lbc_gemm_w4a8")
    return pr.result()


def amx_available() -> bool:
    """lowbit.kernels.amx_available(): the AMX entry points are served by the
    GPU's W4A8 kernels here, so they are always available."""
    return True


def _amx_int4(w) -> Int4Weights:
    """Canonical device weights of AMX-packed ones (unpacked once, cached on the object)."""
    c = getattr(w, "_lbc_int4", None)
    if c is None:
        from .formats import AMXInt4Weights
        if not hasattr(w, "to_int4"):   # a lowbit.AMXInt4Weights: same fields and bytes
            w = AMXInt4Weights(w.qw, w.scales, w.sz, w.zeros, w.n, w.k, w.kp)
        c = w.to_int4().cuda()
        try:
            object.__setattr__(w, "_lbc_int4", c)
        except (AttributeError, TypeError):
            pass
    return c


def gemm_w4a8_amx(x, w, params: Params | None = None, isa=None, threads: int | None = None,
                  _prep: _Prepared | None = None):
    """lowbit's gemm_w4a8_amx (src/lowbit/kernels.py:208-217): W4A8 on weights in
    the AMX repack layout (formats.AMXInt4Weights, or lowbit's own), fp32 X
    quantized per token to int8 inside the call; the same results as
    gemm_w4a8 on the unpacked weights (exact int32 group sums)."""
    return gemm_w4a8(x, _amx_int4(w), params, isa, threads, _prep)


def w4a8_group_acc_amx(a: Int8Acts, w):
    """lowbit's w4a8_group_acc_amx (src/lowbit/kernels.py:220-225): exact int32
    accumulators out[m, n, g] for AMX-packed weights."""
    return w4a8_group_acc(a, _amx_int4(w))


def _dev_acts(a: Int8Acts):
    from ._torch import to_cuda
    torch = _torch()
    host = not isinstance(a.xq, torch.Tensor)
    return host, to_cuda(a.xq), to_cuda(a.scale), to_cuda(a.gsum)


def gemm_w4a8_q(a: Int8Acts, w: Int4Weights, params: Params | None = None, isa=None,
                threads: int | None = None):
    """W4A8 GEMM on already-quantized activations."""
    torch = _torch()
    host, xq, xs, gs = _dev_acts(a)
    m = int(xq.shape[0])
    d = _dev_weights(w)
    y = torch.empty((m, w.n), dtype=torch.float32, device=xq.device)
    rc = _call("lbc_gemm_w4a8_q", xq.data_ptr(), xs.data_ptr(), gs.data_ptr(), m, w.kp, d.qw.data_ptr(),
               d.scales.data_ptr(), None if d.zeros is None else d.zeros.data_ptr(), w.n, y.data_ptr(),
               C.byref(_params(params, isa, "w4a8", (m, w.n, w.k))), _stream())
    _check(rc, "lbc_gemm_w4a8_q")
    return y.cpu().numpy() if host else y


def quant_act_int8(x, kp: int) -> Int8Acts:
    """Per-token int8 quantization on the GPU (bit-identical to formats.quantize_act_int8)."""
    torch = _torch()
    pr = _Prepared(np.atleast_2d(x) if not isinstance(x, torch.Tensor) else x, kp, 1)
    m = pr.m
    xq = torch.empty((m, kp), dtype=torch.int8, device=pr.x.device)
    xs = torch.empty((m,), dtype=torch.float32, device=pr.x.device)
    gs = torch.empty((m, kp // GROUP), dtype=torch.int32, device=pr.x.device)
    _check(_call("lbc_quant_act_int8", pr.x.data_ptr(), m, kp, xq.data_ptr(), xs.data_ptr(),
                 gs.data_ptr(), _stream()), "lbc_quant_act_int8")
    if pr.host:
        return Int8Acts(xq.cpu().numpy(), xs.cpu().numpy(), gs.cpu().numpy())
    return Int8Acts(xq, xs, gs)


def w4a8_group_acc(a: Int8Acts, w: Int4Weights, isa=None):
    """Exact int32 accumulators out[m, n, g] = sum_{k in g} (q - z) * xq (debug/test)."""
    torch = _torch()
    host, xq, _, gs = _dev_acts(a)
    m = int(xq.shape[0])
    d = _dev_weights(w)
    out = torch.empty((m, w.n, w.kp // GROUP), dtype=torch.int32, device=xq.device)
    _check(_call("lbc_w4a8_group_acc", xq.data_ptr(), gs.data_ptr(), m, w.kp, d.qw.data_ptr(),
                 None if d.zeros is None else d.zeros.data_ptr(), w.n, out.data_ptr(), -1, _stream()),
           "lbc_w4a8_group_acc")
    return out.cpu().numpy() if host else out


# ---------------------------------------------------------------- on-device quantizers

_QMODE = {("absmax", False): 0, ("absmax", True): 1, ("signed-max", False): 2}


def quantize_int4_cuda(w, asym: bool = False, scale: str = "absmax") -> Int4Weights:
    """formats.quantize_int4 on the GPU, bit for bit: W fp32 [N, K] (numpy or
    torch) -> Int4Weights with CUDA tensors."""
    from ._torch import to_cuda
    torch = _torch()
    if scale not in ("absmax", "signed-max"):
        raise ValueError(f"scale must be 'absmax' or 'signed-max', not {scale!r}")
    if asym and scale != "absmax":
        raise ValueError("scale='signed-max' is a symmetric rule (asym=False)")
    wt = to_cuda(w).to(torch.float32).contiguous()
    n, k = (int(d) for d in wt.shape)
    kp = -(-k // GROUP) * GROUP
    qw = torch.empty((n, kp // 2), dtype=torch.uint8, device=wt.device)
    sc = torch.empty((n, kp // GROUP), dtype=torch.float32, device=wt.device)
    z = torch.empty((n, kp // GROUP), dtype=torch.uint8, device=wt.device) if asym else None
    _check(_call("lbc_quantize_int4", wt.data_ptr(), n, k, _QMODE[(scale, bool(asym))], qw.data_ptr(),
                 sc.data_ptr(), None if z is None else z.data_ptr(), _stream()), "lbc_quantize_int4")
    return Int4Weights(qw, sc, z, k)


def quantize_mxfp4_cuda(w) -> MXFP4Weights:
    """formats.quantize_mxfp4 on the GPU, bit for bit."""
    from ._torch import to_cuda
    torch = _torch()
    wt = to_cuda(w).to(torch.float32).contiguous()
    n, k = (int(d) for d in wt.shape)
    kp = -(-k // 32) * 32
    qw = torch.empty((n, kp // 2), dtype=torch.uint8, device=wt.device)
    e = torch.empty((n, kp // 32), dtype=torch.uint8, device=wt.device)
    _check(_call("lbc_quantize_mxfp4", wt.data_ptr(), n, k, qw.data_ptr(), e.data_ptr(), _stream()),
           "lbc_quantize_mxfp4")
    return MXFP4Weights(qw, e, k)


def describe_plan(kind: str, m: int, n: int, kp: int, params: Params | None = None, isa=None) -> dict:
    """Kernel configuration the library would launch for this GEMM (for tuning / debugging)."""
    import json
    buf = C.create_string_buffer(512)
    rc = lib().lbc_describe_plan(KIND_IDS[kind], m, n, kp, C.byref(_params(params, isa)), buf, 512)
    _check(rc, "lbc_describe_plan")
    return json.loads(buf.value.decode())


def tc_selftest(kind: int):
    """D[128,16] from the tensor-core self-test kernel (kind 0 bf16, 1 int8) as int32 numpy."""
    torch = _torch()
    out = torch.full((128, 16), -12345, dtype=torch.int32, device="cuda")
    _check(lib().lbc_tc_selftest(kind, out.data_ptr(), _stream()), "lbc_tc_selftest")
    return out.cpu().numpy()


def set_wait_cycles(cycles: int) -> None:
    """Limit of every bounded device-side wait on the current device, in SM
    clock cycles (<= 0: the default, about 2 s); for kernels launched afterwards."""
    _check(lib().lbc_set_wait_cycles(int(cycles)), "lbc_set_wait_cycles")


def wait_cycles() -> int:
    return int(lib().lbc_wait_cycles())


def device_status(reset: bool = True) -> int:
    """0, or the error code a bounded device-side wait recorded (synchronous)."""
    return int(lib().lbc_device_status(1 if reset else 0))


GEMMS = {"w4a16": gemm_w4a16, "mxfp4": gemm_mxfp4, "w4a8": gemm_w4a8}
