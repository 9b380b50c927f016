"""Column-parallel (N-sharded) GEMMs over torch.distributed ranks.

Rank p of P owns weight rows ``shard_bounds(N, p, P)`` of every per-row array
(``qw``, ``scales``, ``zeros``, ``e8m0``: no group straddles a row), computes
its Y slice ``[M, N_p]`` with the single-GPU kernels, and one all-gather
assembles ``Y[M, N]`` on every rank. Shards differ by at most one row; the
gather pads every slice to the largest shard so one collective of equal-size
buffers suffices (NCCL over NVLink on GPUs, gloo for CPU tests), then drops the
padding while placing each slice at its row offset.
"""
from __future__ import annotations

from .formats import shard_bounds


def padded_rows(n: int, world: int) -> int:
    """Rows of the largest shard (the gather's slice height)."""
    return -(-n // world)


class ColumnParallel:
    """Gather buffers for one (M, N, world) shape, reused across calls."""

    def __init__(self, m: int, n: int, group=None):
        import torch
        import torch.distributed as dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.m, self.n = m, n
        self.lo, self.hi = shard_bounds(n, self.rank, self.world)
        self.rows = padded_rows(n, self.world)
        self._torch, self._dist = torch, dist
        self.bounds = [shard_bounds(n, r, self.world) for r in range(self.world)]

    def gather(self, y_local, out=None):
        """All-gather the [M, N_p] slices into [M, N] (out, if given)."""
        torch, dist = self._torch, self._dist
        m = self.m
        if tuple(y_local.shape) != (m, self.hi - self.lo):
            raise ValueError(f"local slice has shape {tuple(y_local.shape)}, expected {(m, self.hi - self.lo)}")
        if self.n % self.world == 0 and dist.get_backend(self.group) == "nccl":
            # equal shards: one all-gather into [P, M, N/P], viewed as [M, N]
            buf = torch.empty((self.world, m, self.rows), dtype=y_local.dtype, device=y_local.device)
            dist.all_gather_into_tensor(buf, y_local.contiguous(), group=self.group)
            y = buf.permute(1, 0, 2).reshape(m, self.n)
            if out is None:
                return y if m == 1 else y.contiguous()
            out.copy_(y)
            return out
        send = torch.zeros((m, self.rows), dtype=y_local.dtype, device=y_local.device)
        send[:, : self.hi - self.lo] = y_local
        parts = [torch.empty_like(send) for _ in range(self.world)]
        dist.all_gather(parts, send, group=self.group)
        if out is None:
            out = torch.empty((m, self.n), dtype=y_local.dtype, device=y_local.device)
        for r, (lo, hi) in enumerate(self.bounds):
            out[:, lo:hi] = parts[r][:, : hi - lo]
        return out


def gemm_sharded(kind: str, x, w_local, cp: ColumnParallel, **kw):
    """This rank's slice through the single-GPU kernel, then the all-gather."""
    from . import kernels as K
    y = K.GEMMS[kind](x, w_local, **kw)
    return cp.gather(y)


class _PeerBuffers:
    """Library-owned device buffers of this rank, mapped by every rank of the
    process group over CUDA IPC (`lbc_device_alloc`, zero-filled), plus
    private ones that stay local. `peers(name)` lists a shared buffer's
    address on every rank, in rank order (this rank's own included).
    `close()` is collective: every rank unmaps the peers' buffers, then
    frees its own once nobody maps them."""

    def __init__(self, group, shared: dict, private: dict):
        import ctypes as C
        import torch.distributed as dist
        from . import kernels as K
        self.K, self.C, self.dist, self.group = K, C, dist, group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        L = K.lib()
        self._own, self._opened, self.addr, self._peers = [], [], {}, {}
        for name, nbytes in list(shared.items()) + list(private.items()):
            p = C.c_void_p()
            K._check(L.lbc_device_alloc(nbytes, C.byref(p)), "lbc_device_alloc")
            self._own.append(p.value)
            self.addr[name] = p.value
        handles = []
        for name in shared:
            h = (C.c_char * 64)()
            K._check(L.lbc_ipc_get_handle(self.addr[name], h), "lbc_ipc_get_handle")
            handles.append(bytes(h))
        everyone = [None] * self.world
        dist.all_gather_object(everyone, handles, group=group)
        for i, name in enumerate(shared):
            ptrs = []
            for r in range(self.world):
                if r == self.rank:
                    ptrs.append(self.addr[name])
                    continue
                p = C.c_void_p()
                buf = (C.c_char * 64).from_buffer_copy(everyone[r][i])
                K._check(L.lbc_ipc_open_handle(buf, C.byref(p)), "lbc_ipc_open_handle")
                self._opened.append(p.value)
                ptrs.append(p.value)
            self._peers[name] = ptrs

    def peers(self, name: str) -> list:
        return self._peers[name]

    def close(self):
        L = self.K.lib()
        for p in self._opened:
            L.lbc_ipc_close_handle(p)
        self._opened = []
        self.dist.barrier(group=self.group)  # no rank maps this rank's buffers any more
        for p in self._own:
            L.lbc_device_free(p)
        self._own = []


class FusedColumnParallel:
    """W4A16 decode (one or two tokens) with the all-gather fused into the
    kernel (``lbc_gemm_w4a16_allgather``): every rank's GEMV writes its own Y
    rows and sends each value to every other rank over NVLink (CUDA IPC peer
    pointers) as one 8-byte word tagged with the call's epoch; each rank's
    CTAs wait for the words of this epoch in its own landing buffer and copy
    them into its Y. No separate collective runs and no fence or flag sits
    between the GEMV and the exchange.

    The landing buffers alternate halves by call parity: a rank writes call
    e + 2 into a peer's buffer only after its own call e + 1 received that
    peer's call e + 1 rows, which that peer produced after its call e ended.
    The call counter lives on the device (CUDA-graph replays stay correct).
    ``__call__`` returns this rank's Y, alternating between two buffers by the
    host's count of calls, so the previous call's result stays readable.
    """

    def __init__(self, m: int, n: int, group=None):
        import ctypes as C
        import torch
        import torch.distributed as dist
        from . import kernels as K
        if m > 2:
            raise ValueError("the fused all-gather decode serves one or two tokens")
        self.K, self.C, self.torch = K, C, torch
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the fused all-gather decode serves at most 8 ranks")
        self.m, self.n = m, n
        self.lo, self.hi = shard_bounds(n, self.rank, self.world)
        # landing buffer: LBC_GATHER_LAND_BYTES(n); counters: byte 0 the CTA
        # counter, byte 128 the call epoch
        self._buf = _PeerBuffers(group, {"land": n * 2 * 2 * 8}, {"counter": 256})
        self._counter = self._buf.addr["counter"]
        lands = self._buf.peers("land")
        dev = torch.cuda.current_device()
        self._lptrs = torch.tensor(lands, dtype=torch.int64, device=dev)
        self._ys = [torch.empty((m, n), dtype=torch.float32, device=dev) for _ in range(2)]
        self.epoch = 0
        dist.barrier(group=group)

    def __call__(self, x, w_local, params=None, _prep=None):
        K, C = self.K, self.C
        self.epoch += 1
        y = self._ys[self.epoch & 1]
        pr = _prep or K._Prepared(x, w_local.kp, w_local.n)
        d = K._dev_weights(w_local)
        rc = K.lib().lbc_gemm_w4a16_allgather(
            pr.x.data_ptr(), pr.m, w_local.kp, d.qw.data_ptr(), d.scales.data_ptr(),
            None if d.zeros is None else d.zeros.data_ptr(), w_local.n, self.lo, self.n,
            y.data_ptr(), self._lptrs.data_ptr(), self._counter, self._counter + 128,
            self.rank, self.world, C.byref(K._params(params, None)), K._stream())
        K._check(rc, "lbc_gemm_w4a16_allgather")
        return y

    def resync(self):
        """Re-read the device call counter (after CUDA-graph replays of these calls)."""
        torch = self.torch
        torch.cuda.synchronize()
        self.epoch = int(_u32_view(torch, self._counter + 128).item())

    def close(self):
        self.torch.cuda.synchronize()
        self._buf.close()


class FusedColumnParallelGemm:
    """Many-token GEMM (64+ tokens, any of the three formats) with the
    all-gather fused into the tcgen05 prefill kernel's store
    (``lbc_gemm_allgather``): every finished output tile goes to every rank's
    Y over NVLink while later tiles are computed, so the exchange overlaps the
    GEMM instead of following it. Y is double-buffered by call parity (a rank
    can start call e + 1 while a peer still reads Y(e); call e + 2 waits for
    every rank's call e + 1, which follows that rank's reads of Y(e) in its
    stream); each rank's device call counter (CUDA-graph replays stay correct)
    and one call counter per rank pair signal completion. ``__call__`` returns
    the Y of the call it launched (by the host's count of calls)."""

    KINDS = {"w4a16": 0, "mxfp4": 1, "w4a8": 2}

    def __init__(self, kind: str, m: int, n: int, group=None):
        import ctypes as C
        import torch
        import torch.distributed as dist
        from . import kernels as K
        if kind not in self.KINDS:
            raise ValueError(f"kind must be one of {sorted(self.KINDS)}")
        if m < 64:
            raise ValueError("the fused all-gather GEMM serves 64 or more tokens")
        self.K, self.C, self.torch = K, C, torch
        self.kind, self.group = kind, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.m, self.n = m, n
        self.lo, self.hi = shard_bounds(n, self.rank, self.world)
        half = m * n * 4
        # Y of both parities, the call counters [world] of the rank pairs, and
        # this rank's CTA counter (byte 0) and call epoch (byte 128)
        self._buf = _PeerBuffers(group, {"y": 2 * half, "flags": max(16, 4 * self.world)}, {"counter": 256})
        self._y, self._counter = self._buf.addr["y"], self._buf.addr["counter"]
        ys, fs = self._buf.peers("y"), self._buf.peers("flags")
        dev = torch.cuda.current_device()
        self._yptrs = torch.tensor([y + par * half for par in (0, 1) for y in ys], dtype=torch.int64, device=dev)
        self._fptrs = torch.tensor(fs, dtype=torch.int64, device=dev)
        self._yview = [_f32_view(torch, self._y + par * half, (m, n)) for par in (0, 1)]
        self.epoch = 0
        dist.barrier(group=group)

    def __call__(self, x, w_local, params=None, _prep=None):
        K, C = self.K, self.C
        self.epoch += 1
        pr = _prep or K._Prepared(x, w_local.kp, w_local.n)
        d = K._dev_weights(w_local)
        ptr = (lambda t: None if t is None else t.data_ptr())
        rc = K.lib().lbc_gemm_allgather(
            self.KINDS[self.kind], pr.x.data_ptr(), pr.m, w_local.kp, d.qw.data_ptr(),
            ptr(getattr(d, "scales", None)), ptr(getattr(d, "zeros", None)), ptr(getattr(d, "e8m0", None)),
            w_local.n, self.lo, self.n, self._yptrs.data_ptr(), self._fptrs.data_ptr(), self._counter,
            self._counter + 128, self.rank, self.world, C.byref(K._params(params, None)), K._stream())
        K._check(rc, "lbc_gemm_allgather")
        return self._yview[self.epoch & 1]

    def resync(self):
        """Re-read the device call counter (after CUDA-graph replays of these calls)."""
        torch = self.torch
        torch.cuda.synchronize()
        self.epoch = int(_u32_view(torch, self._counter + 128).item())

    def close(self):
        self.torch.cuda.synchronize()
        self._buf.close()


def _f32_view(torch, ptr, shape):
    """A float32 CUDA tensor aliasing library-owned device memory."""
    class _Arr:
        __cuda_array_interface__ = {"shape": shape, "typestr": "<f4", "data": (ptr, False), "version": 3,
                                    "strides": None}
    return torch.as_tensor(_Arr(), device="cuda")


def _u32_view(torch, ptr):
    class _Arr:
        __cuda_array_interface__ = {"shape": (1,), "typestr": "<u4", "data": (ptr, False), "version": 3,
                                    "strides": None}
    return torch.as_tensor(_Arr(), device="cuda").to(torch.int64)
