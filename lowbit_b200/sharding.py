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


class FusedColumnParallel:
    """W4A16 decode (one or two tokens) with the all-gather fused into the
    kernel: every rank's GEMV stores its Y rows straight into the Y buffer of
    every rank over NVLink (CUDA IPC peer pointers) and signals completion
    with a per-call epoch flag, so no separate collective runs.

    Y is double-buffered by call parity: a rank may start call e + 2 only
    after every rank finished call e + 1, and a rank's call e + 1 reads its X
    only after whatever consumed Y(e) on that GPU, so no store lands in a
    buffer still being read. The call counter lives on the device (CUDA-graph
    replays stay correct); ``__call__`` returns a view of the Y buffer of the
    call it launched, by the host's own count of calls, so read it only when
    every call went through ``__call__`` (not a graph replay).
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
        self.m, self.n = m, n
        self.lo, self.hi = shard_bounds(n, self.rank, self.world)
        L = K.lib()
        ybytes = 2 * m * n * 4
        self._own = []

        def alloc(nbytes):
            p = C.c_void_p()
            K._check(L.lbc_device_alloc(nbytes, C.byref(p)), "lbc_device_alloc")
            self._own.append(p.value)
            return p.value

        self._y = alloc(ybytes)
        self._flags = alloc(4 * self.world)
        self._counter = alloc(256)  # byte 0: CTA counter, byte 128: call epoch
        handles = []
        for ptr in (self._y, self._flags):
            h = (C.c_char * 64)()
            K._check(L.lbc_ipc_get_handle(ptr, h), "lbc_ipc_get_handle")
            handles.append(bytes(h))
        everyone = [None] * self.world
        dist.all_gather_object(everyone, handles, group=group)
        self._opened = []
        ys, fs = [], []
        for r, (hy, hf) in enumerate(everyone):
            if r == self.rank:
                ys.append(self._y)
                fs.append(self._flags)
                continue
            for h, out in ((hy, ys), (hf, fs)):
                p = C.c_void_p()
                buf = (C.c_char * 64).from_buffer_copy(h)
                K._check(L.lbc_ipc_open_handle(buf, C.byref(p)), "lbc_ipc_open_handle")
                self._opened.append(p.value)
                out.append(p.value)
        dev = torch.cuda.current_device()
        half = m * n * 4
        self._yptrs = torch.tensor([y + par * half for par in (0, 1) for y in ys], dtype=torch.int64, device=dev)
        self._fptrs = torch.tensor(fs, dtype=torch.int64, device=dev)
        self.epoch = 0
        self._yview = [self._as_tensor(self._y + par * half, (m, n)) for par in (0, 1)]
        dist.barrier(group=group)

    def _as_tensor(self, ptr, shape):
        """A float32 CUDA tensor aliasing library-owned device memory."""
        torch = self.torch

        class _Arr:
            __cuda_array_interface__ = {"shape": shape, "typestr": "<f4", "data": (ptr, False), "version": 3,
                                        "strides": None}
        return torch.as_tensor(_Arr(), device="cuda")

    def __call__(self, x, w_local, params=None, _prep=None):
        K, C = self.K, self.C
        self.epoch += 1
        par = self.epoch & 1
        pr = _prep or K._Prepared(x, w_local.kp, w_local.n)
        d = K._dev_weights(w_local)
        rc = K.lib().lbc_gemm_w4a16_allgather(
            pr.x.data_ptr(), pr.m, w_local.kp, d.qw.data_ptr(), d.scales.data_ptr(),
            None if d.zeros is None else d.zeros.data_ptr(), w_local.n, self.lo, self.n,
            self._yptrs.data_ptr(), self._fptrs.data_ptr(), self._counter, self._counter + 128,
            self.rank, self.world, C.byref(K._params(params, None)), K._stream())
        K._check(rc, "lbc_gemm_w4a16_allgather")
        return self._yview[par]

    def resync(self):
        """Re-read the device call counter (after CUDA-graph replays of these calls)."""
        torch = self.torch
        torch.cuda.synchronize()
        e = self._as_u32(self._counter + 128)
        self.epoch = int(e.item())

    def _as_u32(self, ptr):
        torch = self.torch

        class _Arr:
            __cuda_array_interface__ = {"shape": (1,), "typestr": "<u4", "data": (ptr, False), "version": 3,
                                        "strides": None}
        return torch.as_tensor(_Arr(), device="cuda").to(torch.int64)

    def close(self):
        torch = self.torch
        torch.cuda.synchronize()
        L = self.K.lib()
        for p in self._opened:
            L.lbc_ipc_close_handle(p)
        self._opened = []
        for p in self._own:
            L.lbc_device_free(p)
        self._own = []
