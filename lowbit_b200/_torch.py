"""torch plumbing: device placement, raw pointers and the current stream.

torch is used only for device memory, streams and torch.distributed; every
computation on the hot path runs in liblowbit_b200.so.
"""
from __future__ import annotations

import numpy as np
import torch

_NP2T = {np.dtype(np.float32): torch.float32, np.dtype(np.uint8): torch.uint8,
         np.dtype(np.int8): torch.int8, np.dtype(np.int32): torch.int32}


def require_cuda() -> None:
    if not torch.cuda.is_available():
        raise RuntimeError("lowbit_b200 needs a CUDA device (sm_100a); there is no CPU path")


def to_cuda(a, device=None) -> torch.Tensor:
    """Contiguous CUDA tensor holding `a` (numpy array or tensor); copies at most once."""
    require_cuda()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if isinstance(a, torch.Tensor):
        t = a if a.device == dev else a.to(dev)
        return t.contiguous()
    arr = np.ascontiguousarray(a)
    if not arr.flags.writeable:
        # a read-only view (a packed file's memory map): torch only reads it
        # for the copy to the device
        import warnings
        with warnings.catch_warnings():
            warnings.simplefilter("ignore", UserWarning)
            return torch.from_numpy(arr).to(dev, non_blocking=False).contiguous()
    return torch.from_numpy(arr).to(dev, non_blocking=False).contiguous()


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else int(t.data_ptr())


def stream_handle(stream=None) -> int:
    s = torch.cuda.current_stream() if stream is None else stream
    return int(s.cuda_stream)
