"""lbc_gemm_w4a8_noalloc, the W4A8 entry point for callers that cannot allocate
device memory (its scratch is a fixed array inside the library), must give the
same results as the regular lbc_gemm_w4a8 with a caller workspace, call after
call, although every call reuses the array the previous call left behind.
Called through the C ABI with device pointers. This file is collected last."""
import ctypes as C

import numpy as np
import pytest

import lowbit_b200 as lb
from lowbit_b200 import kernels as K
from oracle import lbref as R

pytestmark = pytest.mark.gpu

RTOL = 1e-5  # the W4A8 tolerance of the other GPU tests


def _lib():
    L = K.lib()
    vp, i = C.c_void_p, C.c_int
    L.lbc_gemm_w4a8_noalloc.argtypes = [vp, i, i, vp, vp, vp, i, vp, C.c_void_p, vp]
    L.lbc_gemm_w4a8_noalloc.restype = i
    return L


def _run_both(L, x, W, isa=None):
    import torch
    dev = torch.device("cuda", torch.cuda.current_device())
    m, kp, n = x.shape[0], W.kp, W.n
    xp = np.zeros((m, kp), np.float32)
    xp[:, : x.shape[1]] = x
    xd = torch.from_numpy(xp).to(dev)
    qw = torch.from_numpy(W.qw).to(dev)
    sc = torch.from_numpy(W.scales).to(dev)
    zz = None if W.zeros is None else torch.from_numpy(W.zeros).to(dev)
    y_ref = torch.full((m, n), float("nan"), device=dev)
    y_na = torch.full((m, n), float("nan"), device=dev)
    ws = torch.empty(int(L.lbc_gemm_w4a8_workspace_size(m, kp)), dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    zp = None if zz is None else zz.data_ptr()
    p = None if isa is None else C.byref(K._params(None, isa))
    rc = L.lbc_gemm_w4a8(xd.data_ptr(), m, kp, qw.data_ptr(), sc.data_ptr(), zp, n, y_ref.data_ptr(),
                         p, ws.data_ptr(), st)
    assert rc >= 0, L.lbc_last_error()
    rc = L.lbc_gemm_w4a8_noalloc(xd.data_ptr(), m, kp, qw.data_ptr(), sc.data_ptr(), zp, n,
                                 y_na.data_ptr(), p, st)
    assert rc >= 0, L.lbc_last_error()
    torch.cuda.synchronize()
    return y_ref.cpu().numpy(), y_na.cpu().numpy()


# (M, N, K, asym, isa): the automatic paths (16 and 32 tokens: the int8 mma
# kernel; 3 tokens: the SIMT decode kernel) and, asked for explicitly at 32
# tokens on a 4096 x 4096 matrix, the tensor-core exact kernel, whose
# partial-row slots and epoch flags also live in the static scratch
CASES = [(16, 256, 4096, False, None), (3, 96, 640, True, None), (32, 4096, 4096, True, "tcgen05"),
         (16, 256, 4096, False, None), (32, 4096, 4096, True, "tcgen05"), (32, 4096, 4096, True, None)]


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls():
    L = _lib()
    rng = np.random.default_rng(99)
    # different problems in a row: each reuses (and must not depend on) what
    # the one before left in the static scratch
    for (m, n, k, asym, isa) in CASES:
        x = (rng.standard_normal((m, k)) * rng.uniform(0.1, 10)).astype(np.float32)
        W = lb.quantize_int4(rng.standard_normal((n, k)).astype(np.float32), asym=asym)
        y_ref, y_na = _run_both(L, x, W, isa)
        a = lb.quantize_act_int8(x)
        bound = R.w4a8_bound(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros)
        R.assert_close(y_na, y_ref.astype(np.float64), bound, RTOL)
        R.assert_close(y_na, R.gemm_w4a8_ref(a.xq, a.scale, a.gsum, W.qw, W.scales, W.zeros), bound, RTOL)


def test_noalloc_rejects_problems_beyond_its_scratch():
    L = _lib()
    limit = 4 << 20
    m, kp = 1024, 8192  # 8 MiB of int8 codes alone
    assert L.lbc_gemm_w4a8_workspace_size(m, kp) > limit
    rc = L.lbc_gemm_w4a8_noalloc(None, m, kp, None, None, None, 16, None, None, None)
    assert rc == -1
    assert b"static buffer" in L.lbc_last_error()


def test_noalloc_allocates_nothing():
    """After a first round (which may load kernels lazily), more calls leave the
    device's free memory and torch's allocator unchanged."""
    import torch
    L = _lib()
    rng = np.random.default_rng(7)
    dev = torch.device("cuda", torch.cuda.current_device())
    st = torch.cuda.current_stream().cuda_stream
    probs = []
    for (m, n, k, asym, isa) in CASES[:3]:
        W = lb.quantize_int4(rng.standard_normal((n, k)).astype(np.float32), asym=asym)
        xd = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).to(dev)
        probs.append((m, n, k, xd, torch.from_numpy(W.qw).to(dev), torch.from_numpy(W.scales).to(dev),
                      None if W.zeros is None else torch.from_numpy(W.zeros).to(dev),
                      torch.empty((m, n), device=dev), None if isa is None else C.byref(K._params(None, isa))))

    def round_():
        for (m, n, k, xd, qw, sc, zz, y, p) in probs:
            rc = L.lbc_gemm_w4a8_noalloc(xd.data_ptr(), m, k, qw.data_ptr(), sc.data_ptr(),
                                         None if zz is None else zz.data_ptr(), n, y.data_ptr(), p, st)
            assert rc >= 0, L.lbc_last_error()
        torch.cuda.synchronize()

    round_()
    free0, alloc0 = torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()
    for _ in range(3):
        round_()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.cuda.memory_allocated() == alloc0


def test_noalloc_bad_shape_sets_error_text():
    L = _lib()
    rc = L.lbc_gemm_w4a8_noalloc(None, 0, 128, None, None, None, 16, None, None, None)
    assert rc == -1
    assert b"bad shape" in L.lbc_last_error()
