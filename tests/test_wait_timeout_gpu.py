"""Bounded device-side waits run out cleanly (on one GPU, without a fault):
the fused all-gather decode is launched for rank 0 of a world of 2 whose
"rank 1" never runs (both ranks' landing buffers live on this GPU), so the
tagged words it waits for never come. With a short wait limit
(lbc_set_wait_cycles) the kernel gives up, records LBC_ERR_TIMEOUT in the
device status and returns; after the status is reset and the default limit
restored, a normal call on the same context succeeds."""
import ctypes as C

import numpy as np
import pytest

import lowbit_b200 as lb
from lowbit_b200 import kernels as K
from oracle import lbref as R

pytestmark = pytest.mark.gpu
LBC_ERR_TIMEOUT = -7


def test_allgather_wait_times_out_and_context_stays_usable():
    import torch
    dev = torch.device("cuda", torch.cuda.current_device())
    L = K.lib()
    n_total, k, world = 1024, 512, 2
    rng = np.random.default_rng(3)
    W = lb.quantize_int4(rng.standard_normal((n_total, k)).astype(np.float32), asym=True)
    Wh = W.shard(0, world)
    Wl = Wh.cuda()
    x = torch.from_numpy(rng.standard_normal((1, k)).astype(np.float32)).to(dev)
    y = torch.zeros((1, n_total), device=dev)
    lands = [torch.zeros(2 * 2 * n_total, dtype=torch.int64, device=dev) for _ in range(world)]
    counter = torch.zeros(64, dtype=torch.int32, device=dev)
    epoch = torch.zeros(64, dtype=torch.int32, device=dev)
    lptrs = torch.tensor([t.data_ptr() for t in lands], dtype=torch.int64, device=dev)
    K.device_status(reset=True)
    K.set_wait_cycles(2_000_000)   # about 1 ms
    try:
        assert K.wait_cycles() == 2_000_000
        rc = L.lbc_gemm_w4a16_allgather(x.data_ptr(), 1, W.kp, Wl.qw.data_ptr(), Wl.scales.data_ptr(),
                                        Wl.zeros.data_ptr(), Wl.n, 0, n_total, y.data_ptr(), lptrs.data_ptr(),
                                        counter.data_ptr(), epoch.data_ptr(), 0, world, None, K._stream())
        assert rc >= 0, L.lbc_last_error()
        torch.cuda.synchronize()
        assert K.device_status(reset=True) == LBC_ERR_TIMEOUT
        # the call still completed: epoch advanced, rank 0's own rows are right
        # in its Y and were sent to "rank 1" as words tagged with epoch 1
        # (call parity 1: the second half of the landing buffer)
        assert int(epoch[0].item()) == 1 and int(counter[0].item()) == 0
        xh = x.cpu().numpy()
        lo, hi = 0, Wh.n
        own = R.gemm_w4a16_ref(xh, Wh.qw, Wh.scales, Wh.zeros)[0]
        got = y[0, lo:hi].cpu().numpy()
        R.assert_close(got, own, R.abs_bound(xh, R.dequant_int4(Wh.qw, Wh.scales, Wh.zeros))[0], 1e-5)
        words = lands[1][2 * n_total + lo: 2 * n_total + hi].cpu().numpy().view(np.uint64)
        assert np.all((words >> np.uint64(32)) == 1)
        np.testing.assert_array_equal((words & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32), got)
    finally:
        K.set_wait_cycles(0)
    assert K.wait_cycles() == 4_000_000_000
    # the context is intact: a normal call gives the right answer, status clean
    y = K.gemm_w4a16(xh, W)
    R.assert_close(y, R.gemm_w4a16_ref(xh, W.qw, W.scales, W.zeros),
                   R.abs_bound(xh, R.dequant_int4(W.qw, W.scales, W.zeros)), 1e-5)
    assert K.device_status(reset=False) == 0


@pytest.mark.parametrize("fmt", ["w4a16", "w4a8"])
def test_gemm_allgather_wait_times_out(fmt):
    """The fused all-gather prefill GEMM (lbc_gemm_allgather) launched for rank
    0 of a world of 2 whose "rank 1" never runs: rank 0's tiles land in both
    ranks' Y buffers and it counts its call in "rank 1"'s counters, then its
    wait for rank 1's call runs out (short limit): LBC_ERR_TIMEOUT, the call
    counter still advances, and the context stays usable."""
    import torch
    dev = torch.device("cuda", torch.cuda.current_device())
    L = K.lib()
    m, n_total, k, world = 192, 640, 512, 2
    rng = np.random.default_rng(4)
    W = lb.quantize_int4(rng.standard_normal((n_total, k)).astype(np.float32), asym=(fmt == "w4a16"))
    Wh = W.shard(0, world)
    Wl = Wh.cuda()
    x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).to(dev)
    ys = [torch.full((m, n_total), -1.0, device=dev) for _ in range(2 * world)]   # [parity][rank]
    flags = [torch.zeros(4, dtype=torch.int32, device=dev) for _ in range(world)]
    counter = torch.zeros(64, dtype=torch.int32, device=dev)
    epoch = torch.zeros(64, dtype=torch.int32, device=dev)
    yptrs = torch.tensor([y.data_ptr() for y in ys], dtype=torch.int64, device=dev)
    fptrs = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64, device=dev)
    K.device_status(reset=True)
    K.set_wait_cycles(2_000_000)
    try:
        rc = L.lbc_gemm_allgather({"w4a16": 0, "w4a8": 2}[fmt], x.data_ptr(), m, W.kp, Wl.qw.data_ptr(),
                                  Wl.scales.data_ptr(), None if Wl.zeros is None else Wl.zeros.data_ptr(), None,
                                  Wl.n, 0, n_total, yptrs.data_ptr(), fptrs.data_ptr(), counter.data_ptr(),
                                  epoch.data_ptr(), 0, world, None, K._stream())
        assert rc >= 0, L.lbc_last_error()
        torch.cuda.synchronize()
        assert K.device_status(reset=True) == LBC_ERR_TIMEOUT
    finally:
        K.set_wait_cycles(0)
    assert int(epoch[0].item()) == 1 and int(counter[0].item()) == 0
    assert int(flags[1][0].item()) == 1 and int(flags[0][0].item()) == 1 and int(flags[0][1].item()) == 0
    # call 1 has parity 1: rank 0's rows, the same bits in both ranks'
    # buffers, within the prefill contract of the oracle; the other rows and
    # the other parity untouched
    xh = x.cpu().numpy()
    got = ys[2].cpu().numpy()
    np.testing.assert_array_equal(ys[3].cpu().numpy(), got)
    if fmt == "w4a16":
        R.assert_close(got[:, :Wh.n], R.gemm_w4a16_ref(xh, Wh.qw, Wh.scales, Wh.zeros),
                       R.abs_bound(xh, R.dequant_int4(Wh.qw, Wh.scales, Wh.zeros)), 4e-3)
    else:
        xq, xs, asum = R.quant_act_int8_ref(xh, W.kp)
        R.assert_close(got[:, :Wh.n], R.gemm_w4a8_ref(xq, xs, asum, Wh.qw, Wh.scales, None),
                       R.w4a8_bound(xq, xs, asum, Wh.qw, Wh.scales, None), 1e-5)
    assert np.all(got[:, Wh.n:] == -1.0)
    for r in range(world):
        assert np.all(ys[r].cpu().numpy() == -1.0)
    assert K.device_status(reset=False) == 0


@pytest.mark.parametrize("fmt", ["w4a16", "mxfp4", "w4a8"])
def test_gemm_allgather_world1_equals_gemm(fmt):
    """World 1: the fused all-gather GEMM is the prefill GEMM with its store
    redirected; values equal the plain call bit for bit (a shape whose plain
    call does not split K: 10 row tiles x 8 token tiles fill more than half
    the SMs), call after call (the parity buffers alternate), also when
    replayed from a CUDA graph."""
    import torch
    dev = torch.device("cuda", torch.cuda.current_device())
    L = K.lib()
    m, n, k = 1000, 1270, 256
    rng = np.random.default_rng(5)
    w = rng.standard_normal((n, k)).astype(np.float32)
    W = lb.quantize_mxfp4(w) if fmt == "mxfp4" else lb.quantize_int4(w, asym=(fmt == "w4a16"))
    Wd = W.cuda()
    gemm = {"w4a16": K.gemm_w4a16, "mxfp4": K.gemm_mxfp4, "w4a8": K.gemm_w4a8}[fmt]
    ys = [torch.zeros((m, n), device=dev) for _ in range(2)]
    flags = torch.zeros(4, dtype=torch.int32, device=dev)
    counter = torch.zeros(64, dtype=torch.int32, device=dev)
    epoch = torch.zeros(64, dtype=torch.int32, device=dev)
    yptrs = torch.tensor([y.data_ptr() for y in ys], dtype=torch.int64, device=dev)
    fptrs = torch.tensor([flags.data_ptr()], dtype=torch.int64, device=dev)
    xs = [torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).to(dev) for _ in range(3)]

    def call(x):
        p = lambda t: None if t is None else t.data_ptr()
        rc = L.lbc_gemm_allgather({"w4a16": 0, "mxfp4": 1, "w4a8": 2}[fmt], x.data_ptr(), m, W.kp, Wd.qw.data_ptr(),
                                  p(getattr(Wd, "scales", None)), p(getattr(Wd, "zeros", None)),
                                  p(getattr(Wd, "e8m0", None)), n, 0, n, yptrs.data_ptr(), fptrs.data_ptr(),
                                  counter.data_ptr(), epoch.data_ptr(), 0, 1, None, K._stream())
        assert rc >= 0, L.lbc_last_error()

    for i, x in enumerate(xs):
        call(x)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(ys[(i + 1) & 1].cpu().numpy(), gemm(x, Wd).cpu().numpy())
    assert int(epoch[0].item()) == 3 and int(flags[0].item()) == 3
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            call(xs[0])
    torch.cuda.current_stream().wait_stream(s)
    for i in range(2):
        g.replay()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(ys[(4 + i) & 1].cpu().numpy(), gemm(xs[0], Wd).cpu().numpy())
    assert int(epoch[0].item()) == 5
    assert K.device_status(reset=False) == 0
