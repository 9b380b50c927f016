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
