"""Host-buffer entry points (lbc_gemm_w4a16_host / _mxfp4_host / _w4a8_host),
the path lowbit's own numpy API takes here: X and Y in host memory, weights
on the device. They run the same kernels as the device-pointer entry points
(their first call with a given shape and weights eagerly, later ones as a
cached CUDA graph), so their results must equal the device path's bit for
bit, and the oracle's within the usual bound."""
import ctypes as C
import threading

import numpy as np
import pytest

import lowbit_b200 as lb
from lowbit_b200 import kernels as K
from oracle import lbref as R

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

KINDS = {"w4a16": (lambda w: lb.quantize_int4(w, asym=True), K.gemm_w4a16),
         "w4a8": (lambda w: lb.quantize_int4(w, asym=True), K.gemm_w4a8),
         "mxfp4": (lambda w: lb.quantize_mxfp4(w), K.gemm_mxfp4)}


def _device(fn, x, W):
    """The device-pointer path: torch CUDA X in, torch CUDA Y out."""
    xd = torch.from_numpy(np.pad(x, ((0, 0), (0, W.kp - x.shape[1])))).cuda()
    return fn(xd, W.cuda()).cpu().numpy()


@pytest.mark.parametrize("kind", list(KINDS))
@pytest.mark.parametrize("m,n,k", [(1, 333, 4096), (2, 1001, 1000), (5, 257, 2048), (96, 300, 640),
                                   (1, 11008, 4096), (3, 7, 128)])
def test_host_equals_device(rng, kind, m, n, k):
    quant, fn = KINDS[kind]
    x = rng.standard_normal((m, k)).astype(np.float32)
    W = quant(rng.standard_normal((n, k)).astype(np.float32))
    ref = _device(fn, x, W)
    for _ in range(3):          # eager first call, then the captured graph
        y = fn(x, W)
        assert isinstance(y, np.ndarray) and y.shape == (m, n)
        np.testing.assert_array_equal(y, ref)
    if kind == "w4a16" and m <= 2:   # the exact SIMT path (tensor-core paths: their own tests)
        R.assert_close(y, R.gemm_w4a16_ref(x, W.qw, W.scales, W.zeros),
                       R.abs_bound(x, R.dequant_int4(W.qw, W.scales, W.zeros)), 1e-5)


def test_host_fresh_inputs_every_call(rng):
    """A cached graph reads each call's X: every call's Y matches its own X."""
    W = lb.quantize_int4(rng.standard_normal((513, 1024)).astype(np.float32), asym=True)
    Wd = W.cuda()
    for i in range(6):
        x = rng.standard_normal((2, 1024)).astype(np.float32)
        y = K.gemm_w4a16(x, Wd)
        np.testing.assert_array_equal(y, K.gemm_w4a16(torch.from_numpy(x).cuda(), Wd).cpu().numpy())


def test_host_many_weights_and_shapes(rng):
    """More (shape, weights) keys than one stream's graph cache holds."""
    Ws = [lb.quantize_int4(rng.standard_normal((64 + i, 256)).astype(np.float32)).cuda() for i in range(70)]
    x = rng.standard_normal((1, 256)).astype(np.float32)
    for rep in range(2):
        for W in Ws:
            np.testing.assert_array_equal(K.gemm_w4a16(x, W),
                                          K.gemm_w4a16(torch.from_numpy(x).cuda(), W).cpu().numpy())


def test_host_threads_and_streams(rng):
    """Two host threads on two streams, each with its own staging."""
    W = lb.quantize_int4(rng.standard_normal((2048, 2048)).astype(np.float32), asym=True).cuda()
    xs = [rng.standard_normal((1, 2048)).astype(np.float32) for _ in range(2)]
    refs = [K.gemm_w4a16(torch.from_numpy(x).cuda(), W).cpu().numpy() for x in xs]
    errors = []

    def worker(i):
        try:
            with torch.cuda.stream(torch.cuda.Stream()):
                for _ in range(50):
                    np.testing.assert_array_equal(K.gemm_w4a16(xs[i], W), refs[i])
        except Exception as e:  # noqa: BLE001
            errors.append(e)

    ts = [threading.Thread(target=worker, args=(i,)) for i in range(2)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errors, errors


def test_host_entry_refuses_capture(rng):
    """The host-buffer entry synchronises its stream, so it refuses a capturing
    stream with LBC_ERR_PARAMS, enqueuing nothing."""
    W = lb.quantize_int4(rng.standard_normal((64, 128)).astype(np.float32)).cuda()
    x = np.ones((1, 128), np.float32)
    y = np.zeros((1, 64), np.float32)
    L = K.lib()
    buf = torch.zeros(4, device="cuda")
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        rc = L.lbc_gemm_w4a16_host(x.ctypes.data, 1, 128, W.qw.data_ptr(), W.scales.data_ptr(), None, 64,
                                   y.ctypes.data, None, torch.cuda.current_stream().cuda_stream)
        buf.add_(1)
    assert rc == -2
    g.replay()
    torch.cuda.synchronize()
    assert float(buf[0]) == 1.0
    assert not y.any()


def test_host_entry_bad_arguments():
    L = K.lib()
    assert L.lbc_gemm_w4a16_host(None, 1, 128, None, None, None, 16, None, None, None) == -1
    x = np.ones((1, 100), np.float32)
    assert L.lbc_gemm_w4a16_host(x.ctypes.data, 1, 100, None, None, None, 16, x.ctypes.data, None, None) == -1
    assert L.lbc_gemm_mxfp4_host(x.ctypes.data, 1, 100, None, None, 16, x.ctypes.data, None, None) == -1
    assert L.lbc_gemm_w4a8_host(x.ctypes.data, 0, 128, None, None, None, 16, x.ctypes.data, None, None) == -1
    assert C.c_int(L.lbc_device_status(1)).value == 0


@pytest.mark.parametrize("kind", ["w4a16", "mxfp4"])
def test_host_scratch_growth_keeps_cached_graphs_valid(rng, kind):
    """A cached host-call graph holds the address of the per-stream scratch its
    capture used (tensor-core fixup slots, few-token K-range partial sums). A
    later call that needs more scratch grows it; the earlier graph must still
    see valid memory when it is replayed: small key, big key, small key
    again, each equal to the device path. Shapes: few-token kernel with K
    ranges (8 tokens on 896 x 4864, then 16 tokens on 1152 x 4864) and the
    tensor-core exact kernel (32 tokens on 4096 x 4096, then 48 on 11008 x 4096)."""
    quant, fn = KINDS[kind]
    for (m1, n1, k1), (m2, n2, k2) in (((8, 896, 4864), (16, 1152, 4864)),
                                       ((32, 4096, 4096), (48, 11008, 4096))):
        xs = rng.standard_normal((m1, k1)).astype(np.float32)
        xb = rng.standard_normal((m2, k2)).astype(np.float32)
        Ws = quant(rng.standard_normal((n1, k1)).astype(np.float32))
        Wb = quant(rng.standard_normal((n2, k2)).astype(np.float32))
        ref_s, ref_b = _device(fn, xs, Ws), _device(fn, xb, Wb)
        for _ in range(2):      # eager + capture of the small key
            np.testing.assert_array_equal(fn(xs, Ws), ref_s)
        for _ in range(2):      # the big key grows the scratch
            np.testing.assert_array_equal(fn(xb, Wb), ref_b)
        for _ in range(3):      # the small key's cached graph again
            np.testing.assert_array_equal(fn(xs, Ws), ref_s)
