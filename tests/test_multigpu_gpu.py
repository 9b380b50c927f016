"""Column-parallel decode on two GPUs (skipped with fewer): the fused kernel
(GEMV + all-gather by NVLink peer stores, lbc_gemm_w4a16_allgather) and the
NCCL all-gather path both assemble the unsharded result on every rank, call
after call (the device epoch and the double-buffered Y advance together)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, m, n, k, q):
    import torch.distributed as dist
    from datetime import timedelta

    import lowbit_b200 as lb
    from lowbit_b200 import kernels as K
    from lowbit_b200.sharding import ColumnParallel, FusedColumnParallel
    from oracle import lbref as R
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    errs = []
    try:
        rng = np.random.default_rng(11)
        w = rng.standard_normal((n, k)).astype(np.float32)
        W = lb.quantize_int4(w, asym=True)
        Wl = W.shard(rank, world).cuda()
        bound = R.abs_bound
        fused = FusedColumnParallel(m, n)
        cp = ColumnParallel(m, n)
        for call in range(4):
            x = rng.standard_normal((m, k)).astype(np.float32)
            ref = R.gemm_w4a16_ref(x, W.qw, W.scales, W.zeros)
            b = bound(x, R.dequant_int4(W.qw, W.scales, W.zeros))
            xd = torch.from_numpy(x).cuda()
            y = fused(xd, Wl).cpu().numpy()
            err = np.max(np.abs(y - ref) / (b + 1e-30))
            errs.append(("fused", call, float(err)))
            y2 = cp.gather(K.gemm_w4a16(xd, Wl)).cpu().numpy()
            errs.append(("nccl", call, float(np.max(np.abs(y2 - ref) / (b + 1e-30)))))
        status = K.device_status(reset=True)
        fused.close()
        q.put((rank, errs, status))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, [("exception", -1, repr(e))], -1))
    finally:
        dist.destroy_process_group()


def _run(world, m, n, k):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, m, n, k, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for rank, errs, status in results:
        assert status == 0, (rank, errs)
        for kind, call, err in errs:
            assert kind != "exception", err
            assert err <= 1e-5, (rank, kind, call, err)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("m,n,k", [(1, 11008, 4096), (2, 301, 640)])
def test_two_gpu_fused_allgather(m, n, k):
    _run(2, m, n, k)


@pytest.mark.skipif(torch.cuda.device_count() < 3, reason="needs more than two GPUs")
@pytest.mark.parametrize("m,n,k", [(1, 11008, 4096), (2, 1001, 384)])
def test_all_gpus_fused_allgather(m, n, k):
    _run(min(torch.cuda.device_count(), 8), m, n, k)


def _gemm_rank_main(rank, world, port, q):
    """Every rank: the fused all-gather prefill GEMM of its shard, three calls
    per format: the assembled Y against the oracle (the prefill contract
    4e-3 * (|X| . |W|^T), the W4A8 bound), and bit-identical on every rank
    (each value is stored once by its owner into every rank's buffer)."""
    import torch.distributed as dist
    from datetime import timedelta

    import lowbit_b200 as lb
    from lowbit_b200 import kernels as K
    from lowbit_b200.sharding import FusedColumnParallelGemm
    from oracle import lbref as R
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    out = []
    try:
        m, n, k = 200, 1001, 512
        rng = np.random.default_rng(12)
        w = rng.standard_normal((n, k)).astype(np.float32)
        for fmt in ("w4a16", "mxfp4", "w4a8"):
            W = lb.quantize_mxfp4(w) if fmt == "mxfp4" else lb.quantize_int4(w, asym=(fmt == "w4a16"))
            Wl = W.shard(rank, world).cuda()
            fc = FusedColumnParallelGemm(fmt, m, n)
            for call in range(3):
                xh = rng.standard_normal((m, k)).astype(np.float32)
                y = fc(torch.from_numpy(xh).cuda(), Wl)
                torch.cuda.synchronize()
                everyone = [torch.empty_like(y) for _ in range(world)]
                dist.all_gather(everyone, y.contiguous())
                same = all(bool(torch.equal(everyone[0], e)) for e in everyone)
                yh = y.cpu().numpy()
                if fmt == "mxfp4":
                    err = R.assert_close(yh, R.gemm_mxfp4_ref(xh, W.qw, W.e8m0),
                                         R.abs_bound(xh, R.dequant_mxfp4(W.qw, W.e8m0)), 4e-3)
                elif fmt == "w4a16":
                    err = R.assert_close(yh, R.gemm_w4a16_ref(xh, W.qw, W.scales, W.zeros),
                                         R.abs_bound(xh, R.dequant_int4(W.qw, W.scales, W.zeros)), 4e-3)
                else:
                    xq, xs, asum = R.quant_act_int8_ref(xh, W.kp)
                    err = R.assert_close(yh, R.gemm_w4a8_ref(xq, xs, asum, W.qw, W.scales, None),
                                         R.w4a8_bound(xq, xs, asum, W.qw, W.scales, None), 1e-5)
                out.append((fmt, call, 0 if (same and err <= 1.0) else f"same={same} err={err}"))
            fc.close()
        out.append(("status", 0, K.device_status(reset=True)))
    except Exception as e:  # reported to the parent
        out.append(("exception", -1, repr(e)))
    finally:
        dist.destroy_process_group()
    q.put((rank, out))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_fused_allgather_gemm():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gemm_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for rank, out in results:
        for kind, call, v in out:
            assert kind != "exception", (rank, v)
            assert v == 0, (rank, kind, call, v)
