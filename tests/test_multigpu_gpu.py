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
