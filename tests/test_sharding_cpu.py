"""N-sharded (column-parallel) GEMM host logic on two gloo ranks (CPU): every
rank computes its weight-row slice (here with the oracle, the GPU kernels need
a device), the all-gather assembles Y, and the result equals the unsharded
oracle bit for bit; shards of unequal height (N % world != 0) included."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import lowbit_b200 as lb
from lowbit_b200.sharding import ColumnParallel, padded_rows
from oracle import lbref as R


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, m, n, k, kind, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        rng = np.random.default_rng(5)
        x = rng.standard_normal((m, k)).astype(np.float32)
        w = rng.standard_normal((n, k)).astype(np.float32)
        if kind == "mxfp4":
            W = lb.quantize_mxfp4(w)
            Wl = W.shard(rank, world)
            y_local = R.gemm_mxfp4_ref(x, Wl.qw, Wl.e8m0).astype(np.float32)
            ref = R.gemm_mxfp4_ref(x, W.qw, W.e8m0).astype(np.float32)
        else:
            W = lb.quantize_int4(w, asym=True)
            Wl = W.shard(rank, world)
            y_local = R.gemm_w4a16_ref(x, Wl.qw, Wl.scales, Wl.zeros).astype(np.float32)
            ref = R.gemm_w4a16_ref(x, W.qw, W.scales, W.zeros).astype(np.float32)
        cp = ColumnParallel(m, n)
        y = cp.gather(torch.from_numpy(y_local)).numpy()
        q.put((rank, bool(np.array_equal(y, ref)), y.shape))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("m,n,k,kind", [(1, 64, 256, "w4a16"), (3, 37, 384, "w4a16"), (2, 33, 96, "mxfp4")])
def test_two_rank_gather_matches_unsharded(m, n, k, kind):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, m, n, k, kind, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, equal, shape in results:
        assert shape == (m, n)
        assert equal, f"rank {rank}: gathered Y differs from the unsharded oracle"


def test_padded_rows():
    assert padded_rows(11008, 8) == 1376
    assert padded_rows(37, 2) == 19
    assert [lb.formats.shard_bounds(37, r, 2) for r in range(2)] == [(0, 19), (19, 37)]


def _tp_shard_rank(rank, world, port, q):
    import os

    import numpy as np
    import torch
    import torch.distributed as dist

    from lowbit_b200.model import tp_shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = np.random.default_rng(5).standard_normal((151936 // 64, 24)).astype(np.float32)
        part = torch.from_numpy(tp_shard(w, rank, world))
        parts = [None] * world
        dist.all_gather_object(parts, part)
        q.put((rank, bool(np.array_equal(torch.cat(parts).numpy(), w))))
    finally:
        dist.destroy_process_group()


def test_tp_shards_reassemble_the_weight_gloo():
    """Tensor-parallel model: every rank's column-parallel shard of a weight
    (tp_shard) concatenated in rank order is the whole weight (gloo, world 2)."""
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_shard_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res[0] and res[1]
