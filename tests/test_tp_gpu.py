"""Tensor-parallel decoder forward (column-parallel linears: the prompt's
GEMMs with an NCCL all-gather, the decode GEMVs with the all-gather fused
into the kernel; everything else replicated) on two GPUs, skipped with fewer: the
logits of a prompt and of greedy decode steps (CUDA-graph replays with the
collectives captured) equal the one-GPU model's within 1e-4 * max|logit|
(the shards change only the split points of a few kernels' sums), and the
greedy tokens are the same."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg():
    from lowbit_b200 import model as PM
    return PM.ModelConfig(vocab_size=1024, hidden_size=256, intermediate_size=512, num_layers=2, num_heads=4,
                          num_kv_heads=2, head_dim=64, rms_norm_eps=1e-6, rope_theta=1e6,
                          tie_word_embeddings=True, qkv_bias=True, max_position=128)


def _rank_main(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta

    from lowbit_b200 import model as PM
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    out = {}
    m = None
    try:
        cfg = _cfg()
        W = PM.random_weights(cfg, seed=0, scale=0.05)
        m = PM.Model(cfg, W, backend="w4a16", asym=True, group=dist.group.WORLD)
        prompt = np.random.default_rng(0).integers(0, cfg.vocab_size, 8)
        c = m.new_cache(32)
        out["prefill"] = m.forward(prompt, c)
        out["step"] = m.forward([int(np.argmax(out["prefill"]))], c)
        c.reset()
        out["tokens"] = m.generate(prompt, 6, cache=c)
        if rank == 0:
            ref = PM.Model(cfg, W, backend="w4a16", asym=True)
            rc = ref.new_cache(32)
            out["ref_prefill"] = ref.forward(prompt, rc)
            out["ref_step"] = ref.forward([int(np.argmax(out["ref_prefill"]))], rc)
            rc.reset()
            out["ref_tokens"] = ref.generate(prompt, 6, cache=rc)
        torch.cuda.synchronize()
    except Exception as e:  # reported to the parent
        out["error"] = repr(e)
    finally:
        if m is not None:
            m.release_graphs()
        dist.barrier()
        dist.destroy_process_group()
    q.put((rank, out))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp_model_equals_single_gpu():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        assert "error" not in res[r], res[r].get("error")
    r0 = res[0]
    for key in ("prefill", "step"):
        ref = r0["ref_" + key]
        for r in range(world):
            err = np.max(np.abs(res[r][key] - ref)) / np.max(np.abs(ref))
            assert err <= TOL, (key, r, err)
    for r in range(world):
        assert res[r]["tokens"] == r0["ref_tokens"]
