#!/usr/bin/env python
"""Headline benchmark: lowbit's W4A16 decode GEMM (M=1, N=11008, K=4096, int4 g128 asym)
on B200, reported as weight GB/s (BASELINE.json metric and configs[0]).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Our arm ("ours"):
  * a step = one fused dequant+GEMM of the step's weight matrix (11008x4096
    int4) against X [1, 4096] fp32; with N>1 ranks each rank owns N/P weight
    rows and the step ends with an NCCL all-gather of Y (column parallelism);
  * inputs resident in HBM; consecutive steps read different copies of the
    weights from a rotating pool larger than 2x L2 (every step streams its
    weights from HBM, like successive layers in decode);
  * the K timed steps are captured in one CUDA graph and replayed, bracketed
    by barrier + synchronize, timed with CUDA events, max over ranks;
  * `e2e`: the same step through the public API the reference's users call,
    lowbit_b200.gemm_w4a16(x_numpy, W): X in host memory, Y returned as a new
    host array, the call synchronous (lbc_gemm_w4a16_host underneath); with
    N>1 ranks the fused all-gather call with X copied from pinned host memory
    and Y read back to pinned host memory, synchronised per step.
Reference arm: lowbit's own CPU kernels (compiled from the reference's sources
into oracle/_ref) on all host cores, same config, same metric.

    python bench.py --workload model [--steps K] [--warmup W]
    python bench.py --workload gemm --fmt w4a16|w4a8|mxfp4 --m M --n N --k K
    python bench.py --workload sweep
    python bench.py --workload tune

GEMM workloads: one GEMM per step on seeded inputs (the BASELINE shape sweep
of configs[3] for `sweep`), weights quantized on the GPU, a CUDA graph of the
steps over rotating weight copies; each line carries its roofline (tensor or
HBM, whichever bounds the shape).

Model workload: the Qwen2-0.5B-shaped decoder (24
layers, hidden 896, 14/2 heads, SwiGLU 4864, vocabulary 151936, tied
embeddings), random weights (random_weights(seed 0, scale 0.02): N(0, 0.02)
linears, the generator's x20 embedding and 1 + r norms), every linear int4
g128 asym; a 128-token prompt then 128 greedy tokens at batch 1 and 16.
Reports decode and prefill tokens/s and max |delta logit| against the
reference's computation on the host (its C kernels for every linear, the
numpy glue restated in oracle/model_ref.py), whose decode is also timed as
the CPU baseline.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

M, N, K = 1, 11008, 4096
L2_BYTES = 126 * 2**20
METRIC = "M=1 decode weight GB/s (W4A16 int4-g128 asym, N=11008, K=4096)"
WORKLOAD = "W4A16 decode GEMM M=1 N=11008 K=4096, int4 g128 asym (BASELINE configs[0])"
PUBLISHED_GBPS = 22.4  # reference README: W4A16 M=1 N=11008 K=4096 cold, AVX-512, 4 threads
FALLBACK_HBM_GBS = 6650.0
REPLAYS = 10  # timed replays of the step graph; the line reports their median


def peaks() -> tuple[float, float, float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return (float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", 0)),
                "measured (MEASURED_PEAKS.json)")
    return FALLBACK_HBM_GBS, 1590.0, 1400.0, "fallback (profiling recipe)"


def inputs(m=M, n=N, k=K):
    w = np.random.default_rng(0).standard_normal((n, k)).astype(np.float32)
    x = np.random.default_rng(1).standard_normal((m, k)).astype(np.float32)
    return x, w


def _sha(*arrays) -> str:
    """SHA-256 of arrays as tests/golden/make_golden.py records them."""
    import hashlib
    h = hashlib.sha256()
    for a in arrays:
        if a is None:
            h.update(b"none")
        else:
            a = np.ascontiguousarray(a)
            h.update(str(a.dtype).encode() + str(a.shape).encode())
            h.update(a.tobytes())
    return h.hexdigest()


def reference_weights(name: str, fmt: str, w: np.ndarray, asym: bool = False):
    """Packed weights for the reference's CPU kernels, in the bytes lowbit's own
    quantizer produces: quantized here, then checked against the SHA-256 the
    reference recorded for the same BASELINE input (tests/golden/
    golden_meta.json, written by tests/golden/make_golden.py from lowbit).
    Returns (weights, note); the note says whether the digest matched."""
    from lowbit_b200 import quantize_int4, quantize_mxfp4
    W = quantize_mxfp4(w) if fmt == "mxfp4" else quantize_int4(w, asym=asym)
    arrays = (W.qw, W.e8m0) if fmt == "mxfp4" else (W.qw, W.scales, W.zeros)
    try:
        want = json.loads((ROOT / "tests" / "golden" / "golden_meta.json").read_text())["digests"][name + "_packed"]
    except (OSError, KeyError, ValueError):
        return W, "packed bytes not checked (no golden digest)"
    if _sha(*arrays) != want:
        raise SystemExit(f"packed {name} weights differ from the reference quantizer's (digest mismatch)")
    return W, "packed bytes equal to lowbit's quantizer output (SHA-256 of tests/golden/golden_meta.json)"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while the GPU is busy."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, pw, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [s.strip() for s in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
                pw.append(float(f[3]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None, "samples": len(sm), "reasons": sorted(reasons)}


# ---------------------------------------------------------------- reference arm
def run_reference(args) -> dict:
    from oracle import ref_lib
    if not ref_lib.available():
        return {"impl": "reference", "unavailable": "oracle/_ref/liblowbit_ref.so not built "
                "(make -C oracle ref needs the reference sources)"}
    x, w = inputs()
    W, wnote = reference_weights("w4a16_decode", "w4a16", w, asym=True)
    threads = os.cpu_count() or 1
    g = ref_lib.RefGemm("w4a16", x, W, threads)
    info = g.info()
    g.tune(budget_s=3.0)
    pool = _host_pool(W)
    for i in range(args.warmup):
        g.w = pool[i % len(pool)]
        g()
    ts = []
    for i in range(args.steps):
        g.w = pool[i % len(pool)]
        t0 = time.perf_counter()
        g()
        ts.append(time.perf_counter() - t0)
    total = sum(ts)
    gbps = W.nbytes / (total / args.steps) / 1e9
    sample = (f"lowbit lb_gemm_w4a16 ({info['isa']}, openmp={info['openmp']}) M=1 N=11008 K=4096, "
              f"{args.steps} calls, cold: {len(pool)} weight copies rotated, tuned params "
              f"mr={g.params.mr} nr={g.params.nr} nb={g.params.nb} kb={g.params.kb}; {wnote}")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbps, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / args.steps, 5), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": round(gbps / PUBLISHED_GBPS, 3), "dtype": "f32",
        "data": "synthetic: W~N(0,1) seed 0, X~N(0,1) seed 1 (BASELINE configs[0])",
        "config": {"workload": WORKLOAD, "M": M, "N": N, "K": K, "format": "w4a16",
                   "parallelism": f"OpenMP {threads} threads on the host", "l2": "cold (rotating copies)"},
        "cpu_baseline": {"value": round(gbps, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": round(gbps, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    return line


def _host_pool(W):
    """Host weight copies exceeding 2x a generous LLC (the reference's cold mode, lb/bench.py:169-178)."""
    from dataclasses import replace
    copies = int(max(2, min(24, np.ceil((512 << 20) / W.nbytes))))
    return [W] + [replace(W, qw=W.qw.copy(), scales=W.scales.copy(),
                          zeros=None if W.zeros is None else W.zeros.copy()) for _ in range(copies - 1)]


def cpu_baseline(budget_s: float = 10.0) -> dict:
    """The reference's CPU kernel on the host cores, bounded sample (rank 0, N=1)."""
    from oracle import ref_lib
    if not ref_lib.available():
        return {"value": None, "unit": "GB/s", "cores": 0, "kind": "reference",
                "sample": "unavailable: oracle/_ref/liblowbit_ref.so not built"}
    x, w = inputs()
    W, wnote = reference_weights("w4a16_decode", "w4a16", w, asym=True)
    threads = os.cpu_count() or 1
    g = ref_lib.RefGemm("w4a16", x, W, threads)
    info = g.info()
    g.tune(budget_s=3.0)
    pool = _host_pool(W)
    ts = []
    t_end = time.perf_counter() + budget_s
    i = 0
    while time.perf_counter() < t_end or len(ts) < 5:
        g.w = pool[i % len(pool)]
        t0 = time.perf_counter()
        g()
        ts.append(time.perf_counter() - t0)
        i += 1
    med = statistics.median(ts)
    return {"value": round(W.nbytes / med / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
            "sample": f"lowbit lb_gemm_w4a16 ({info['isa']}, openmp={info['openmp']}) M=1 N=11008 K=4096, "
                      f"median of {len(ts)} cold calls over {budget_s:.0f} s, tuned mr={g.params.mr} "
                      f"nr={g.params.nr} nb={g.params.nb} kb={g.params.kb}; {wnote}"}


# ---------------------------------------------------------------- our arm
def run_ours(args) -> dict | None:
    import torch
    import torch.distributed as dist

    import lowbit_b200 as lb
    from lowbit_b200 import kernels as Kn

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    x, w = inputs()
    W = lb.quantize_int4(w, asym=True)
    Wl = W.shard(rank, world)
    n_loc = Wl.n
    wbytes_total = W.nbytes
    wbytes_local = Wl.nbytes
    copies = int(max(2, min(64, np.ceil(2 * L2_BYTES / wbytes_local) + 1)))
    base = Wl.cuda(dev)
    pool = [base] + [lb.Int4Weights(base.qw.clone(), base.scales.clone(), base.zeros.clone(), base.k)
                     for _ in range(copies - 1)]
    pool_mb = copies * wbytes_local / 2**20
    xd = torch.from_numpy(x).to(dev)
    prep = Kn._Prepared(xd, W.kp, n_loc)
    cp = fused = None
    if world > 1:
        from lowbit_b200.sharding import ColumnParallel, FusedColumnParallel
        cp = ColumnParallel(M, N)              # NCCL all-gather (reported beside)
        fused = FusedColumnParallel(M, N)      # GEMV + NVLink peer-store gather in one kernel

    def gemv(i):
        Kn.gemm_w4a16(prep.x, pool[i % copies], _prep=prep)

    def step(i):
        if world > 1:
            fused(prep.x, pool[i % copies], _prep=prep)
        else:
            gemv(i)

    def step_nccl(i):
        gemv(i)
        cp.gather(prep.y)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    # correctness of the configuration being timed (oracle check, outside the timing)
    if rank == 0:
        from oracle import lbref as R
        gemv(0)
        torch.cuda.synchronize()
        ref = R.gemm_w4a16_ref(x, Wl.qw, Wl.scales, Wl.zeros)
        R.assert_close(prep.y.cpu().numpy(), ref, R.abs_bound(x, R.dequant_int4(Wl.qw, Wl.scales, Wl.zeros)), 1e-5)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    barrier()

    def capture(fn, steps):
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
                for i in range(steps):
                    fn(i)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        return g

    g_step = capture(step, args.steps)
    g_gemv = capture(gemv, args.steps) if world > 1 else g_step
    g_nccl = capture(step_nccl, args.steps) if world > 1 else None
    g_step.replay()  # graph warm-up (not timed)
    torch.cuda.synchronize()

    clocks = ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local])
                          if "CUDA_VISIBLE_DEVICES" in os.environ else local)
    clocks.start()
    # keep the GPU busy ~1.5 s so the sampler sees the clocks under this load
    t_soak = time.perf_counter() + 1.5
    while time.perf_counter() < t_soak:
        g_gemv.replay()
        torch.cuda.synchronize()

    def timed(graph, reps=REPLAYS):
        """Median over `reps` replays of a graph of args.steps steps, ms per step
        (CUDA events on the replaying stream, barrier + synchronize around each)."""
        out = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            barrier()
            torch.cuda.synchronize()
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize()
            out.append(e0.elapsed_time(e1) / args.steps)
        barrier()
        return statistics.median(out)

    ms_step_local = timed(g_step)
    # kernel-only duration (no collective) for the roofline
    ms_kernel_local = timed(g_gemv)
    ms_nccl_local = 0.0
    if g_nccl is not None:
        ms_nccl_local = timed(g_nccl)
    clk = clocks.stop()

    t = torch.tensor([ms_step_local, ms_kernel_local, ms_nccl_local], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step, ms_kernel, ms_nccl = float(t[0]), float(t[1]), float(t[2])

    # end to end through the public API, host buffers (pinned) in and out every step
    if fused is not None:
        fused.resync()
    xh = torch.from_numpy(x).pin_memory()
    yh = torch.empty((M, N), dtype=torch.float32).pin_memory()
    xdev = torch.empty((M, K), dtype=torch.float32, device=dev)
    e2e_steps = max(args.steps, 100)

    def e2e_step(i):
        if world == 1:
            lb.gemm_w4a16(x, pool[i % copies])
            return
        xdev.copy_(xh, non_blocking=True)
        y = fused(xdev, pool[i % copies])
        yh.copy_(y, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for i in range(copies + 5):     # every weight copy once: first calls capture their graphs
        e2e_step(i)
    barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        e2e_step(i)
    e2e_local = (time.perf_counter() - t0) / e2e_steps
    te = torch.tensor([e2e_local], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_s = float(te[0])

    del g_step, g_gemv, g_nccl
    status = Kn.device_status(reset=True)
    if fused is not None:
        fused.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return None

    hbm, _, _, peak_src = peaks()
    alg_bytes = wbytes_local + Kn_x_bytes(W.kp) + M * n_loc * 4
    achieved = alg_bytes / (ms_kernel * 1e-3) / 1e9
    value = wbytes_total / (ms_step * 1e-3) / 1e9
    traffic = _ncu_traffic("w4a16_decode") if world == 1 else None
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 6),
        "higher_is_better": True, "scaling": "strong",
        "vs_baseline": round(value / PUBLISHED_GBPS, 2), "dtype": "f32",
        "data": "synthetic: W~N(0,1) seed 0, X~N(0,1) seed 1, quantized by quantize_int4(asym=True)",
        "config": {"workload": WORKLOAD, "M": M, "N": N, "K": K, "format": "w4a16",
                   "parallelism": f"N-shard x{world}" + (" + all-gather of Y fused into the GEMV (NVLink peer stores)"
                                                        if world > 1 else ""),
                   "l2": f"inputs larger than L2: {copies} rotating weight copies ({pool_mb:.0f} MB/rank)",
                   "timing": f"K steps in one CUDA graph, CUDA events, median of {REPLAYS} replays, max over ranks"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": traffic, "peak_source": peak_src,
                     "alg_bytes_per_launch": alg_bytes, "kernel_us": round(ms_kernel * 1e3, 3)},
        "e2e": {"value": round(wbytes_total / e2e_s / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": M * K * 4, "d2h_bytes_per_step": M * N * 4,
                "us_per_step": round(e2e_s * 1e6, 2)},
        "gpu_launches": args.steps,
        "multi_gpu": ({"fused_step_us": round(ms_step * 1e3, 3), "gemv_only_us": round(ms_kernel * 1e3, 3),
                       "nccl_allgather_step_us": round(ms_nccl * 1e3, 3)} if world > 1 else None),
        "clocks": clk,
        "device_status": status,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(budget_s=args.cpu_seconds)
    if world == 1 and not args.no_secondary:
        line["secondary"] = secondary_lines(args)
    return line


# BASELINE configs[1] and [2] and the prefill kernel's target shape, reported
# beside the headline: (name, format, M, N, K, golden digest name, asym)
SECONDARY = (("w4a8_m16", "w4a8", 16, 4096, 4096, "w4a8_m16", False),
             ("mxfp4_m64", "mxfp4", 64, 11008, 4096, "mxfp4_m64", False),
             ("w4a16_prefill_m4096", "w4a16", 4096, 11008, 4096, "w4a16_decode", True))


def _median_time(fn, budget_s: float, min_calls: int = 3) -> tuple[float, int]:
    fn()
    ts = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(ts) < min_calls:
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts), len(ts)


def secondary_cpu(name: str, fmt: str, m: int, n: int, k: int, digest: str, asym: bool, budget_s: float) -> dict:
    """The reference's best CPU path for one secondary shape on all host cores,
    median over a bounded sample: W4A8 both the VNNI kernel (tuned) and the
    AMX kernel (when this host has AMX), reporting the faster; MXFP4 its
    AVX-512 kernel (tuned); W4A16 at 4096 tokens its AVX-512 kernel with the
    default tiles (one call takes seconds: no tuning)."""
    from lowbit_b200.formats import pack_amx
    from oracle import ref_lib
    if not ref_lib.available():
        return {"value": None, "unit": "us", "cores": 0, "kind": "reference",
                "sample": "unavailable: oracle/_ref/liblowbit_ref.so not built"}
    w = np.random.default_rng(0).standard_normal((n, k)).astype(np.float32)
    x = np.random.default_rng(1).standard_normal((m, k)).astype(np.float32)
    W, wnote = reference_weights(digest, fmt, w, asym=asym)
    threads = os.cpu_count() or 1
    g = ref_lib.RefGemm(fmt, x, W, threads)
    info = g.info()
    paths = {}
    if m <= 64:
        g.tune(budget_s=min(3.0, budget_s / 2))
    t, calls = _median_time(g, budget_s / 2)
    paths[f"{info['isa']}{'+vnni' if fmt == 'w4a8' and info['vnni'] else ''}"] = (t, calls)
    if fmt == "w4a8" and ref_lib.amx_available():
        ga = ref_lib.RefGemmAMX(x, pack_amx(W), threads)
        paths["amx"] = _median_time(ga, budget_s / 2)
    best = min(paths, key=lambda p: paths[p][0])
    return {"value": round(paths[best][0] * 1e6, 1), "unit": "us", "cores": threads, "kind": "reference",
            "path": best, "paths_us": {p: round(v[0] * 1e6, 1) for p, v in paths.items()},
            "sample": f"lowbit {fmt} M={m} N={n} K={k} on {threads} threads: median of "
                      f"{', '.join(f'{v[1]} {p} calls' for p, v in paths.items())} (openmp={info['openmp']}); {wnote}"}


def secondary_lines(args) -> dict:
    out = {}
    for name, fmt, m, n, k, digest, asym in SECONDARY:
        steps = max(5, min(args.steps, int(2e6 / (m * n * k / 1e6 + 50))))
        line = gemm_line(fmt, m, n, k, steps, 3)
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = secondary_cpu(name, fmt, m, n, k, digest, asym, args.cpu_seconds / 2)
        out[name] = line
    return out


def Kn_x_bytes(kp: int) -> int:
    return M * kp * 4


def _ncu_traffic(workload: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text()).get(workload)
    except (OSError, ValueError):
        return None


# ---------------------------------------------------------------- GEMM workloads (BASELINE configs[1..3])
SWEEP_M = (1, 16, 64, 512, 4096)
SWEEP_NK = ((4096, 4096), (11008, 4096), (4096, 11008), (14336, 4096))


_INPUTS: dict = {}


def _gemm_inputs(m: int, n: int, k: int):
    """BASELINE.json's inputs: W [N, K] ~ N(0, 1) from numpy default_rng(0), X
    [M, K] ~ N(0, 1) from default_rng(1), generated on the host (cached per
    shape within a run)."""
    if (n, k) not in _INPUTS:
        _INPUTS[(n, k)] = np.random.default_rng(0).standard_normal((n, k)).astype(np.float32)
    if (m, k) not in _INPUTS:
        _INPUTS[(m, k)] = np.random.default_rng(1).standard_normal((m, k)).astype(np.float32)
    return _INPUTS[(n, k)], _INPUTS[(m, k)]


def _gemm_check(fmt: str, x: np.ndarray, W, y, plan: dict) -> float:
    """One oracle check of a timed GEMM (outside the timing): up to 64 sampled
    weight rows x 256 sampled tokens in float64; tolerance 4e-3 * (|X| . |W|^T)
    on the bf16 prefill kernel (W4A16 / MXFP4 from 64 tokens), 1e-5 on the
    exact paths, the W4A8 magnitude bound for W4A8. Returns max err / limit."""
    from oracle import lbref as R
    rng = np.random.default_rng(3)
    m, n = y.shape
    rows = np.sort(rng.choice(n, min(n, 64), replace=False))
    toks = np.sort(rng.choice(m, min(m, 256), replace=False))
    import torch
    ti, ri = torch.as_tensor(toks, device=y.device), torch.as_tensor(rows, device=y.device)
    ys = y[ti][:, ri].cpu().numpy()
    xs = x[toks]
    qw = W.qw[ri].cpu().numpy()
    if fmt == "mxfp4":
        e = W.e8m0[ri].cpu().numpy()
        tol = 4e-3 if plan.get("kernel") == "prefill" else 1e-5
        return R.assert_close(ys, R.gemm_mxfp4_ref(xs, qw, e), R.abs_bound(xs, R.dequant_mxfp4(qw, e)), tol)
    sc = W.scales[ri].cpu().numpy()
    z = None if W.zeros is None else W.zeros[ri].cpu().numpy()
    if fmt == "w4a16":
        tol = 4e-3 if plan.get("kernel") == "prefill" else 1e-5
        return R.assert_close(ys, R.gemm_w4a16_ref(xs, qw, sc, z), R.abs_bound(xs, R.dequant_int4(qw, sc, z)), tol)
    xq, xsc, asum = R.quant_act_int8_ref(xs, W.kp)
    return R.assert_close(ys, R.gemm_w4a8_ref(xq, xsc, asum, qw, sc, z), R.w4a8_bound(xq, xsc, asum, qw, sc, z), 1e-5)


def _dist():
    """(world, rank, device) of this process: torch.distributed over NCCL when
    launched with WORLD_SIZE > 1 (one rank per GPU), else one GPU."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    return world, rank, dev


def gemm_line(fmt: str, m: int, n: int, k: int, steps: int, warmup: int, reps: int = 10) -> dict:
    """One GEMM of `fmt` (w4a16 asym / w4a8 sym / mxfp4) on BASELINE's seeded
    inputs (numpy seeds 0 / 1, quantized on the GPU bit-identically to the
    reference's quantizers), device-resident, checked once against the
    oracle, then timed as a CUDA graph of `steps` calls over rotating weight
    copies (inputs + copies larger than L2), CUDA events, median of `reps`
    replays.

    Under torch.distributed (WORLD_SIZE = P > 1, one rank per GPU) W is
    column-sharded as BASELINE configs[3] asks: rank p keeps rows
    shard_bounds(N, p, P) of the packed arrays, and a step is its slice's GEMM
    plus the all-gather that assembles Y [M, N] on every rank (W4A16 with one
    or two tokens: the GEMV with the all-gather fused in; otherwise NCCL
    all_gather). The step time is the max over ranks; the oracle check runs on
    rank 0's assembled Y; the GEMM alone and the gather's share are reported
    beside it."""
    import torch
    import torch.distributed as dist
    from lowbit_b200 import kernels as Kn
    from lowbit_b200.formats import shard_bounds
    from lowbit_b200.kernels import quantize_int4_cuda, quantize_mxfp4_cuda
    world, rank, dev = _dist()
    hbm, tf_burst, tf_sust, src = peaks()
    wh, xh = _gemm_inputs(m, n, k)
    w = torch.from_numpy(wh).to(dev)
    x = torch.from_numpy(xh).to(dev)
    Wfull = (quantize_mxfp4_cuda(w) if fmt == "mxfp4" else quantize_int4_cuda(w, asym=(fmt == "w4a16")))
    del w
    fields = ("qw", "scales", "zeros", "e8m0")
    from dataclasses import replace
    lo, hi = shard_bounds(n, rank, world)
    W = Wfull if world == 1 else replace(Wfull, **{f: getattr(Wfull, f)[lo:hi].contiguous() for f in fields
                                                   if getattr(Wfull, f, None) is not None})
    n_loc = hi - lo
    wbytes = int(sum(getattr(W, f).numel() * getattr(W, f).element_size() for f in fields
                     if getattr(W, f, None) is not None))
    copies = int(max(1, min(16, np.ceil(2 * L2_BYTES / max(1, wbytes + 4 * m * (k + n_loc))))))
    pool = [W] + [replace(W, **{f: getattr(W, f).clone() for f in fields
                                if getattr(W, f, None) is not None}) for _ in range(copies - 1)]
    fn = {"w4a16": Kn.gemm_w4a16, "w4a8": Kn.gemm_w4a8, "mxfp4": Kn.gemm_mxfp4}[fmt]
    prep = Kn._Prepared(x, W.kp, n_loc)
    plan = Kn.describe_plan(fmt, m, n_loc, W.kp)
    gather, fused = None, None
    if world > 1:
        from lowbit_b200.sharding import ColumnParallel, FusedColumnParallel, FusedColumnParallelGemm
        gather = ColumnParallel(m, n)          # NCCL all-gather (timed beside)
        if fmt == "w4a16" and m <= 2:
            fused = FusedColumnParallel(m, n)
        elif plan.get("kernel") == "prefill":
            fused = FusedColumnParallelGemm(fmt, m, n)

    def gemm(i):
        fn(x, pool[i % copies], _prep=prep)

    def step_nccl(i):
        gemm(i)
        return gather.gather(prep.y) if gather is not None else prep.y

    def step(i):
        if fused is not None:
            return fused(x, pool[i % copies], _prep=prep)
        return step_nccl(i)

    y = step(0)
    torch.cuda.synchronize()
    parity = _gemm_check(fmt, xh, Wfull, y, plan) if rank == 0 else 0.0
    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()

    def capture(f):
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
                for i in range(steps):
                    f(i)
        torch.cuda.current_stream().wait_stream(s)
        g.replay()
        torch.cuda.synchronize()
        return g

    def timed(g):
        ts = []
        for _ in range(reps):
            if world > 1:
                dist.barrier(device_ids=[dev.index])
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3 / steps)
        return statistics.median(ts)

    g_step = capture(step)
    t = [timed(g_step)]
    if world > 1:
        t.append(timed(capture(gemm)))
        t.append(timed(capture(step_nccl)) if fused is not None else t[0])
        tt = torch.tensor(t, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t = [float(v) for v in tt]
    us = t[0]
    flops = 2.0 * m * n * k
    wbytes_all = wbytes if world == 1 else int(sum(getattr(Wfull, f).numel() * getattr(Wfull, f).element_size()
                                                   for f in fields if getattr(Wfull, f, None) is not None))
    byts = wbytes_all + 4 * m * W.kp + 4 * m * n
    peak_t = tf_burst * (2 if fmt == "w4a8" else 1)
    # the roofline of one rank's kernel: its FLOPs / bytes over its GEMM time
    us_k = t[1] if world > 1 else us
    f_loc, b_loc = 2.0 * m * n_loc * k, wbytes + 4 * m * W.kp + 4 * m * n_loc
    tensor_bound = f_loc / (peak_t * 1e12) > b_loc / (hbm * 1e9)
    ach = f_loc / us_k / 1e6 if tensor_bound else b_loc / us_k / 1e3
    peak = peak_t if tensor_bound else hbm
    line = {"fmt": fmt, "M": m, "N": n, "K": k, "us": round(us, 3), "TFLOP/s": round(flops / us / 1e6, 2),
            "GB/s": round(byts / us / 1e3, 1), "kernel": plan.get("kernel", plan.get("path")),
            "parity": {"max_err_over_limit": round(parity, 4), "sample": "64 weight rows x 256 tokens, float64 oracle"
                       + (", rank 0's assembled Y" if world > 1 else "")},
            "roofline": {"bound": "tensor" if tensor_bound else "hbm", "achieved": round(ach, 2),
                         "peak": peak, "unit": "TFLOP/s" if tensor_bound else "GB/s", "frac": round(ach / peak, 4),
                         "peak_source": src + (" (int8: 2x the bf16 figure, assumed: not measured)"
                                               if tensor_bound and fmt == "w4a8" else "")},
            "weight_copies": copies}
    if world > 1:
        line["n_gpus"] = world
        line["gemm_only_us"] = round(t[1], 3)
        line["nccl_step_us"] = round(t[2], 3)
        line["gather"] = ("fused into the GEMV (NVLink tagged-word stores)" if fused is not None and m <= 2
                          else "fused into the prefill GEMM's store (NVLink peer stores per output tile)"
                          if fused is not None else "NCCL all_gather of the [M, N/P] slices")
        line["roofline"]["scope"] = "one rank's GEMM on its N/P rows"
        if fused is not None:
            fused.close()
    del g_step
    return line


def run_gemm(args) -> dict | None:
    line = gemm_line(args.fmt, args.m, args.n, args.k, args.steps, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if int(os.environ.get("RANK", "0")) != 0:
        return None
    return {"metric": f"{args.fmt} GEMM time (M={args.m}, N={args.n}, K={args.k})", "value": line["us"],
            "unit": "us", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": line["us"] / 1e3,
            "higher_is_better": False, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": {"w4a16": "f32 (bf16 from 64 tokens)", "w4a8": "int8/int32",
                      "mxfp4": "f32 (bf16 from 64 tokens)"}[args.fmt],
            "data": "synthetic: W ~ N(0,1) numpy default_rng(0), X ~ N(0,1) default_rng(1), quantized on the GPU "
                    "bit-identically to the reference's quantizers",
            "config": {"workload": f"{args.fmt} GEMM M={args.m} N={args.n} K={args.k}",
                       "parallelism": f"N-shard x{world} + all-gather of Y" if world > 1 else "1 GPU",
                       "timing": "CUDA graph of `steps` calls over rotating weight copies, CUDA events, "
                                 "median of 10 replays" + (", max over ranks" if world > 1 else "")},
            "detail": line}


def run_sweep(args) -> dict | None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rows = []
    for fmt in ("w4a16", "w4a8", "mxfp4"):
        for m in SWEEP_M:
            for n, k in SWEEP_NK:
                steps = max(3, min(args.steps, int(2e6 / (m * n * k / 1e6 + 50))))
                rows.append(gemm_line(fmt, m, n, k, steps, 3))
    if int(os.environ.get("RANK", "0")) != 0:
        return None
    return {"metric": f"GEMM shape sweep (BASELINE configs[3], {world} GPU{'s' if world > 1 else ''})",
            "n_gpus": world, "rows": rows}


def run_tune(args) -> dict:
    """The autotuner over BASELINE's sweep shapes at decode and small-batch token
    counts (M in 1, 2, 16, 64; all three formats; the four (N, K) of configs[3]):
    tuned vs default time per shape, and their median ratio (the reference
    reports its own tuner's median gain, README.md:377-379)."""
    import tempfile

    from lowbit_b200 import tune
    rows = []
    cache = Path(tempfile.mkdtemp()) / "tune.json"
    for fmt in ("w4a16", "w4a8", "mxfp4"):
        for m in (1, 2, 16, 64):
            for n, k in SWEEP_NK:
                e = tune.tune(fmt, m, n, k, reps=5, steps=20, path=cache)
                rows.append({"fmt": fmt, "M": m, "N": n, "K": k, "default_us": round(e["default_time_s"] * 1e6, 3),
                             "tuned_us": round(e["time_s"] * 1e6, 3), "params": e["params"],
                             "speedup": round(e["default_time_s"] / e["time_s"], 3), "n_configs": e["n_configs"]})
    sp = [r["speedup"] for r in rows]
    return {"metric": "autotuner speedup over default params (median over shapes)", "value": round(statistics.median(sp), 3),
            "unit": "x", "higher_is_better": True, "n_gpus": 1,
            "data": "the tuner's own problem: W ~ 0.02 N(0,1), X ~ N(0,1) (src/lowbit/tune.py:81-86)",
            "config": {"workload": "tune: 3 formats x M in {1,2,16,64} x 4 (N,K) of BASELINE configs[3]",
                       "timing": "CUDA graph of 20 calls over rotating weight copies, median of 5 replays"},
            "max_speedup": max(sp), "rows": rows}


# ---------------------------------------------------------------- model workload
MODEL_METRIC = "Qwen2-0.5B-shape greedy decode tokens/s (w4a16 int4-g128 asym, batch 1)"


def run_model(args) -> dict:
    import torch
    from lowbit_b200 import model as PM
    from oracle import model_ref as O
    from oracle import ref_lib

    # tensor parallelism under torch.distributed.run: every linear column
    # parallel over the ranks (one GPU each), the rest replicated
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    group = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
        group = dist.group.WORLD
    cfg = PM.qwen2_0_5b_config()
    t_build = time.perf_counter()
    W = PM.random_weights(cfg, seed=0, scale=0.02)
    m = PM.Model(cfg, W, backend="w4a16", asym=True, group=group)
    t_build = time.perf_counter() - t_build
    V, P, NEW = cfg.vocab_size, 128, 128
    prompt = np.random.default_rng(0).integers(0, V, P)
    packed = None
    if world == 1:
        # the packed-weight file: write the quantized model, read it back
        # (no quantization), check the logits are the same
        import tempfile
        with tempfile.TemporaryDirectory() as td:
            pk = Path(td) / "model.safetensors"
            t0 = time.perf_counter()
            PM.save_packed(m, pk)
            t_save = time.perf_counter() - t0
            t0 = time.perf_counter()
            m_pk = PM.load_packed(pk)
            torch.cuda.synchronize()
            t_load = time.perf_counter() - t0
            packed = {"bytes": pk.stat().st_size, "save_s": round(t_save, 2), "load_s": round(t_load, 2),
                      "logits_identical": bool(np.array_equal(m_pk.forward(prompt[:16], logits="all"),
                                                              m.forward(prompt[:16], logits="all")))}
            del m_pk
    prompts16 = np.random.default_rng(1).integers(0, V, (16, P))
    c1, c16 = m.new_cache(P + NEW), m.new_cache(P + NEW, batch=16)
    for _ in range(args.warmup):  # builds plans, workspaces and the decode graphs
        c1.reset()
        m.generate(prompt, 4, cache=c1)
        c16.reset()
        m.generate_batch(prompts16, 4, cache=c16)
    clk = ClockSampler(torch.cuda.current_device())
    clk.start()
    runs1, runs16, toks = [], [], None
    for _ in range(args.steps):
        c1.reset()
        t = {}
        toks = m.generate(prompt, NEW, cache=c1, timings=t)
        runs1.append(t)
        c16.reset()
        t = {}
        m.generate_batch(prompts16, NEW, cache=c16, timings=t)
        runs16.append(t)
    clocks = clk.stop()
    # one decode step of each batch inside an NVTX range, for profilers
    # (ncu --nvtx --nvtx-include "model_decode_step_b1/" ...); untimed
    for cache, rng_name in ((c1, "model_decode_step_b1"), (c16, "model_decode_step_b16")):
        g, _ = m._decode_graph(cache)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push(rng_name)
        g.replay()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    del g  # a graph holding NCCL calls must be gone before the process group

    # per-section device time (Model.prof, the reference's linear / attention /
    # lm_head / other split) of one profiled generation, untimed: the prompt's
    # prefill, then the graph-replayed decode steps (event-record nodes at the
    # section boundaries: a profiled step is slower than the timed ones)
    m.prof.enabled = True
    m.prof.reset()
    c1.reset()
    tp = {}
    m.generate(prompt, NEW, cache=c1, timings=tp)
    m.prof.enabled = False
    m.prof.reset()
    steps_d = NEW - 1
    profile = {"unit": "us",
               "prefill_128": {k: round(v * 1e6, 1) for k, v in sorted(tp["prof_prefill"].items())},
               "decode_per_step": {k: round(v * 1e6 / steps_d, 2) for k, v in sorted(tp["prof_decode"].items())},
               "decode_step_wall_us_profiled": round(tp["decode_s"] * 1e6 / steps_d, 2),
               "note": "device time from each section boundary to the next (CUDA events); fused decode GEMVs "
                       "(input norm, SiLU*up inside) count as linear"}

    def med(runs, key):
        return statistics.median(r[key] for r in runs)

    d1, d16, p1, p16 = med(runs1, "decode_s"), med(runs16, "decode_s"), med(runs1, "prefill_s"), med(runs16, "prefill_s")
    if world > 1:  # the slowest rank's times
        tt = torch.tensor([d1, d16, p1, p16], dtype=torch.float64, device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        d1, d16, p1, p16 = (float(v) for v in tt)
    dec1 = (NEW - 1) / d1
    dec16 = 16 * (NEW - 1) / d16
    line = {"metric": MODEL_METRIC, "value": round(dec1, 1), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 / dec1, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: random_weights(seed 0, scale 0.02), prompt default_rng(0).integers(0, 151936, 128)",
            "config": {"workload": "Qwen2-0.5B-shaped decoder, w4a16 asym linears, prompt 128, 128 greedy tokens "
                                   "(BASELINE configs[4])", "layers": cfg.num_layers, "hidden": cfg.hidden_size,
                       "vocab": V, "prompt": P, "new_tokens": NEW,
                       "parallelism": (f"tensor parallel x{world}: column-parallel linears (decode GEMVs with the "
                                       "all-gather fused in, NCCL all-gather otherwise), norms / RoPE / attention "
                                       "replicated" if world > 1 else "one GPU"),
                       "timing": "decode: 127 CUDA-graph replays of a whole decode step (host clock around "
                                 "synchronised loops, max over ranks); a step = one token for every sequence "
                                 "of the batch"},
            "prefill_tok_s": round(P / p1, 1),
            "batch16": {"decode_tok_s": round(dec16, 1), "prefill_tok_s": round(16 * P / p16, 1),
                        "ms_per_step": round(1e3 * d16 / (NEW - 1), 4)},
            "build_s": round(t_build, 1), "packed_file": packed, "clocks": clocks, "profile_b1": profile}
    # parity and CPU baseline: the reference's computation on the host (its C
    # kernels for every linear), prefill then 3 teacher-forced decode steps
    if ref_lib.available() and not args.no_cpu_baseline and world == 1:
        threads = os.cpu_count() or 1
        ocfg = O.Cfg(**{k: getattr(cfg, k) for k in O.Cfg.__dataclass_fields__})
        lin = {}
        for key, (w, b) in O.concat_weights(ocfg, W).items():
            lin[key] = O.lin_ref_c("w4a16", (m.lm_head if key == "lm_head" else
                                             getattr(m.layers[key[0]], key[1])).wq, b, threads)
        ref = O.Model(ocfg, W, lin)
        oc = O.new_cache(ocfg, P + 8)
        c1.reset()
        feed = [int(t) for t in toks[:3]]
        d_abs, scale = 0.0, 0.0
        t0 = time.perf_counter()
        lo = ref.forward(prompt, oc)
        t_pre = time.perf_counter() - t0
        lg = m.forward(prompt, c1)
        d_abs, scale = max(d_abs, float(np.abs(lg - lo).max())), max(scale, float(np.abs(lo).max()))
        td = []
        for tk in feed:
            t0 = time.perf_counter()
            lo = ref.forward([tk], oc)
            td.append(time.perf_counter() - t0)
            lg = m.forward([tk], c1)
            d_abs, scale = max(d_abs, float(np.abs(lg - lo).max())), max(scale, float(np.abs(lo).max()))
        cpu_dec = 1.0 / statistics.median(td)
        line["max_abs_dlogit"] = round(d_abs, 6)
        line["rel_dlogit"] = float(f"{d_abs / scale:.3e}")
        line["parity_note"] = ("logits of the 128-token prefill (bf16 prefill GEMMs, 4e-3 contract) and 3 decode "
                               "steps (exact fp32 decode GEMMs) vs the reference's C kernels + numpy glue")
        line["cpu_baseline"] = {"value": round(cpu_dec, 2), "unit": "tok/s", "cores": threads, "kind": "reference",
                                "sample": f"3 decode steps after a 128-token prefill ({t_pre:.1f} s): lowbit "
                                          "lb_gemm_w4a16 for every linear (oracle/_ref) with the numpy glue, "
                                          "default tiles"}
    else:
        why = ("skipped (--no-cpu-baseline)" if args.no_cpu_baseline else
               "the one-GPU run reports it" if world > 1 else "unavailable: oracle/_ref/liblowbit_ref.so not built")
        line["cpu_baseline"] = {"value": None, "unit": "tok/s", "cores": 0, "kind": "reference", "sample": why}
    if world > 1:
        import gc
        m.release_graphs()  # they hold NCCL calls
        gc.collect()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
        if rank != 0:
            return None
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="omit the secondary block (configs[1], configs[2], M=4096 prefill)")
    ap.add_argument("--workload", choices=["decode", "model", "gemm", "sweep", "tune"], default="decode")
    ap.add_argument("--fmt", choices=["w4a16", "w4a8", "mxfp4"], default="w4a16")
    # --M/--N/--K are the spellings torch.distributed.run passes through
    # (it takes --m, --n, --k for abbreviations of its own options)
    ap.add_argument("--m", "--M", dest="m", type=int, default=4096)
    ap.add_argument("--n", "--N", dest="n", type=int, default=11008)
    ap.add_argument("--k", "--K", dest="k", type=int, default=4096)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload in ("gemm", "sweep"):
        line = run_gemm(args) if args.workload == "gemm" else run_sweep(args)
        if line is not None:
            print(json.dumps(line), flush=True)
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()
        return
    if args.workload == "tune":
        print(json.dumps(run_tune(args)), flush=True)
        return
    if args.workload == "model":
        if args.steps > 50:
            args.steps = 3  # a step is a whole 128-token generation here
        line = run_model(args)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return
        print(json.dumps(run_reference(args)), flush=True)
        return
    line = run_ours(args)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
