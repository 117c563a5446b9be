"""Benchmark of the B200 k-quant path (BASELINE.json metric: weight GB/s and % of HBM peak for the
Q4_K / Q6_K matvec; decode tokens/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl kq|reference]

One JSON line on rank 0. Workloads:

  stack70b   configs[4]  Llama-70B-shaped decode matvec stack, rows sharded over the N GPUs
                         (default): a step is one decode token
  stack7b    configs[2]  Llama-7B-shaped decode matvec stack, a step is one token
  q6k_head   configs[1]  Q6_K 32000 x 4096, batch 1: a step is one matvec
  q4k        configs[0]  Q4_K 4096 x 4096, batch 1
  sweep      configs[3]  Q4_K 14336 x 4096, batch --batch (1..64)
  q5k                    Q5_K 14336 x 4096, batch 1 (the next k-quant type)

Stacks: one token is one replay of a CUDA graph of the token's launches; by default chains of
the warp-MMA kernel (per layer one launch for q|k|v, o and gate|up, one for down; the head),
whose outputs, with N GPUs, are pushed into every rank's full vectors inside those launches
(`--exchange nccl` times one launch per projection with NCCL all-gathers instead). `scaling` is
"strong" (the model is fixed, its rows split over the N GPUs). Before timing, a 2-layer copy of
the stack, sharded and exchanged the same way, is checked on every rank against the unsharded
CPU reference ("parity" in the line); rank 0 at N=1 also times the Q6_K head matvec alone
(configs[1], "matvec_q6k_head") and the CPU baseline.

Single matvecs: a step is one launch over one weight matrix, its weights rotating over enough
copies that their total exceeds twice the 126 MB L2, so every step streams from DRAM. With N GPUs
every rank runs its own replica ("replicas only": `scaling` "weak", `value` sums the ranks'
bytes over the slowest rank's time).

`--impl reference` times the CPU implementation of the path (the oracle's AVX2 C port, all host
threads) on the same workload; under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024
# Host threads, read before torch / CUDA initialise (they may narrow the affinity mask).
try:
    HOST_THREADS = len(os.sched_getaffinity(0))
except AttributeError:  # pragma: no cover
    HOST_THREADS = os.cpu_count() or 1
FALLBACK_HBM_GBS = 6650.0

WORKLOADS = {
    "q6k_head": dict(qtype=6, rows=32000, k=4096, batch=1, source="BASELINE configs[1]"),
    "q4k": dict(qtype=4, rows=4096, k=4096, batch=1, source="BASELINE configs[0]"),
    "sweep": dict(qtype=4, rows=14336, k=4096, batch=None, source="BASELINE configs[3]"),
    "q5k": dict(qtype=5, rows=14336, k=4096, batch=1, source="next k-quant type, sweep shape"),
}


STACKS = {"stack7b": "7b", "stack70b": "70b"}


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default 200 tokens for stacks, 20000 launches for a matvec)")
    ap.add_argument("--warmup", type=int, default=None, help="untimed steps (default 5 / 200)")
    ap.add_argument("--workload", default="stack70b", choices=sorted(WORKLOADS) + sorted(STACKS))
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--path", default="auto", choices=["auto", "tc", "cc", "wm"],
                    help="tensor cores (tcgen05), CUDA cores, warp-level MMA, or the library's choice")
    ap.add_argument("--extra-flags", type=lambda v: int(v, 0), default=0,
                    help="more descriptor flag bits OR-ed into every timed launch (A/B tests)")
    ap.add_argument("--impl", default="kq", choices=["kq", "reference"])
    ap.add_argument("--exchange", default="auto", choices=["auto", "nccl", "push", "chain"],
                    help="stacks: NCCL all-gathers after one launch per projection, the warp-MMA "
                         "matvec's own push to peer memory (one launch per projection), or chains of "
                         "the warp-MMA kernel (up to three projections a launch, outputs pushed to "
                         "peer memory at N > 1); auto (default): one launch per projection, with "
                         "the push at N > 1")
    ap.add_argument("--e2e-steps", type=int, default=2000, help="steps of the end-to-end leg")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU-baseline time budget")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=None,
                    help="stacks: run only the first N layers (smaller cases for profiling; the "
                         "line's config says so); default: the config's layer count")
    args = ap.parse_args(argv)
    stack = args.workload in STACKS
    if args.steps is None:
        args.steps = 200 if stack else 20000
    if args.warmup is None:
        args.warmup = 5 if stack else 200
    if args.exchange == "auto":
        # measured on B200 (70B stack): one launch per projection with programmatic dependent
        # launch beats chains on one GPU (67.8 vs 63.0 tokens/s); the push beats NCCL on two
        args.exchange = "push" if int(os.environ.get("WORLD_SIZE", "1")) > 1 else "nccl"
    return args


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            v = float(json.load(f)["hbm_gbs"])
        return v, "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(name: str, unit: str = "launch"):
    """DRAM bytes (read + write) per launch of the dominant kernel (per token for a stack) from
    the committed ncu summary for this workload, or None."""
    path = os.path.join(ROOT, "profiles", f"{name}.md")
    try:
        text = open(path).read()
    except OSError:
        return None
    m = re.search(r"traffic_bytes_per_" + unit + r":\s*([0-9]+)", text)
    return int(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="kq_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.15)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons,
                "samples": len(rows)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def matvec_launches(qtype, batch, path):
    """Kernels one matvec call launches: the tensor-core path (Q4_K/Q5_K above batch 8, or when
    asked) runs an X pre-pass before the matmul; the other paths are one kernel."""
    tc = path == "tc" or (path == "auto" and batch > 8 and qtype in (4, 5))
    return 2 if tc else 1


def workload_shape(args):
    w = dict(WORKLOADS[args.workload])
    if w["batch"] is None:
        w["batch"] = args.batch
    return w


def cpu_model():
    """The host CPU's model name (/proc/cpuinfo), or the platform's processor string."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def cpu_matvec_timing(qtype, Wh, x, rows, K, seconds, threads):
    """Repeats the CPU matvec on a row sample until `seconds` pass; returns (GB/s, sample)."""
    import oracle

    rb = (K // 256) * oracle.block_bytes(qtype)
    t0 = time.perf_counter()
    oracle.matvec_cpu(qtype, Wh, x, rows, K, threads)
    one = time.perf_counter() - t0
    # sample rows so that one call is ~ seconds / 8, at least 256 rows
    sample_rows = max(256, min(rows, int(rows * (seconds / 8) / max(one, 1e-6))))
    reps = 0
    t0 = time.perf_counter()
    while True:
        oracle.matvec_cpu(qtype, Wh[: sample_rows * rb], x, sample_rows, K, threads)
        reps += 1
        if time.perf_counter() - t0 >= seconds:
            break
    el = time.perf_counter() - t0
    gbs = sample_rows * rb * reps / el / 1e9
    sample = f"{reps} x {sample_rows} rows of the {rows}x{K} Q{qtype}_K matrix, batch {x.shape[0]}, {el:.1f} s"
    return gbs, sample


def run_reference(args):
    """The reference arm: the CPU implementation of the path (the oracle's AVX2 port)."""
    import numpy as np

    import oracle

    world, rank, _ = dist_setup()
    if rank != 0:
        return 0
    w = workload_shape(args)
    qtype, rows, K, batch = w["qtype"], w["rows"], w["k"], w["batch"]
    threads = HOST_THREADS
    rb = (K // 256) * oracle.block_bytes(qtype)
    Wh = oracle.fill(qtype, oracle.stream_key(2026, qtype), 0, rows * K // 256)
    x = np.random.default_rng(0).standard_normal((batch, K), dtype=np.float32)
    t0 = time.perf_counter()
    oracle.matvec_cpu(qtype, Wh, x, rows, K, threads)
    one = time.perf_counter() - t0
    total_budget = 90.0
    per_step = total_budget / max(1, args.steps + args.warmup)
    sample_rows = max(64, min(rows, int(rows * per_step / max(one, 1e-6))))
    for _ in range(args.warmup):
        oracle.matvec_cpu(qtype, Wh[: sample_rows * rb], x, sample_rows, K, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.matvec_cpu(qtype, Wh[: sample_rows * rb], x, sample_rows, K, threads)
    el = time.perf_counter() - t0
    gbs = sample_rows * rb * args.steps / el / 1e9
    sample = (f"each step {sample_rows} of {rows} rows of the Q{qtype}_K {rows}x{K} matrix, "
              f"batch {batch}")
    line = {
        "impl": "reference", "metric": "weight GB/s", "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_of(args, w, world),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample, "cpu_model": cpu_model()},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
        "note": "fxeqxmulfx/kernite has no k-quant path and no Rust toolchain here; the CPU "
                "implementation timed is this repo's AVX2+FMA C port (oracle/kq_cpu.c)",
    }
    print(json.dumps(line), flush=True)
    return 0


def rotation_copies(wbytes: int) -> int:
    """Weight copies a single-matvec run rotates over: their total exceeds twice the L2."""
    return max(2, -(-2 * L2_BYTES // wbytes) + 1)


def config_of(args, w, world):
    """The workload description of a single-matvec run, the same in both arms."""
    import oracle

    wbytes = w["rows"] * (w["k"] // 256) * oracle.block_bytes(w["qtype"])
    copies = rotation_copies(wbytes)
    return {
        "workload": f"{args.workload}: Q{w['qtype']}_K {w['rows']}x{w['k']} batch {w['batch']} ({w['source']})",
        "qtype": f"Q{w['qtype']}_K", "rows": w["rows"], "k": w["k"], "batch": w["batch"],
        "path": args.path,
        "parallelism": f"replicas x{world}" if world > 1 else "single",
        "l2": f"weights rotate over {copies} copies ({copies * wbytes / 1e6:.0f} MB > 2x L2)",
    }


def main(argv=None):
    args = parse_args(argv)
    if args.workload in STACKS:
        return run_stack(args)
    if args.impl == "reference":
        return run_reference(args)

    import numpy as np
    import torch

    import kernite_b200 as kb

    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    kernels = kb.Kernels.load(local)
    w = workload_shape(args)
    qtype, rows, K, batch = w["qtype"], w["rows"], w["k"], w["batch"]
    wbytes = kb.matrix_bytes(qtype, rows, K)
    algo_bytes = wbytes + batch * K * 4 + batch * rows * 4
    copies = rotation_copies(wbytes)
    nblk = rows * K // 256
    Ws = []
    for c in range(copies):
        W = torch.empty(wbytes, dtype=torch.uint8, device="cuda")
        kernels.fill(qtype, W, 0, nblk, kb.stream_key(2026 + c, qtype))
        Ws.append(W)
    rng = np.random.default_rng(rank)
    x = torch.from_numpy(rng.standard_normal((batch, K), dtype=np.float32)).cuda()
    y = torch.empty(batch, rows, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()

    path_flag = {"auto": 0, "tc": kb.FLAG_TENSOR_CORES, "cc": kb.FLAG_CUDA_CORES,
                 "wm": kb.FLAG_WARP_MMA}[args.path]

    def step(i, s):
        kernels.matvec(qtype, y, Ws[i % copies], x, rows, K, batch,
                       flags=kb.FLAG_WEIGHTS_STATIC | path_flag | args.extra_flags, stream=s)

    # The timed loop replays CUDA graphs of launches (captured with their programmatic-
    # dependent-launch edges): a graph of G steps, G a multiple of the weight copies so that
    # consecutive replays keep rotating, and one of the remaining K mod G steps.
    G = copies * max(1, 64 // copies) if copies < 64 else copies

    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n):
                step(i, stream)
        return g

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i, stream)
    torch.cuda.synchronize()
    kernels.device_error()
    g_full = capture(G) if args.steps >= G else None
    rem = args.steps % G if args.steps >= G else args.steps
    g_rem = capture(rem) if rem else None
    with torch.cuda.stream(stream):  # graph warm-up (not timed)
        (g_full or g_rem).replay()
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    sampler.start()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(args.steps // G if g_full else 0):
            g_full.replay()
        if g_rem:
            g_rem.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1)
    kernels.device_error()
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    value = world * wbytes * args.steps / (ms / 1e3) / 1e9
    del g_full, g_rem

    # end to end through the public API: pinned x in, y out, every step
    e2e = run_e2e(kernels, kb, torch, qtype, Ws, rows, K, batch, args.e2e_steps, dist)

    peak, peak_kind = measured_peak()
    achieved = algo_bytes / (ms_step / 1e3) / 1e9
    if args.workload == "sweep" and matvec_launches(qtype, batch, args.path) == 2:
        traffic = profiled_traffic("sweep_tc", f"launch_b{batch}")  # the tensor-core kernel
    else:
        traffic = profiled_traffic(args.workload if args.workload != "sweep" else f"sweep_b{batch}")
    roofline = {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                else "fallback 6650 GB/s", "algorithmic_bytes_per_launch": algo_bytes}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle

        Wh = Ws[0].cpu().numpy()
        xh = x.cpu().numpy()
        threads = HOST_THREADS
        # sanity: the CPU port computes the same y as the GPU on this matrix
        kernels.matvec(qtype, y, Ws[0], x, rows, K, batch)
        torch.cuda.synchronize()
        y_cpu = oracle.matvec_cpu(qtype, Wh, xh, rows, K, threads)
        y_ref, bound = oracle.matvec_ref(qtype, Wh, xh, K, 0, min(rows, 256))
        ok = bool((abs(y_cpu[:, :256] - y_ref) <= 1e-3 * bound).all()
                  and (abs(y.cpu().numpy()[:, :256] - y_ref) <= 1e-3 * bound).all())
        gbs, sample = cpu_matvec_timing(qtype, Wh, xh, rows, K, args.cpu_seconds, threads)
        gbs1, sample1 = cpu_matvec_timing(qtype, Wh, xh, rows, K, args.cpu_seconds / 4, 1)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": sample, "checked_against_oracle": ok,
               "single_thread": {"value": round(gbs1, 3), "sample": sample1},
               "cpu_model": cpu_model()}

    if rank == 0:
        cfg = config_of(args, w, world)
        line = {
            "metric": "weight GB/s", "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 6),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": cfg,
            "hbm_frac": round(achieved / peak, 4),
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": args.steps * matvec_launches(qtype, batch, args.path), "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    kernels.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_e2e(kernels, kb, torch, qtype, Ws, rows, K, batch, steps, dist):
    """The same matvec through kernite_b200's public API with host buffers (kq_matvec_host): each
    step copies its x from pinned host memory, launches, reads y back into pinned host memory
    and waits for it."""
    import numpy as np

    copies = len(Ws)
    xh = torch.from_numpy(np.random.default_rng(1).standard_normal((batch, K), dtype=np.float32)).pin_memory()
    yh = torch.empty(batch, rows).pin_memory()
    s = torch.cuda.Stream()

    def step(i):
        # one library call: x to the device, the matvec, y back (kq_matvec_host), then the wait
        kernels.matvec_host(qtype, yh, Ws[i % copies], xh, rows, K, batch, stream=s)
        s.synchronize()

    for i in range(20):
        step(i)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for i in range(steps):
        step(i)
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    world = dist.get_world_size() if dist else 1
    wbytes = kb.matrix_bytes(qtype, rows, K)
    return {"value": round(world * wbytes * steps / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": batch * K * 4, "d2h_bytes_per_step": batch * rows * 4,
            "steps": steps, "ms_per_step": round(ms / steps, 5)}


def _init_dist(torch, world, local):
    if world == 1:
        return None
    import datetime

    import torch.distributed as dist

    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                            device_id=torch.device("cuda", local))
    return dist


def stack_cpu_seconds_per_token(cfg, threads, also_single=False, layers_timed=3):
    """CPU baseline for a stack: the matvecs of the first `layers_timed` layers (each matrix its
    own weights, timed once after a warm-up call) and the head, with the AVX2 port, the layers
    scaled to the stack's layer count. Returns (seconds per token, sample), and with
    `also_single` the seconds per token on one thread as well (same matrices, timed after)."""
    import numpy as np

    import oracle

    from kernite_b200 import stack as st

    rng = np.random.default_rng(0)
    counts = [threads, 1] if also_single else [threads]
    t = {n: 0.0 for n in counts}
    nl = max(1, min(layers_timed, cfg.layers))

    def timed(qtype, W, x, rows, k, scale):
        for n in counts:
            if n == threads:
                oracle.matvec_cpu(qtype, W, x, rows, k, n)  # warm
            t0 = time.perf_counter()
            oracle.matvec_cpu(qtype, W, x, rows, k, n)
            t[n] += scale * (time.perf_counter() - t0)

    for layer in range(nl):
        for name, qtype, rows, k in cfg.matrices():
            W = oracle.fill(qtype, oracle.stream_key(cfg.seed, cfg.tensor_id(layer, name)), 0, rows * k // st.QK)
            timed(qtype, W, rng.standard_normal((1, k), dtype=np.float32), rows, k, cfg.layers / nl)
            del W
    H = oracle.fill(6, oracle.stream_key(cfg.seed, cfg.tensor_id(cfg.layers, "head")), 0,
                    cfg.vocab * cfg.hidden // st.QK)
    timed(6, H, rng.standard_normal((1, cfg.hidden), dtype=np.float32), cfg.vocab, cfg.hidden, 1)
    sample = (f"layers 0..{nl - 1} (4 matvecs each, own weights) and the head, each timed once after "
              f"a warm-up call; layers scaled to {cfg.layers}")
    if also_single:
        return t[threads], sample, t[1]
    return t[threads], sample


def stack_config(args, cfg, world, chain):
    """The workload description of a stack run, the same in both arms."""
    return {"workload": f"{args.workload}: {cfg.name}", "layers": cfg.layers, "hidden": cfg.hidden,
            "ffn": cfg.ffn, "kv": cfg.kv, "vocab": cfg.vocab, "batch": 1,
            "parallelism": (f"rows sharded x{world}, " + (
                "chains, push to peer memory" if chain else "push to peer memory"
                if args.exchange == "push" else "NCCL all-gather")) if world > 1 else
            ("single, chains" if chain else "single"),
            "graph": True,
            "l2": f"{cfg.weight_bytes() / world / 1e9:.1f} GB of weights per GPU per token > L2"}


def stack_parity(cfg, kernels, rank, world, chain, push, dist):
    """On-run parity of the stack exactly as timed (same sharding, exchange and kernels) on its
    first two layers: every rank runs one token of a 2-layer copy (same seed, shapes and shards)
    on seeded input; every rank's logits must be identical (checked by an all-reduce of max and
    min), and rank 0 checks them against the unsharded f64 CPU reference within
    1e-3 * sum_k |w_head x_k| per logit (x = the reference's normalised head input)."""
    import dataclasses

    import numpy as np
    import torch

    import oracle

    from kernite_b200 import stack as st

    c2 = dataclasses.replace(cfg, layers=min(2, cfg.layers))
    stream = torch.cuda.Stream()
    s = st.make_cuda_stack(c2, kernels, rank, world, stream=stream, push=push, chain=chain)
    x = np.random.default_rng(31).standard_normal(c2.hidden).astype(np.float32)
    s.buf["x"].copy_(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        s.forward()
    torch.cuda.synchronize()
    kernels.device_error()
    got = s.buf["logits"].clone()
    same = True
    if dist:
        hi, lo = got.clone(), got.clone()
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        same = bool(torch.equal(hi, lo))
    if s.be.peers:
        s.be.close()
    del s
    if rank != 0:
        return None
    ref, bound = st.reference_logits(c2, x, with_bound=True)
    err = np.abs(got.cpu().numpy().astype(np.float64) - ref)
    ratio = float((err / (1e-3 * bound)).max())
    return {"parity_ok": bool(same and ratio <= 1.0), "worst_error_ratio": round(ratio, 5),
            "ranks_identical": same,
            "checked": f"2-layer copy of the stack, one token, {world} rank(s), against the f64 CPU "
                       "reference: |logit - ref| <= 1e-3 * sum|w_head x|"}


def time_lone_matvec(kernels, qtype, rows, K, steps=2000):
    """The Q6_K head-shaped single matvec timed as the q6k_head workload
    is, for the stack line's extra keys: weights rotating over copies totalling > 2x L2, graph-
    replayed launches, CUDA events on the launching stream."""
    import numpy as np
    import torch

    import kernite_b200 as kb

    wbytes = kb.matrix_bytes(qtype, rows, K)
    copies = rotation_copies(wbytes)
    Ws = []
    for c in range(copies):
        W = torch.empty(wbytes, dtype=torch.uint8, device="cuda")
        kernels.fill(qtype, W, 0, rows * K // 256, kb.stream_key(2026 + c, qtype))
        Ws.append(W)
    x = torch.from_numpy(np.random.default_rng(0).standard_normal((1, K), dtype=np.float32)).cuda()
    y = torch.empty(1, rows, device="cuda")
    stream = torch.cuda.Stream()
    G = copies * max(1, 64 // copies)
    with torch.cuda.stream(stream):
        for i in range(3 * G):
            kernels.matvec(qtype, y, Ws[i % copies], x, rows, K, 1, flags=kb.FLAG_WEIGHTS_STATIC, stream=stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(G):
            kernels.matvec(qtype, y, Ws[i % copies], x, rows, K, 1, flags=kb.FLAG_WEIGHTS_STATIC, stream=stream)
    reps = max(1, steps // G)
    with torch.cuda.stream(stream):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    kernels.device_error()
    ms = e0.elapsed_time(e1) / (reps * G)
    algo = wbytes + K * 4 + rows * 4
    peak, kind = measured_peak()
    del g
    return {"workload": f"Q{qtype}_K {rows}x{K} batch 1 (BASELINE configs[1])", "launches": reps * G,
            "us_per_launch": round(ms * 1e3, 3), "weight_gbs": round(wbytes / (ms / 1e3) / 1e9, 2),
            "roofline": {"bound": "hbm", "achieved": round(algo / (ms / 1e3) / 1e9, 2), "peak": peak,
                         "unit": "GB/s", "frac": round(algo / (ms / 1e3) / 1e9 / peak, 4),
                         "peak_source": kind, "traffic": profiled_traffic("q6k_head"),
                         "algorithmic_bytes_per_launch": algo}}


def run_stack(args):
    """Decode tokens/s of a Llama-shaped matvec stack: one token = one replay of a CUDA graph
    holding every launch of the token (chains by default: per layer one launch for q|k|v, o and
    gate|up and one for down, then the head; for N > 1 the outputs pushed to every rank's full
    vectors inside those launches)."""
    import numpy as np

    from kernite_b200 import stack as st

    cfg = st.CONFIGS[STACKS[args.workload]]
    if args.layers is not None:
        import dataclasses

        cfg = dataclasses.replace(cfg, layers=args.layers, name=f"{cfg.name}, first {args.layers} layers")
    world, rank, local = dist_setup()
    chain = args.exchange == "chain"
    if args.impl == "reference":
        if rank != 0:
            return 0
        sec, sample = stack_cpu_seconds_per_token(cfg, HOST_THREADS)
        tps = 1.0 / sec
        line = {"impl": "reference", "metric": "decode tokens/s", "value": round(tps, 4),
                "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": stack_config(args, cfg, world, chain),
                "cpu_baseline": {"value": round(tps, 4), "unit": "tokens/s", "cores": HOST_THREADS,
                                 "kind": "port", "sample": sample, "cpu_model": cpu_model()},
                "e2e": {"value": round(tps, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0},
                "gpu_launches": 0,
                "note": "fxeqxmulfx/kernite has no k-quant path and no Rust toolchain here; the CPU "
                        "implementation timed is this repo's AVX2+FMA C port (oracle/kq_cpu.c) on the "
                        "host's cores, one process whatever the GPU count"}
        print(json.dumps(line), flush=True)
        return 0

    import torch

    import kernite_b200 as kb

    torch.cuda.set_device(local)
    dist = _init_dist(torch, world, local)
    kernels = kb.Kernels.load(local)
    push = args.exchange == "push" and world > 1
    parity = stack_parity(cfg, kernels, rank, world, chain, push, dist)
    stream = torch.cuda.Stream()
    stack = st.make_cuda_stack(cfg, kernels, rank, world, stream=stream, push=push, chain=chain)
    x = torch.from_numpy(np.random.default_rng(0).standard_normal(cfg.hidden).astype(np.float32))
    stack.buf["x"].copy_(x.cuda())
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            stack.forward()
    torch.cuda.synchronize()
    kernels.device_error()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        stack.forward()

    with torch.cuda.stream(stream):
        for _ in range(3):
            graph.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    kernels.device_error()
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_tok = ms / args.steps
    tps = 1e3 / ms_tok
    wbytes = cfg.weight_bytes()

    # end to end: x in from pinned memory, one token, logits out, every step
    xh = x.pin_memory()
    lh = torch.empty(cfg.vocab).pin_memory()
    e2e_steps = max(3, min(args.e2e_steps, args.steps))
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        f0.record(stream)
        for _ in range(e2e_steps):
            stack.buf["x"].copy_(xh, non_blocking=True)
            graph.replay()
            lh.copy_(stack.buf["logits"], non_blocking=True)
            stream.synchronize()
        f1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = f0.elapsed_time(f1)
    if dist:
        t = torch.tensor([ms_e2e], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t.item())
    e2e = {"value": round(e2e_steps / (ms_e2e / 1e3), 3), "unit": "tokens/s",
           "h2d_bytes_per_step": cfg.hidden * 4, "d2h_bytes_per_step": cfg.vocab * 4,
           "steps": e2e_steps}

    peak, peak_kind = measured_peak()
    per_gpu_gbs = wbytes / world / (ms_tok / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": round(per_gpu_gbs, 2), "peak": peak, "unit": "GB/s",
                "frac": round(per_gpu_gbs / peak, 4),
                "traffic": profiled_traffic(args.workload, "token") if world == 1 and args.layers is None else None,
                "traffic_note": "DRAM bytes per token on one GPU: 80 layers at the per-layer bytes of a "
                                "2-layer ncu capture, plus the head (profiles/stack70b.md)",
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                else "fallback 6650 GB/s",
                "note": "achieved = the stack's weight bytes per GPU per token / token time"}
    # A graph holding NCCL calls must be released before the process group goes, or the
    # teardown waits for good.
    torch.cuda.synchronize()
    graph.reset()
    graph = None
    lone = None
    cpu = None
    if rank == 0 and world == 1:
        lone = time_lone_matvec(kernels, 6, 32000, 4096)
        if not args.no_cpu_baseline:
            sec, sample, sec1 = stack_cpu_seconds_per_token(cfg, HOST_THREADS, also_single=True)
            cpu = {"value": round(1.0 / sec, 4), "unit": "tokens/s", "cores": HOST_THREADS,
                   "kind": "port", "sample": sample, "cpu_model": cpu_model(),
                   "single_thread": {"value": round(1.0 / sec1, 4), "sample": sample}}
    if rank == 0:
        line = {
            "metric": "decode tokens/s", "value": round(tps, 3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_tok, 5), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": stack_config(args, cfg, world, chain),
            "weight_gbs": round(wbytes * tps / 1e9, 2),
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "parity": parity,
            "gpu_launches": args.steps * stack.launches_per_token(), "clocks": clocks,
        }
        if lone is not None:
            line["matvec_q6k_head"] = lone
        print(json.dumps(line), flush=True)
    if stack.be.peers:
        stack.be.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    kernels.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
