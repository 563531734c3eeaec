#!/usr/bin/env python3
"""Benchmark of the B200 FP8 block-scaled GEMM (one JSON line on rank 0).

Metric: FP8 blockscale GEMM TFLOPS (2*M*N*K per call), with HBM GB/s and the
roofline fraction of the GEMM kernel, and us/call.

Default workload: the prefill layer M=8192, N=7168, K=16384 (e4m3 operands,
fp32 block scales, bf16 output), the configuration the benchmark quotes at
1, 2, 4 and 8 GPUs.  At N=1 a step is one call of the reference's timed
operator, ``gemm_a8w8_blockscale_bpreshuffle_asm(a, packed_b, out, packed_sa,
sb, ...)`` (client/aiter/hsa/gfx942/driver.py:26-29: pre-packed weight,
transposed-contiguous x_scale).  Under torchrun (``--gpus N``) the output
columns are sharded over the ranks (strong scaling): rank r holds WQ rows
[r*N/g, (r+1)*N/g), and each step is one launch per rank whose epilogue
stores every bf16 tile into every rank's Y over NVLink peer mappings and
whose CTAs complete the exchange on the device (``--gather fused``,
the default), or the blocks are all-gathered over NCCL and interleaved
(``--gather nccl``).  The decode shape M=256, N=3072, K=7168 is measured
beside it on every rank (key ``decode``) and can be the headline with
``--workload decode``; ``--workload`` selects any benchmark config.

Steps rotate over enough distinct input sets that the rotation exceeds 2.5x
the 126 MB L2 (one set when a set alone is larger), and are timed as
CUDA-graph replays with CUDA events on the launch stream, max over ranks
(client/aiter/runner.py:160-189 times graph replays the same way).

``--impl reference`` times the reference's own algorithm for this path -- the
fp32 dequantise-then-matmul of client/aiter/hsa/gfx942/driver.py:18-20 -- on
the host cores (the oracle port; the reference's GPU path needs gfx942 and the
absent aiter submodule), on the same workload, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

L2_BYTES = 126 * 1024 * 1024
METRIC = "FP8 blockscale GEMM TFLOPS & HBM GB/s (% roofline), us/call"
from fack_b200.data import SHARDED  # noqa: E402  (workloads sharded by output columns)


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ---------------------------------------------------------------- clocks --
class ClockSampler:
    """NVML sampler (SM clock, max clock, clock-event reasons) for one GPU."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index: int, period_s: float = 0.01):
        self.samples = []
        self.ok = False
        self.period = period_s
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # NVML missing: report no clocks rather than guess
            self.err = str(e)

    def _sample(self):
        nv = self.nv
        try:
            reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:
            reasons = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
        self.samples.append((time.time(), nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM), int(reasons)))

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.period)

    def start(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        if self.ok:
            self._stop.set()
            self._t.join()
            self._sample()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "note": getattr(self, "err", "no samples")}
        mask = 0
        for _, _, r in self.samples:
            mask |= r
        reasons = [name for bit, name in self.REASONS.items() if mask & bit and bit != 0x1]
        return {"sm_mhz": statistics.median(s[1] for s in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples)}


# ------------------------------------------------------------- workloads --
def env_ranks():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def make_sets(wl, n_sets, dev, shard):
    """n_sets distinct device copies of (a, packed_b, out, packed_sa, sb)."""
    from fack_b200 import data
    import fack_b200 as fb
    xq, xs = data.make_activations(wl.M, wl.K, wl.x_dist, seed=0, device=dev)
    wq, ws = data.make_weights(wl.N, wl.K, wl.w_dist, seed=1, device=dev)
    if shard is not None:
        from fack_b200.dist import shard_weight
        wq, ws = shard_weight(wq, ws, *shard)
    packed = fb.shuffle_weight(wq)
    del wq
    sa = data.to_aiter_xscale(xs)
    sets = []
    for i in range(n_sets):
        cp = (lambda t: t.clone()) if i else (lambda t: t)
        b = cp(packed)
        b.is_shuffled = True
        sets.append({"a": cp(xq), "b": b, "sa": cp(sa), "sa_logical": cp(xs), "sb": cp(ws),
                     "out": torch.empty((wl.M, packed.shape[0]), dtype=torch.bfloat16, device=dev)})
    return sets


def capture(fn_steps, stream, keep):
    """Capture fn_steps() into a CUDA graph (kept in `keep`); returns its replay."""
    g = torch.cuda.CUDAGraph()
    keep.append(g)
    with torch.cuda.graph(g, stream=stream):
        fn_steps()
    return g.replay


def timed_graph_replay(plan, stream):
    """Run [(fn, times)] (graph replays or eager step loops), bracketed by CUDA
    events on `stream`; ms."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):  # replay() and eager launches use the current stream
        start.record(stream)
        for fn, times in plan:
            for _ in range(times):
                fn()
        end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)


def max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def load_traffic(workload: str):
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        return d.get(workload, {}).get("bytes_per_launch")
    except Exception:
        return None


def cpu_oracle_rate(wl, budget_s: float, max_steps: int = 3):
    """Time the CPU oracle on a bounded column sample of `wl`; TFLOPS and sample text."""
    from fack_b200 import data
    from oracle.blockscale import reference_gemm
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    xq, xs = data.make_activations(wl.M, wl.K, wl.x_dist, seed=0)
    n_cols = 128
    wq, ws = data.make_weights(n_cols, wl.K, "normal", seed=1)
    t0 = time.perf_counter()
    reference_gemm(xq, wq, xs, ws)
    t1 = time.perf_counter() - t0
    # grow the column sample to fill ~budget/steps per call, up to the full N
    per_call = budget_s / max_steps
    n_cols = int(min(wl.N, max(128, 128 * math.floor(per_call / max(t1, 1e-4)))))
    n_cols -= n_cols % 128
    wq, ws = data.make_weights(n_cols, wl.K, "normal", seed=1)
    times = []
    for _ in range(max_steps):
        t0 = time.perf_counter()
        reference_gemm(xq, wq, xs, ws)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    tflops = data.flops(wl.M, n_cols, wl.K) / t / 1e12
    sample = (f"M={wl.M} x N={n_cols} (of {wl.N}) x K={wl.K} of workload {wl.name}: dequantise both operands + "
              f"fp32 matmul + bf16 round (driver.py:18-20), median of {max_steps} calls, {t * 1e3:.1f} ms/call")
    return tflops, threads, sample


# ------------------------------------------------------------- our arm --
def roofline(k_bytes, k_flops, k_us, peaks, clk, region_ms):
    """Roofline of one GEMM launch of k_us: the bound (HBM or tensor) whose
    time is the larger.  The tensor peak that applies is the one at the clocks
    the timed region ran at: the burst GEMM figure while the SM clock held its
    maximum, the sustained (power-capped) figure once it dropped below 95 % of
    it; without clock samples, the sustained figure for a region over 0.2 s."""
    if clk and clk.get("samples") and clk.get("sm_mhz") and clk.get("sm_max_mhz"):
        sustained = clk["sm_mhz"] < 0.95 * clk["sm_max_mhz"]
        why = f"median SM clock {clk['sm_mhz']:.0f} of {clk['sm_max_mhz']} MHz"
    else:
        sustained = region_ms > 200.0
        why = f"timed region {region_ms:.0f} ms"
    bf16_peak = peaks["bf16_tflops_sustained"] if sustained else peaks["bf16_tflops"]
    fp8_peak = 2.0 * bf16_peak
    t_mem = k_bytes / (peaks["hbm_gbs"] * 1e3)        # us
    t_tc = k_flops / (fp8_peak * 1e6)                 # us
    hbm_gbs = k_bytes / (k_us * 1e3)
    tflops_k = k_flops / (k_us * 1e6)
    if t_mem >= t_tc:
        roof = {"bound": "hbm", "achieved": round(hbm_gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(hbm_gbs / peaks["hbm_gbs"], 4)}
    else:
        roof = {"bound": "tensor", "achieved": round(tflops_k, 1), "peak": round(fp8_peak, 1), "unit": "TFLOP/s",
                "frac": round(tflops_k / fp8_peak, 4)}
    roof.update({"algorithmic_bytes": k_bytes, "kernel_us": round(k_us, 3), "peak_source": (
        f"{peaks['source']} MEASURED_PEAKS.json: hbm_gbs copy bandwidth; fp8 dense = 2 x bf16 "
        f"{'sustained' if sustained else 'burst'} {bf16_peak} TFLOP/s ({why})"),
        "t_mem_us": round(t_mem, 3), "t_tc_us": round(t_tc, 3),
        "frac_of_max_roof": round(max(t_mem, t_tc) / k_us, 4)})
    return roof


def measure_unsharded(name, steps, dev, stream, world, peaks, local):
    """Kernel time of an unsharded workload on this rank's GPU (replicas when
    world > 1): CUDA-graph replays of the reference's call form over rotating
    input sets, max over ranks.  The secondary record of the bench line."""
    import fack_b200 as fb
    from fack_b200 import data
    wl = data.WORKLOADS[name]
    set_bytes = data.algorithmic_bytes(wl.M, wl.N, wl.K)
    n_sets = max(1, math.ceil(2.5 * L2_BYTES / set_bytes))
    sets = make_sets(wl, n_sets, dev, None)
    cfg = fb.get_config(wl.M, wl.N, wl.K)

    def call(s):
        fb.gemm_a8w8_blockscale_bpreshuffle_asm(s["a"], s["b"], s["out"], s["sa"], s["sb"], None,
                                                cfg["splitK"], cfg["kernelName"], True)
    with torch.cuda.stream(stream):
        for i in range(3):
            call(sets[i % n_sets])
    torch.cuda.synchronize(dev)
    chunk = n_sets * max(1, 256 // n_sets)
    graphs = []
    with torch.cuda.stream(stream):
        run = capture(lambda: [call(sets[i % n_sets]) for i in range(chunk)], stream, graphs)
    reps = max(3, math.ceil(steps / chunk))
    sampler = ClockSampler(local)
    sampler.start()
    timed_graph_replay([(run, 2)], stream)
    barrier(world)
    ms = max_over_ranks(timed_graph_replay([(run, reps)], stream), world, dev)
    sampler.stop()
    for g in graphs:
        g.reset()
    us = ms * 1e3 / (reps * chunk)
    clk = sampler.summary()
    roof = roofline(set_bytes, data.flops(wl.M, wl.N, wl.K), us, peaks, clk, ms)
    del sets
    return {"workload": f"{wl.name} M={wl.M} N={wl.N} K={wl.K}", "kernel": cfg["kernelName"],
            "us_per_call": round(us, 3), "tflops": round(data.flops(wl.M, wl.N, wl.K) / (us * 1e6), 2),
            "hbm_gbs": round(set_bytes / (us * 1e3), 1), "calls_timed": reps * chunk,
            "l2": f"rotate {n_sets} input sets x {set_bytes / 1e6:.1f} MB", "roofline": roof,
            "clocks": clk, "parallelism": "single GPU" if world == 1 else f"{world} independent replicas"}


def run_ours(args):
    import fack_b200 as fb
    from fack_b200 import data
    rank, world, local = env_ranks()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=90), device_id=dev)
    wl = data.WORKLOADS[args.workload]
    sharded = args.workload in SHARDED and world > 1
    shard = (rank, world) if sharded else None
    n_local = wl.N // world if sharded else wl.N
    set_bytes = data.algorithmic_bytes(wl.M, n_local, wl.K)
    n_sets = args.rotate or max(1, math.ceil(2.5 * L2_BYTES / set_bytes))
    sets = make_sets(wl, n_sets, dev, shard)
    cfg = fb.get_config(wl.M, n_local, wl.K)
    stream = torch.cuda.Stream(dev)

    sharder = None
    if sharded:
        from fack_b200.dist import ShardedBlockscaleGemm
        sharder = ShardedBlockscaleGemm(mode=args.gather)
        # two outputs alternate, so a peer never stores into the Y of the
        # step before (the fused path then needs no extra exchange step)
        full_out = [torch.empty((wl.M, wl.N), dtype=torch.bfloat16, device=dev) for _ in range(2)]

    def gemm_call(s):
        fb.gemm_a8w8_blockscale_bpreshuffle_asm(s["a"], s["b"], s["out"], s["sa"], s["sb"], None,
                                                cfg["splitK"], cfg["kernelName"], True)

    def step(i):
        s = sets[i % n_sets]
        if sharded:
            sharder(s["a"], s["b"], s["sa_logical"], s["sb"], out=full_out[i % 2])
        else:
            gemm_call(s)

    log(f"[bench rank {rank}] {wl.name}: {n_sets} input sets, plan {cfg['kernelName']}, sharded={sharded}")
    # warm-up (eager: sizes the split-K workspace, registers the outputs and
    # the exchange state); an even count ends on the second output
    warm = args.warmup + (args.warmup % 2)
    with torch.cuda.stream(stream):
        for i in range(warm):
            step(i)
    barrier(world)

    period = n_sets if n_sets % 2 == 0 else 2 * n_sets   # a graph starts on output 0 and set 0
    chunk = max(period, (min(args.steps, 1024) // period) * period)
    full, rem = divmod(args.steps, chunk)
    graphs = []
    timing = "CUDA-graph replay"

    def steps_fn(n):
        return lambda: [step(i) for i in range(n)]

    def gemm_fn(n):
        return lambda: [gemm_call(sets[i % n_sets]) for i in range(n)]

    try:
        with torch.cuda.stream(stream):
            run_chunk = capture(steps_fn(chunk), stream, graphs) if full else None
            run_rem = capture(steps_fn(rem), stream, graphs) if rem else None
            run_gemm = capture(gemm_fn(chunk), stream, graphs) if sharded else None  # GEMM-only: kernel roofline
    except Exception as e:  # collectives that cannot be captured: time eager launches instead
        log(f"graph capture failed ({e}); timing eager launches")
        for g in graphs:
            g.reset()
        graphs = []
        timing = "eager launches"
        run_chunk, run_rem = steps_fn(chunk), steps_fn(rem)
        run_gemm = gemm_fn(chunk) if sharded else None
    if world > 1:  # all ranks must time the same way (captured steps hold exchange steps)
        flag = torch.tensor([1 if graphs else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if flag.item() == 0 and graphs:
            for g in graphs:
                g.reset()
            graphs = []
            timing = "eager launches"
            run_chunk, run_rem = steps_fn(chunk), steps_fn(rem)
            run_gemm = gemm_fn(chunk) if sharded else None
    log(f"[bench rank {rank}] timing via {timing}")
    plan = [(run_chunk, full)] if full else []
    if rem:
        plan.append((run_rem, 1))

    # keep the GPU busy ~0.3 s before timing so clocks are sampled under load
    sampler = ClockSampler(local)
    sampler.start()
    probe = run_chunk or run_rem
    # every rank must replay the same number of steps (the sharded steps wait
    # on each other), so the warm-up count comes from the slowest rank's probe
    t_probe = max_over_ranks(timed_graph_replay([(probe, 1)], stream) / 1e3, world, dev)
    log(f"[bench rank {rank}] probe {t_probe * 1e3:.3f} ms per chunk; warming, then timing {args.steps} steps")
    timed_graph_replay([(probe, max(1, int(0.3 / max(t_probe, 1e-6))))], stream)
    barrier(world)
    ms = timed_graph_replay(plan, stream)
    sampler.stop()
    barrier(world)
    ms = max_over_ranks(ms, world, dev)
    clk = sampler.summary()

    us_call = ms * 1e3 / args.steps
    ranks_work = world if not sharded else 1
    total_flops = data.flops(wl.M, wl.N, wl.K) * ranks_work * args.steps
    value = total_flops / (ms / 1e3) / 1e12

    # roofline of the GEMM kernel (per launch on one GPU): for a sharded step
    # the same rank's launch without peer stores or exchange, timed alone
    if sharded:
        k_ms = timed_graph_replay([(run_gemm, 1)], stream)
        k_us = max_over_ranks(k_ms * 1e3 / chunk, world, dev)
    else:
        k_us = us_call
    peaks = measured_peaks()
    k_bytes = data.algorithmic_bytes(wl.M, n_local, wl.K)
    roof = roofline(k_bytes, data.flops(wl.M, n_local, wl.K), k_us, peaks, clk, ms)
    roof["step_us"] = round(us_call, 3)
    # ncu DRAM bytes of the workload's launch on one GPU; a column shard reads
    # its share of the weights and writes its share of Y, so its launch is
    # reported as that scaled by n_local / N
    traffic = load_traffic(args.workload)
    if traffic is not None and sharded:
        traffic = int(round(traffic * n_local / wl.N))
    roof = {**{k: roof[k] for k in ("bound", "achieved", "peak", "unit", "frac")}, "traffic": traffic,
            **{k: v for k, v in roof.items() if k not in ("bound", "achieved", "peak", "unit", "frac")}}

    # e2e through the public API with pinned host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, wl, sets[0], dev, stream, sharder, world, cfg)

    # the decode shape beside the headline (replicas at N > 1)
    decode = None
    if args.workload != "decode" and not args.no_decode:
        del sets
        torch.cuda.empty_cache()
        decode = measure_unsharded("decode", 2000, dev, stream, world, peaks, local)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tfl, cores, sample = cpu_oracle_rate(wl, budget_s=args.cpu_budget)
        cpu = {"value": round(tfl, 4), "unit": "TFLOPS", "cores": cores, "kind": "port", "sample": sample}

    # our launches per step: the GEMM (plus the fix-up of its tail split when
    # the plan has one; the last of them runs the fused exchange), plus the
    # interleave of the NCCL-gather path (NCCL's own kernels not counted)
    tail_split = cfg["splitK"] == 1 and fb.tail_workspace_size(wl.M, n_local, wl.K, cfg["tile_m"], cfg["tile_n"], 1) > 0
    per_step_launches = (2 if tail_split else 1) + (1 if sharded and args.gather == "nccl" else 0)
    extra = sharder.barriers if sharder is not None and args.gather == "fused" else 0
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 6), "higher_is_better": True,
        "scaling": "strong" if sharded or args.workload in SHARDED else "weak", "vs_baseline": None,
        "dtype": "fp8_e4m3 (fp32 accumulate, bf16 out)",
        "data": "synthetic (seeded; benchmark-config construction, scale = amax/240)",
        "config": {"workload": f"{wl.name} M={wl.M} N={wl.N} K={wl.K}", "M": wl.M, "N": wl.N, "K": wl.K,
                   "x_dist": wl.x_dist, "w_dist": wl.w_dist, "tile_m": cfg["tile_m"], "split_k": cfg["splitK"],
                   "kernel": cfg["kernelName"], "n_local": n_local, "tail_split": tail_split,
                   "weights": "prepacked (bpreshuffle=True)",
                   "l2": f"rotate {n_sets} input sets x {set_bytes / 1e6:.1f} MB = {n_sets * set_bytes / 1e6:.0f} MB"
                         f" (> 126 MB L2)",
                   "timing": f"{timing}, CUDA events on the launch stream, max over ranks",
                   "parallelism": ((f"N-shard g={world}: one launch per rank per step; its epilogue stores every "
                                    "tile to all ranks' Y over NVLink peer mappings (CUDA IPC); each CTA counts its "
                                    "landed stores into every peer's exchange state and CTA 0 waits for the "
                                    "peers' counts (no collective on the stream)"
                                    if args.gather == "fused" else f"N-shard g={world} + NCCL all-gather")
                                   if sharded else
                                   ("single GPU" if world == 1 else f"{world} independent replicas"))},
        "us_per_call": round(us_call, 3), "hbm_gbs": round(k_bytes / (k_us * 1e3), 1),
        "roofline": roof, "e2e": e2e, "cpu_baseline": cpu, "clocks": clk, "decode": decode,
        "gpu_launches": per_step_launches * args.steps,
        "gpu_launches_note": f"{extra} stand-alone exchange steps outside the timed region" if extra else None,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    status = fb.device_status()
    if status:
        log(f"device status flags set: {status:#x}")
    for g in graphs:
        g.reset()
    del graphs, plan, probe, run_chunk, run_rem, run_gemm
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        if sharder is not None:
            sharder.close()  # release the peer mappings before the group goes
        dist.barrier()
        dist.destroy_process_group()
    if status:
        sys.exit(3)


def run_e2e(args, wl, s0, dev, stream, sharder, world, cfg):
    """Public API, host inputs: per step the pinned H2D of XQ + x_scale, the
    call, the D2H of Y, on three streams over rotating buffers (step i's
    inputs cross PCIe while step i-1 computes and step i-2's result comes
    back; each step still moves its own bytes), captured in CUDA graphs as the
    reference's runner captures its timed launches (client/aiter/runner.py:
    169-172), at least three graphs."""
    import fack_b200 as fb
    from fack_b200 import data
    a_h = s0["a"].cpu().pin_memory()
    sa_h = (s0["sa_logical"] if sharder else s0["sa"]).cpu().pin_memory()
    y_h = torch.empty((wl.M, wl.N), dtype=torch.bfloat16).pin_memory()
    h2d = a_h.numel() * a_h.element_size() + sa_h.numel() * 4
    d2h = y_h.numel() * 2
    # outputs rotate over nb buffers; GEMM i waits for the copy-out of step
    # i - w.  Sharded: a peer stores into buffer i % 3 once every rank has
    # finished step i - 1, whose GEMM waited for the copy-out of step i - 3,
    # the buffer's previous use.
    nb, w = (3, 2) if sharder else (2, 2)
    per_graph = 64 if h2d + d2h < 32e6 else 15
    per_graph -= per_graph % nb
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    a_b = [torch.empty_like(s0["a"]) for _ in range(2)]
    sa_b = [torch.empty_like(sa_h, device=dev) for _ in range(2)]
    out_b = [torch.empty((wl.M, wl.N), dtype=torch.bfloat16, device=dev) for _ in range(nb)]

    def call(i, b, o):
        if sharder:
            sharder(a_b[b], s0["b"], sa_b[b], s0["sb"], out=out_b[o])
        else:
            fb.gemm_a8w8_blockscale_bpreshuffle_asm(a_b[b], s0["b"], out_b[o], sa_b[b], s0["sb"], None,
                                                    cfg["splitK"], cfg["kernelName"], True)

    def steps_graph(n):
        fork = torch.cuda.Event()
        fork.record(stream)                        # the side streams join the capture here
        s_in.wait_event(fork)
        s_out.wait_event(fork)
        comp, outd, ev_in = [], [], None
        for i in range(n):
            b, o = i % 2, i % nb
            if i >= 2:
                s_in.wait_event(comp[i - 2])       # step i-2's call has read these inputs
            ev_in = torch.cuda.Event()
            with torch.cuda.stream(s_in):
                a_b[b].copy_(a_h, non_blocking=True)
                sa_b[b].copy_(sa_h, non_blocking=True)
                ev_in.record(s_in)
            stream.wait_event(ev_in)
            if i >= w:
                stream.wait_event(outd[i - w])
            call(i, b, o)
            ev_c = torch.cuda.Event()
            ev_c.record(stream)
            comp.append(ev_c)
            s_out.wait_event(ev_c)
            ev_o = torch.cuda.Event()
            with torch.cuda.stream(s_out):
                y_h.copy_(out_b[o], non_blocking=True)
                ev_o.record(s_out)
            outd.append(ev_o)
        stream.wait_event(outd[-1])                # join both side streams back
        stream.wait_event(ev_in)

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        steps_graph(nb)                            # eager warm-up outside capture (registers every output)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            steps_graph(per_graph)
        g.replay()                                 # warm replay
        torch.cuda.synchronize(dev)
        barrier(world)
        reps = max(3, math.ceil(min(args.steps, args.e2e_steps) / per_graph))
        start.record(stream)
        for _ in range(reps):
            g.replay()
        end.record(stream)
        end.synchronize()
    g.reset()
    steps = reps * per_graph
    ms = max_over_ranks(start.elapsed_time(end), world, dev)
    us = ms * 1e3 / steps
    work = data.flops(wl.M, wl.N, wl.K) * (1 if sharder else world) * steps
    return {"value": round(work / (ms / 1e3) / 1e12, 4), "unit": "TFLOPS",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps, "us_per_step": round(us, 2),
            "h2d_gbs": round(h2d / (us * 1e3), 2), "d2h_gbs": round(d2h / (us * 1e3), 2),
            "api": ("fack_b200.dist.ShardedBlockscaleGemm (fused all-gather)" if sharder else
                    "fack_b200.gemm_a8w8_blockscale_bpreshuffle_asm with the plan of get_config") +
                   f"; per step: pinned copy-in, call, copy-out on three streams over {nb} output buffers, "
                   f"{reps} CUDA graphs of {per_graph} steps"}


# ------------------------------------------------------- reference arm --
def run_reference(args):
    rank, world, _ = env_ranks()
    if rank != 0:
        return
    from fack_b200 import data
    from oracle.blockscale import reference_gemm
    wl = data.WORKLOADS[args.workload]
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    xq, xs = data.make_activations(wl.M, wl.K, wl.x_dist, seed=0)
    # size the per-step column sample so warm-up + steps fit the time budget
    wq, ws = data.make_weights(128, wl.K, "normal" if wl.w_dist == "normal" else wl.w_dist, seed=1)
    t128 = float("inf")
    for _ in range(2):  # the first call is cold
        t0 = time.perf_counter()
        reference_gemm(xq, wq, xs, ws)
        t128 = min(t128, time.perf_counter() - t0)
    per_step = args.ref_budget / max(1, args.steps + args.warmup)
    n_cols = int(min(wl.N, max(128, 128 * math.floor(per_step / max(t128, 1e-5)))))
    n_cols -= n_cols % 128
    # below one 128-column weight block per step, sample fewer tokens too (the
    # oracle's time is mostly the fp32 matmul, linear in the token count); the
    # weight block's dequantisation (~2 ms at K = 7168 on 8 cores) is the
    # floor of a step
    m_rows = wl.M if per_step >= t128 else max(1, min(wl.M, int(wl.M * per_step / max(t128, 1e-9))))
    xq, xs = xq[:m_rows], xs[:m_rows]
    wq, ws = data.make_weights(n_cols, wl.K, "normal" if wl.w_dist == "normal" else wl.w_dist, seed=1)
    for _ in range(args.warmup):
        reference_gemm(xq, wq, xs, ws)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        reference_gemm(xq, wq, xs, ws)
    dt = time.perf_counter() - t0
    value = data.flops(m_rows, n_cols, wl.K) * args.steps / dt / 1e12
    sample = (f"M={m_rows} (of {wl.M}) x N={n_cols} (of {wl.N}) x K={wl.K} per step of workload {wl.name}: "
              f"fp32 dequantise + "
              f"matmul + bf16 (client/aiter/hsa/gfx942/driver.py:18-20 restated), torch CPU, {threads} threads")
    line = {"metric": METRIC, "value": round(value, 5), "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt * 1e3 / args.steps, 3), "higher_is_better": True,
            "scaling": "strong" if args.workload in SHARDED else "weak", "vs_baseline": None,
            "dtype": "fp32 (dequantised e4m3)",
            "data": "synthetic (seeded; benchmark-config construction)", "impl": "reference",
            "config": {"workload": f"{wl.name} M={wl.M} N={wl.N} K={wl.K}", "M": wl.M, "N": wl.N, "K": wl.K,
                       "parallelism": "host CPU, rank 0 only"},
            "cpu_baseline": {"value": round(value, 5), "unit": "TFLOPS", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 5), "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "gpu_launches": 0}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="prefill")
    ap.add_argument("--gather", choices=["fused", "nccl"], default="fused",
                    help="sharded workloads: peer stores from the GEMM epilogue, or NCCL all-gather + interleave")
    ap.add_argument("--rotate", type=int, default=0, help="input sets to rotate (0 = enough to exceed L2)")
    ap.add_argument("--e2e-steps", type=int, default=192, help="e2e steps (at least three CUDA graphs)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the secondary decode-shape measurement")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU oracle work for cpu_baseline")
    ap.add_argument("--ref-budget", type=float, default=90.0, help="seconds for the reference arm's steps")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.steps < 1:
        ap.error("--steps must be >= 1")
    from fack_b200 import data
    if args.workload not in data.WORKLOADS:
        ap.error(f"unknown workload; choose from {sorted(data.WORKLOADS)}")
    _, world, _ = env_ranks()
    if world != args.gpus:
        ap.error(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
