"""Exact-shape plan tuner for the FP8 block-scaled GEMM.

``python -m fack_b200.tune [--family blockscale|bf16|i8|siblings] [--shapes M,N,K;M,N,K...] [--out CSV]
[--log JSONL] [--verbose]``

For every (M, N, K) the tuner times each valid plan of the kernel --
token tile 128 (one CTA) or 256 (a CTA pair), weight tile 64, 128 or 256
dividing N, split-K 1..min(8, K/128) (pairs: 1..4), the 224-wide weight tile
(one K slice) when 224 divides N, for M <= 64 the swapped
16/32/64-token tiles, and for M <= 16 the warp-MMA kernel's 16-row weight
tiles -- through the same entry
the reference calls (pre-packed weight, transposed x_scale, split-K slices
combined in distributed shared memory), checks each plan's output against an
fp32 dequantise-then-matmul on the device, and writes the fastest plan per
shape as a row of the exact-shape table that ``fack_gemm_bs_plan`` consults
(``fack_b200/configs/a8w8_blockscale_bpreshuffle_tuned_gemm.csv``).

This is the B200 counterpart of the reference's per-shape tuning records: the
reference keys its kernel choice by exact (cu_num, M, N, K) rows of a tuned
CSV carrying kernelName, splitK, us, tflops, bw and errRatio
(client/aiter/dispatch.py:23-35; a row with a non-zero errRatio is refused,
dispatch.py:135-137).  The rows written here carry the same columns plus
``heuristic_kernelName`` / ``heuristic_us``, the cost model's plan and its
time, so the gain of every override is on record.  ``--log`` also writes one
JSON line per timed plan -- measured µs, errRatio and the cost model's
estimate in SM cycles (``fack_gemm_bs_plan_estimate``) -- the data for
calibrating the model's rates against the hardware.

``--family bf16|i8|siblings`` tunes the sibling families instead
(``fack_gemm_tn``: BF16 TN and INT8 per token) over the same kind of plan
list -- token tile 128 or 256, weight tile 64/128/256, split-K -- into the
sibling table (``configs/gemm_tn_tuned_gemm.csv``, read by
``fack_gemm_tn_tuned_load``); INT8 plans must match the exact epilogue
bitwise, BF16 plans an fp32 matmul within 1e-2.

Timing: each plan is captured in a CUDA graph of ``launches`` calls rotating
over input sets larger than 2.5 x the 126 MB L2 together, replayed once to
warm up, then ``repeats`` timed replays (CUDA events on the launch stream);
the median per-call time is kept.  errRatio = fraction of outputs with
|y - ref| > 1e-2 + 1e-2 * |ref|; only plans with errRatio 0 are eligible.
"""
from __future__ import annotations

import argparse
import csv
import json
import math
import statistics
import sys
from pathlib import Path

import torch

from . import _lib, data, ops

L2_BYTES = 126e6
KEEP_MARGIN = 0.02  # a plan must beat the cost model's by more than this to replace it
HEADER = ["cu_num", "M", "N", "K", "kernelName", "splitK", "us", "tflops", "bw", "errRatio",
          "heuristic_kernelName", "heuristic_us"]

# The exact (M, N, K) workloads tuned in the reference's records
# (client/aiter/co_out/records/*.json, 43 records of the blockscale family).
RECORD_SHAPES = (
    (1024, 1536, 4096), (1152, 1536, 4096), (128, 1536, 4096), (2304, 1536, 4096), (256, 1536, 4096),
    (128, 3072, 6144), (384, 3072, 6144), (48, 4096, 2048), (64, 4096, 2048),
    (144, 3072, 7168), (208, 3072, 7168), (224, 3072, 7168), (240, 3072, 7168), (256, 3072, 7168),
    (288, 3072, 7168), (320, 3072, 7168), (480, 3072, 7168), (512, 3072, 7168), (736, 3072, 7168),
    (768, 3072, 7168), (800, 3072, 7168),
    (144, 4096, 7168), (160, 4096, 7168), (176, 4096, 7168), (320, 4096, 7168), (352, 4096, 7168),
    (192, 4608, 7168), (208, 4608, 7168), (224, 4608, 7168), (240, 4608, 7168), (256, 4608, 7168),
    (672, 4608, 7168), (1408, 4608, 7168),
    (128, 7168, 7168), (288, 7168, 7168), (320, 7168, 7168), (352, 7168, 7168),
    (32, 8192, 7168), (80, 8192, 7168), (112, 8192, 7168), (128, 8192, 7168), (144, 8192, 7168),
    (240, 11264, 7168),
)


def default_shapes() -> list:
    """The reference's tuned workloads plus the benchmark workloads of this
    library (decode M sweep, plumbing, prefill, wide layer) and one rank's
    column shard of the sharded ones at 2, 4 and 8 GPUs."""
    shapes = list(RECORD_SHAPES)
    for wl in data.WORKLOADS.values():
        shapes.append((wl.M, wl.N, wl.K))
    shapes += data.shard_shapes()
    out, seen = [], set()
    for s in shapes:
        if s not in seen:
            seen.add(s)
            out.append(s)
    return out


def candidates(M: int, N: int, K: int) -> list:
    """Every (tile_m, tile_n, split_k) the planner accepts for the shape."""
    KB = K // ops.BLOCK
    plans = []
    for tm in (16, 32, 64):                      # swapped small-M tiles hold all M tokens
        if M <= tm:
            plans += [(tm, 128, sk) for sk in range(1, min(8, KB) + 1) if -(-KB // sk) <= 128]
    for tm in (128, 256):
        for tn in (256, 128, 64):
            if N % tn:
                continue
            for sk in range(1, min(8 if tm == 128 else 4, KB) + 1):
                plans.append((tm, tn, sk))
    if N % 224 == 0:                             # 224-wide tiles: persistent kernel, one K slice
        plans.append((128, 224, 1))
    if M <= 16 and KB <= 256:                    # the warp-MMA small-M kernel: 16-row weight tiles
        plans.append((16, 16, 1))
    return plans


def _sets_for(M: int, N: int, K: int) -> int:
    per_set = M * K + N * K + 4 * M * (K // 128) + 4 * (N // 128) * (K // 128)
    return max(1, math.ceil(2.5 * L2_BYTES / per_set))


def _reference(xq, xs, wq, ws):
    """fp32 dequantise-then-matmul on the device (TF32 off)."""
    xd = xq.float() * xs.repeat_interleave(128, dim=1)
    wd = wq.float() * ws.repeat_interleave(128, dim=0).repeat_interleave(128, dim=1)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return xd @ wd.T
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def err_ratio(y: torch.Tensor, ref: torch.Tensor) -> float:
    d = (y.float() - ref).abs()
    bad = (d > 1e-2 + 1e-2 * ref.abs()) | ~torch.isfinite(y.float())
    return float(bad.float().mean())


class ShapeBench:
    """Input sets, packed weights and the fp32 reference for one shape."""

    def __init__(self, M: int, N: int, K: int, seed: int = 0, launches: int = 24):
        dev = torch.device("cuda")
        self.M, self.N, self.K = M, N, K
        self.sets = []
        for i in range(_sets_for(M, N, K)):
            xq, xs = data.make_activations(M, K, "normal", seed + 2 * i, dev)
            wq, ws = data.make_weights(N, K, "normal", seed + 2 * i + 1, dev)
            self.sets.append((xq, data.to_aiter_xscale(xs), ops.shuffle_weight(wq), ws, xq, xs, wq))
        xq, _, _, ws, _, xs, wq = self.sets[0]
        # rows checked: all of them, or 512 spread over a large M
        self.rows = torch.arange(M, device=dev) if M <= 1024 else torch.linspace(0, M - 1, 512, device=dev).long()
        self.ref = _reference(xq[self.rows], xs[self.rows], wq, ws)
        self.out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        self.launches = max(launches, len(self.sets))

    def call(self, i: int, name: str):
        xq, xsa, wp, ws = self.sets[i % len(self.sets)][:4]
        ops.gemm_a8w8_blockscale_bpreshuffle_asm(xq, wp, self.out, xsa, ws, None, None, name, True)

    def check(self, name: str) -> float:
        self.call(0, name)
        torch.cuda.synchronize()
        return err_ratio(self.out[self.rows], self.ref)

    def time_us(self, name: str, repeats: int = 3) -> float:
        return _graph_time(lambda i: self.call(i, name), len(self.sets), self.launches, repeats)


def _graph_time(call, n_sets: int, launches: int, repeats: int = 3) -> float:
    """Median µs per call of ``call(i)`` captured ``launches`` times in a CUDA
    graph (i rotating over the input sets), replayed once to warm up, then
    ``repeats`` timed replays (CUDA events on the launch stream)."""
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(n_sets):  # first calls outside capture
            call(i)
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(launches):
            call(i % n_sets)
    times = []
    with torch.cuda.stream(stream):
        g.replay()
        for _ in range(repeats):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            g.replay()
            b.record(stream)
            b.synchronize()
            times.append(a.elapsed_time(b) * 1e3 / launches)
    g.reset()
    return statistics.median(times)


def choose(results: list, heuristic_name: str, shape=None) -> tuple:
    """The winning (us, kernelName, splitK, errRatio) of one shape's results:
    the fastest plan with errRatio 0, unless the cost model's own plan passes
    and is within KEEP_MARGIN of it (timing noise), which then stays.  Raises
    RuntimeError if no plan passes the check."""
    ok = [r for r in results if r[3] == 0.0]
    if not ok:
        raise RuntimeError(f"no plan of shape {shape} passed the output check: "
                           + ", ".join(f"{r[1]} errRatio {r[3]}" for r in results))
    best = min(ok)
    heur_row = next((r for r in ok if r[1] == heuristic_name), None)
    if heur_row and heur_row[0] <= best[0] * (1.0 + KEEP_MARGIN):
        best = heur_row
    return best


def tune_shape(M: int, N: int, K: int, log=None) -> dict:
    """Time every plan of one shape; the fastest plan with errRatio 0 wins."""
    sb = ShapeBench(M, N, K)
    heur = ops.get_config(M, N, K)
    results, plans = [], []
    for tm, tn, sk in candidates(M, N, K):
        name = ops.kernel_name(tm, tn, sk)
        er = sb.check(name)
        us = sb.time_us(name) if er == 0.0 else float("inf")
        results.append((us, name, sk, er))
        plans.append(plan_record(M, N, K, name, us, er, ops.plan_estimate(M, N, K, tm, tn, sk)))
        if log:
            log(f"  {name:28s} {us:9.2f} us  errRatio {er}")
    best = choose(results, heur["kernelName"], (M, N, K))
    heur_row = next((r for r in results if r[1] == heur["kernelName"]), None)
    heur_us = heur_row[0] if heur_row else float("nan")
    us = best[0]
    return {"cu_num": torch.cuda.get_device_properties(0).multi_processor_count, "M": M, "N": N, "K": K,
            "kernelName": best[1], "splitK": best[2], "us": round(us, 3),
            "tflops": round(data.flops(M, N, K) / us / 1e6, 1),
            "bw": round(data.algorithmic_bytes(M, N, K) / us / 1e3, 1), "errRatio": 0,
            "heuristic_kernelName": heur["kernelName"], "heuristic_us": round(heur_us, 3),
            "bad_plans": [r[1] for r in results if r[3] != 0.0], "plans": plans}


def plan_record(M: int, N: int, K: int, name: str, us: float, err: float, model_cycles) -> dict:
    """One --log line: a timed plan with the cost model's estimate (None =
    the model would not offer it; us None = failed the output check)."""
    return {"M": M, "N": N, "K": K, "kernelName": name, "us": round(us, 3) if math.isfinite(us) else None,
            "errRatio": err, "model_cycles": None if model_cycles is None else round(model_cycles, 1)}


def model_report(records: list, margin: float = KEEP_MARGIN) -> dict:
    """How well the cost model ranks plans, from --log records: per shape the
    model's pick (lowest estimate among plans it offers and that passed), the
    measured best, and the regret = pick's time / best time - 1.  Shapes whose
    regret exceeds ``margin`` are listed worst first."""
    shapes: dict = {}
    for r in records:
        if r["us"] is None:
            continue
        shapes.setdefault((r["M"], r["N"], r["K"]), []).append(r)
    per = []
    for key, rs in sorted(shapes.items()):
        best = min(rs, key=lambda r: r["us"])
        offered = [r for r in rs if r["model_cycles"] is not None]
        if not offered:
            continue
        pick = min(offered, key=lambda r: r["model_cycles"])
        per.append({"shape": "x".join(map(str, key)), "model_pick": pick["kernelName"], "pick_us": pick["us"],
                    "best": best["kernelName"], "best_us": best["us"], "regret": pick["us"] / best["us"] - 1.0})
    misses = sorted((p for p in per if p["regret"] > margin), key=lambda p: -p["regret"])
    regrets = [p["regret"] for p in per]
    return {"shapes": len(per), "mean_regret": sum(regrets) / len(regrets) if regrets else 0.0,
            "max_regret": max(regrets, default=0.0), "misses": misses, "per_shape": per}


def write_log(rows: list, path: Path) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    with open(path, "w") as f:
        for r in rows:
            for rec in r.get("plans", []):
                f.write(json.dumps(rec) + "\n")


# ------------------------------------------- sibling families (fack_gemm_tn) --

SIBLING_FAMILIES = ("bf16", "i8")


def sibling_default_shapes() -> list:
    """The decode layer's M sweep at N = 3072, K = 7168 and a large 8192^3 problem."""
    return [(m, 3072, 7168) for m in data.SWEEP_M] + [(8192, 8192, 8192)]


def sibling_candidates(family: str, M: int, N: int, K: int) -> list:
    """Every (tile_m, tile_n, split_k) fack_gemm_tn_plan accepts for the shape:
    tile_m 128 or 256 (a CTA pair), tile_n 64/128/256 dividing N, split-K up to
    min(8, K chunks of 128 bytes), 4 for pairs."""
    chunks = K * (2 if family == "bf16" else 1) // 128
    plans = []
    for tm in (128, 256):
        for tn in (256, 128, 64):
            if N % tn:
                continue
            for sk in range(1, min(8 if tm == 128 else 4, chunks) + 1):
                plans.append((tm, tn, sk))
    return plans


class SiblingShapeBench:
    """Input sets and the reference for one sibling shape: INT8 checked
    bitwise against the exact epilogue ((float(acc) * sa) * sb, each an fp32
    rounding), BF16 within 1e-2 of an fp32 matmul."""

    def __init__(self, family: str, M: int, N: int, K: int, seed: int = 0, launches: int = 24):
        from . import siblings
        self.siblings = siblings
        dev = torch.device("cuda")
        self.family = family
        es = 2 if family == "bf16" else 1
        n_sets = max(1, math.ceil(2.5 * L2_BYTES / ((M + N) * K * es)))
        self.sets = []
        for i in range(n_sets):
            g = torch.Generator(device=dev).manual_seed(seed + i)
            if family == "bf16":
                a = (torch.randn((M, K), generator=g, device=dev) * 0.25).bfloat16()
                b = (torch.randn((N, K), generator=g, device=dev) * 0.25).bfloat16()
                sa = sb = None
            else:
                a = torch.randint(-128, 128, (M, K), generator=g, device=dev, dtype=torch.int8)
                b = torch.randint(-128, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
                sa = 0.001 + 0.01 * torch.rand(M, generator=g, device=dev)
                sb = 0.001 + 0.01 * torch.rand(N, generator=g, device=dev)
            self.sets.append((a, ops.shuffle_weight(b), b, sa, sb))
        a, _, b, sa, sb = self.sets[0]
        self.rows = torch.arange(M, device=dev) if M <= 1024 else torch.linspace(0, M - 1, 512, device=dev).long()
        if family == "bf16":
            prev = torch.backends.cuda.matmul.allow_tf32
            torch.backends.cuda.matmul.allow_tf32 = False
            try:
                self.ref = a[self.rows].float() @ b.float().T
            finally:
                torch.backends.cuda.matmul.allow_tf32 = prev
        else:
            acc = a[self.rows].double() @ b.double().T        # exact: |sum| <= 2^14 * K < 2^53
            self.ref = ((acc.float() * sa[self.rows, None]) * sb[None, :]).bfloat16()
        self.out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        self.launches = max(launches, len(self.sets))

    def call(self, i: int, plan: tuple):
        a, bp, _, sa, sb = self.sets[i % len(self.sets)]
        tm, tn, sk = plan
        self.siblings.gemm_tn(a, bp, self.out, a_scale=sa, b_scale=sb, tile_m=tm, tile_n=tn, split_k=sk)

    def check(self, plan: tuple) -> float:
        self.call(0, plan)
        torch.cuda.synchronize()
        y = self.out[self.rows]
        if self.family == "i8":
            return float((y.view(torch.int16) != self.ref.view(torch.int16)).float().mean())
        return err_ratio(y, self.ref)

    def time_us(self, plan: tuple, repeats: int = 3) -> float:
        return _graph_time(lambda i: self.call(i, plan), len(self.sets), self.launches, repeats)


def tune_sibling_shape(family: str, M: int, N: int, K: int, log=None) -> dict:
    """Time every plan of one sibling shape; the fastest plan that passes wins
    (the cost model's own plan stays when within KEEP_MARGIN of it)."""
    from . import siblings
    kind = siblings.KINDS[torch.bfloat16 if family == "bf16" else torch.int8]
    sb = SiblingShapeBench(family, M, N, K)
    heur = siblings.get_config(kind, M, N, K)
    results, plans = [], []
    for plan in sibling_candidates(family, M, N, K):
        name = siblings.kernel_name(kind, *plan)
        er = sb.check(plan)
        us = sb.time_us(plan) if er == 0.0 else float("inf")
        results.append((us, name, plan[2], er))
        plans.append(plan_record(M, N, K, name, us, er, None))
        if log:
            log(f"  {name:32s} {us:9.2f} us  errRatio {er}")
    best = choose(results, heur["kernelName"], (family, M, N, K))
    heur_row = next((r for r in results if r[1] == heur["kernelName"]), None)
    es = 2 if family == "bf16" else 1
    algo = (M * K + N * K) * es + 2 * M * N + (4 * (M + N) if family == "i8" else 0)
    us = best[0]
    return {"cu_num": torch.cuda.get_device_properties(0).multi_processor_count, "M": M, "N": N, "K": K,
            "kernelName": best[1], "splitK": best[2], "us": round(us, 3),
            "tflops": round(data.flops(M, N, K) / us / 1e6, 1), "bw": round(algo / us / 1e3, 1), "errRatio": 0,
            "heuristic_kernelName": heur["kernelName"],
            "heuristic_us": round(heur_row[0], 3) if heur_row else float("nan"),
            "bad_plans": [r[1] for r in results if r[3] != 0.0], "plans": plans}


def write_csv(rows: list, path: Path, planner: str = "fack_gemm_bs_plan") -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    with open(path, "w", newline="") as f:
        f.write(f"# Exact-shape plans for {planner}, measured on B200 by python -m fack_b200.tune\n")
        w = csv.DictWriter(f, fieldnames=HEADER, extrasaction="ignore")
        w.writeheader()
        for r in sorted(rows, key=lambda r: (r["N"], r["K"], r["M"])):
            w.writerow(r)


def parse_shapes(text: str) -> list:
    out = []
    for part in text.replace(" ", "").split(";"):
        if part:
            m, n, k = (int(v) for v in part.split(","))
            out.append((m, n, k))
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--family", choices=["blockscale", "bf16", "i8", "siblings"], default="blockscale",
                    help="the FP8 block-scaled GEMM (default) or the sibling BF16 / INT8 families (both: siblings)")
    ap.add_argument("--shapes", default="", help="M,N,K;M,N,K... (default: the tuned workloads)")
    ap.add_argument("--out", default="", help="table to write (default: the family's table in configs/)")
    ap.add_argument("--log", default="", help="write every timed plan with the cost model's estimate (JSONL)")
    ap.add_argument("--report", default="", help="summarise a --log file (the model's regret per shape; no GPU)")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args(argv)
    if args.report:
        records = [json.loads(ln) for ln in Path(args.report).read_text().splitlines() if ln.strip()]
        rep = model_report(records)
        print(json.dumps({k: rep[k] for k in ("shapes", "mean_regret", "max_regret", "misses")}, indent=1))
        return 0
    if not torch.cuda.is_available():
        print("tune: needs a CUDA device", file=sys.stderr)
        return 2
    lib = _lib.load()
    sibling = args.family != "blockscale"
    # time the cost model's plans, not an older table's
    (lib.fack_gemm_tn_tuned_clear if sibling else lib.fack_gemm_bs_tuned_clear)()
    out = args.out or str(_lib.TN_TUNED_TABLE if sibling else _lib.TUNED_TABLE)
    if sibling:
        families = SIBLING_FAMILIES if args.family == "siblings" else (args.family,)
        shapes = parse_shapes(args.shapes) if args.shapes else sibling_default_shapes()
        jobs = [(fam, s) for fam in families for s in shapes]
    else:
        jobs = [(None, s) for s in (parse_shapes(args.shapes) if args.shapes else default_shapes())]
    rows = []
    log = (lambda s: print(s, file=sys.stderr, flush=True)) if args.verbose else None
    for fam, (M, N, K) in jobs:
        row = tune_sibling_shape(fam, M, N, K, log) if fam else tune_shape(M, N, K, log)
        rows.append(row)
        print(json.dumps({k: row[k] for k in ("M", "N", "K", "kernelName", "us", "heuristic_kernelName",
                                              "heuristic_us", "bad_plans")}), flush=True)
        torch.cuda.empty_cache()
    write_csv(rows, Path(out), "fack_gemm_tn_plan" if sibling else "fack_gemm_bs_plan")
    if args.log:
        write_log(rows, Path(args.log))
    bad = sum(len(r["bad_plans"]) for r in rows)
    print(json.dumps({"rows": len(rows), "out": out, "plans_failing_check": bad}))
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
