"""Throughput of the sibling GEMM families (``fack_gemm_tn``).

``python -m fack_b200.sibling_bench`` prints one JSON line per (family,
shape): microseconds per call (CUDA-graph replay, CUDA events on the launch
stream, operand sets rotated over more than 2.5 x the 126 MB L2), TFLOP/s
against the measured dense bf16 peak in MEASURED_PEAKS.json (the INT8 tensor
rate is twice that on B200), algorithmic GB/s against the measured HBM
copy bandwidth, and for context the same GEMM through torch's library path
(``torch.matmul`` for bf16, ``torch._int_mm`` for int8 without the epilogue).
Shapes: the decode layer 256 x 3072 x 7168 (bandwidth-bound) and a large
8192 x 8192 x 8192 problem (tensor-bound).
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import torch

from . import ops, siblings

L2_BYTES = 126e6


def _peaks() -> dict:
    p = Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def _time(fn, sets: int, launches: int) -> float:
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(sets):
            fn(i)
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(launches):
            fn(i % sets)
    with torch.cuda.stream(stream):
        g.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        g.replay()
        b.record(stream)
    b.synchronize()
    g.reset()
    return a.elapsed_time(b) * 1e3 / launches


def measure(family: str, M: int, N: int, K: int) -> dict:
    dev = torch.device("cuda")
    es = 2 if family == "bf16" else 1
    algo = (M * K + N * K) * es + 2 * M * N + (4 * (M + 2 * N) if family == "i8" else 0)
    sets = max(1, math.ceil(2.5 * L2_BYTES / ((M + N) * K * es)))
    data = []
    for i in range(sets):
        g = torch.Generator(device=dev).manual_seed(i)
        if family == "bf16":
            a = (torch.randn((M, K), generator=g, device=dev) * 0.25).bfloat16()
            b = (torch.randn((N, K), generator=g, device=dev) * 0.25).bfloat16()
            data.append((a, ops.shuffle_weight(b), b, None, None, torch.empty((M, N), dtype=torch.bfloat16, device=dev)))
        else:
            a = torch.randint(-16, 17, (M, K), generator=g, device=dev, dtype=torch.int8)
            b = torch.randint(-16, 17, (N, K), generator=g, device=dev, dtype=torch.int8)
            sa = 0.02 + 0.03 * torch.rand((M, 1), generator=g, device=dev)
            sb = 0.02 + 0.03 * torch.rand((N, 1), generator=g, device=dev)
            data.append((a, ops.shuffle_weight(b), b, sa, sb, torch.empty((M, N), dtype=torch.bfloat16, device=dev)))
    cfg = siblings.get_config(siblings.KINDS[torch.bfloat16 if family == "bf16" else torch.int8], M, N, K)

    def ours(i):
        a, bp, _, sa, sb, out = data[i]
        if family == "bf16":
            siblings.gemm_a16w16_asm(a, bp, out, bpreshuffle=True)
        else:
            siblings.gemm_a8w8_asm(a, bp, sa, sb, out)

    def library(i):
        a, _, b, _, _, _ = data[i]
        if family == "bf16":
            torch.matmul(a, b.T)
        else:
            torch._int_mm(a, b.T)

    launches = max(20, sets)
    us = _time(ours, sets, launches)
    try:
        lib_us = round(_time(library, sets, launches), 3)
    except RuntimeError as e:  # the library path may not take this shape / layout
        lib_us = f"unavailable: {str(e).splitlines()[0][:80]}"
    pk = _peaks()
    tensor_peak = pk["bf16_tflops"] * (1 if family == "bf16" else 2)
    tflops = 2.0 * M * N * K / us / 1e6
    gbs = algo / us / 1e3
    return {"op": f"fack_gemm_tn/{family}", "M": M, "N": N, "K": K, "kernelName": cfg["kernelName"],
            "us_per_call": round(us, 3), "tflops": round(tflops, 1),
            "tensor_peak_tflops": tensor_peak, "tensor_frac": round(tflops / tensor_peak, 4),
            "algorithmic_bytes": algo, "achieved_gbs": round(gbs, 1), "hbm_frac": round(gbs / pk["hbm_gbs"], 4),
            "peak_source": pk["source"], "library_us": lib_us,
            "library_path": "torch.matmul" if family == "bf16" else "torch._int_mm (s32 out, no epilogue)",
            "input_sets": sets}


def main() -> None:
    for family in ("bf16", "i8"):
        for M, N, K in ((256, 3072, 7168), (8192, 8192, 8192)):
            print(json.dumps(measure(family, M, N, K)), flush=True)


if __name__ == "__main__":
    main()
