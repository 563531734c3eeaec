"""Throughput of the fused activation quantisation (``fack_quant_act``).

``python -m fack_b200.quant_bench`` prints one JSON line per shape: the
activation shapes of the prefill (8192 x 16384) and decode (256 x 7168)
configs, fp32 and bf16 input.  Timing: CUDA-graph replay of many launches,
CUDA events on the launch stream, inputs rotated over more than twice the
126 MB L2.  Algorithmic bytes per launch = M*K*(input bytes + 1) (read X,
write the codes) + 4*M*K/128 (scales); the roofline is the measured HBM copy
bandwidth in MEASURED_PEAKS.json.
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import torch

from . import ops

L2_BYTES = 126e6


def _hbm_gbs() -> tuple:
    p = Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measure(M: int, K: int, dtype: torch.dtype, launches: int = 200) -> dict:
    dev = torch.device("cuda")
    in_bytes = torch.finfo(dtype).bits // 8
    algo = M * K * (in_bytes + 1) + 4 * M * K // 128
    sets = max(1, math.ceil(2.5 * L2_BYTES / algo))
    xs = [torch.randn((M, K), device=dev).to(dtype) for _ in range(sets)]
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for x in xs:
            ops.quantize_activations(x)
    torch.cuda.synchronize()
    reps = max(launches, sets)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(reps):
            ops.quantize_activations(xs[i % sets])
    with torch.cuda.stream(stream):
        g.replay()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        g.replay()
        end.record(stream)
    end.synchronize()
    us = start.elapsed_time(end) * 1e3 / reps
    peak, src = _hbm_gbs()
    gbs = algo / (us * 1e3)
    g.reset()
    return {"op": "fack_quant_act", "M": M, "K": K, "dtype": str(dtype).replace("torch.", ""),
            "us_per_call": round(us, 3), "algorithmic_bytes": algo, "achieved_gbs": round(gbs, 1),
            "peak_gbs": peak, "peak_source": src, "frac": round(gbs / peak, 4), "input_sets": sets}


def main() -> None:
    for M, K in ((8192, 16384), (256, 7168)):
        for dtype in (torch.float32, torch.bfloat16):
            print(json.dumps(measure(M, K, dtype)), flush=True)


if __name__ == "__main__":
    main()
