"""Run one FP8 block-scaled GEMM shape a few times: the case driver of ncu
captures and quick checks.

``python -m fack_b200.case_bench M N K [--calls C] [--x-dist D] [--plan TM,TN,S]``

Synthetic inputs of the benchmark construction (seeded; scale = amax/240)
rotate over enough input sets to exceed 2.5 x the 126 MB L2 (one set when a
set alone is larger).  Three warm-up calls, then ``--calls`` more, each through
the reference's call form (``gemm_a8w8_blockscale_bpreshuffle_asm``:
pre-packed weight, transposed x_scale) with the library's plan for the shape,
or the plan ``--plan`` fixes (token tile, weight tile, split-K) -- e.g. to
profile the persistent kernel on a smaller case than the workload it serves.
Eager launches (no graph), so a profiler sees each one; prints the plan and the
device status word.
"""
from __future__ import annotations

import argparse
import math
import sys

import torch


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("M", type=int)
    ap.add_argument("N", type=int)
    ap.add_argument("K", type=int)
    ap.add_argument("--calls", type=int, default=2, help="calls after the three warm-up calls")
    ap.add_argument("--x-dist", default="normal", choices=["normal", "outlier", "constant", "uniform"])
    ap.add_argument("--plan", default="", help="tile_m,tile_n,split_k (default: the library's plan)")
    args = ap.parse_args(argv)
    if not torch.cuda.is_available():
        print("case_bench: needs a CUDA device", file=sys.stderr)
        return 2
    from . import data, ops
    M, N, K = args.M, args.N, args.K
    dev = torch.device("cuda", torch.cuda.current_device())
    per_set = data.algorithmic_bytes(M, N, K)
    n_sets = max(1, math.ceil(2.5 * 126e6 / per_set))
    sets = []
    for i in range(n_sets):
        xq, xs = data.make_activations(M, K, args.x_dist, seed=2 * i, device=dev)
        wq, ws = data.make_weights(N, K, "normal", seed=2 * i + 1, device=dev)
        sets.append((xq, ops.shuffle_weight(wq), data.to_aiter_xscale(xs), ws,
                     torch.empty((M, N), dtype=torch.bfloat16, device=dev)))
        del wq
    if args.plan:
        tm, tn, sk = (int(v) for v in args.plan.split(","))
        name, split = ops.kernel_name(tm, tn, sk), sk
    else:
        cfg = ops.get_config(M, N, K)
        name, split = cfg["kernelName"], cfg["splitK"]
    for i in range(3 + args.calls):
        xq, b, sa, ws, out = sets[i % n_sets]
        ops.gemm_a8w8_blockscale_bpreshuffle_asm(xq, b, out, sa, ws, None, split, name, True)
    torch.cuda.synchronize()
    status = ops.device_status()
    print(f"{M}x{N}x{K} plan {name}: {3 + args.calls} calls over {n_sets} input sets, device status {status:#x}")
    return 1 if status else 0


if __name__ == "__main__":
    sys.exit(main())
