"""torchrun worker for tests/test_dist_gpu.py (one process per GPU, NCCL).

For every case each rank holds its column shard of the weights, and both
exchange modes assemble the replicated Y[M, N]:

* ``nccl``: local GEMM into this rank's slot, NCCL all-gather, interleave;
* ``fused``: the GEMM's epilogue stores every tile into every rank's Y over
  NVLink and the launch completes once every rank's block has landed
  (three calls over two alternating outputs, then the same output twice in a
  row, which adds one exchange step).

Checks on every rank: each column block of Y is bitwise the unsharded GPU
kernel run on that rank's shard; the fused Y is bitwise the NCCL Y; sampled
rows x one 128-column block of every rank's shard agree with the CPU oracle
(the reference's fp32 dequantise-then-matmul) within rtol = atol = 1e-2; no
device status flag is set.  Rank 0 prints one JSON line per case (plans,
timings of one fused call) and DIST_GPU_OK / DIST_GPU_FAIL.
"""
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

RTOL = ATOL = 1e-2

# (name, M, N, K, x distribution, w distribution, rows sampled for the oracle)
CASES = [
    ("small_wide", 32, 8192, 1024, "uniform", "uniform_logscale", 32),
    ("tiny_m", 5, 4096, 2048, "normal", "normal", 5),          # the warp-MMA small-M kernel with peers
    ("small_ragged", 300, 2048, 768, "outlier", "normal", 300),
    ("prefill", 8192, 7168, 16384, "outlier", "normal", 24),
    ("wide_constant", 32, 65536, 7168, "constant", "uniform_logscale", 32),
    ("wide_uniform", 32, 65536, 7168, "uniform", "uniform_logscale", 32),
]


def oracle_sample(xq, xs, wq, ws, rows, n0):
    """The oracle on rows x columns [n0, n0 + 128) (host copies of the inputs)."""
    from oracle.blockscale import reference_gemm
    return reference_gemm(xq[rows].cpu(), wq[n0:n0 + 128].cpu(), xs[rows].cpu(), ws[n0 // 128:n0 // 128 + 1].cpu())


def run_case(name, M, N, K, xd, wd, n_rows, rank, world, dev):
    import fack_b200 as fb
    from fack_b200 import data
    from fack_b200.dist import ShardedBlockscaleGemm, shard_bounds, shard_weight
    ok = True
    why = []
    xq, xs = data.make_activations(M, K, xd, seed=1, device=dev)
    wq, ws = data.make_weights(N, K, wd, seed=2, device=dev)
    wq_r, ws_r = shard_weight(wq, ws, rank, world)
    packed_r = fb.shuffle_weight(wq_r)
    ns = N // world
    cfg = fb.get_config(M, ns, K)

    # NCCL all-gather + interleave
    gemm = ShardedBlockscaleGemm()
    y = gemm(xq, packed_r, xs, ws_r)
    torch.cuda.synchronize()
    # each column block is that rank's unsharded local GEMM, bit for bit
    for r in range(world):
        n0, n1 = shard_bounds(N, world, r)
        wr, sr = shard_weight(wq, ws, r, world)
        local_r = fb.gemm_blockscale(xq, wr, xs, sr)
        if not torch.equal(y[:, n0:n1].view(torch.int16), local_r.view(torch.int16)):
            ok = False
            why.append(f"nccl block {r} differs from rank {r}'s local GEMM")
        del wr, sr, local_r

    # fused: alternating outputs, then one output twice in a row
    fused = ShardedBlockscaleGemm(mode="fused")
    outs = [torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    times = []
    for i, o in enumerate((0, 1, 0, 0)):
        outs[o].fill_(float("nan"))
        dist.barrier()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        fused(xq, packed_r, xs, ws_r, out=outs[o])
        t1.record()
        t1.synchronize()
        times.append(t0.elapsed_time(t1) * 1e3)
        if not torch.equal(outs[o].view(torch.int16), y.view(torch.int16)):
            ok = False
            bad = (outs[o].view(torch.int16) != y.view(torch.int16)).sum().item()
            why.append(f"fused call {i}: {bad} elements differ from the NCCL result")
    if fused.barriers != 1:
        ok = False
        why.append(f"fused path ran {fused.barriers} extra exchange steps, expected 1")
    dist.barrier()
    fused.close()

    # the oracle on sampled rows x one 128-column block of every rank's shard
    g = torch.Generator().manual_seed(1000 + world)
    rows = torch.randperm(M, generator=g)[:n_rows].sort().values
    worst = 0.0
    for r in range(world):
        n0, _ = shard_bounds(N, world, r)
        blk = n0 + 128 * int(torch.randint(0, ns // 128, (1,), generator=g))
        ref = oracle_sample(xq, xs, wq, ws, rows, blk).float()
        got = y[rows.to(dev)][:, blk:blk + 128].float().cpu()
        if not torch.isfinite(got).all() or not torch.allclose(got, ref, rtol=RTOL, atol=ATOL):
            ok = False
            why.append(f"rank {r}'s block at column {blk} differs from the oracle "
                       f"(max abs {float((got - ref).abs().max()):.4g})")
        worst = max(worst, float(((got - ref).abs() / (ATOL + RTOL * ref.abs())).max()))
    if fb.device_status() != 0:
        ok = False
        why.append("device status flags set")
    # every rank's plan, gathered to rank 0
    plans = [None] * world
    dist.all_gather_object(plans, cfg["kernelName"])
    rec = {"case": name, "M": M, "N": N, "K": K, "x": xd, "w": wd, "world": world, "ok": ok,
           "plans": plans, "fused_call_us": [round(t, 1) for t in times],
           "oracle_rows": int(n_rows), "oracle_worst_err_over_tol": round(worst, 4), "why": why}
    del xq, xs, wq, ws, wq_r, ws_r, packed_r, y, outs
    torch.cuda.empty_cache()
    return ok, rec


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    only = os.environ.get("FACK_DIST_CASES")
    ok = True
    for case in CASES:
        if only and case[0] not in only.split(","):
            continue
        if case[2] % (128 * world):
            continue
        c_ok, rec = run_case(*case, rank, world, dev)
        flags = [None] * world
        dist.all_gather_object(flags, rec)
        if rank == 0:
            for r, f in enumerate(flags):
                if not f["ok"]:
                    print(f"rank {r}: {f['why']}", flush=True)
            rec["ok"] = all(f["ok"] for f in flags)
            print("DIST_CASE " + json.dumps(rec), flush=True)
        ok &= all(f["ok"] for f in flags)
        dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("DIST_GPU_OK" if ok else "DIST_GPU_FAIL", flush=True)
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
