"""torchrun worker for tests/test_dist_gpu.py (one process per GPU, NCCL)."""
import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    import fack_b200 as fb
    from fack_b200 import data
    from fack_b200.dist import ShardedBlockscaleGemm, shard_bounds, shard_weight
    ok = True
    for (M, N, K, xd, wd) in ((32, 8192, 1024, "uniform", "uniform_logscale"), (300, 2048, 768, "outlier", "normal")):
        xq, xs = data.make_activations(M, K, xd, seed=1, device=dev)
        wq, ws = data.make_weights(N, K, wd, seed=2, device=dev)
        full = fb.gemm_blockscale(xq, wq, xs, ws)                 # unsharded, on this GPU
        wq_r, ws_r = shard_weight(wq, ws, rank, world)
        gemm = ShardedBlockscaleGemm()
        y = gemm(xq, fb.shuffle_weight(wq_r), xs, ws_r)
        torch.cuda.synchronize()
        for r in range(world):                                     # each slice == that rank's local GEMM
            n0, n1 = shard_bounds(N, world, r)
            wr, sr = shard_weight(wq, ws, r, world)
            local_r = fb.gemm_blockscale(xq, wr, xs, sr)
            ok &= torch.equal(y[:, n0:n1].view(torch.int16), local_r.view(torch.int16))
        ok &= bool(torch.allclose(y.float(), full.float(), rtol=1e-2, atol=1e-2))
        ok &= fb.device_status() == 0
        # fused: the GEMM's epilogue stores into every rank's Y over NVLink
        fused = ShardedBlockscaleGemm(mode="fused")
        y_f = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
        for _ in range(2):                                         # registered once, reused
            fused(xq, fb.shuffle_weight(wq_r), xs, ws_r, out=y_f)
            torch.cuda.synchronize()
            ok &= torch.equal(y_f.view(torch.int16), y.view(torch.int16))
            y_f.fill_(float("nan"))
            dist.barrier()
        fused.close()
        ok &= fb.device_status() == 0
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    if rank == 0:
        print("DIST_GPU_OK" if flag.item() == 1 else "DIST_GPU_FAIL", flush=True)
    sys.exit(0 if flag.item() == 1 else 1)


if __name__ == "__main__":
    main()
