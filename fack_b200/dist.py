"""N-sharded (column-parallel) blockscale GEMM over several GPUs.

The reference runs one GPU per process and has no collective
(client/aiter/docs/validation.md:42-46).  For the wide and prefill layers this
library shards the output columns: rank r owns WQ rows [r*N/g, (r+1)*N/g) and
the matching w_scale rows, the activations are replicated, each rank computes
its [M, N/g] block with the single-GPU kernel straight into its slot of a
[g, M, N/g] gather buffer, an in-place all-gather (NCCL over NVLink) fills the
other slots, and a column-interleave kernel assembles row-major Y[M, N].

Only the bf16 output crosses NVLink; N/g stays a multiple of 128, so every
shard is made of whole 128x128 weight-scale blocks.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

BLOCK = 128


def shard_bounds(N: int, world: int, rank: int):
    """Column range [n0, n1) owned by `rank`; N must split into whole 128-blocks."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    if N % (BLOCK * world):
        raise ValueError(f"N={N} does not split into {world} shards of whole 128-column blocks")
    ns = N // world
    return rank * ns, (rank + 1) * ns


def shard_weight(wq: torch.Tensor, w_scale: torch.Tensor, rank: int, world: int):
    """This rank's (WQ rows, w_scale rows) of a full weight."""
    n0, n1 = shard_bounds(wq.shape[0], world, rank)
    return wq[n0:n1].contiguous(), w_scale[n0 // BLOCK:n1 // BLOCK].contiguous()


def _default_local_gemm(xq, wq, x_scale, w_scale, out):
    from .ops import gemm_blockscale
    return gemm_blockscale(xq, wq, x_scale, w_scale, out=out)


def _default_interleave(gathered, out):
    from .ops import gather_interleave
    return gather_interleave(gathered, out)


class ShardedBlockscaleGemm:
    """Y[M, N] = blockscale(XQ, WQ) with WQ column-sharded over a process group.

    ``local_gemm(xq, wq_shard, x_scale, ws_shard, out)`` and
    ``interleave(gathered, out)`` default to this library's CUDA kernels; the
    CPU tests substitute checkers to exercise the sharding and gather logic
    on gloo ranks.
    """

    def __init__(self, group=None, local_gemm: Optional[Callable] = None,
                 interleave: Optional[Callable] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.local_gemm = local_gemm or _default_local_gemm
        self.interleave = interleave or _default_interleave
        self._gather = None

    def gather_buffer(self, M: int, ns: int, device) -> torch.Tensor:
        g = self._gather
        if g is None or g.shape != (self.world, M, ns) or g.device != torch.device(device):
            if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
                raise RuntimeError("gather buffer must be sized before CUDA-graph capture")
            g = torch.empty((self.world, M, ns), dtype=torch.bfloat16, device=device)
            self._gather = g
        return g

    def __call__(self, xq, wq_shard, x_scale, ws_shard, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        M = xq.shape[0]
        ns = wq_shard.shape[0]
        if ns % BLOCK:
            raise ValueError("weight shard must hold whole 128-row blocks")
        gathered = self.gather_buffer(M, ns, xq.device)
        mine = gathered[self.rank]
        self.local_gemm(xq, wq_shard, x_scale, ws_shard, mine)
        if self.world > 1:
            if dist.get_backend(self.group) == "nccl":
                # in place: this rank's input is its own slot of the output
                dist.all_gather_into_tensor(gathered.view(-1), mine.view(-1), group=self.group)
            else:
                dist.all_gather(list(gathered.unbind(0)), mine.clone(), group=self.group)
        if out is None:
            out = torch.empty((M, self.world * ns), dtype=torch.bfloat16, device=xq.device)
        self.interleave(gathered, out)
        return out
