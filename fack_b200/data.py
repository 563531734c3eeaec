"""Block quantisation and the seeded synthetic workloads of the benchmark configs.

Quantisation (per the benchmark construction): activations get one fp32 scale
per token per 128-wide K group, weights one per 128x128 block, each
``scale = amax / 240`` and ``q = cast_e4m3fn(v / scale)``.  With |q| <= 240
every code is exactly representable both in e4m3fn (B200) and in the
reference's e4m3fnuz (gfx942), so the same bytes mean the same numbers on both.

Workloads (name -> shape, distribution), all seeded:

* ``plumbing``  M=32,  N=8192,  K=7168; X~N(0,1), W~N(0,0.02)
* ``decode``    M=256, N=3072,  K=7168; same distributions
* ``sweep``     N=3072, K=7168, M in SWEEP_M; same distributions
* ``prefill``   M=8192, N=7168, K=16384; X~N(0,1) with 0.1% entries x50, W~N(0,0.02)
* ``wide``      M=32, N=65536, K=7168; X all ones ("constant") or U(-1,1)
  ("uniform"), W~U(-0.05,0.05) quantised per block, then every block scale
  replaced by 2^u, u~U(-12,2)

Generation runs on whatever device the generator lives on (CPU for fixtures
and the oracle, the GPU for the benchmark's large inputs).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

FP8 = torch.float8_e4m3fn
QMAX = 240.0
BLOCK = 128
SWEEP_M = (1, 16, 32, 144, 208, 224, 240, 288, 320, 480, 512)


@dataclass(frozen=True)
class Workload:
    name: str
    M: int
    N: int
    K: int
    x_dist: str = "normal"       # normal | outlier | constant | uniform
    w_dist: str = "normal"       # normal | uniform_logscale


WORKLOADS = {
    "plumbing": Workload("plumbing", 32, 8192, 7168),
    "decode": Workload("decode", 256, 3072, 7168),
    "prefill": Workload("prefill", 8192, 7168, 16384, "outlier", "normal"),
    "wide_constant": Workload("wide_constant", 32, 65536, 7168, "constant", "uniform_logscale"),
    "wide_uniform": Workload("wide_uniform", 32, 65536, 7168, "uniform", "uniform_logscale"),
}
for _m in SWEEP_M:
    WORKLOADS[f"sweep_m{_m}"] = Workload(f"sweep_m{_m}", _m, 3072, 7168)

# Workloads whose output columns are sharded over the GPUs of one node
# (rank r computes Y[:, r*N/g : (r+1)*N/g]); the others run as replicas.
SHARDED = ("prefill", "wide_constant", "wide_uniform")
SHARD_COUNTS = (2, 4, 8)


def shard_shapes() -> list:
    """(M, N/g, K) of one rank's GEMM for every sharded workload and g in SHARD_COUNTS."""
    out = []
    for name in SHARDED:
        wl = WORKLOADS[name]
        for g in SHARD_COUNTS:
            if wl.N % (BLOCK * g) == 0 and (wl.M, wl.N // g, wl.K) not in out:
                out.append((wl.M, wl.N // g, wl.K))
    return out


def _safe_scale(amax: torch.Tensor) -> torch.Tensor:
    s = amax / QMAX
    return torch.where(amax > 0, s, torch.ones_like(s))


def quantize_act(x: torch.Tensor):
    """fp32 [M,K] -> (e4m3 [M,K], fp32 x_scale [M,K/128]) per token per 128-K group."""
    M, K = x.shape
    g = x.reshape(M, K // BLOCK, BLOCK)
    scale = _safe_scale(g.abs().amax(dim=2))
    q = (g / scale.unsqueeze(2)).clamp(-QMAX, QMAX).to(FP8)
    return q.reshape(M, K), scale.contiguous()


def quantize_weight(w: torch.Tensor):
    """fp32 [N,K] -> (e4m3 [N,K], fp32 w_scale [N/128,K/128]) per 128x128 block."""
    N, K = w.shape
    b = w.reshape(N // BLOCK, BLOCK, K // BLOCK, BLOCK)
    scale = _safe_scale(b.abs().amax(dim=(1, 3)))
    q = (b / scale[:, None, :, None]).clamp(-QMAX, QMAX).to(FP8)
    return q.reshape(N, K), scale.contiguous()


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def make_activations(M: int, K: int, dist: str, seed: int, device="cpu", chunk_rows: int = 2048):
    g = _gen(seed, device)
    xq = torch.empty((M, K), dtype=FP8, device=device)
    xs = torch.empty((M, K // BLOCK), dtype=torch.float32, device=device)
    for r0 in range(0, M, chunk_rows):
        r1 = min(M, r0 + chunk_rows)
        shape = (r1 - r0, K)
        if dist == "normal":
            x = torch.randn(shape, generator=g, device=device)
        elif dist == "outlier":
            x = torch.randn(shape, generator=g, device=device)
            hit = torch.rand(shape, generator=g, device=device) < 1e-3
            x = torch.where(hit, x * 50.0, x)
        elif dist == "constant":
            x = torch.ones(shape, device=device)
        elif dist == "uniform":
            x = torch.rand(shape, generator=g, device=device) * 2.0 - 1.0
        else:
            raise ValueError(f"unknown activation distribution {dist!r}")
        xq[r0:r1], xs[r0:r1] = quantize_act(x)
    return xq, xs


def make_weights(N: int, K: int, dist: str, seed: int, device="cpu", chunk_rows: int = 2048):
    g = _gen(seed, device)
    wq = torch.empty((N, K), dtype=FP8, device=device)
    ws = torch.empty((N // BLOCK, K // BLOCK), dtype=torch.float32, device=device)
    chunk_rows = max(BLOCK, chunk_rows // BLOCK * BLOCK)
    for r0 in range(0, N, chunk_rows):
        r1 = min(N, r0 + chunk_rows)
        shape = (r1 - r0, K)
        if dist == "normal":
            w = torch.randn(shape, generator=g, device=device) * 0.02
            q, s = quantize_weight(w)
        elif dist == "uniform_logscale":
            w = (torch.rand(shape, generator=g, device=device) * 2.0 - 1.0) * 0.05
            q, _ = quantize_weight(w)
            u = torch.rand(((r1 - r0) // BLOCK, K // BLOCK), generator=g, device=device) * 14.0 - 12.0
            s = torch.exp2(u)
        else:
            raise ValueError(f"unknown weight distribution {dist!r}")
        wq[r0:r1], ws[r0 // BLOCK:r1 // BLOCK] = q, s
    return wq, ws


def make_inputs(wl: Workload, seed: int = 0, device="cpu", M: Optional[int] = None):
    """(XQ, x_scale, WQ, w_scale) for a workload; x_scale is logical row-major.

    Activations use ``seed`` and weights ``seed + 1``, so shapes that share N
    and K (the decode sweep) share their weights."""
    m = wl.M if M is None else M
    xq, xs = make_activations(m, wl.K, wl.x_dist, seed, device)
    wq, ws = make_weights(wl.N, wl.K, wl.w_dist, seed + 1, device)
    return xq, xs, wq, ws


def to_aiter_xscale(x_scale: torch.Tensor) -> torch.Tensor:
    """Logical [M,K/128] -> the reference's transposed-contiguous view
    (``sa.T.contiguous().view_as(sa)``, client/aiter/hsa/gfx942/driver.py:22)."""
    return x_scale.t().contiguous().view(x_scale.shape)


def algorithmic_bytes(M: int, N: int, K: int) -> int:
    """Bytes a GEMM call must move at minimum: XQ + WQ + scales + Y (bf16)."""
    return M * K + N * K + 4 * M * (K // BLOCK) + 4 * (N // BLOCK) * (K // BLOCK) + 2 * M * N


def flops(M: int, N: int, K: int) -> int:
    """2*M*N*K, the reference's FLOP count (client/aiter/hsa/gfx942/driver.py:34)."""
    return 2 * M * N * K
