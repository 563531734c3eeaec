"""CPU oracle for the FP8 block-scaled GEMM -- test infrastructure only.

This module is the checker.  Only the tests, the smoke check and the
benchmark's CPU-baseline / reference arm may import it; the product path
(fack_b200) never does, and has no CPU fallback.

It restates the reference's own fp32 oracle,
client/aiter/hsa/gfx942/driver.py:18-20:

    reference = ((a.float() * sa.repeat_interleave(128, dim=1)) @
                 (b.float() * sb.repeat_interleave(128, dim=0).repeat_interleave(128, dim=1)).T
                ).bfloat16()

i.e. dequantise both e4m3 operands with their fp32 block scales, one fp32
matmul, round to bf16.  ``sa`` is the LOGICAL row-major [M, K/128] scale (the
driver keeps it that way for its reference, driver.py:31-33), ``sb`` the
[N/128, K/128] block scale.

Pinned against golden vectors produced by executing the reference's own
``prepare()`` (tests/golden/make_golden.py), so this restatement is checked
bit-for-bit against the reference code on the reference's input construction.
"""
from __future__ import annotations

import torch

BLOCK = 128


def dequant_act(xq: torch.Tensor, x_scale: torch.Tensor) -> torch.Tensor:
    """a.float() * sa.repeat_interleave(128, dim=1)  (driver.py:19)."""
    return xq.float() * x_scale.repeat_interleave(BLOCK, dim=1)


def dequant_weight(wq: torch.Tensor, w_scale: torch.Tensor) -> torch.Tensor:
    """b.float() * sb.repeat_interleave(128, 0).repeat_interleave(128, 1)  (driver.py:20)."""
    return wq.float() * w_scale.repeat_interleave(BLOCK, dim=0).repeat_interleave(BLOCK, dim=1)


def reference_gemm(xq: torch.Tensor, wq: torch.Tensor, x_scale: torch.Tensor,
                   w_scale: torch.Tensor) -> torch.Tensor:
    """bf16 [M,N] = (dequant(XQ) @ dequant(WQ).T).bfloat16(), fp32 on the CPU."""
    xq, wq, x_scale, w_scale = (t.cpu() for t in (xq, wq, x_scale, w_scale))
    return (dequant_act(xq, x_scale) @ dequant_weight(wq, w_scale).T).bfloat16()


def reference_gemm_rows(xq, wq, x_scale, w_scale, rows) -> torch.Tensor:
    """The same formula for a subset of output rows (for large shapes)."""
    rows = torch.as_tensor(rows, dtype=torch.long)
    return reference_gemm(xq.cpu()[rows], wq, x_scale.cpu()[rows], w_scale)


def exact_gemm_f64(xq, wq, x_scale, w_scale) -> torch.Tensor:
    """float64 [M,N] of the same expression, unrounded (error analysis only)."""
    xq, wq, x_scale, w_scale = (t.cpu() for t in (xq, wq, x_scale, w_scale))
    a = xq.double() * x_scale.double().repeat_interleave(BLOCK, dim=1)
    b = wq.double() * w_scale.double().repeat_interleave(BLOCK, dim=0).repeat_interleave(BLOCK, dim=1)
    return a @ b.T


def unpack_aiter_xscale(packed_sa: torch.Tensor) -> torch.Tensor:
    """Logical [M,K/128] scales from the reference's transposed-contiguous view
    (inverse of ``sa.T.contiguous().view_as(sa)``, driver.py:22)."""
    M, KB = packed_sa.shape
    return packed_sa.contiguous().view(KB, M).t().contiguous()


QMAX = 240.0


def quantize_activations_ref(x: torch.Tensor):
    """(XQ e4m3 [M,K], logical x_scale fp32 [M,K/128]) from fp32 or bf16 X.

    The activation construction of the benchmark workloads ("quantised per
    row per 128-K group with x_scale = amax/240"): per token
    and 128-wide K group, scale = amax(|x|)/240 (1 for an all-zero group),
    code = e4m3fn(clamp(x/scale, -240, 240)) rounded to nearest even; bf16
    input is widened to fp32 first.  The reference takes X already quantised
    (client/aiter/hsa/gfx942/driver.py:14-17); this restates the step before
    its GEMM, which fack_quant_act fuses into one kernel.
    """
    x = x.float().cpu()
    M, K = x.shape
    g = x.reshape(M, K // BLOCK, BLOCK)
    amax = g.abs().amax(dim=2)
    scale = torch.where(amax > 0, amax / QMAX, torch.ones_like(amax))
    q = (g / scale.unsqueeze(2)).clamp(-QMAX, QMAX).to(torch.float8_e4m3fn)
    return q.reshape(M, K), scale.contiguous()
