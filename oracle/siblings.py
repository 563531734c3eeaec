"""CPU oracle for the sibling GEMM families -- test infrastructure only.

Only the tests and the benchmark's CPU legs may import it; the product path
(fack_b200) never does.

Restates the references of the reference's sibling driver,
client/aiter/hsa/gfx942/gemm_driver.py:

* BF16 TN (line 50): ``(a.float() @ b.float().T).bfloat16()``;
* INT8 per token (line 73):
  ``((a.float() @ b.float().T) * sa * sb.T + bias).bfloat16()`` with
  ``sa`` [M, 1], ``sb`` [N, 1] and ``bias`` [1, N] fp32.  The integer sum is
  formed exactly (int64) and rounded once to fp32, which equals the
  reference's fp32 matmul whenever that one is exact -- the driver's inputs
  (|values| <= 16) guarantee it (gemm_driver.py:60, :66, :69).

Pinned by tests/golden/make_golden_siblings.py, which runs the driver's own
``prepare()`` and keeps its references.
"""
from __future__ import annotations

from typing import Optional

import torch


def reference_bf16_tn(a: torch.Tensor, b: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bf16 [M, N] = (A.float() @ B.float().T (+ bias)).bfloat16() on the CPU."""
    y = a.cpu().float() @ b.cpu().float().T
    if bias is not None:
        y = y + bias.cpu().float().reshape(1, -1)
    return y.bfloat16()


def exact_i8_sum(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """int64 [M, N] = A . B^T, exact: formed in float64, where every product
    (|p| <= 2^14) and every partial sum of fewer than 2^39 of them is an
    integer below 2^53, so no rounding occurs."""
    if a.shape[1] >= 1 << 39:
        raise ValueError("K too large for an exact float64 sum")
    return (a.cpu().double() @ b.cpu().double().T).to(torch.int64)


def reference_i8_per_token(a: torch.Tensor, b: torch.Tensor, sa: torch.Tensor, sb: torch.Tensor,
                           bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bf16 [M, N] = ((float(A . B^T) * sa) * sb (+ bias)).bfloat16(), every
    step rounded in fp32 in the reference's order."""
    y = exact_i8_sum(a, b).to(torch.float32)
    y = y * sa.cpu().float().reshape(-1, 1)
    y = y * sb.cpu().float().reshape(1, -1)
    if bias is not None:
        y = y + bias.cpu().float().reshape(1, -1)
    return y.bfloat16()
