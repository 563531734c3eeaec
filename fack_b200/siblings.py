"""PyTorch surface of the sibling GEMM families (``fack_gemm_tn``).

The reference drives two more GEMM families through the same client as the
block-scaled FP8 path (client/aiter/hsa/gfx942/gemm_driver.py:32-79):

* ``gemm_a16w16_asm(a, b, out, bias=None, splitK=None, kernelName=None,
  bpreshuffle=False)`` -- BF16 TN, Y = bf16(A . B^T) (gemm_driver.py:50, call :54);
* ``gemm_a8w8_asm(a, b, sa, sb, out, kernelName=None, bias=None,
  bpreshuffle=True, splitK=None)`` -- INT8 with per-token activation scales
  ``sa`` [M, 1], per-channel weight scales ``sb`` [N, 1] and an fp32 bias
  [1, N]: Y = bf16((A . B^T) * sa * sb^T + bias) (gemm_driver.py:73).

Both take ``b`` either row-major or from :func:`fack_b200.shuffle_weight`
(``bpreshuffle`` must say which, as in aiter).  ``kernelName`` may be one of
the reference's gfx942 symbols (the library then picks its own tile) or this
library's ``fack_tn_sm100_{bf16|i8}_t{128|256}x{64|128|256}_s{S}`` (token tile
256 = a pair of CTAs sharing each MMA; S <= 4 then).  ``splitK``
None lets the library choose; an explicit value is honoured.  Contract
violations raise ``ValueError`` before any launch.
"""
from __future__ import annotations

import ctypes
import re
from typing import Optional

import torch

from . import _lib

KINDS = {torch.bfloat16: _lib.FACK_GEMM_BF16, torch.int8: _lib.FACK_GEMM_I8}
PREFIX = "fack_tn_sm100"
# substrings of the reference's gfx942 catalog symbols (gemm_driver.py:46, :58)
AITER_PATTERNS = {_lib.FACK_GEMM_BF16: "bf16gemm_fp32bf16_", _lib.FACK_GEMM_I8: "I8gemm_bf16_perTokenI8_BpreShuffle_"}


def _family(kind: int) -> str:
    return "bf16" if kind == _lib.FACK_GEMM_BF16 else "i8"


def kernel_name(kind: int, tile_m: int, tile_n: int, split_k: int) -> str:
    return f"{PREFIX}_{_family(kind)}_t{tile_m}x{tile_n}_s{split_k}"


def parse_kernel_name(kind: int, name) -> tuple:
    """(tile_m, tile_n, split_k) fixed by a kernel name, (0, 0, 0) for the library's choice."""
    if not name or AITER_PATTERNS[kind] in str(name):
        return 0, 0, 0
    m = re.fullmatch(PREFIX + r"_(bf16|i8)_t(128|256)x(64|128|256)_s([1-8])", str(name))
    if not m or m.group(1) != _family(kind) or (m.group(2) == "256" and int(m.group(4)) > 4):
        raise ValueError(f"unknown {_family(kind)} kernel {name!r}")
    return int(m.group(2)), int(m.group(3)), int(m.group(4))


def plan(kind: int, M: int, N: int, K: int, tile_m: int = 0, tile_n: int = 0, split_k: int = 0) -> tuple:
    """(tile_m, tile_n, split_k) the library uses; 0 = library choice."""
    lib = _lib.load()
    tm, tn, sk = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    _lib.check(lib.fack_gemm_tn_plan(kind, M, N, K, tile_m, tile_n, split_k, ctypes.byref(tm), ctypes.byref(tn),
                                     ctypes.byref(sk)), "fack_gemm_tn_plan")
    return tm.value, tn.value, sk.value


def get_config(kind: int, M: int, N: int, K: int) -> dict:
    tm, tn, sk = plan(kind, M, N, K)
    return {"libtype": "asm", "kernelName": kernel_name(kind, tm, tn, sk), "splitK": sk, "tile_m": tm,
            "tile_n": tn}


def _vec(t: Optional[torch.Tensor], n: int, name: str, dev) -> Optional[torch.Tensor]:
    if t is None:
        return None
    if not isinstance(t, torch.Tensor) or t.dtype != torch.float32 or t.device != dev or t.numel() != n \
            or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous float32 tensor of {n} elements on {dev}")
    return t


def gemm_tn(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None,
            a_scale: Optional[torch.Tensor] = None, b_scale: Optional[torch.Tensor] = None,
            bias: Optional[torch.Tensor] = None, packed: Optional[bool] = None, tile_n: int = 0,
            split_k: int = 0, tile_m: int = 0) -> torch.Tensor:
    """Native entry: Y[M, N] bf16 from A[M, K] and B[N, K] (bf16, or int8 with
    a_scale [M] / b_scale [N]); ``packed`` defaults to ``b.is_shuffled``."""
    for nm, t in (("a", a), ("b", b)):
        if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dim() != 2:
            raise ValueError(f"{nm} must be a 2-D CUDA tensor")
    if a.dtype not in KINDS or b.dtype != a.dtype:
        raise ValueError("a and b must both be bfloat16 or both int8")
    kind = KINDS[a.dtype]
    M, K = a.shape
    N = b.shape[0]
    if b.shape[1] != K or a.stride(1) != 1 or b.stride(1) != 1 or a.device != b.device:
        raise ValueError(f"shape/layout mismatch: a {tuple(a.shape)}, b {tuple(b.shape)}")
    dev = a.device
    if kind == _lib.FACK_GEMM_I8:
        if a_scale is None or b_scale is None:
            raise ValueError("the INT8 family needs a_scale [M] and b_scale [N]")
    elif a_scale is not None or b_scale is not None:
        raise ValueError("the BF16 family takes no scales")
    a_scale, b_scale = _vec(a_scale, M, "a_scale", dev), _vec(b_scale, N, "b_scale", dev)
    bias = _vec(bias, N, "bias", dev)
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    if out.dtype != torch.bfloat16 or tuple(out.shape) != (M, N) or out.stride(1) != 1 or out.device != dev:
        raise ValueError(f"out must be a bfloat16 [{M}, {N}] tensor with unit column stride on {dev}")
    packed = bool(getattr(b, "is_shuffled", False)) if packed is None else bool(packed)
    if packed and not b.is_contiguous():
        raise ValueError("a packed weight must be contiguous")
    lib = _lib.load()
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    with torch.cuda.device(dev):
        st = lib.fack_gemm_tn(kind, a.data_ptr(), a.stride(0), b.data_ptr(), int(packed), b.stride(0),
                              ptr(a_scale), ptr(b_scale), ptr(bias), out.data_ptr(), out.stride(0), M, N, K,
                              int(tile_m), int(tile_n), int(split_k), torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(st, "fack_gemm_tn")
    return out


def _check_shuffle_flag(b, bpreshuffle):
    shuffled = bool(getattr(b, "is_shuffled", False))
    if bool(bpreshuffle) != shuffled:
        raise ValueError("bpreshuffle={} but the weight {} a shuffle_weight() output".format(
            bool(bpreshuffle), "is" if shuffled else "is not"))
    return shuffled


def gemm_a16w16_asm(a, b, out, bias=None, splitK=None, kernelName=None, bpreshuffle=False):
    """Drop-in for aiter's ``gemm_a16w16_asm`` (BF16 TN; writes and returns ``out``)."""
    if a.dtype != torch.bfloat16:
        raise ValueError("gemm_a16w16_asm takes bfloat16 operands")
    tile_m, tile_n, name_split = parse_kernel_name(_lib.FACK_GEMM_BF16, kernelName)
    shuffled = _check_shuffle_flag(b, bpreshuffle)
    split = name_split if splitK is None else int(splitK)
    return gemm_tn(a, b, out, bias=None if bias is None else bias.reshape(-1), packed=shuffled, tile_n=tile_n,
                   split_k=split, tile_m=tile_m)


def gemm_a8w8_asm(a, b, sa, sb, out, kernelName=None, bias=None, bpreshuffle=True, splitK=None):
    """Drop-in for aiter's ``gemm_a8w8_asm`` (INT8, per-token scales, fp32 bias;
    writes and returns ``out``)."""
    if a.dtype != torch.int8:
        raise ValueError("gemm_a8w8_asm takes int8 operands")
    tile_m, tile_n, name_split = parse_kernel_name(_lib.FACK_GEMM_I8, kernelName)
    shuffled = _check_shuffle_flag(b, bpreshuffle)
    split = name_split if splitK is None else int(splitK)
    flat = lambda t: None if t is None else t.reshape(-1)  # noqa: E731  ([M,1] / [N,1] / [1,N] views)
    return gemm_tn(a, b, out, a_scale=flat(sa), b_scale=flat(sb), bias=flat(bias), packed=shuffled,
                   tile_n=tile_n, split_k=split, tile_m=tile_m)


def _public_plan(kind: int, a, b, name: str):
    """(M, N, K, config) for a public entry, after the checks that need no device."""
    for nm, t in (("a", a), ("b", b)):
        if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dim() != 2:
            raise ValueError(f"{name}: {nm} must be a 2-D CUDA tensor")
    M, K = a.shape
    N = b.shape[0]
    with torch.cuda.device(a.device):
        return M, N, K, get_config(kind, M, N, K)


def gemm_a8w8_ASM(a, b, sa, sb, bias=None, dtype=torch.bfloat16):
    """Drop-in for aiter's public INT8 entry ``gemm_a8w8_ASM`` (the call the
    reference's dispatch check makes, client/aiter/hsa/gfx942/dispatch_driver.py:55-56):
    picks the plan for (M, N, K) (exact-shape table first, then the cost
    model), allocates ``out`` and makes one :func:`gemm_a8w8_asm` call with
    that kernelName and splitK."""
    if dtype != torch.bfloat16:
        raise ValueError("only bfloat16 output is supported")
    if not isinstance(a, torch.Tensor) or a.dtype != torch.int8:
        raise ValueError("gemm_a8w8_ASM takes int8 operands")
    M, N, K, cfg = _public_plan(KINDS[torch.int8], a, b, "gemm_a8w8_ASM")
    out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    return gemm_a8w8_asm(a, b, sa, sb, out, kernelName=cfg["kernelName"], bias=bias,
                         bpreshuffle=bool(getattr(b, "is_shuffled", False)), splitK=cfg["splitK"])


def gemm_a16w16(a, b, bias=None, otype=torch.bfloat16):
    """Drop-in for aiter's public BF16 entry ``tuned_gemm.gemm_a16w16`` (the
    call the reference's dispatch check makes,
    client/aiter/hsa/gfx942/dispatch_driver.py:86-87): picks the plan,
    allocates ``out`` and makes one :func:`gemm_a16w16_asm` call."""
    if otype != torch.bfloat16:
        raise ValueError("only bfloat16 output is supported")
    if not isinstance(a, torch.Tensor) or a.dtype != torch.bfloat16:
        raise ValueError("gemm_a16w16 takes bfloat16 operands")
    M, N, K, cfg = _public_plan(KINDS[torch.bfloat16], a, b, "gemm_a16w16")
    out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    return gemm_a16w16_asm(a, b, out, bias=bias, splitK=cfg["splitK"], kernelName=cfg["kernelName"],
                           bpreshuffle=bool(getattr(b, "is_shuffled", False)))
