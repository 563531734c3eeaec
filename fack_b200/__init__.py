"""fack_b200 -- B200 (sm_100a) FP8 block-scaled GEMM.

Drop-in for the one data-parallel path of feifei14119/FACK: aiter's
``gemm_a8w8_blockscale_bpreshuffle`` operator, with the sibling BF16 TN and
INT8 per-token GEMMs the same client drives and the fused activation
quantisation in front of it.  The arithmetic is a
hand-written tcgen05/TMA kernel behind a C ABI (include/fack_gemm.h); this
package is the PyTorch-facing operator surface and the N-sharded multi-GPU
wrapper.
"""
from .ops import (  # noqa: F401
    AITER_SYMBOLS,
    device_status,
    gather_interleave,
    gemm_a8w8_blockscale_bpreshuffle,
    gemm_a8w8_blockscale_bpreshuffle_asm,
    gemm_a8w8_blockscale_bpreshuffle_ck,
    gemm_blockscale,
    get_config,
    quantize_activations,
    shuffle_weight,
    tail_workspace_size,
    workspace_size,
)
from .siblings import gemm_a8w8_ASM, gemm_a8w8_asm, gemm_a16w16, gemm_a16w16_asm, gemm_tn  # noqa: F401

__all__ = [
    "AITER_SYMBOLS",
    "device_status",
    "gather_interleave",
    "gemm_a16w16",
    "gemm_a16w16_asm",
    "gemm_a8w8_ASM",
    "gemm_a8w8_asm",
    "gemm_tn",
    "gemm_a8w8_blockscale_bpreshuffle",
    "gemm_a8w8_blockscale_bpreshuffle_asm",
    "gemm_a8w8_blockscale_bpreshuffle_ck",
    "gemm_blockscale",
    "get_config",
    "quantize_activations",
    "shuffle_weight",
    "tail_workspace_size",
    "workspace_size",
]
