"""GPU: the no-allocation entry point, fack_gemm_bs_noalloc.

Some callers cannot call cudaMalloc at the moment they run the GEMM (a plugin's
enqueue path that must not allocate or synchronise, a process whose device
memory another allocator owns).  For them
the library keeps its split-K scratch in a fixed 16 MiB buffer compiled into
the library.  These tests call that entry point through the C ABI and check
it against the regular entry point with a caller-owned workspace, twice in a
row (the buffer is reused and keeps the previous call's contents), and check
that a problem needing more scratch is refused before any launch.

This file sorts last so that a run stopping at the first failure has already
run every other test; it also passes on its own in a fresh process.
"""
import ctypes

import pytest
import torch

from fack_b200 import _lib, data

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-2
SCRATCH_BYTES = 16 << 20


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _args(xq, xs, wq, ws, out):
    M, K = xq.shape
    N = wq.shape[0]
    # logical row-major x_scale: element (m, kb) at m*(K/128) + kb
    return (xq.data_ptr(), xq.stride(0), wq.data_ptr(), _lib.FACK_W_ROW_MAJOR, xs.data_ptr(), K // 128, 1,
            ws.data_ptr(), out.data_ptr(), out.stride(0), M, N, K)


def test_noalloc_matches_workspace_entry_point_twice(cuda_device):
    lib = _lib.load()
    M, N, K = 256, 3072, 7168   # the decode shape: the library's plan splits K, so the scratch is used
    tm, tn, sk, nb = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()
    assert lib.fack_gemm_bs_plan(M, N, K, 0, 0, 0, ctypes.byref(tm), ctypes.byref(tn), ctypes.byref(sk),
                                 ctypes.byref(nb)) == 0
    assert sk.value > 1 and 0 < nb.value <= SCRATCH_BYTES

    xq, xs, wq, ws = data.make_inputs(data.Workload("noalloc", M, N, K), seed=17, device=cuda_device)
    expected = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_device)
    workspace = torch.empty(nb.value, dtype=torch.uint8, device=cuda_device)
    st = lib.fack_gemm_bs(*_args(xq, xs, wq, ws, expected), 0, workspace.data_ptr(), workspace.numel(), _stream())
    assert st == 0, _lib.status_string(st)
    torch.cuda.synchronize()

    for call in range(2):
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        st = lib.fack_gemm_bs_noalloc(*_args(xq, xs, wq, ws, out), 0, _stream())
        assert st == 0, _lib.status_string(st)
        torch.cuda.synchronize()
        y, ref = out.float(), expected.float()
        assert torch.isfinite(y).all(), f"call {call}: unwritten output elements"
        assert torch.allclose(y, ref, rtol=RTOL, atol=ATOL), (
            f"call {call}: max abs diff {float((y - ref).abs().max()):.4g}")

    flags = ctypes.c_uint()
    assert lib.fack_device_status(_stream(), ctypes.byref(flags), 0) == 0 and flags.value == 0


def test_noalloc_refuses_problems_beyond_its_scratch(cuda_device):
    lib = _lib.load()
    M, N, K = 8192, 7168, 16384  # split 8 would need ~1.9 GB of partials
    tm, tn, sk, nb = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()
    assert lib.fack_gemm_bs_plan(M, N, K, 0, 0, 8, ctypes.byref(tm), ctypes.byref(tn), ctypes.byref(sk),
                                 ctypes.byref(nb)) == 0
    assert nb.value > SCRATCH_BYTES
    fake = 1 << 20  # never dereferenced: the size check comes first
    st = lib.fack_gemm_bs_noalloc(fake, K, fake, 0, fake, K // 128, 1, fake, fake, N, M, N, K, 8, _stream())
    assert st == _lib.FACK_ERR_SCRATCH_LIMIT
    assert "16 MiB" in _lib.status_string(st)
