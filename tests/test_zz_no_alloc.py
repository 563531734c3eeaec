"""GPU: the no-allocation entry point, fack_gemm_bs_noalloc.

Some callers cannot call cudaMalloc at the moment they run the GEMM (a plugin's
enqueue path that must not allocate or synchronise, a process whose device
memory another allocator owns).  For them
the library keeps its split-K scratch in a fixed 16 MiB buffer compiled into
the library.  These tests call that entry point through the C ABI and check
it against the regular entry point with a caller-owned workspace, bit for
bit, twice in a row (the buffer is reused and keeps the previous call's
contents), and against the oracle on sampled rows; that a shape whose own
plan needs more scratch gets the best plan that fits; and that an explicit
split needing more scratch is refused before any launch.

This file sorts last so that a run stopping at the first failure has already
run every other test; it also passes on its own in a fresh process.
"""
import ctypes

import pytest
import torch

from fack_b200 import _lib, data
from oracle.blockscale import reference_gemm

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


def _plan(lib, M, N, K, tm=0, tn=0, sk=0):
    a, b, c, nb = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()
    st = lib.fack_gemm_bs_plan(M, N, K, tm, tn, sk, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c),
                               ctypes.byref(nb))
    assert st == 0, _lib.status_string(st)
    return a.value, b.value, c.value, nb.value


def _oracle_rows(xq, xs, wq, ws, y, n_rows=16):
    rows = torch.linspace(0, xq.shape[0] - 1, n_rows).long()
    ref = reference_gemm(xq[rows.to(xq.device)].cpu(), wq.cpu(), xs[rows.to(xs.device)].cpu(), ws.cpu()).float()
    got = y[rows.to(y.device)].float().cpu()
    assert torch.allclose(got, ref, rtol=RTOL, atol=ATOL), f"max abs diff {float((got - ref).abs().max()):.4g}"


def test_noalloc_matches_workspace_entry_point_twice(cuda_device):
    lib = _load_with_tables()
    M, N, K = 256, 3072, 7168   # the decode shape: the library's plan splits K, so the scratch is used
    _, _, sk, nb = _plan(lib, M, N, K)
    assert sk > 1 and 0 < nb <= SCRATCH_BYTES

    xq, xs, wq, ws = data.make_inputs(data.Workload("noalloc", M, N, K), seed=17, device=cuda_device)
    expected = torch.empty((M, N), dtype=torch.bfloat16, device=cuda_device)
    workspace = torch.empty(nb, dtype=torch.uint8, device=cuda_device)
    st = lib.fack_gemm_bs(*_args(xq, xs, wq, ws, expected), 0, workspace.data_ptr(), workspace.numel(), _stream())
    assert st == 0, _lib.status_string(st)
    torch.cuda.synchronize()

    for call in range(2):
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        st = lib.fack_gemm_bs_noalloc(*_args(xq, xs, wq, ws, out), 0, _stream())
        assert st == 0, _lib.status_string(st)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all(), f"call {call}: unwritten output elements"
        # the same kernel, plan and split-K combine as the workspace entry point: the same bits
        assert torch.equal(out.view(torch.int16), expected.view(torch.int16)), (
            f"call {call}: {int((out.view(torch.int16) != expected.view(torch.int16)).sum())} elements differ")
        _oracle_rows(xq, xs, wq, ws, out)

    flags = ctypes.c_uint()
    assert lib.fack_device_status(_stream(), ctypes.byref(flags), 0) == 0 and flags.value == 0


def _load_with_tables():
    lib = _lib.load()
    if lib.fack_gemm_bs_tuned_count() == 0:   # a test before this one cleared the shipped table
        for t in _lib.tuned_tables():
            _lib.load_tuned(t, lib)
    return lib


def test_noalloc_replans_when_the_own_plan_needs_more_scratch(cuda_device):
    """With the exact-shape table cleared the cost model's plan for these
    shapes splits K 2-3 ways and needs more than 16 MiB of partials; the
    entry point then takes the best plan that fits.  Its output must be bit
    for bit that of one explicit plan whose workspace fits, run through the
    workspace entry point, and agree with the oracle."""
    lib = _lib.load()
    lib.fack_gemm_bs_tuned_clear()
    try:
        shape = None
        for M, N, K in ((800, 3072, 7168), (1408, 4608, 7168), (640, 4096, 7168), (1024, 3072, 7168)):
            if _plan(lib, M, N, K)[3] > SCRATCH_BYTES:
                shape = (M, N, K)
                break
        assert shape is not None, "no candidate shape's automatic plan exceeds the built-in scratch"
        M, N, K = shape
        xq, xs, wq, ws = data.make_inputs(data.Workload("noalloc_replan", M, N, K), seed=23, device=cuda_device)
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        st = lib.fack_gemm_bs_noalloc(*_args(xq, xs, wq, ws, out), 0, _stream())
        assert st == 0, _lib.status_string(st)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        _oracle_rows(xq, xs, wq, ws, out)
        matches = []
        for tn in (256, 128, 64):
            if N % tn:
                continue
            for sk in range(1, 9):
                if K // 128 // sk < 2:
                    break
                _, _, _, need = _plan(lib, M, N, K, 128, tn, sk)
                if need > SCRATCH_BYTES:
                    continue
                ref = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda_device)
                ws_buf = torch.empty(max(need, 16), dtype=torch.uint8, device=cuda_device)
                st = lib.fack_gemm_bs_ex(*_args(xq, xs, wq, ws, ref), 128, tn, sk,
                                         ws_buf.data_ptr() if need else None, ws_buf.numel() if need else 0,
                                         _stream())
                assert st == 0, _lib.status_string(st)
                torch.cuda.synchronize()
                if torch.equal(ref.view(torch.int16), out.view(torch.int16)):
                    matches.append((tn, sk, need))
        assert matches, f"{shape}: the no-allocation output matches no plan whose partials fit 16 MiB"
    finally:
        lib.fack_gemm_bs_tuned_clear()
        for t in _lib.tuned_tables():
            _lib.load_tuned(t, lib)


def test_noalloc_refuses_problems_beyond_its_scratch(cuda_device):
    lib = _load_with_tables()
    M, N, K = 8192, 7168, 16384  # split 8 would need ~1.9 GB of partials
    _, _, _, nb = _plan(lib, M, N, K, 0, 0, 8)
    assert nb > SCRATCH_BYTES
    # NULL operands: the size check refuses the call first; were it ever to come
    # later, the pointer checks would still refuse it on the host (BAD_ALIGN),
    # so nothing is launched either way
    st = lib.fack_gemm_bs_noalloc(None, K, None, 0, None, K // 128, 1, None, None, N, M, N, K, 8, _stream())
    assert st == _lib.FACK_ERR_SCRATCH_LIMIT
    assert "16 MiB" in _lib.status_string(st)
