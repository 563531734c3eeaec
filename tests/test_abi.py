"""CPU: the C-ABI library loads, exports every symbol the header declares, and
rejects contract violations on the host before touching a device."""
import ctypes
import re
from pathlib import Path

import pytest

from fack_b200 import _lib
from fack_b200.build import LIB

HEADER = Path(__file__).resolve().parents[1] / "include" / "fack_gemm.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(fack_\w+)\s*\(", text, flags=re.M)))


def test_library_built_in_tree():
    assert LIB.exists(), "run python -m fack_b200.build"
    assert LIB.parent.name == "fack_b200"


def test_every_declared_symbol_is_exported_and_typed():
    names = declared_functions()
    assert len(names) >= 8
    lib = _lib.load()
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(names)


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.fack_version() == 100
    for code in range(10):
        s = lib.fack_status_string(code).decode()
        assert s and s != "unknown status"
    assert lib.fack_status_string(99).decode() == "unknown status"


@pytest.mark.parametrize("m,n,k", [(0, 128, 128), (4, 100, 128), (4, 128, 100), (4, 0, 128), (4, 128, -128)])
def test_bad_shapes_rejected(m, n, k):
    lib = _lib.load()
    tm, sk = ctypes.c_int(), ctypes.c_int()
    assert lib.fack_gemm_bs_select(m, n, k, 1, ctypes.byref(tm), ctypes.byref(sk)) == _lib.FACK_ERR_BAD_SHAPE
    st = lib.fack_gemm_bs(16, k, 16, 0, 16, 1, 1, 16, 16, n, m, n, k, 1, None, 0, None)
    assert st == _lib.FACK_ERR_BAD_SHAPE


def test_explicit_split_plan_and_workspace_without_device():
    lib = _lib.load()
    tn, sk = ctypes.c_int(), ctypes.c_int()
    # 2 token tiles x 12 weight tiles of 256 x 6 slices = 144 CTAs -> 256-row weight tiles
    assert lib.fack_gemm_bs_select(256, 3072, 7168, 6, ctypes.byref(tn), ctypes.byref(sk)) == 0
    assert (tn.value, sk.value) == (256, 6)
    # one token tile x 12 tiles = too few CTAs for 256 or 128 at split 1 -> 64-row tiles
    assert lib.fack_gemm_bs_select(1, 3072, 7168, 1, ctypes.byref(tn), ctypes.byref(sk)) == 0
    assert tn.value == 64
    # N = 384 is not a multiple of 256
    assert lib.fack_gemm_bs_select(300, 384, 7168, 8, ctypes.byref(tn), ctypes.byref(sk)) == 0
    assert tn.value in (64, 128)
    nb = ctypes.c_size_t()
    assert lib.fack_gemm_bs_workspace_size(256, 3072, 7168, 6, ctypes.byref(nb)) == 0
    assert nb.value == (2 * 12) * 6 * 128 * 256 * 4
    assert lib.fack_gemm_bs_workspace_size(256, 3072, 7168, 1, ctypes.byref(nb)) == 0
    assert nb.value == 0
    # split beyond the cluster limit or beyond K/128 is refused
    assert lib.fack_gemm_bs_select(256, 3072, 7168, 9, ctypes.byref(tn), ctypes.byref(sk)) == _lib.FACK_ERR_BAD_ARG
    assert lib.fack_gemm_bs_select(256, 3072, 256, 3, ctypes.byref(tn), ctypes.byref(sk)) == _lib.FACK_ERR_BAD_ARG


def test_pointer_and_stride_checks_before_device():
    lib = _lib.load()
    M, N, K = 32, 256, 512
    ok = 1 << 20  # a 16-byte aligned fake address: never dereferenced on these paths
    # NULL / misaligned pointers
    assert lib.fack_gemm_bs(None, K, ok, 0, ok, 1, 1, ok, ok, N, M, N, K, 1, None, 0, None) == _lib.FACK_ERR_BAD_ALIGN
    assert lib.fack_gemm_bs(ok + 8, K, ok, 0, ok, 1, 1, ok, ok, N, M, N, K, 1, None, 0, None) == _lib.FACK_ERR_BAD_ALIGN
    assert lib.fack_gemm_bs(ok, K, ok, 0, ok + 2, 1, 1, ok, ok, N, M, N, K, 1, None, 0, None) == _lib.FACK_ERR_BAD_ALIGN
    # strides
    assert lib.fack_gemm_bs(ok, K - 16, ok, 0, ok, 1, 1, ok, ok, N, M, N, K, 1, None, 0, None) == _lib.FACK_ERR_BAD_STRIDE
    assert lib.fack_gemm_bs(ok, K + 8, ok, 0, ok, 1, 1, ok, ok, N, M, N, K, 1, None, 0, None) == _lib.FACK_ERR_BAD_STRIDE
    assert lib.fack_gemm_bs(ok, K, ok, 0, ok, 1, 1, ok, ok, N + 4, M, N, K, 1, None, 0, None) == _lib.FACK_ERR_BAD_STRIDE
    assert lib.fack_gemm_bs(ok, K, ok, 0, ok, 0, 1, ok, ok, N, M, N, K, 1, None, 0, None) == _lib.FACK_ERR_BAD_STRIDE
    # layout / split arguments
    assert lib.fack_gemm_bs(ok, K, ok, 2, ok, 1, 1, ok, ok, N, M, N, K, 1, None, 0, None) == _lib.FACK_ERR_BAD_ARG
    assert lib.fack_gemm_bs(ok, K, ok, 0, ok, 1, 1, ok, ok, N, M, N, K, 9, None, 0, None) == _lib.FACK_ERR_BAD_ARG
    # prepack and interleave validation
    assert lib.fack_gemm_bs_prepack_w(ok, K, None, 100, K, ok, None, None) == _lib.FACK_ERR_BAD_SHAPE
    assert lib.fack_gemm_bs_prepack_w(ok, K - 16, None, N, K, ok, None, None) == _lib.FACK_ERR_BAD_STRIDE
    assert lib.fack_gather_interleave(ok, 2, 4, 12, ok, 24, None) == _lib.FACK_ERR_BAD_SHAPE
    assert lib.fack_gather_interleave(ok, 2, 4, 128, ok, 200, None) == _lib.FACK_ERR_BAD_STRIDE
    assert lib.fack_device_status(None, None, 0) == _lib.FACK_ERR_BAD_ARG


def test_check_maps_contract_violations_to_valueerror():
    with pytest.raises(ValueError):
        _lib.check(_lib.FACK_ERR_BAD_SHAPE, "x")
    with pytest.raises(_lib.FackError):
        _lib.check(_lib.FACK_ERR_LAUNCH, "x")
    _lib.check(_lib.FACK_OK, "x")
