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
    for code in range(_lib.FACK_ERR_SCRATCH_LIMIT + 1):
        s = lib.fack_status_string(code).decode()
        assert s and s != "unknown status"
    assert lib.fack_status_string(99).decode() == "unknown status"


@pytest.mark.parametrize("m,n,k", [(0, 128, 128), (4, 100, 128), (4, 128, 100), (4, 0, 128), (4, 128, -128),
                                   (65535 * 128 + 1, 128, 128)])   # more token tiles than gridDim.y holds
def test_bad_shapes_rejected(m, n, k):
    lib = _lib.load()
    tm, sk = ctypes.c_int(), ctypes.c_int()
    assert lib.fack_gemm_bs_select(m, n, k, 1, ctypes.byref(tm), ctypes.byref(sk)) == _lib.FACK_ERR_BAD_SHAPE
    st = lib.fack_gemm_bs(16, k, 16, 0, 16, 1, 1, 16, 16, n, m, n, k, 1, None, 0, None)
    assert st == _lib.FACK_ERR_BAD_SHAPE


def test_explicit_split_plan_and_workspace_without_device():
    lib = _lib.load()
    tm, tn, sk, nb = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()

    def plan(M, N, K, m=0, n=0, s=0):
        st = lib.fack_gemm_bs_plan(M, N, K, m, n, s, ctypes.byref(tm), ctypes.byref(tn), ctypes.byref(sk),
                                   ctypes.byref(nb))
        return st, tm.value, tn.value, sk.value, nb.value

    # requested pairs, split 4: 12 x 2 x 4 = 96 CTAs < 120 -> 128-wide weight tiles
    assert plan(256, 3072, 7168, m=256, s=4)[:4] == (0, 256, 128, 4)
    # 256 tokens, split 6: 12 x 2 x 6 = 144 CTAs with single-CTA 256-wide tiles
    assert plan(256, 3072, 7168, s=6)[:4] == (0, 128, 256, 6)
    # one token: single-CTA tiles; 12 CTAs at 256 -> smallest weight tile
    assert plan(1, 3072, 7168, s=1)[1:3] == (128, 64)
    # N = 384 is not a multiple of 256
    assert plan(300, 384, 7168, s=8)[2] in (64, 128)
    # workspace = tiles x split x 128 x tile_n x 4
    st, m, n, s, ws = plan(256, 3072, 7168, m=128, n=256, s=6)
    assert st == 0 and ws == (12 * 2) * 6 * 128 * 256 * 4
    st, m, n, s, ws = plan(200, 3072, 7168, m=256, n=256, s=2)
    assert st == 0 and ws == (12 * 2) * 2 * 128 * 256 * 4   # a pair: two 128-token tiles
    assert plan(256, 3072, 7168, m=128, n=256, s=1)[4] == 0
    assert lib.fack_gemm_bs_workspace_size(256, 3072, 7168, 1, ctypes.byref(nb)) == 0 and nb.value == 0
    # refused: split beyond the cluster limit, beyond K/128, pairs with split > 4, odd tiles
    assert plan(256, 3072, 7168, s=9)[0] == _lib.FACK_ERR_BAD_ARG
    assert plan(256, 3072, 256, s=3)[0] == _lib.FACK_ERR_BAD_ARG
    assert plan(256, 3072, 7168, m=256, s=5)[0] == _lib.FACK_ERR_BAD_ARG
    assert plan(256, 3072, 7168, m=64, s=1)[0] == _lib.FACK_ERR_BAD_ARG
    assert plan(256, 384, 7168, n=256, s=1)[0] == _lib.FACK_ERR_BAD_ARG
    # 224-wide weight tiles: 128-token tiles and one K slice, filled in when not given (no device query)
    assert plan(8192, 896, 16384, n=224) == (0, 128, 224, 1, 0)
    assert plan(8192, 896, 16384, m=128, n=224, s=1) == (0, 128, 224, 1, 0)
    assert plan(8192, 896, 16384, n=224, s=2)[0] == _lib.FACK_ERR_BAD_ARG
    assert plan(8192, 896, 16384, m=256, n=224)[0] == _lib.FACK_ERR_BAD_ARG
    assert plan(8192, 1024, 16384, n=224)[0] == _lib.FACK_ERR_BAD_ARG
    # the warp-MMA small-M kernel (16-row weight tiles): up to 16 tokens, one slice, K <= 256 blocks
    assert plan(1, 3072, 7168, n=16) == (0, 16, 16, 1, 0)
    assert plan(16, 3072, 7168, m=16, n=16, s=1) == (0, 16, 16, 1, 0)
    assert plan(17, 3072, 7168, n=16)[0] == _lib.FACK_ERR_BAD_ARG
    assert plan(8, 3072, 7168, m=32, n=16)[0] == _lib.FACK_ERR_BAD_ARG
    assert plan(8, 3072, 7168, n=16, s=2)[0] == _lib.FACK_ERR_BAD_ARG
    assert plan(8, 3072, 257 * 128, n=16)[0] == _lib.FACK_ERR_BAD_ARG
    assert plan(8, 3072, 7168, m=16, s=1)[2] == 128          # a 16-token tile alone is the swapped kernel
    tn2, sk2 = ctypes.c_int(), ctypes.c_int()
    assert lib.fack_gemm_bs_select(256, 3072, 7168, 6, ctypes.byref(tn2), ctypes.byref(sk2)) == 0
    assert (tn2.value, sk2.value) == (256, 6)


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
    # activation quantisation validation
    f32, bf16 = _lib.FACK_DTYPE_F32, _lib.FACK_DTYPE_BF16
    assert lib.fack_quant_act(ok, f32, K, M, 100, ok, K, ok, 1, M, None) == _lib.FACK_ERR_BAD_SHAPE
    assert lib.fack_quant_act(ok, 7, K, M, K, ok, K, ok, 1, M, None) == _lib.FACK_ERR_BAD_ARG
    assert lib.fack_quant_act(ok + 4, bf16, K, M, K, ok, K, ok, 1, M, None) == _lib.FACK_ERR_BAD_ALIGN
    assert lib.fack_quant_act(ok, f32, K + 4, M, K, ok, K, ok, 1, M, None) == _lib.FACK_ERR_BAD_STRIDE
    assert lib.fack_quant_act(ok, f32, K, M, K, ok, K + 8, ok, 1, M, None) == _lib.FACK_ERR_BAD_STRIDE


def test_sibling_gemm_validation_before_device():
    lib = _lib.load()
    ok = 1 << 20
    BF, I8 = _lib.FACK_GEMM_BF16, _lib.FACK_GEMM_I8
    M, N, K = 32, 256, 256

    def tn(kind=I8, a=ok, lda=K, b=ok, packed=0, ldb=K, sa=ok, sb=ok, bias=None, out=ok, ldo=N, m=M, n=N, k=K,
           tm=0, tile=0, split=1):
        return lib.fack_gemm_tn(kind, a, lda, b, packed, ldb, sa, sb, bias, out, ldo, m, n, k, tm, tile, split, None)

    assert tn(kind=2) == _lib.FACK_ERR_BAD_ARG
    assert tn(n=192 + 32) == _lib.FACK_ERR_BAD_SHAPE            # N % 64
    assert tn(k=192) == _lib.FACK_ERR_BAD_SHAPE                 # int8: K % 128
    assert tn(kind=BF, sa=None, sb=None, k=96, lda=96, ldb=96) == _lib.FACK_ERR_BAD_SHAPE
    assert tn(m=0) == _lib.FACK_ERR_BAD_SHAPE
    assert tn(a=ok + 8) == _lib.FACK_ERR_BAD_ALIGN
    assert tn(sa=None) == _lib.FACK_ERR_BAD_ALIGN               # int8 needs both scale vectors
    assert tn(bias=ok + 2) == _lib.FACK_ERR_BAD_ALIGN
    assert tn(kind=BF) == _lib.FACK_ERR_BAD_ARG                 # bf16 takes no scales
    assert tn(lda=K + 8) == _lib.FACK_ERR_BAD_STRIDE            # int8 rows: 16-byte multiple
    assert tn(kind=BF, sa=None, sb=None, lda=K + 4) == _lib.FACK_ERR_BAD_STRIDE
    assert tn(ldo=N + 4) == _lib.FACK_ERR_BAD_STRIDE
    assert tn(packed=2) == _lib.FACK_ERR_BAD_ARG
    assert tn(split=9) == _lib.FACK_ERR_BAD_ARG
    assert tn(tile=96) == _lib.FACK_ERR_BAD_ARG
    assert tn(tm=192) == _lib.FACK_ERR_BAD_ARG
    assert tn(tm=256, split=5) == _lib.FACK_ERR_BAD_ARG        # a pair's cluster is 2 x split <= 8
    tm_, tn_, sk = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()

    def plan(kind, m, n, k, t_m, t_n, s):
        st = lib.fack_gemm_tn_plan(kind, m, n, k, t_m, t_n, s, ctypes.byref(tm_), ctypes.byref(tn_), ctypes.byref(sk))
        return st, (tm_.value, tn_.value, sk.value)

    # a fully explicit plan needs no device
    assert plan(I8, M, N, K, 128, 128, 2) == (0, (128, 128, 2))
    assert plan(I8, M, N, K, 256, 64, 2) == (0, (256, 64, 2))
    assert plan(I8, M, 320, K, 128, 256, 1)[0] == _lib.FACK_ERR_BAD_ARG
    assert plan(BF, M, N, 128, 128, 64, 3)[0] == _lib.FACK_ERR_BAD_ARG
    assert plan(BF, M, N, 192, 128, 64, 3)[0] == 0                # bf16: K % 64
    assert plan(BF, M, N, 1024, 256, 64, 5)[0] == _lib.FACK_ERR_BAD_ARG


def test_swapped_tiles_peer_outputs_and_ipc_validation_before_device():
    lib = _lib.load()
    ok = 1 << 20  # fake 16-byte aligned address: every call below fails validation first
    tm, tn, sk, nb = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()

    def plan(M, N, K, m=0, n=0, s=0):
        st = lib.fack_gemm_bs_plan(M, N, K, m, n, s, ctypes.byref(tm), ctypes.byref(tn), ctypes.byref(sk),
                                   ctypes.byref(nb))
        return st, tm.value, tn.value, sk.value, nb.value

    # swapped small-M tiles: all M tokens in one tile, 128 weight rows, no workspace
    assert plan(16, 3072, 7168, m=16, s=5) == (0, 16, 128, 5, 0)
    assert plan(33, 3072, 7168, m=64, n=128, s=8) == (0, 64, 128, 8, 0)
    assert plan(17, 3072, 7168, m=16, s=5)[0] == _lib.FACK_ERR_BAD_ARG       # 17 tokens do not fit 16
    assert plan(16, 3072, 7168, m=16, n=256, s=5)[0] == _lib.FACK_ERR_BAD_ARG  # weight tile is 128
    assert plan(16, 3072, 131072, m=16, s=1)[0] == _lib.FACK_ERR_BAD_ARG      # 1024 K blocks > 128 per slice
    assert plan(16, 3072, 7168, m=48, s=1)[0] == _lib.FACK_ERR_BAD_ARG        # not a tile size
    # peer outputs of the fused multi-GPU path
    M, N, K = 32, 256, 512
    peers8 = (ctypes.c_void_p * 8)(*([ok] * 8))
    peers_bad = (ctypes.c_void_p * 2)(ok, ok + 8)

    def bcast(peers, n):
        return lib.fack_gemm_bs_bcast(ok, K, ok, 0, ok, 1, 1, ok, ok, N, peers, n, M, N, K, 0, 0, 1, None, 0, None)

    assert bcast(peers8, 8) == _lib.FACK_ERR_BAD_ARG                      # at most 7 peers
    assert bcast(None, 1) == _lib.FACK_ERR_BAD_ARG
    assert bcast(peers_bad, 2) == _lib.FACK_ERR_BAD_ALIGN
    assert bcast(peers8, -1) == _lib.FACK_ERR_BAD_ARG
    # CUDA IPC entry points reject missing arguments before any CUDA call
    off = ctypes.c_size_t()
    assert lib.fack_ipc_get_handle(None, ctypes.create_string_buffer(64), 64, ctypes.byref(off)) == _lib.FACK_ERR_BAD_ARG
    assert lib.fack_ipc_get_handle(ok, ctypes.create_string_buffer(64), 32, ctypes.byref(off)) == _lib.FACK_ERR_BAD_ARG
    assert lib.fack_ipc_open_handle(None, ctypes.byref(ctypes.c_void_p())) == _lib.FACK_ERR_BAD_ARG
    assert lib.fack_ipc_close_handle(None) == _lib.FACK_ERR_BAD_ARG


def test_check_maps_contract_violations_to_valueerror():
    with pytest.raises(ValueError):
        _lib.check(_lib.FACK_ERR_BAD_SHAPE, "x")
    with pytest.raises(_lib.FackError):
        _lib.check(_lib.FACK_ERR_LAUNCH, "x")
    _lib.check(_lib.FACK_OK, "x")
