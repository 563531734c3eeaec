"""ctypes binding of the C-ABI library ``libfack_gemm.so`` (include/fack_gemm.h).

Loading fails loudly: there is no CPU or library fallback for the GEMM, so a
missing or stale build raises instead of silently computing something else.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libfack_gemm.so"

# Exact-shape plan table shipped with the library (rows measured on B200 by
# ``python -m fack_b200.tune``), loaded into the C table with the library.
# More tables, separated by os.pathsep, are merged on top of it from this
# variable, later rows replacing earlier ones -- the counterpart of aiter's
# AITER_CONFIG_GEMM_A8W8_BLOCKSCALE_BPRESHUFFLE (client/aiter/dispatch.py:29-30).
TUNED_TABLE = _HERE / "configs" / "a8w8_blockscale_bpreshuffle_tuned_gemm.csv"
TUNED_ENV = "FACK_CONFIG_GEMM_A8W8_BLOCKSCALE_BPRESHUFFLE"
# The sibling families' (BF16 TN, INT8 per token) table, same form; the
# shipped file is optional, more tables come from this variable.
TN_TUNED_TABLE = _HERE / "configs" / "gemm_tn_tuned_gemm.csv"
TN_TUNED_ENV = "FACK_CONFIG_GEMM_TN"

# Status codes, mirrored from enum fack_status.
FACK_OK = 0
FACK_ERR_BAD_SHAPE = 1
FACK_ERR_BAD_ALIGN = 2
FACK_ERR_BAD_STRIDE = 3
FACK_ERR_WS_TOO_SMALL = 4
FACK_ERR_LAUNCH = 5
FACK_ERR_UNSUPPORTED_ARCH = 6
FACK_ERR_BAD_ARG = 7
FACK_ERR_DEVICE_TIMEOUT = 8
FACK_ERR_CUDA = 9
FACK_ERR_SCRATCH_LIMIT = 10

# Bytes of one rank's exchange state (fack_gemm_bs_allgather, fack_xchg_barrier).
FACK_XCHG_BYTES = 128
# Device status bits (fack_device_status).
FACK_DEVICE_EXCHANGE = 32

FACK_W_ROW_MAJOR = 0
FACK_W_PACKED = 1

FACK_DTYPE_F32 = 0
FACK_DTYPE_BF16 = 1

FACK_GEMM_BF16 = 0
FACK_GEMM_I8 = 1

# Every symbol the header declares, with its ctypes signature.
_c_int, _c_i64, _c_p, _c_sz = ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t
SIGNATURES = {
    "fack_status_string": (ctypes.c_char_p, [_c_int]),
    "fack_version": (_c_int, []),
    "fack_last_error": (ctypes.c_char_p, []),
    "fack_gemm_bs_select": (_c_int, [_c_int, _c_int, _c_int, _c_int,
                                     ctypes.POINTER(_c_int), ctypes.POINTER(_c_int)]),
    "fack_gemm_bs_plan_estimate": (_c_int, [_c_int] * 6 + [ctypes.POINTER(ctypes.c_double)]),
    "fack_gemm_bs_workspace_size": (_c_int, [_c_int, _c_int, _c_int, _c_int, ctypes.POINTER(_c_sz)]),
    "fack_gemm_bs_tail_workspace_size": (_c_int, [_c_int] * 6 + [ctypes.POINTER(_c_sz)]),
    "fack_gemm_bs_plan": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int, ctypes.POINTER(_c_int),
                                   ctypes.POINTER(_c_int), ctypes.POINTER(_c_int), ctypes.POINTER(_c_sz)]),
    "fack_gemm_bs_ex": (_c_int, [_c_p, _c_i64, _c_p, _c_int, _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_i64,
                                 _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_p, _c_sz, _c_p]),
    "fack_gemm_bs_prepack_w": (_c_int, [_c_p, _c_i64, _c_p, _c_int, _c_int, _c_p, _c_p, _c_p]),
    "fack_gemm_bs": (_c_int, [_c_p, _c_i64, _c_p, _c_int, _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_i64,
                              _c_int, _c_int, _c_int, _c_int, _c_p, _c_sz, _c_p]),
    "fack_gemm_bs_noalloc": (_c_int, [_c_p, _c_i64, _c_p, _c_int, _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_i64,
                                      _c_int, _c_int, _c_int, _c_int, _c_p]),
    "fack_gather_interleave": (_c_int, [_c_p, _c_int, _c_int, _c_int, _c_p, _c_i64, _c_p]),
    "fack_quant_act": (_c_int, [_c_p, _c_int, _c_i64, _c_int, _c_int, _c_p, _c_i64, _c_p, _c_i64, _c_i64, _c_p]),
    "fack_device_status": (_c_int, [_c_p, ctypes.POINTER(ctypes.c_uint), _c_int]),
    "fack_gemm_tn_plan": (_c_int, [_c_int] * 7 + [ctypes.POINTER(_c_int)] * 3),
    "fack_gemm_tn": (_c_int, [_c_int, _c_p, _c_i64, _c_p, _c_int, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_i64,
                              _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_p]),
    "fack_gemm_bs_bcast": (_c_int, [_c_p, _c_i64, _c_p, _c_int, _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_i64,
                                    ctypes.POINTER(_c_p), _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                    _c_p, _c_sz, _c_p]),
    "fack_gemm_bs_allgather": (_c_int, [_c_p, _c_i64, _c_p, _c_int, _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_i64,
                                        ctypes.POINTER(_c_p), _c_p, ctypes.POINTER(_c_p), _c_int, _c_int,
                                        _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_p, _c_sz, _c_p]),
    "fack_xchg_barrier": (_c_int, [_c_p, ctypes.POINTER(_c_p), _c_int, _c_int, _c_p]),
    "fack_ipc_get_handle": (_c_int, [_c_p, _c_p, _c_sz, ctypes.POINTER(_c_sz)]),
    "fack_ipc_open_handle": (_c_int, [_c_p, ctypes.POINTER(_c_p)]),
    "fack_ipc_close_handle": (_c_int, [_c_p]),
    "fack_gemm_bs_tuned_set": (_c_int, [_c_int] * 7),
    "fack_gemm_bs_tuned_lookup": (_c_int, [_c_int] * 4 + [ctypes.POINTER(_c_int)] * 3),
    "fack_gemm_bs_tuned_count": (_c_int, []),
    "fack_gemm_bs_tuned_clear": (_c_int, []),
    "fack_gemm_bs_tuned_load": (_c_int, [ctypes.c_char_p, ctypes.POINTER(_c_int), ctypes.POINTER(_c_int)]),
    "fack_gemm_tn_tuned_set": (_c_int, [_c_int] * 8),
    "fack_gemm_tn_tuned_lookup": (_c_int, [_c_int] * 5 + [ctypes.POINTER(_c_int)] * 3),
    "fack_gemm_tn_tuned_count": (_c_int, []),
    "fack_gemm_tn_tuned_clear": (_c_int, []),
    "fack_gemm_tn_tuned_load": (_c_int, [ctypes.c_char_p, ctypes.POINTER(_c_int), ctypes.POINTER(_c_int)]),
}

_lib = None


def load(path: os.PathLike | str | None = None) -> ctypes.CDLL:
    """Load (once) and type the C-ABI library; raises if it is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"{p} is not built; run `python -m fack_b200.build` (nvcc, sm_100a). "
            "The FP8 block-scaled GEMM has no fallback implementation.")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        if path is not None and not hasattr(lib, name):
            continue  # another build (e.g. an older one under comparison) may predate this entry
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
        for table in tuned_tables():
            load_tuned(table, lib)
        for table in tuned_tables(sibling=True):
            load_tuned(table, lib, sibling=True)
    return lib


def tuned_tables(sibling: bool = False) -> list:
    """The plan tables loaded with the library, in merge order (the FP8
    table's, or with ``sibling`` the BF16 / INT8 families')."""
    shipped, env = (TN_TUNED_TABLE, TN_TUNED_ENV) if sibling else (TUNED_TABLE, TUNED_ENV)
    tables = [shipped] if shipped.exists() else []
    extra = os.environ.get(env, "")
    return tables + [Path(p) for p in extra.split(os.pathsep) if p]


def load_tuned(path: os.PathLike | str, lib: ctypes.CDLL | None = None, sibling: bool = False) -> tuple:
    """Merge a tuned-plan CSV into the library's FP8 table (or with
    ``sibling`` the BF16 / INT8 table); returns (rows loaded, rows skipped
    because they name another kernel family).  Raises ValueError naming the
    file and line of the first bad row (the table is then unchanged)."""
    lib = lib or load()
    n, skipped = ctypes.c_int(), ctypes.c_int()
    fn = lib.fack_gemm_tn_tuned_load if sibling else lib.fack_gemm_bs_tuned_load
    st = fn(os.fsencode(str(path)), ctypes.byref(n), ctypes.byref(skipped))
    if st != FACK_OK:
        raise ValueError(f"tuned table {path}: {lib.fack_status_string(st).decode()}: "
                         f"{lib.fack_last_error().decode()}")
    return n.value, skipped.value


def status_string(code: int) -> str:
    return load().fack_status_string(int(code)).decode()


class FackError(RuntimeError):
    """Raised for a non-zero status from the C ABI."""

    def __init__(self, code: int, what: str):
        self.code = int(code)
        detail = load().fack_last_error().decode()
        super().__init__(f"{what}: {status_string(code)} (status {code})" + (f" [{detail}]" if detail else ""))


def check(code: int, what: str) -> None:
    if code == FACK_OK:
        return
    if code in (FACK_ERR_BAD_SHAPE, FACK_ERR_BAD_STRIDE, FACK_ERR_BAD_ARG, FACK_ERR_BAD_ALIGN):
        # contract violations are ValueError before any launch, as in the
        # reference driver (client/aiter/hsa/gfx942/driver.py:11-12)
        raise ValueError(f"{what}: {status_string(code)} (status {code})")
    raise FackError(code, what)
