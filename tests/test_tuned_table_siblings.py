"""CPU: the exact-shape plan table of the sibling families (BF16 TN, INT8 per
token; fack_gemm_tn_tuned_*): rows keyed by (kind, SM count, M, N, K), checked
by the sibling planner's explicit-plan rules, kept apart from the FP8 rows,
and loaded from the same CSV form (kernelName fack_tn_sm100_{bf16|i8}_...)."""
import ctypes
import os
import subprocess
import sys
from pathlib import Path

import pytest

from fack_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
BF, I8 = _lib.FACK_GEMM_BF16, _lib.FACK_GEMM_I8


@pytest.fixture()
def lib():
    lib = _lib.load()
    lib.fack_gemm_tn_tuned_clear()
    lib.fack_gemm_bs_tuned_clear()
    yield lib
    lib.fack_gemm_tn_tuned_clear()
    lib.fack_gemm_bs_tuned_clear()
    for sibling in (False, True):  # leave the tables as the library loaded them
        for table in _lib.tuned_tables(sibling=sibling):
            _lib.load_tuned(table, lib, sibling=sibling)


def lookup(lib, kind, cu, M, N, K):
    tm, tn, sk = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    assert lib.fack_gemm_tn_tuned_lookup(kind, cu, M, N, K, ctypes.byref(tm), ctypes.byref(tn),
                                         ctypes.byref(sk)) == 0
    return tm.value, tn.value, sk.value


def test_rows_per_kind_and_apart_from_the_fp8_table(lib):
    assert lib.fack_gemm_tn_tuned_set(BF, 148, 256, 3072, 7168, 128, 256, 5) == 0
    assert lib.fack_gemm_tn_tuned_set(I8, 148, 256, 3072, 7168, 256, 128, 2) == 0
    assert lib.fack_gemm_bs_tuned_set(148, 256, 3072, 7168, 128, 64, 1) == 0
    assert lookup(lib, BF, 148, 256, 3072, 7168) == (128, 256, 5)
    assert lookup(lib, I8, 148, 256, 3072, 7168) == (256, 128, 2)
    assert lookup(lib, BF, 132, 256, 3072, 7168) == (0, 0, 0)
    assert lib.fack_gemm_tn_tuned_count() == 2 and lib.fack_gemm_bs_tuned_count() == 1
    assert lib.fack_gemm_tn_tuned_clear() == 0
    assert lib.fack_gemm_tn_tuned_count() == 0 and lib.fack_gemm_bs_tuned_count() == 1   # FP8 rows untouched
    lib.fack_gemm_bs_tuned_clear()
    assert lib.fack_gemm_bs_tuned_count() == 0


@pytest.mark.parametrize("row,status", [
    ((7, 148, 256, 3072, 7168, 128, 256, 1), _lib.FACK_ERR_BAD_ARG),    # not a sibling kind
    ((BF, 0, 256, 3072, 7168, 128, 256, 1), _lib.FACK_ERR_BAD_ARG),     # cu_num
    ((BF, 148, 256, 3072, 7168, 64, 128, 1), _lib.FACK_ERR_BAD_ARG),    # no swapped tiles in this family
    ((BF, 148, 256, 3072, 7168, 128, 96, 1), _lib.FACK_ERR_BAD_ARG),
    ((BF, 148, 256, 3072, 7168, 256, 128, 5), _lib.FACK_ERR_BAD_ARG),   # pair: 2 x split > 8
    ((BF, 148, 256, 3072, 7168, 128, 256, 0), _lib.FACK_ERR_BAD_ARG),   # every field given
    ((I8, 148, 256, 3072, 7104, 128, 256, 1), _lib.FACK_ERR_BAD_SHAPE), # int8: K % 128
    ((BF, 148, 256, 3000, 7168, 128, 64, 1), _lib.FACK_ERR_BAD_SHAPE),  # N % 64
])
def test_invalid_rows_refused(lib, row, status):
    assert lib.fack_gemm_tn_tuned_set(*row) == status
    assert lib.fack_gemm_tn_tuned_count() == 0


def test_bf16_k_multiple_of_64_accepted(lib):
    assert lib.fack_gemm_tn_tuned_set(BF, 148, 256, 3072, 7104, 128, 256, 1) == 0    # 7104 = 111 x 64


def write(tmp_path, text, name="tn.csv"):
    p = tmp_path / name
    p.write_text(text)
    return p


def test_csv_load_kind_from_name_and_skips(lib, tmp_path):
    p = write(tmp_path, "\n".join([
        "# sibling plans",
        "kernelName,cu_num,M,N,K,splitK,errRatio,us",
        "fack_tn_sm100_bf16_t128x256_s5,148,256,3072,7168,5,0,18.4",
        "fack_tn_sm100_i8_t256x256_s1,148,8192,8192,8192,1,0,420.7",
        "fack_bs_sm100_t128x256_s5,148,256,3072,7168,5,0,14.5",                       # FP8 row: skipped
        "_ZN5aiter35bf16gemm_fp32bf16_tn_48x64_pf3_splitkE,80,256,3072,7168,1,0,30",   # gfx942: skipped
    ]) + "\n")
    assert _lib.load_tuned(p, lib, sibling=True) == (2, 2)
    assert lookup(lib, BF, 148, 256, 3072, 7168) == (128, 256, 5)
    assert lookup(lib, I8, 148, 8192, 8192, 8192) == (256, 256, 1)
    assert lookup(lib, I8, 148, 256, 3072, 7168) == (0, 0, 0)
    assert lib.fack_gemm_bs_tuned_count() == 0


@pytest.mark.parametrize("bad,why", [
    ("fack_tn_sm100_fp8_t128x256_s1,148,256,3072,7168", "malformed"),
    ("fack_tn_sm100_bf16_t0128x256_s1,148,256,3072,7168", "malformed"),
    ("fack_tn_sm100_i8_t256x256_s8,148,256,3072,7168", "invalid for this shape"),
    ("fack_tn_sm100_i8_t128x256_s1,148,256,3072,7104", "invalid for this shape"),
])
def test_bad_rows_leave_the_table_unchanged(lib, tmp_path, bad, why):
    good = "fack_tn_sm100_bf16_t128x64_s1,148,1,3072,7168"
    p = write(tmp_path, "kernelName,cu_num,M,N,K\n" + good + "\n" + bad + "\n")
    with pytest.raises(ValueError) as e:
        _lib.load_tuned(p, lib, sibling=True)
    assert why in str(e.value) and f"{p}:3:" in str(e.value)
    assert lib.fack_gemm_tn_tuned_count() == 0


def test_environment_table_loads_with_the_library(tmp_path):
    p = write(tmp_path, "cu_num,M,N,K,kernelName\n148,7,3072,7168,fack_tn_sm100_i8_t256x64_s2\n")
    code = ("import ctypes; from fack_b200 import _lib; lib = _lib.load(); r = [ctypes.c_int() for _ in range(3)];"
            "lib.fack_gemm_tn_tuned_lookup(1, 148, 7, 3072, 7168, *map(ctypes.byref, r)); print([x.value for x in r])")
    env = dict(os.environ, **{_lib.TN_TUNED_ENV: str(p)})
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True, check=True)
    assert out.stdout.strip() == "[256, 64, 2]"


@pytest.mark.parametrize("family,shape", [("bf16", (256, 3072, 7168)), ("i8", (256, 3072, 7168)),
                                          ("bf16", (33, 384, 640)), ("i8", (33, 384, 640)), ("i8", (8, 192, 256))])
def test_sibling_tuner_candidates_are_exactly_the_valid_plans(family, shape):
    from fack_b200 import tune
    lib = _lib.load()
    kind = BF if family == "bf16" else I8
    M, N, K = shape
    cands = set(tune.sibling_candidates(family, M, N, K))
    assert cands
    out = [ctypes.c_int() for _ in range(3)]
    for tm in (64, 128, 256):
        for tn in (64, 128, 256):
            for sk in range(1, 10):
                ok = lib.fack_gemm_tn_plan(kind, M, N, K, tm, tn, sk, *map(ctypes.byref, out)) == 0
                assert ok == ((tm, tn, sk) in cands), (family, shape, tm, tn, sk)


def test_sibling_tuner_csv_loads_into_the_sibling_table(lib, tmp_path):
    from fack_b200 import tune
    rows = [{"cu_num": 148, "M": 256, "N": 3072, "K": 7168, "kernelName": "fack_tn_sm100_bf16_t128x256_s5",
             "splitK": 5, "us": 18.4, "tflops": 612.0, "bw": 2675.0, "errRatio": 0,
             "heuristic_kernelName": "fack_tn_sm100_bf16_t128x256_s5", "heuristic_us": 18.4, "bad_plans": []},
            {"cu_num": 148, "M": 256, "N": 3072, "K": 7168, "kernelName": "fack_tn_sm100_i8_t128x128_s6",
             "splitK": 6, "us": 15.9, "tflops": 709.0, "bw": 1600.0, "errRatio": 0,
             "heuristic_kernelName": "fack_tn_sm100_i8_t128x256_s5", "heuristic_us": 16.5, "bad_plans": []}]
    p = tmp_path / "tn.csv"
    tune.write_csv(rows, p, "fack_gemm_tn_plan")
    assert p.read_text().startswith("# Exact-shape plans for fack_gemm_tn_plan")
    assert _lib.load_tuned(p, lib, sibling=True) == (2, 0)
    assert lookup(lib, BF, 148, 256, 3072, 7168) == (128, 256, 5)
    assert lookup(lib, I8, 148, 256, 3072, 7168) == (128, 128, 6)
