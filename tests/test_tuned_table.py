"""CPU: the exact-shape plan table (fack_gemm_bs_tuned_*), its CSV loader and
the tuner's candidate set.  No device is touched: every call here is host-only."""
import csv
import json
import ctypes
import os
import subprocess
import sys
from pathlib import Path

import pytest

from fack_b200 import _lib, tune

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture()
def lib():
    lib = _lib.load()
    lib.fack_gemm_bs_tuned_clear()
    yield lib
    lib.fack_gemm_bs_tuned_clear()
    for table in _lib.tuned_tables():  # leave the table as the library loaded it
        _lib.load_tuned(table, lib)


def lookup(lib, cu, M, N, K):
    tm, tn, sk = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    assert lib.fack_gemm_bs_tuned_lookup(cu, M, N, K, ctypes.byref(tm), ctypes.byref(tn), ctypes.byref(sk)) == 0
    return tm.value, tn.value, sk.value


def test_set_lookup_replace_clear(lib):
    assert lib.fack_gemm_bs_tuned_count() == 0
    assert lookup(lib, 148, 256, 3072, 7168) == (0, 0, 0)
    assert lib.fack_gemm_bs_tuned_set(148, 256, 3072, 7168, 128, 256, 5) == 0
    assert lookup(lib, 148, 256, 3072, 7168) == (128, 256, 5)
    assert lookup(lib, 132, 256, 3072, 7168) == (0, 0, 0)      # another SM count: no row
    assert lookup(lib, 148, 255, 3072, 7168) == (0, 0, 0)      # exact M only, no padding
    assert lib.fack_gemm_bs_tuned_set(148, 256, 3072, 7168, 256, 128, 4) == 0
    assert lookup(lib, 148, 256, 3072, 7168) == (256, 128, 4)  # replaced
    assert lib.fack_gemm_bs_tuned_count() == 1
    assert lib.fack_gemm_bs_tuned_clear() == 0 and lib.fack_gemm_bs_tuned_count() == 0


@pytest.mark.parametrize("row,status", [
    ((148, 256, 3072, 7168, 96, 256, 1), _lib.FACK_ERR_BAD_ARG),    # token tile
    ((148, 256, 3072, 7168, 128, 96, 1), _lib.FACK_ERR_BAD_ARG),    # weight tile
    ((148, 256, 384, 7168, 128, 256, 1), _lib.FACK_ERR_BAD_ARG),    # 256 does not divide 384
    ((148, 256, 3072, 7168, 128, 256, 9), _lib.FACK_ERR_BAD_ARG),   # beyond the cluster limit
    ((148, 256, 3072, 7168, 256, 256, 5), _lib.FACK_ERR_BAD_ARG),   # pair: 2 x split > 8
    ((148, 256, 3072, 256, 128, 256, 3), _lib.FACK_ERR_BAD_ARG),    # split > K/128
    ((148, 256, 3072, 7168, 128, 256, 0), _lib.FACK_ERR_BAD_ARG),
    ((0, 256, 3072, 7168, 128, 256, 1), _lib.FACK_ERR_BAD_ARG),     # cu_num
    ((148, 0, 3072, 7168, 128, 256, 1), _lib.FACK_ERR_BAD_SHAPE),
    ((148, 256, 3000, 7168, 128, 256, 1), _lib.FACK_ERR_BAD_SHAPE),
    ((148, 65535 * 128 + 1, 3072, 7168, 128, 256, 1), _lib.FACK_ERR_BAD_SHAPE),   # beyond 65535 token tiles
    ((148, 8192, 896, 16384, 128, 224, 2), _lib.FACK_ERR_BAD_ARG),  # 224-wide tiles: one K slice only
    ((148, 8192, 896, 16384, 256, 224, 1), _lib.FACK_ERR_BAD_ARG),  # 224-wide tiles: single CTAs only
    ((148, 8192, 1024, 16384, 128, 224, 1), _lib.FACK_ERR_BAD_ARG),  # 224 does not divide 1024
    ((148, 17, 3072, 7168, 16, 16, 1), _lib.FACK_ERR_BAD_ARG),      # small-M kernel: at most 16 tokens
    ((148, 8, 3072, 7168, 32, 16, 1), _lib.FACK_ERR_BAD_ARG),       # small-M kernel: 16-token tile only
    ((148, 8, 3072, 7168, 16, 16, 2), _lib.FACK_ERR_BAD_ARG),       # small-M kernel: no split
    ((148, 8, 3072, 257 * 128, 16, 16, 1), _lib.FACK_ERR_BAD_ARG),  # small-M kernel: K <= 256 blocks
])
def test_invalid_rows_refused(lib, row, status):
    assert lib.fack_gemm_bs_tuned_set(*row) == status
    assert lib.fack_gemm_bs_tuned_count() == 0


def write(tmp_path, text, name="t.csv"):
    p = tmp_path / name
    p.write_text(text)
    return p


def test_largest_m_accepted(lib):
    assert lib.fack_gemm_bs_tuned_set(148, 65535 * 128, 3072, 7168, 128, 256, 1) == 0


def test_csv_load_by_column_name(lib, tmp_path):
    p = write(tmp_path, "\n".join([
        "# comment lines and blank lines are ignored",
        "",
        "M,N,K,cu_num,us,kernelName,splitK,errRatio,extra",
        "256,3072,7168,148,15.2,fack_bs_sm100_t128x256_s5,5,0,x",
        "32,8192,7168,148,9.1,fack_bs_sm100_t256x128_s4,4,0.0,y",
        '"144", "3072", "7168", "80", "20", "_ZN5aiter42fp8gemm_bf16_blockscale_BpreShuffle_64x128E", "1", "0", z',
        "256,3072,7168,148,15.0,fack_bs_sm100_t128x128_s6,6,0,later row wins",
    ]) + "\n")
    assert _lib.load_tuned(p, lib) == (3, 1)
    assert lookup(lib, 148, 256, 3072, 7168) == (128, 128, 6)
    assert lookup(lib, 148, 32, 8192, 7168) == (256, 128, 4)
    assert lookup(lib, 80, 144, 3072, 7168) == (0, 0, 0)       # another library's kernel: skipped
    assert lib.fack_gemm_bs_tuned_count() == 2


GOOD = "148,1,3072,7168,fack_bs_sm100_t128x64_s1"


@pytest.mark.parametrize("rows,why", [
    (["cu_num,M,N,K,kernelName,splitK", GOOD + ",1", "148,256,3072,7168,fack_bs_sm100_t128x256_s5,4"],
     "splitK disagrees"),
    (["cu_num,M,N,K,kernelName,errRatio", GOOD + ",0", "148,256,3072,7168,fack_bs_sm100_t128x256_s5,0.01"],
     "errRatio"),
    (["cu_num,M,N,kernelName", "148,256,3072,fack_bs_sm100_t128x256_s5"], "header lacks"),
    (["cu_num,M,N,K,kernelName", GOOD, "148,256,3072,7168"], "field count"),
    (["cu_num,M,N,K,kernelName", GOOD, "148,256,3072,7168.5,fack_bs_sm100_t128x256_s5"], "integers"),
    (["cu_num,M,N,K,kernelName", GOOD, "148,256,384,7168,fack_bs_sm100_t128x256_s5"], "invalid for this shape"),
    (["cu_num,M,N,K,kernelName", GOOD, "148,256,3072,7168,fack_bs_sm100_t0128x256_s5"], "malformed"),
    (["cu_num,M,N,K,kernelName", GOOD, "148,256,3072,7168,fack_bs_sm100_t128x256_s+5"], "malformed"),
])
def test_bad_file_leaves_table_unchanged(lib, tmp_path, rows, why):
    assert lib.fack_gemm_bs_tuned_set(148, 1, 128, 128, 128, 64, 1) == 0
    p = write(tmp_path, "\n".join(rows) + "\n")
    with pytest.raises(ValueError) as e:
        _lib.load_tuned(p, lib)
    line = 1 if why == "header lacks" else len(rows)     # the first bad line is named
    assert why in str(e.value) and f"{p}:{line}:" in str(e.value)
    assert lib.fack_gemm_bs_tuned_count() == 1                 # nothing of the bad file was added
    assert lookup(lib, 148, 1, 3072, 7168) == (0, 0, 0)


def test_missing_file_and_empty_file(lib, tmp_path):
    with pytest.raises(ValueError):
        _lib.load_tuned(tmp_path / "absent.csv", lib)
    with pytest.raises(ValueError):
        _lib.load_tuned(write(tmp_path, "# only a comment\n"), lib)


def test_environment_tables_merge_over_the_shipped_one(tmp_path):
    p = write(tmp_path, "cu_num,M,N,K,kernelName\n148,7,3072,7168,fack_bs_sm100_t256x64_s2\n")
    code = ("import ctypes; from fack_b200 import _lib; lib = _lib.load(); r = [ctypes.c_int() for _ in range(3)];"
            "lib.fack_gemm_bs_tuned_lookup(148, 7, 3072, 7168, *map(ctypes.byref, r)); print([x.value for x in r])")
    env = dict(os.environ, **{_lib.TUNED_ENV: str(p)})
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True, check=True)
    assert out.stdout.strip() == "[256, 64, 2]"


def test_tuner_candidates_are_exactly_the_valid_plans():
    lib = _lib.load()
    tm, tn, sk, nb = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()
    for M, N, K in ((256, 3072, 7168), (48, 4096, 2048), (33, 384, 640), (1, 128, 256), (16, 3072, 7168),
                    (64, 1024, 40960), (8192, 896, 16384), (300, 1792, 1024)):
        cands = tune.candidates(M, N, K)
        assert len(set(cands)) == len(cands)
        for c in cands:
            assert lib.fack_gemm_bs_plan(M, N, K, *c, ctypes.byref(tm), ctypes.byref(tn), ctypes.byref(sk),
                                         ctypes.byref(nb)) == 0
            assert (tm.value, tn.value, sk.value) == c
        for t_m in (16, 32, 64, 128, 256):
            for t_n in (16, 64, 128, 224, 256):
                for s in range(1, 9):
                    ok = lib.fack_gemm_bs_plan(M, N, K, t_m, t_n, s, ctypes.byref(tm), ctypes.byref(tn),
                                               ctypes.byref(sk), ctypes.byref(nb)) == 0
                    assert ok == ((t_m, t_n, s) in cands), (M, N, K, t_m, t_n, s)


def test_default_shapes_cover_the_reference_records_and_workloads():
    shapes = tune.default_shapes()
    assert len(tune.RECORD_SHAPES) == 43 and len(set(tune.RECORD_SHAPES)) == 43
    assert set(tune.RECORD_SHAPES) <= set(shapes)
    assert (256, 3072, 7168) in shapes and (8192, 7168, 16384) in shapes and (32, 65536, 7168) in shapes
    # one rank's shard of the column-sharded workloads at 2, 4 and 8 GPUs
    for s in ((32, 32768, 7168), (32, 16384, 7168), (32, 8192, 7168),
              (8192, 3584, 16384), (8192, 1792, 16384), (8192, 896, 16384)):
        assert s in shapes, s
    assert len(shapes) == len(set(shapes))
    assert all(n % 128 == 0 and k % 128 == 0 for _, n, k in shapes)


def test_shipped_table_is_valid():
    if not _lib.TUNED_TABLE.exists():
        pytest.skip("no shipped table")
    rows = list(csv.DictReader(line for line in _lib.TUNED_TABLE.read_text().splitlines()
                               if not line.startswith("#")))
    assert rows
    shapes = set(tune.default_shapes())
    for r in rows:
        M, N, K = int(r["M"]), int(r["N"]), int(r["K"])
        assert (M, N, K) in shapes
        assert int(r["cu_num"]) == 148 and float(r["errRatio"]) == 0
        assert r["kernelName"].endswith(f"_s{r['splitK']}")
        assert float(r["us"]) <= float(r["heuristic_us"]) + 1e-6   # never slower than the cost model's plan
    lib = _lib.load()
    assert lib.fack_gemm_bs_tuned_count() >= len({(r["M"], r["N"], r["K"]) for r in rows})


def test_tuner_choice_rule():
    r = [(10.0, "fack_bs_sm100_t128x256_s5", 5, 0.0), (9.0, "fack_bs_sm100_t128x128_s6", 6, 0.0),
         (5.0, "fack_bs_sm100_t128x64_s8", 8, 0.25)]                  # fastest, but fails the check
    assert tune.choose(r, "fack_bs_sm100_t64x128_s1")[1] == "fack_bs_sm100_t128x128_s6"
    # the cost model's plan within KEEP_MARGIN of the best stays
    near = [(9.0 * (1 + tune.KEEP_MARGIN / 2), "fack_bs_sm100_t128x256_s5", 5, 0.0)] + r[1:]
    assert tune.choose(near, "fack_bs_sm100_t128x256_s5")[1] == "fack_bs_sm100_t128x256_s5"
    assert tune.choose(r, "fack_bs_sm100_t128x256_s5")[1] == "fack_bs_sm100_t128x128_s6"   # 11 % slower: replaced
    assert tune.choose(r, "fack_bs_sm100_t128x64_s8")[1] == "fack_bs_sm100_t128x128_s6"    # failing plan never kept
    with pytest.raises(RuntimeError, match="no plan"):
        tune.choose([r[2]], "fack_bs_sm100_t128x64_s8", (256, 3072, 7168))


def test_tuner_csv_loads_into_the_c_table(lib, tmp_path):
    """write_csv's output is what fack_gemm_bs_tuned_load reads."""
    rows = [{"cu_num": 148, "M": 256, "N": 3072, "K": 7168, "kernelName": "fack_bs_sm100_t128x256_s5",
             "splitK": 5, "us": 14.5, "tflops": 777.0, "bw": 1758.0, "errRatio": 0,
             "heuristic_kernelName": "fack_bs_sm100_t128x256_s5", "heuristic_us": 14.5, "bad_plans": []},
            {"cu_num": 148, "M": 32, "N": 3072, "K": 7168, "kernelName": "fack_bs_sm100_t32x128_s5",
             "splitK": 5, "us": 9.3, "tflops": 47.4, "bw": 2372.0, "errRatio": 0,
             "heuristic_kernelName": "fack_bs_sm100_t128x256_s8", "heuristic_us": 10.4, "bad_plans": []}]
    p = tmp_path / "tuned.csv"
    tune.write_csv(rows, p)
    assert _lib.load_tuned(p, lib) == (2, 0)
    assert lookup(lib, 148, 256, 3072, 7168) == (128, 256, 5)
    assert lookup(lib, 148, 32, 3072, 7168) == (32, 128, 5)


def test_plan_estimate_validates_before_any_device_query(lib):
    cyc = ctypes.c_double(-1.0)
    assert lib.fack_gemm_bs_plan_estimate(0, 3072, 7168, 128, 256, 5, ctypes.byref(cyc)) == _lib.FACK_ERR_BAD_SHAPE
    assert lib.fack_gemm_bs_plan_estimate(256, 3072, 7168, 0, 256, 5, ctypes.byref(cyc)) == _lib.FACK_ERR_BAD_ARG
    assert lib.fack_gemm_bs_plan_estimate(256, 3072, 7168, 128, 96, 5, ctypes.byref(cyc)) == _lib.FACK_ERR_BAD_ARG
    assert lib.fack_gemm_bs_plan_estimate(65, 3072, 7168, 64, 128, 5, ctypes.byref(cyc)) == _lib.FACK_ERR_BAD_ARG
    assert lib.fack_gemm_bs_plan_estimate(256, 3072, 7168, 128, 256, 5, None) == _lib.FACK_ERR_BAD_ARG
    assert cyc.value == -1.0


def test_tuner_log_lines(tmp_path):
    rec = tune.plan_record(256, 3072, 7168, "fack_bs_sm100_t128x256_s5", 14.4861, 0.0, 27311.26)
    bad = tune.plan_record(256, 3072, 7168, "fack_bs_sm100_t128x64_s8", float("inf"), 0.25, None)
    p = tmp_path / "plans.jsonl"
    tune.write_log([{"plans": [rec, bad]}, {"plans": []}], p)
    lines = [json.loads(ln) for ln in p.read_text().splitlines()]
    assert lines == [{"M": 256, "N": 3072, "K": 7168, "kernelName": "fack_bs_sm100_t128x256_s5", "us": 14.486,
                      "errRatio": 0.0, "model_cycles": 27311.3},
                     {"M": 256, "N": 3072, "K": 7168, "kernelName": "fack_bs_sm100_t128x64_s8", "us": None,
                      "errRatio": 0.25, "model_cycles": None}]


def test_model_report_regret(tmp_path):
    rec = tune.plan_record
    log = [rec(256, 3072, 7168, "fack_bs_sm100_t128x256_s5", 14.5, 0.0, 26000.0),     # model's pick, 10 % slow
           rec(256, 3072, 7168, "fack_bs_sm100_t128x128_s6", 13.18, 0.0, 27000.0),    # measured best
           rec(256, 3072, 7168, "fack_bs_sm100_t128x64_s8", float("inf"), 0.5, 1.0),  # failed: ignored
           rec(32, 3072, 7168, "fack_bs_sm100_t32x128_s5", 9.3, 0.0, 17000.0),        # pick = best
           rec(32, 3072, 7168, "fack_bs_sm100_t32x128_s1", 8.0, 0.0, None)]           # not offered
    rep = tune.model_report(log)
    assert rep["shapes"] == 2
    by = {p["shape"]: p for p in rep["per_shape"]}
    assert by["256x3072x7168"]["regret"] == pytest.approx(14.5 / 13.18 - 1)
    assert by["32x3072x7168"]["model_pick"] == "fack_bs_sm100_t32x128_s5"
    assert by["32x3072x7168"]["regret"] == pytest.approx(9.3 / 8.0 - 1)   # the unoffered plan was faster
    assert [m["shape"] for m in rep["misses"]] == ["32x3072x7168", "256x3072x7168"]
    p = tmp_path / "plans.jsonl"
    tune.write_log([{"plans": log}], p)
    assert tune.main(["--report", str(p)]) == 0
