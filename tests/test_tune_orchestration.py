"""CPU: the tuner's orchestration with the GPU pieces replaced by fakes --
family selection, the table each family clears and writes, the row a shape
produces, the --log lines and the exit status."""
import csv
import json
import types

import pytest
import torch

from fack_b200 import _lib, siblings, tune


class FakeBench:
    """Times every plan from its tile sizes; one plan fails the check."""

    def __init__(self, family, M, N, K, *a, **kw):
        self.family = family

    def check(self, plan):
        return 0.5 if plan == (128, 64, 8) else 0.0

    def time_us(self, plan, repeats=3):
        tm, tn, sk = plan
        return 10.0 + abs(tn - 128) / 64 + abs(sk - 3) * 0.5 + (tm == 256) * 0.25


@pytest.fixture()
def fakes(monkeypatch):
    monkeypatch.setattr(tune, "SiblingShapeBench", FakeBench)
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda i: types.SimpleNamespace(multi_processor_count=148))
    monkeypatch.setattr(siblings, "get_config",
                        lambda kind, M, N, K: {"kernelName": siblings.kernel_name(kind, 128, 256, 5)})
    monkeypatch.setattr(torch.cuda, "empty_cache", lambda: None)
    yield
    lib = _lib.load()
    for sibling in (False, True):
        for table in _lib.tuned_tables(sibling=sibling):
            _lib.load_tuned(table, lib, sibling=sibling)


def test_sibling_shape_row(fakes):
    row = tune.tune_sibling_shape("i8", 256, 3072, 7168)
    assert row["kernelName"] == "fack_tn_sm100_i8_t128x128_s3" and row["splitK"] == 3 and row["us"] == 10.0
    assert row["heuristic_kernelName"] == "fack_tn_sm100_i8_t128x256_s5" and row["heuristic_us"] == 13.0
    assert row["bad_plans"] == ["fack_tn_sm100_i8_t128x64_s8"] and row["cu_num"] == 148
    assert len(row["plans"]) == len(tune.sibling_candidates("i8", 256, 3072, 7168))
    assert row["tflops"] == round(2 * 256 * 3072 * 7168 / 10.0 / 1e6, 1)


def test_main_siblings_writes_both_families(fakes, tmp_path):
    lib = _lib.load()
    assert lib.fack_gemm_tn_tuned_set(_lib.FACK_GEMM_BF16, 148, 1, 3072, 7168, 128, 64, 1) == 0
    out, log = tmp_path / "tn.csv", tmp_path / "plans.jsonl"
    assert tune.main(["--family", "siblings", "--shapes", "256,3072,7168", "--out", str(out),
                      "--log", str(log)]) == 1          # one plan per shape failed its check
    assert lib.fack_gemm_tn_tuned_count() == 0           # the old sibling rows were cleared before timing
    lines = [ln for ln in out.read_text().splitlines() if not ln.startswith("#")]
    rows = list(csv.DictReader(lines))
    assert [r["kernelName"] for r in rows] == ["fack_tn_sm100_bf16_t128x128_s3", "fack_tn_sm100_i8_t128x128_s3"]
    assert out.read_text().startswith("# Exact-shape plans for fack_gemm_tn_plan")
    assert _lib.load_tuned(out, lib, sibling=True) == (2, 0)
    recs = [json.loads(ln) for ln in log.read_text().splitlines()]
    assert {r["kernelName"].split("_")[3] for r in recs} == {"bf16", "i8"}
    assert all(r["model_cycles"] is None for r in recs)


def test_main_family_defaults(fakes, tmp_path, monkeypatch):
    calls = []
    monkeypatch.setattr(tune, "tune_sibling_shape", lambda fam, M, N, K, log=None: calls.append((fam, M, N, K)) or
                        {"cu_num": 148, "M": M, "N": N, "K": K, "kernelName": "fack_tn_sm100_bf16_t128x256_s1",
                         "splitK": 1, "us": 1.0, "tflops": 1.0, "bw": 1.0, "errRatio": 0,
                         "heuristic_kernelName": "x", "heuristic_us": 1.0, "bad_plans": [], "plans": []})
    assert tune.main(["--family", "bf16", "--out", str(tmp_path / "t.csv")]) == 0
    assert [c[1:] for c in calls] == tune.sibling_default_shapes() and {c[0] for c in calls} == {"bf16"}
