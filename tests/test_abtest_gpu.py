"""GPU: the paired A/B harness on real timings (decode shape 256x3072x7168)."""
import pytest

from fack_b200 import _lib, abtest as ab

pytestmark = pytest.mark.gpu

SHAPE = [(256, 3072, 7168)]


def policy(n=8, min_gain=0.01):
    return {"method": ab.SIGN, "confirm_pairs": n, "final_pairs": n, "min_gain": min_gain,
            "alpha": 0.05, "max_confirmations": 1}


def test_clearly_faster_plan_is_confirmed(cuda_device):
    # one K slice of 64-wide weight tiles (96 CTAs, 56 K blocks each) against the tuned 128x256 split-5 plan
    ev = ab.make_evaluator("fack_bs_sm100_t128x64_s1", "fack_bs_sm100_t128x256_s5", SHAPE)
    rep = ab.run_pairs(ev, policy())
    r = rep["results"]["256x3072x7168"]
    assert r["verdict"] == "confirmed_gain", r
    assert r["candidate_median_us"] < r["baseline_median_us"]
    # and the reverse order is a regression
    rep = ab.run_pairs(ab.make_evaluator("fack_bs_sm100_t128x256_s5", "fack_bs_sm100_t128x64_s1", SHAPE), policy())
    assert rep["results"]["256x3072x7168"]["verdict"] == "regression"


def test_library_build_against_its_own_plan_is_not_a_change(cuda_device):
    # the built library's automatic plan for this shape is the tuned 128x256 split 5
    ev = ab.make_evaluator(str(_lib.LIB_PATH), "fack_bs_sm100_t128x256_s5", SHAPE)
    r = ab.run_pairs(ev, policy(min_gain=0.05))["results"]["256x3072x7168"]
    assert r["verdict"] == "inconclusive", r
    assert 0.95 < r["median_ratio"] < 1.05
