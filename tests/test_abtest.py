"""CPU: the paired A/B statistics (exact ranks against brute-force
enumeration, verdicts, sequential looks, policy validation) and the trial
driver with a fake evaluator."""
import itertools
import math
import random

import pytest

from fack_b200 import abtest as ab


def sign_policy(n, alpha=0.05, min_gain=0.01, max_conf=1):
    return {"method": ab.SIGN, "confirm_pairs": n, "final_pairs": n, "min_gain": min_gain,
            "alpha": alpha, "max_confirmations": max_conf}


def seq_policy(looks, statistic="signed_rank", alpha=0.05, min_gain=0.01, futility=True):
    return {"method": ab.SEQUENTIAL, "statistic": statistic, "confirm_looks": looks, "final_looks": looks,
            "min_gain": min_gain, "alpha": alpha, "max_confirmations": 1, "futility_stop": futility}


@pytest.mark.parametrize("alpha", [0.01, 0.025, 0.05, 0.1, 0.2])
def test_sign_rank_is_the_exact_binomial_bound(alpha):
    for n in range(1, 25):
        # brute force: largest r <= n/2 with P(#negatives <= r-1) <= alpha
        want = 0
        for r in range(1, n // 2 + 1):
            p = sum(math.comb(n, j) for j in range(r)) / 2 ** n
            if p <= alpha:
                want = r
        assert ab.sign_rank(n, alpha) == want, (n, alpha)


@pytest.mark.parametrize("alpha", [0.01, 0.05, 0.1])
def test_signed_rank_rank_matches_enumerated_null(alpha):
    for n in range(1, 13):
        sums = [sum(k + 1 for k in range(n) if pattern[k]) for pattern in itertools.product((0, 1), repeat=n)]
        want = 0
        for t in range(n * (n + 1) // 2 + 1):
            if sum(s <= t for s in sums) / 2 ** n <= alpha:
                want = t + 1
            else:
                break
        assert ab.signed_rank_rank(n, alpha) == want, (n, alpha)


def test_pair_order_alternates():
    assert [ab.pair_order(i) for i in range(4)] == [("baseline", "candidate"), ("candidate", "baseline")] * 2


@pytest.mark.parametrize("policy", [
    sign_policy(7),                                   # odd: order not balanced
    sign_policy(4),                                   # rank 0 at alpha 0.05
    sign_policy(8, alpha=0.5),
    sign_policy(8, min_gain=-0.1),
    sign_policy(8, alpha=float("nan")),
    dict(sign_policy(8), extra=1),
    sign_policy(8, max_conf=0),
    sign_policy(8, max_conf=20),                      # confirm alpha 0.0025 < 1/256: no rank
    seq_policy([{"pairs": 8, "alpha_share": 0.5}, {"pairs": 16, "alpha_share": 0.4}]),   # shares != 1
    seq_policy([{"pairs": 16, "alpha_share": 0.5}, {"pairs": 8, "alpha_share": 0.5}]),   # not increasing
    seq_policy([{"pairs": 2, "alpha_share": 1.0}]),                                      # too small
    seq_policy([{"pairs": 8, "alpha_share": 1.0}], statistic="t"),
    {"method": "bayes"},
])
def test_invalid_policies_refused(policy):
    with pytest.raises(ValueError):
        ab.validate_policy(policy)


def pairs_from_ratios(ratios):
    """candidate score / baseline score per pair."""
    return [{"baseline": 1.0, "candidate": r} for r in ratios]


def test_sign_verdicts_and_bounds():
    gain = [1.05, 1.04, 1.06, 1.05, 1.03, 1.07, 1.05, 1.045]
    r = ab.assess(pairs_from_ratios(gain), sign_policy(8))
    assert r["verdict"] == "confirmed_gain" and r["rank"] == 2
    s = sorted(gain)
    assert r["lower_ratio_bound"] == pytest.approx(s[1]) and r["upper_ratio_bound"] == pytest.approx(s[-2])
    r = ab.assess(pairs_from_ratios([1 / g for g in gain]), sign_policy(8))
    assert r["verdict"] == "regression"
    r = ab.assess(pairs_from_ratios([1.05, 0.95, 1.02, 0.99, 1.0, 1.01, 0.98, 1.03]), sign_policy(8))
    assert r["verdict"] == "inconclusive"
    # a 0.5 % gain is real but below min_gain = 1 %: not confirmed
    r = ab.assess(pairs_from_ratios([1.005] * 8), sign_policy(8))
    assert r["verdict"] == "inconclusive"
    with pytest.raises(ValueError):
        ab.assess(pairs_from_ratios(gain[:6]), sign_policy(8))         # every planned pair
    with pytest.raises(ValueError):
        ab.assess([{"baseline": 1.0, "candidate": 0.0}] * 8, sign_policy(8))


def test_sequential_stops_at_first_decisive_look():
    looks = [{"pairs": 8, "alpha_share": 0.5}, {"pairs": 16, "alpha_share": 0.5}]
    pol = seq_policy(looks)
    strong = [1.1] * 16
    r = ab.assess(pairs_from_ratios(strong[:8]), pol)
    assert r["verdict"] == "confirmed_gain" and r["stop_reason"] == "confirmed_gain" and r["pairs"] == 8
    with pytest.raises(ValueError):
        ab.assess(pairs_from_ratios(strong), pol)                      # should have stopped at 8
    with pytest.raises(ab.NotStopped):
        ab.assess(pairs_from_ratios([1.0, 1.02, 0.98, 1.01, 0.99, 1.0, 1.03, 0.97]),
                  seq_policy(looks, futility=False))
    # half the pairs 10 % slower, half equal: bounds [log 0.9, 0] -- no verdict, but the
    # upper bound is below log(1.01), so the futility rule stops at the first look
    slow = [0.9, 1.0] * 4
    r = ab.assess(pairs_from_ratios(slow), seq_policy(looks, statistic="sign"))
    assert (r["verdict"], r["stop_reason"], r["pairs"]) == ("inconclusive", "futility", 8)
    assert r["upper_ratio_bound"] == pytest.approx(1.0) and r["lower_ratio_bound"] == pytest.approx(0.9)


def test_null_false_gain_rate_within_alpha():
    rng = random.Random(5)
    pol = sign_policy(16, alpha=0.05, min_gain=0.0)
    hits = 0
    trials = 3000
    for _ in range(trials):
        ratios = [math.exp(rng.gauss(0, 0.02)) for _ in range(16)]
        hits += ab.assess(pairs_from_ratios(ratios), pol)["verdict"] == "confirmed_gain"
    assert hits / trials <= 0.05 + 0.01


def test_run_pairs_with_fake_evaluator():
    calls = []
    rng = random.Random(1)

    def evaluate(side):
        calls.append(side)
        base = {"a": 10.0, "b": 20.0}
        f = {"a": 0.9, "b": 1.0} if side == "candidate" else {"a": 1.0, "b": 1.0}
        return {k: v * f[k] * math.exp(rng.gauss(0, 0.003)) for k, v in base.items()}

    rep = ab.run_pairs(evaluate, sign_policy(8))
    assert calls[:4] == ["baseline", "candidate", "candidate", "baseline"] and len(calls) == 16
    assert rep["results"]["a"]["verdict"] == "confirmed_gain"
    assert rep["results"]["b"]["verdict"] == "inconclusive"
    assert rep["results"]["a"]["candidate_median_us"] < rep["results"]["a"]["baseline_median_us"]


def test_run_pairs_sequential_names_stop_independently():
    looks = [{"pairs": 8, "alpha_share": 0.5}, {"pairs": 16, "alpha_share": 0.5}]
    n = {"i": 0}

    def evaluate(side):
        n["i"] += 1
        jitter = 1.0 + 0.001 * (n["i"] % 5)
        return {"fast": (5.0 if side == "candidate" else 10.0) * jitter,
                "same": 10.0 * (1.0 + 0.002 * ((n["i"] * 7) % 3 - 1))}

    rep = ab.run_pairs(evaluate, seq_policy(looks, futility=False))
    assert rep["results"]["fast"]["pairs"] == 8 and rep["results"]["fast"]["verdict"] == "confirmed_gain"
    assert rep["results"]["same"]["pairs"] == 16 and rep["results"]["same"]["stop_reason"] == "max_pairs"
    assert len(rep["records"]) == 16


def test_run_pairs_refuses_changing_timing_names():
    k = {"i": 0}

    def evaluate(side):
        k["i"] += 1
        return {"a": 1.0} if k["i"] < 3 else {"b": 1.0}

    with pytest.raises(ValueError):
        ab.run_pairs(evaluate, sign_policy(8))


def test_version_specs_per_family():
    """Plans must belong to the compared family; library paths work for every family."""
    from fack_b200 import _lib
    v = ab._Version("fack_tn_sm100_i8_t128x256_s5", "i8")
    assert v.plan == (128, 256, 5) and v.kind == _lib.FACK_GEMM_I8
    assert ab._Version("fack_bs_sm100_t32x128_s5").plan == (32, 128, 5)
    assert ab._Version(str(_lib.LIB_PATH), "bf16").plan == (0, 0, 0)
    for spec, family in (("fack_tn_sm100_bf16_t128x256_s5", "blockscale"),   # sibling plan, FP8 comparison
                         ("fack_bs_sm100_t128x256_s5", "i8"),                 # FP8 plan, sibling comparison
                         ("fack_tn_sm100_bf16_t128x256_s5", "i8"),            # the other sibling
                         ("fack_tn_sm100_i8_t256x256_s8", "i8"),              # pair: split <= 4
                         ("/no/such/libfack_gemm.so", "bf16"),
                         ("fack_bs_sm100_t128x256_s5", "fp4")):
        with pytest.raises(ValueError):
            ab._Version(spec, family)
