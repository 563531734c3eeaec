"""Paired A/B comparison of two versions of the GEMM on B200.

``python -m fack_b200.abtest <baseline> <candidate> --shape M,N,K [--shape ...]
--pairs 8 --min-gain 0.01 --alpha 0.05``

A version is either a build of the library (a path to a ``libfack_gemm.so``)
or a plan of the current build (a kernel name ``fack_bs_sm100_t..x.._s..``;
with ``--family bf16|i8`` the sibling GEMMs are timed instead and plans are
``fack_tn_sm100_{bf16|i8}_t..x.._s..``).
Each trial times both versions on the same resident inputs, in alternating
order (baseline first on even trials, candidate first on odd ones), and the
pair of scores (1 / time) is reduced to a log ratio.  The verdict follows the
reference's acceptance statistics (harness/comparison.py:1-30, assess_pairs
:239; client/aiter/compare.py:51-69 pairs per-distribution timings the same
way):

* ``paired_sign_v1``: a fixed, even number of pairs.  The lower and upper
  bounds of the median log ratio are the r-th smallest and r-th largest log
  ratio, r the largest rank whose one-sided binomial(n, 1/2) tail is <= alpha
  (a distribution-free confidence bound for a median).  Verdict:
  ``confirmed_gain`` if the lower bound exceeds log(1 + min_gain),
  ``regression`` if the upper bound is below -log(1 + min_gain), else
  ``inconclusive``.
* ``paired_sequential_v1``: predeclared looks (even, increasing pair counts),
  each spending a share of alpha (Bonferroni), statistic ``sign`` or
  ``signed_rank`` (bounds from the Walsh averages with the exact Wilcoxon
  signed-rank distribution); the comparison stops at the first decisive look,
  or for futility when the upper bound falls below the threshold.
* In the ``confirm`` stage alpha is divided by ``max_confirmations``; the
  ``final`` stage uses alpha itself.

Timing of one evaluation: a CUDA graph of ``launches`` calls over input sets
larger than 2.5 x the 126 MB L2, replayed once to warm up and once timed with
CUDA events on the launch stream.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import statistics
import sys
from functools import lru_cache
from pathlib import Path
from typing import Callable, Dict, List

SIGN = "paired_sign_v1"
SEQUENTIAL = "paired_sequential_v1"
LOG_TOL = 1e-12


# ---------------------------------------------------------------- statistics --

def sign_rank(n: int, alpha: float) -> int:
    """Largest r <= n/2 with P(Binomial(n, 1/2) <= r - 1) <= alpha, else 0: the
    r-th order statistic of n paired log ratios is a lower confidence bound of
    their median with one-sided non-coverage <= alpha."""
    best, tail = 0, 0
    for r in range(1, n // 2 + 1):
        tail += math.comb(n, r - 1)
        if tail > alpha * 2 ** n:
            break
        best = r
    return best


@lru_cache(maxsize=None)
def _wilcoxon_cdf_counts(n: int) -> tuple:
    """c[t] = number of the 2^n sign patterns whose positive-rank sum is <= t."""
    ways = [0] * (n * (n + 1) // 2 + 1)
    ways[0] = 1
    for k in range(1, n + 1):           # add rank k: either positive (shift by k) or not
        for t in range(len(ways) - 1, k - 1, -1):
            ways[t] += ways[t - k]
    out, acc = [], 0
    for w in ways:
        acc += w
        out.append(acc)
    return tuple(out)


def signed_rank_rank(n: int, alpha: float) -> int:
    """Rank r (1-based) into the sorted n(n+1)/2 Walsh averages whose r-th
    smallest value is a lower bound of the pseudo-median with non-coverage <=
    alpha under the symmetric null: r = 1 + max{t : P(T+ <= t) <= alpha}, or 0
    when even t = 0 exceeds alpha."""
    counts = _wilcoxon_cdf_counts(n)
    limit = alpha * 2 ** n
    r = 0
    while r < len(counts) and counts[r] <= limit:
        r += 1
    return r


def _rank(statistic: str, n: int, alpha: float) -> int:
    return sign_rank(n, alpha) if statistic == "sign" else signed_rank_rank(n, alpha)


def stage_alpha(policy: dict, stage: str) -> float:
    return policy["alpha"] / policy["max_confirmations"] if stage == "confirm" else policy["alpha"]


def pair_order(trial: int) -> tuple:
    return ("baseline", "candidate") if trial % 2 == 0 else ("candidate", "baseline")


def _finite(x) -> bool:
    return not isinstance(x, bool) and isinstance(x, (int, float)) and math.isfinite(x)


def validate_policy(policy: dict) -> dict:
    """Every sample size and threshold is explicit; odd pair counts (unbalanced
    order) and samples too small for their alpha are refused."""
    if not isinstance(policy, dict):
        raise ValueError("policy must be a dict")
    common = {"method", "min_gain", "alpha", "max_confirmations"}
    if policy.get("method") == SEQUENTIAL:
        fields = common | {"statistic", "confirm_looks", "final_looks", "futility_stop"}
    elif policy.get("method") == SIGN:
        fields = common | {"confirm_pairs", "final_pairs"}
    else:
        raise ValueError(f"method must be {SIGN} or {SEQUENTIAL}")
    if set(policy) != fields:
        raise ValueError(f"policy needs exactly {sorted(fields)}")
    mc = policy["max_confirmations"]
    if type(mc) is not int or not 1 <= mc <= 1024:
        raise ValueError("max_confirmations must be an integer in [1, 1024]")
    if not _finite(policy["alpha"]) or not _finite(policy["min_gain"]):
        raise ValueError("alpha and min_gain must be finite numbers")
    if not 0 < policy["alpha"] < 0.5 or policy["min_gain"] < 0:
        raise ValueError("need 0 < alpha < 0.5 and min_gain >= 0")
    for stage in ("confirm", "final"):
        if policy["method"] == SIGN:
            n = policy[stage + "_pairs"]
            if type(n) is not int or not 1 <= n <= 1024 or n % 2:
                raise ValueError(f"{stage}_pairs must be an even integer in [2, 1024]")
            if not sign_rank(n, stage_alpha(policy, stage)):
                raise ValueError(f"{stage}: {n} pairs are too few for alpha {stage_alpha(policy, stage)}")
        else:
            if policy["statistic"] not in ("sign", "signed_rank"):
                raise ValueError("statistic must be sign or signed_rank")
            if type(policy["futility_stop"]) is not bool:
                raise ValueError("futility_stop must be a boolean")
            looks, prev, share = policy[stage + "_looks"], 0, 0.0
            if not isinstance(looks, list) or not looks:
                raise ValueError(f"{stage}_looks must be a non-empty list")
            for look in looks:
                if not isinstance(look, dict) or set(look) != {"pairs", "alpha_share"}:
                    raise ValueError("a look is {pairs, alpha_share}")
                n = look["pairs"]
                if type(n) is not int or not prev < n <= 512 or n % 2:
                    raise ValueError("look pair counts must be even and increase within [2, 512]")
                if not _finite(look["alpha_share"]) or look["alpha_share"] <= 0:
                    raise ValueError("alpha_share must be positive")
                if not _rank(policy["statistic"], n, stage_alpha(policy, stage) * look["alpha_share"]):
                    raise ValueError(f"{stage} look of {n} pairs is too small for its alpha")
                prev, share = n, share + look["alpha_share"]
            if abs(share - 1.0) > 1e-9:
                raise ValueError(f"{stage}_looks alpha shares must sum to 1")
    return dict(policy)


def log_ratios(pairs: List[dict]) -> List[float]:
    """log(candidate score) - log(baseline score) per pair; scores = 1 / time."""
    out = []
    for p in pairs:
        b, c = p.get("baseline"), p.get("candidate")
        if not (_finite(b) and _finite(c) and b > 0 and c > 0):
            raise ValueError("scores must be finite and positive")
        out.append(math.log(c) - math.log(b))
    return out


class NotStopped(ValueError):
    """A sequential sample whose last look did not stop."""


def _verdict(lo: float, hi: float, threshold: float) -> str:
    if lo > threshold + LOG_TOL:
        return "confirmed_gain"
    if hi < -threshold - LOG_TOL:
        return "regression"
    return "inconclusive"


def _exp(v: float):
    try:
        return math.exp(v)
    except OverflowError:
        return None


def _bounds(statistic: str, logs: List[float], alpha: float) -> tuple:
    r = _rank(statistic, len(logs), alpha)
    if statistic == "sign":
        values = sorted(logs)
    else:
        values = sorted((logs[i] + logs[j]) / 2 for i in range(len(logs)) for j in range(i, len(logs)))
    return r, values[r - 1], values[-r], statistics.median(values)


def assess(pairs: List[dict], policy: dict, stage: str = "final") -> dict:
    """Verdict for a complete sample (a sequential one must end at its first
    stopping look)."""
    policy = validate_policy(policy)
    if stage not in ("confirm", "final"):
        raise ValueError("stage is confirm or final")
    threshold = math.log1p(policy["min_gain"])
    logs = log_ratios(pairs)
    if policy["method"] == SIGN:
        if len(pairs) != policy[stage + "_pairs"]:
            raise ValueError("every planned pair is required")
        alpha = stage_alpha(policy, stage)
        r, lo, hi, est = _bounds("sign", logs, alpha)
        looks = []
        verdict, reason = _verdict(lo, hi, threshold), None
    else:
        looks = []
        for look in policy[stage + "_looks"]:
            n = look["pairs"]
            if n > len(logs):
                break
            alpha = stage_alpha(policy, stage) * look["alpha_share"]
            r, lo, hi, est = _bounds(policy["statistic"], logs[:n], alpha)
            verdict = _verdict(lo, hi, threshold)
            last = look is policy[stage + "_looks"][-1]
            if verdict != "inconclusive":
                reason = verdict
            elif policy["futility_stop"] and hi < threshold - LOG_TOL:
                reason = "futility"
            else:
                reason = "max_pairs" if last else None
            looks.append({"pairs": n, "alpha_one_sided": alpha, "rank": r, "lower_log_bound": lo,
                          "upper_log_bound": hi, "verdict": verdict, "stop_reason": reason})
            if reason:
                break
        if not looks or looks[-1]["pairs"] != len(logs):
            raise ValueError("a sequential sample ends exactly at one of its looks")
        if looks[-1]["stop_reason"] is None:
            raise NotStopped(f"no stop by look {len(looks)} ({len(logs)} pairs)")
        if any(lk["stop_reason"] for lk in looks[:-1]):
            raise ValueError("a sequential comparison ends at its first stopping look")
    return {"method": policy["method"], "verdict": verdict, "stop_reason": reason, "pairs": len(logs),
            "alpha_one_sided": alpha, "rank": r, "min_gain": policy["min_gain"], "log_ratios": logs,
            "estimate_ratio": _exp(est), "lower_ratio_bound": _exp(lo), "upper_ratio_bound": _exp(hi),
            "median_ratio": _exp(statistics.median(logs)), "looks": looks,
            "scope": "independent pairs assumed; balanced A/B order does not prove it"}


def run_pairs(evaluate: Callable[[str], Dict[str, float]], policy: dict, stage: str = "final") -> dict:
    """Drive the trials: ``evaluate(side)`` times one version ("baseline" or
    "candidate") and returns {timing name: microseconds}.  Each timing name is
    assessed separately; a sequential policy stops at the first look at which
    every name has stopped."""
    policy = validate_policy(policy)
    if policy["method"] == SIGN:
        sizes = [policy[stage + "_pairs"]]
    else:
        sizes = [look["pairs"] for look in policy[stage + "_looks"]]
    records: List[dict] = []
    names: List[str] = []
    results: dict = {}
    for n in sizes:
        while len(records) < n:
            rec = {}
            for side in pair_order(len(records)):
                times = evaluate(side)
                names = names or sorted(times)
                if sorted(times) != names or not all(_finite(t) and t > 0 for t in times.values()):
                    raise ValueError("every evaluation must report the same positive timings")
                rec[side] = times
            records.append(rec)
        for name in names:
            if name in results:
                continue  # stopped at an earlier look
            pairs = [{s: 1.0 / r[s][name] for s in ("baseline", "candidate")} for r in records]
            try:
                res = assess(pairs, policy, stage)
            except NotStopped:
                continue
            for s in ("baseline", "candidate"):
                res[s + "_median_us"] = statistics.median(r[s][name] for r in records)
            results[name] = res
        if len(results) == len(names):
            return {"policy": policy, "stage": stage, "results": results, "records": records}
    raise ValueError("comparison did not stop by its last look")


# ------------------------------------------------------------------ timing --

FAMILIES = ("blockscale", "bf16", "i8")


class _Version:
    """One side of a comparison: a library build and an optional fixed plan,
    for the FP8 block-scaled GEMM (``family="blockscale"``) or one of the
    sibling families (``"bf16"``, ``"i8"``)."""

    def __init__(self, spec: str, family: str = "blockscale"):
        from . import _lib, ops, siblings
        if family not in FAMILIES:
            raise ValueError(f"family must be one of {FAMILIES}")
        self.family, self.plan = family, (0, 0, 0)
        prefix = ops.KERNEL_PREFIX if family == "blockscale" else siblings.PREFIX
        if spec.startswith(ops.KERNEL_PREFIX) or spec.startswith(siblings.PREFIX):
            if not spec.startswith(prefix):
                raise ValueError(f"{spec}: not a plan of the {family} family ({prefix}_...)")
            self.lib = _lib.load()
            self.plan = (ops.parse_kernel_name(spec) if family == "blockscale"
                         else siblings.parse_kernel_name(self.kind, spec))
        else:
            if not Path(spec).is_file():
                raise ValueError(f"{spec}: neither a library file nor a {prefix} kernel name")
            self.lib = _lib.load(spec)  # another build, loaded beside the current one
            sibling = family != "blockscale"
            if hasattr(self.lib, "fack_gemm_tn_tuned_load" if sibling else "fack_gemm_bs_tuned_load"):
                for table in _lib.tuned_tables(sibling=sibling):
                    _lib.load_tuned(table, self.lib, sibling=sibling)
        self.spec = spec

    @property
    def kind(self) -> int:
        from . import _lib
        return _lib.FACK_GEMM_BF16 if self.family == "bf16" else _lib.FACK_GEMM_I8

    def launch(self, s, stream: int):
        if self.family != "blockscale":
            return self._launch_tn(s, stream)
        M, N, K = s["M"], s["N"], s["K"]
        tm, tn, sk, nb = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()
        st = self.lib.fack_gemm_bs_plan(M, N, K, *self.plan, ctypes.byref(tm), ctypes.byref(tn), ctypes.byref(sk),
                                        ctypes.byref(nb))
        if st == 0:
            xq, xsa, wp, ws, out = s["cur"]
            st = self.lib.fack_gemm_bs_ex(xq.data_ptr(), xq.stride(0), wp.data_ptr(), 1, xsa.data_ptr(), 1, M,
                                          ws.data_ptr(), out.data_ptr(), out.stride(0), M, N, K, tm.value, tn.value,
                                          sk.value, None, 0, ctypes.c_void_p(stream))
        if st != 0:
            raise RuntimeError(f"{self.spec}: status {st}: {self.lib.fack_last_error().decode()}")

    def _launch_tn(self, s, stream: int):
        M, N, K = s["M"], s["N"], s["K"]
        a, bp, sa, sb, out = s["cur"]
        ptr = (lambda t: None if t is None else t.data_ptr())  # noqa: E731
        st = self.lib.fack_gemm_tn(self.kind, a.data_ptr(), a.stride(0), bp.data_ptr(), 1, K, ptr(sa), ptr(sb),
                                   None, out.data_ptr(), out.stride(0), M, N, K, *self.plan,
                                   ctypes.c_void_p(stream))
        if st != 0:
            raise RuntimeError(f"{self.spec}: status {st}: {self.lib.fack_last_error().decode()}")


def _input_sets(family: str, M: int, N: int, K: int, dev) -> list:
    """Operand sets of one shape, together larger than 2.5 x the 126 MB L2."""
    import torch
    from . import data, ops
    es = 2 if family == "bf16" else 1
    sets = []
    for i in range(max(1, math.ceil(2.5 * 126e6 / ((M + N) * K * es)))):
        out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        if family == "blockscale":
            xq, xs = data.make_activations(M, K, "normal", 2 * i, dev)
            wq, ws = data.make_weights(N, K, "normal", 2 * i + 1, dev)
            sets.append((xq, data.to_aiter_xscale(xs), ops.shuffle_weight(wq), ws, out))
            continue
        g = torch.Generator(device=dev).manual_seed(i)
        if family == "bf16":
            a = (torch.randn((M, K), generator=g, device=dev) * 0.25).bfloat16()
            b = (torch.randn((N, K), generator=g, device=dev) * 0.25).bfloat16()
            sa = sb = None
        else:
            a = torch.randint(-128, 128, (M, K), generator=g, device=dev, dtype=torch.int8)
            b = torch.randint(-128, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
            sa = 0.001 + 0.01 * torch.rand(M, generator=g, device=dev)
            sb = 0.001 + 0.01 * torch.rand(N, generator=g, device=dev)
        sets.append((a, ops.shuffle_weight(b), sa, sb, out))
    return sets


def make_evaluator(baseline: str, candidate: str, shapes: List[tuple], launches: int = 24,
                   family: str = "blockscale"):
    """An ``evaluate(side)`` that times each shape's GEMM for one version
    (microseconds per call), the inputs shared by both versions."""
    import torch
    versions = {"baseline": _Version(baseline, family), "candidate": _Version(candidate, family)}
    dev = torch.device("cuda")
    work = []
    for M, N, K in shapes:
        sets = _input_sets(family, M, N, K, dev)
        work.append({"M": M, "N": N, "K": K, "sets": sets, "launches": max(launches, len(sets))})
    stream = torch.cuda.Stream()

    def evaluate(side: str) -> Dict[str, float]:
        v = versions[side]
        times = {}
        for s in work:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(stream):
                for i in range(len(s["sets"])):  # first calls (attribute setup) outside capture
                    s["cur"] = s["sets"][i]
                    v.launch(s, stream.cuda_stream)
            stream.synchronize()
            with torch.cuda.graph(g, stream=stream):
                for i in range(s["launches"]):
                    s["cur"] = s["sets"][i % len(s["sets"])]
                    v.launch(s, stream.cuda_stream)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                g.replay()
                a.record(stream)
                g.replay()
                b.record(stream)
            b.synchronize()
            g.reset()
            times[f"{s['M']}x{s['N']}x{s['K']}"] = a.elapsed_time(b) * 1e3 / s["launches"]
        return times

    return evaluate


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("baseline", help="libfack_gemm.so path, or a plan: fack_bs_sm100_t..x.._s.. "
                                     "(fack_tn_sm100_{bf16|i8}_t..x.._s.. with --family bf16|i8)")
    ap.add_argument("candidate", help="libfack_gemm.so path or a plan of the same family")
    ap.add_argument("--family", choices=FAMILIES, default="blockscale",
                    help="the FP8 block-scaled GEMM (default) or a sibling family")
    ap.add_argument("--shape", action="append", required=True, help="M,N,K (repeatable)")
    ap.add_argument("--pairs", type=int, required=True, help="even, fixed pair count")
    ap.add_argument("--min-gain", type=float, required=True)
    ap.add_argument("--alpha", type=float, required=True)
    ap.add_argument("--out", default="", help="write the full report (JSON) here")
    args = ap.parse_args(argv)
    policy = {"method": SIGN, "confirm_pairs": args.pairs, "final_pairs": args.pairs,
              "min_gain": args.min_gain, "alpha": args.alpha, "max_confirmations": 1}
    validate_policy(policy)
    shapes = [tuple(int(v) for v in s.split(",")) for s in args.shape]
    report = run_pairs(make_evaluator(args.baseline, args.candidate, shapes, family=args.family), policy)
    report.update(baseline=args.baseline, candidate=args.candidate, family=args.family)
    if args.out:
        Path(args.out).write_text(json.dumps(report, indent=2) + "\n")
    for name, r in report["results"].items():
        print(json.dumps({"shape": name, "verdict": r["verdict"], "baseline_median_us": r["baseline_median_us"],
                          "candidate_median_us": r["candidate_median_us"], "lower_ratio_bound": r["lower_ratio_bound"],
                          "upper_ratio_bound": r["upper_ratio_bound"]}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
