"""Per-kernel summary of an ncu launch list.

``python -m fack_b200.ncu_launches LAUNCHES.csv [--top N]``

Reads the CSV that ``ncu --metrics gpu__time_duration.sum --csv --log-file
LAUNCHES.csv <command>`` writes (one row per captured launch; ``==PROF==``
lines before the header are skipped) and prints a markdown table: kernel,
launches, total µs, µs per launch and share of the listed device time, largest
total first.  With ``--top N`` the kernels after the first N are summed into
one "other" row.  ncu serialises the launches and runs them with cold caches,
so the shares, not the absolute times, are what compare with a live timing.
"""
from __future__ import annotations

import argparse
import csv
import io
import sys
from collections import OrderedDict
from pathlib import Path

METRIC = "gpu__time_duration.sum"
TO_US = {"nsecond": 1e-3, "ns": 1e-3, "usecond": 1.0, "us": 1.0, "msecond": 1e3, "ms": 1e3, "second": 1e6, "s": 1e6}


def short_name(name: str) -> str:
    """A demangled kernel signature without ``void`` and its argument list."""
    name = name.replace("(anonymous namespace)::", "").strip()
    if name.startswith("void "):
        name = name[5:]
    depth = 0
    for i, c in enumerate(name):
        if c == "<":
            depth += 1
        elif c == ">":
            depth -= 1
        elif c == "(" and depth == 0:
            return name[:i].strip()
    return name


def read_launches(text: str) -> list:
    """[(kernel, µs)] for every launch row of an ncu CSV log."""
    lines = text.splitlines()
    start = next((i for i, ln in enumerate(lines) if ln.startswith('"ID"')), None)
    if start is None:
        raise ValueError("no ncu CSV header (a line starting with \"ID\") in the log")
    out = []
    for row in csv.DictReader(io.StringIO("\n".join(lines[start:]))):
        if row.get("Metric Name") != METRIC:
            continue
        unit = (row.get("Metric Unit") or "").strip()
        if unit not in TO_US:
            raise ValueError(f"unknown time unit {unit!r} in ncu log")
        value = float(row["Metric Value"].replace(",", ""))
        out.append((short_name(row["Kernel Name"]), value * TO_US[unit]))
    if not out:
        raise ValueError(f"no {METRIC} rows in the ncu log")
    return out


def summarize(launches: list, top: int = 0) -> list:
    """[(kernel, launches, total µs, µs per launch, share)], largest total first."""
    acc: "OrderedDict[str, list]" = OrderedDict()
    for name, us in launches:
        a = acc.setdefault(name, [0, 0.0])
        a[0] += 1
        a[1] += us
    total = sum(a[1] for a in acc.values())
    rows = sorted(((k, n, t) for k, (n, t) in acc.items()), key=lambda r: -r[2])
    if top and len(rows) > top:
        rest = rows[top:]
        rows = rows[:top] + [(f"other ({len(rest)} kernels)", sum(r[1] for r in rest), sum(r[2] for r in rest))]
    return [(k, n, t, t / n, t / total) for k, n, t in rows]


def markdown(rows: list) -> str:
    out = ["| kernel | launches | total µs | µs/launch | share |", "|---|---|---|---|---|"]
    for k, n, t, per, share in rows:
        out.append(f"| `{k}` | {n} | {t:.1f} | {per:.2f} | {100 * share:.1f} % |")
    return "\n".join(out)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("csv", help="ncu --csv --log-file output")
    ap.add_argument("--top", type=int, default=0, help="list the N largest kernels, sum the rest")
    args = ap.parse_args(argv)
    print(markdown(summarize(read_launches(Path(args.csv).read_text()), args.top)))
    return 0


if __name__ == "__main__":
    sys.exit(main())
