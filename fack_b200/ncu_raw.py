"""Per-launch figures from an ncu capture's raw page.

``python -m fack_b200.ncu_raw RAW.csv [--kernel REGEX] [--traffic NAME]``

RAW.csv is ``ncu -i CAPTURE.ncu-rep --page raw --csv`` output: a header row of
metric names, a row of their units, then one row per captured launch.  Prints
one markdown row per launch -- kernel, device time, DRAM bytes read + written
(the roofline's ``traffic``), DRAM and SM throughput, registers per thread --
for the metrics the capture holds.  ``--traffic NAME`` also prints the entry
for ``profiles/traffic.json``: the mean DRAM bytes per launch of the selected
launches under key NAME (the workload).
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import re
import statistics
import sys
from pathlib import Path

from .ncu_launches import short_name

SCALE = {"byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "Tbyte": 1e12,
         "nsecond": 1e-3, "usecond": 1.0, "msecond": 1e3, "second": 1e6}
FIELDS = {  # output key: (metric name, unit it is reported in)
    "duration_us": ("gpu__time_duration.sum", "us"),
    "dram_read": ("dram__bytes_read.sum", "byte"),
    "dram_write": ("dram__bytes_write.sum", "byte"),
    "dram_pct": ("gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed", "%"),
    "sm_pct": ("sm__throughput.avg.pct_of_peak_sustained_elapsed", "%"),
    "tensor_pct": ("sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active", "%"),
    "registers": ("launch__registers_per_thread", ""),
}


def _value(text: str, unit: str, want: str):
    text = (text or "").replace(",", "").strip()
    if not text or text == "n/a":
        return None
    v = float(text)
    if want in ("byte", "us"):
        if unit not in SCALE:
            raise ValueError(f"unknown unit {unit!r}")
        return v * SCALE[unit]
    return v


def read_raw(text: str) -> list:
    """One dict per launch: kernel, id and the FIELDS the capture holds."""
    lines = text.splitlines()
    start = next((i for i, ln in enumerate(lines) if ln.startswith('"ID"')), None)
    if start is None:
        raise ValueError("no raw-page header (a line starting with \"ID\")")
    rows = list(csv.reader(io.StringIO("\n".join(lines[start:]))))
    header, body = rows[0], rows[1:]
    units = [""] * len(header)
    if body and body[0] and body[0][0] == "":  # the units row
        units, body = body[0], body[1:]
    col = {name: i for i, name in enumerate(header)}
    out = []
    for r in body:
        if len(r) != len(header):
            continue
        rec = {"id": r[col["ID"]], "kernel": short_name(r[col["Kernel Name"]])}
        for key, (metric, want) in FIELDS.items():
            i = col.get(metric)
            rec[key] = None if i is None else _value(r[i], units[i], want)
        rr, ww = rec["dram_read"], rec["dram_write"]
        rec["dram_bytes"] = None if rr is None or ww is None else rr + ww
        out.append(rec)
    if not out:
        raise ValueError("no launches in the raw page")
    return out


def _fmt(v, spec):
    return "—" if v is None else format(v, spec)


def markdown(recs: list) -> str:
    lines = ["| launch | kernel | µs | DRAM MB (read + write) | DRAM % | SM % | tensor % | regs |",
             "|---|---|---|---|---|---|---|---|"]
    for r in recs:
        mb = None if r["dram_bytes"] is None else r["dram_bytes"] / 1e6
        lines.append(f"| {r['id']} | `{r['kernel']}` | {_fmt(r['duration_us'], '.2f')} | {_fmt(mb, '.2f')} | "
                     f"{_fmt(r['dram_pct'], '.1f')} | {_fmt(r['sm_pct'], '.1f')} | {_fmt(r['tensor_pct'], '.1f')} | "
                     f"{_fmt(r['registers'], '.0f')} |")
    return "\n".join(lines)


def traffic_entry(recs: list, name: str, source: str) -> dict:
    """profiles/traffic.json entry: mean DRAM bytes per launch of ``recs``."""
    vals = [r["dram_bytes"] for r in recs if r["dram_bytes"] is not None]
    if not vals:
        raise ValueError("the capture holds no dram__bytes_read.sum / dram__bytes_write.sum")
    kernels = sorted({r["kernel"] for r in recs})
    return {name: {"bytes_per_launch": int(round(statistics.mean(vals))), "kernel": ", ".join(kernels),
                   "source": source}}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("csv", help="ncu -i CAPTURE --page raw --csv output")
    ap.add_argument("--kernel", default="", help="keep launches whose kernel name matches this regex")
    ap.add_argument("--traffic", default="", help="also print a profiles/traffic.json entry under this key")
    args = ap.parse_args(argv)
    recs = read_raw(Path(args.csv).read_text())
    if args.kernel:
        recs = [r for r in recs if re.search(args.kernel, r["kernel"])]
        if not recs:
            raise SystemExit(f"no launch matches {args.kernel!r}")
    print(markdown(recs))
    if args.traffic:
        print(json.dumps(traffic_entry(recs, args.traffic, f"ncu raw page {Path(args.csv).name}"), indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
