"""Summaries of TIMING lines (reference tools/perf_report.py:1-17, 262-268).

Reads logs containing ``TIMING iter=N phase=ms ...`` lines (this framework's
trainer with --timing, or the reference's), keeps the last ``--last``
iterations of each file and prints per-phase median and IQR; with ``--vs`` a
second log is summarised beside it with the relative change of the medians.
"""
from __future__ import annotations

import re
from pathlib import Path

import numpy as np


def parse(path) -> list:
    rows = []
    for line in Path(path).read_text(errors="replace").splitlines():
        m = re.search(r"TIMING iter=(\d+) (.*)", line)
        if not m:
            continue
        d = {"iter": int(m.group(1))}
        for kv in m.group(2).split():
            if "=" in kv:
                k, v = kv.split("=", 1)
                try:
                    d[k] = float(v)
                except ValueError:
                    pass
        rows.append(d)
    return rows


def summarise(rows: list, last: int = 30) -> dict:
    rows = rows[-last:]
    keys = []
    for r in rows:
        keys += [k for k in r if k != "iter" and k not in keys]
    out = {}
    for k in keys:
        v = np.array([r[k] for r in rows if k in r])
        if len(v):
            q1, med, q3 = np.percentile(v, [25, 50, 75])
            out[k] = {"median": float(med), "iqr": float(q3 - q1), "n": int(len(v))}
    return out


def main(args) -> int:
    a = summarise(parse(args.logs[0]) if len(args.logs) == 1 else sum((parse(p) for p in args.logs), []), args.last)
    b = summarise(parse(args.vs), args.last) if args.vs else None
    print(f"{'phase':<16} {'median ms':>10} {'IQR':>8}" + (f" {'vs median':>10} {'change':>8}" if b else ""))
    for k, s in a.items():
        line = f"{k:<16} {s['median']:10.1f} {s['iqr']:8.1f}"
        if b and k in b:
            ch = (s["median"] - b[k]["median"]) / max(b[k]["median"], 1e-9) * 100
            line += f" {b[k]['median']:10.1f} {ch:+7.1f}%"
        print(line)
    return 0
