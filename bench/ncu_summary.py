"""Summarise an ncu report (``--page raw --csv``) as a short markdown profile.

    python bench/ncu_summary.py REPORT.ncu-rep --case NAME --command "..." [--flops F] [--bytes B] > profiles/x.md

Reads the counters this framework's profiles quote (duration, DRAM bytes and
throughput, tensor-pipe activity, occupancy, registers, top warp stalls) and
states achieved bandwidth / FLOP rate as fractions of the pool's measured
peaks (MEASURED_PEAKS.json: STREAM-style copy, cuBLAS bf16 burst).
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
KEYS = {
    "time_us": "gpu__time_duration.sum",
    "dram_read": "dram__bytes_read.sum",
    "dram_write": "dram__bytes_write.sum",
    "dram_pct": "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
    "sm_pct": "sm__throughput.avg.pct_of_peak_sustained_elapsed",
    "tensor_pct": "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed",
    "warps_active_pct": "sm__warps_active.avg.pct_of_peak_sustained_active",
    "regs": "launch__registers_per_thread",
    "grid": "launch__grid_size",
    "block": "launch__block_size",
    "l2_hit_pct": "lts__t_sector_hit_rate.pct",
    "sm_clock": "sm__cycles_elapsed.avg.per_second",
}
UNIT = {"byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "us": 1.0, "ms": 1e3, "ns": 1e-3, "s": 1e6,
        "Ghz": 1e9, "Mhz": 1e6}


def read(report: str) -> dict:
    out = subprocess.run(["ncu", "-i", report, "--page", "raw", "--csv"], capture_output=True, text=True).stdout
    rows = list(csv.reader(io.StringIO(out)))
    hdr, units, vals = rows[0], rows[1], rows[2]
    res = {"kernel": vals[hdr.index("Kernel Name")]}
    for k, m in KEYS.items():
        if m in hdr:
            i = hdr.index(m)
            try:
                res[k] = float(vals[i].replace(",", "")) * UNIT.get(units[i], 1.0)
            except ValueError:
                res[k] = vals[i]
    stalls = []
    for i, h in enumerate(hdr):
        if h.startswith("smsp__pcsamp_warps_issue_stalled_") and not h.endswith("_not_issued"):
            try:
                stalls.append((float(vals[i]), h.replace("smsp__pcsamp_warps_issue_stalled_", "")))
            except ValueError:
                pass
    tot = sum(v for v, _ in stalls) or 1.0
    res["stalls"] = [(n, round(100 * v / tot, 1)) for v, n in sorted(stalls, reverse=True)[:5]]
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("report")
    ap.add_argument("--case", required=True)
    ap.add_argument("--command", required=True)
    ap.add_argument("--flops", type=float, default=0.0, help="algorithmic FLOPs per launch")
    ap.add_argument("--bytes", type=float, default=0.0, help="algorithmic bytes per launch")
    ap.add_argument("--timed-ms", type=float, default=None, help="CUDA-event time per launch outside ncu")
    ap.add_argument("--note", default="")
    a = ap.parse_args()
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() \
        else {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
    r = read(a.report)
    t_us = a.timed_ms * 1e3 if a.timed_ms else r["time_us"]
    traffic = r.get("dram_read", 0.0) + r.get("dram_write", 0.0)
    lines = [f"# {a.case}", "", f"Kernel: `{r['kernel'][:150]}`", "",
             f"Command: `{a.command}`", "",
             "| quantity | value |", "|---|---|",
             f"| duration under ncu | {r['time_us']:.1f} us |"]
    if a.timed_ms:
        lines.append(f"| duration, CUDA events (no profiler) | {a.timed_ms * 1e3:.1f} us |")
    lines += [f"| DRAM read + write | {traffic / 1e6:.1f} MB |",
              f"| DRAM throughput (ncu, % of peak) | {r.get('dram_pct', 0):.1f} % |",
              f"| achieved DRAM bandwidth | {traffic / (r['time_us'] * 1e-6) / 1e9:.0f} GB/s = "
              f"{traffic / (r['time_us'] * 1e-6) / 1e9 / peaks['hbm_gbs']:.2f} of measured {peaks['hbm_gbs']:.0f} GB/s |"]
    if a.bytes:
        lines.append(f"| algorithmic bytes / event time | {a.bytes / (t_us * 1e-6) / 1e9:.0f} GB/s = "
                     f"{a.bytes / (t_us * 1e-6) / 1e9 / peaks['hbm_gbs']:.2f} of measured |")
    if a.flops:
        tf = a.flops / (t_us * 1e-6) / 1e12
        lines.append(f"| FLOP rate | {tf:.1f} TFLOP/s = {tf / peaks['bf16_tflops']:.3f} of measured "
                     f"{peaks['bf16_tflops']:.0f} TFLOP/s |")
    lines += [f"| tensor pipe active | {r.get('tensor_pct', 0):.1f} % |",
              f"| SM throughput | {r.get('sm_pct', 0):.1f} % |",
              f"| warps active (of peak sustained) | {r.get('warps_active_pct', 0):.1f} % |",
              f"| L2 hit rate | {r.get('l2_hit_pct', 0):.1f} % |",
              f"| registers / thread, grid x block | {r.get('regs', 0):.0f}, {r.get('grid', 0):.0f} x {r.get('block', 0):.0f} |",
              f"| SM clock during capture | {r.get('sm_clock', 0) / 1e9:.2f} GHz |",
              "", "Top warp stall reasons (share of sampled stalls): " +
              ", ".join(f"{n} {p}%" for n, p in r["stalls"])]
    if a.note:
        lines += ["", a.note]
    print("\n".join(lines))


if __name__ == "__main__":
    main()
