"""Run directory: run.json, progress.csv and the per-iteration console line.

Reference behaviour (python/train_fast.py:1596-1687, 2293-2300): ``run.json``
holds the full run configuration (the self-describing part a resume reads)
plus run metadata and is finalised at the end; ``progress.csv`` gets one row
per iteration with the 16 columns below (an older file with fewer columns is
migrated by extending its header); ``global_step`` counts physics ticks.
"""
from __future__ import annotations

import csv
import json
import math
import os
import socket
import time
from pathlib import Path
from typing import Optional

CSV_COLS = (
    "time/total_timesteps", "rollout/ep_rew_mean", "rollout/ep_len_mean", "time/fps", "train/loss",
    "train/value_loss", "train/entropy_loss", "train/approx_kl", "eval/fwd_max", "eval/path", "eval/speed_max",
    "train/blend_w", "race/success_rate", "race/finish_s", "race/eval_progress", "race/eval_finish_s",
)


def _num(v) -> str:
    if v is None:
        return ""
    try:
        f = float(v)
    except (TypeError, ValueError):
        return ""
    return "" if math.isnan(f) else f"{f:.6g}"


class RunLogger:
    """Writes a run directory (rank 0 only; other ranks get a no-op logger)."""

    def __init__(self, run_dir, config: dict, enabled: bool = True, meta: Optional[dict] = None):
        self.enabled = enabled
        self.dir = Path(run_dir)
        self.t0 = time.time()
        self.last_t = self.t0
        self.last_step = 0
        self.eval: dict = {}
        if not enabled:
            return
        self.dir.mkdir(parents=True, exist_ok=True)
        self.run_json = self.dir / "run.json"
        doc = {"config": config, "started": time.strftime("%Y-%m-%d %H:%M:%S"), "host": socket.gethostname(),
               "pid": os.getpid(), **(meta or {})}
        if self.run_json.exists():                      # a resumed run keeps its history
            try:
                old = json.loads(self.run_json.read_text())
                doc["resumed_from"] = old.get("started")
                doc["history"] = old.get("history", []) + [{k: old.get(k) for k in ("started", "finished")}]
            except (OSError, ValueError):
                pass
        self._write_json(doc)
        self.csv_path = self.dir / "progress.csv"
        self._migrate_csv()

    def _write_json(self, doc: dict) -> None:
        tmp = self.run_json.with_suffix(".json.tmp")
        tmp.write_text(json.dumps(doc, indent=2, default=str))
        os.replace(tmp, self.run_json)

    def _migrate_csv(self) -> None:
        if not self.csv_path.exists():
            with open(self.csv_path, "w", newline="") as f:
                csv.writer(f).writerow(CSV_COLS)
            return
        with open(self.csv_path, newline="") as f:
            rows = list(csv.reader(f))
        if not rows or tuple(rows[0]) == CSV_COLS:
            return
        header = rows[0]
        extra = [c for c in CSV_COLS if c not in header]
        if extra:
            new_header = header + extra
            with open(self.csv_path, "w", newline="") as f:
                w = csv.writer(f)
                w.writerow(new_header)
                for r in rows[1:]:
                    w.writerow(r + [""] * (len(new_header) - len(r)))
            print(f"progress.csv header extended to {len(new_header)} columns")

    def log(self, stats: dict) -> str:
        """Append one progress row and return the console line."""
        now = time.time()
        step = int(stats.get("global_step", 0))
        fps = (step - self.last_step) / max(now - self.last_t, 1e-9)
        self.last_t, self.last_step = now, step
        pl, vl, ent = stats.get("policy_loss"), stats.get("value_loss"), stats.get("entropy")
        loss = None
        if pl is not None and vl is not None:
            loss = float(pl) + float(stats.get("vf_coef", 0.5)) * float(vl) - float(stats.get("ent_coef", 0.0)) * float(
                ent or 0.0)
        row = {
            "time/total_timesteps": step, "rollout/ep_rew_mean": stats.get("ep_rew_mean"),
            "rollout/ep_len_mean": stats.get("ep_len_mean"), "time/fps": fps, "train/loss": loss,
            "train/value_loss": vl, "train/entropy_loss": None if ent is None else -float(ent),
            "train/approx_kl": stats.get("approx_kl"), "eval/fwd_max": self.eval.get("fwd_max"),
            "eval/path": self.eval.get("path"), "eval/speed_max": self.eval.get("speed_max"),
            "train/blend_w": stats.get("blend_w"), "race/success_rate": stats.get("success_rate"),
            "race/finish_s": stats.get("finish_s"), "race/eval_progress": self.eval.get("progress"),
            "race/eval_finish_s": self.eval.get("finish_s"),
        }
        if self.enabled:
            with open(self.csv_path, "a", newline="") as f:
                csv.writer(f).writerow([_num(row[c]) for c in CSV_COLS])
        line = (f"it {stats.get('iteration', 0):5d} | steps {step:>13,} | {fps / 1e3:8.1f}k ticks/s | "
                f"ep_rew {_num(stats.get('ep_rew_mean')) or '-':>9} | ep_len {_num(stats.get('ep_len_mean')) or '-':>7} | "
                f"pg {_num(pl) or '-':>9} | vf {_num(vl) or '-':>9} | ent {_num(ent) or '-':>7} | "
                f"kl {_num(stats.get('approx_kl')) or '-':>9}")
        return line

    def set_eval(self, summary: dict) -> None:
        self.eval = dict(summary)

    def finish(self, extra: Optional[dict] = None) -> None:
        if not self.enabled:
            return
        try:
            doc = json.loads(self.run_json.read_text())
        except (OSError, ValueError):
            doc = {}
        doc["finished"] = time.strftime("%Y-%m-%d %H:%M:%S")
        doc["wall_s"] = round(time.time() - self.t0, 1)
        doc.update(extra or {})
        self._write_json(doc)
