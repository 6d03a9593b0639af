"""Learning-curve A/B against the reference trainer on the same map.

    python bench/learning_ab.py [--iterations 60] [--json out.json]

Both arms train from random weights for the same number of env ticks on the
benchmark's procedural map (one BSP file, written by a child process): this
framework's trainer in this process (the benchmark configuration with the
curiosity term off, so both pay the same coverage reward), and the
reference's unmodified ``python/train_fast.py`` from ``baseline/_ref`` as a
subprocess with the command line of ``bench.py --impl reference``
(2048 envs, 128 decisions x 3 ticks, 4 epochs x 8 minibatches, 128x64 depth,
ramp drops 400-800u, coverage reward). The reference's curve is read from
its ``progress.csv`` (python/train_fast.py:1665-1690); ours from the
trainer's per-iteration statistics. The networks differ (the reference's
own trunk vs the Nature CNN), so the comparison is "no regression": mean
episode return and length over the last quarter of the ticks, next to the
first quarter's. The reference's curve is an SB3-style moving mean of the
last 100 episodes, ours the mean of the episodes that ended in the
iteration; the quarter means smooth both.
"""
from __future__ import annotations

import argparse
import csv
import importlib.util
import json
import os
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def _ref_module():
    spec = importlib.util.spec_from_file_location("surf_reference_arm", ROOT / "rl_cs1.6_surf_b200" / "baseline_ref.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _quarters(rows, key):
    """mean of `key` over the first and the last quarter of the ticks"""
    pts = [(t, v) for t, v in rows if v == v]          # drop NaN
    if not pts:
        return None, None
    t_end = pts[-1][0]
    first = [v for t, v in pts if t <= t_end / 4]
    last = [v for t, v in pts if t >= 3 * t_end / 4]
    mean = lambda xs: sum(xs) / len(xs) if xs else None
    return mean(first), mean(last)


def run_ours(map_path: Path, iterations: int, seed: int = 0) -> dict:
    import surfb200  # noqa: F401
    from surfb200.trainer.config import bench_config
    from surfb200.trainer.ppo import Trainer
    cfg = bench_config(2048)
    cfg.map = str(map_path)
    cfg.reward.int_coef = 0.0
    # the reference's --spawn ramp: drops 400-800u above scanned surfable
    # faces with a 100-400 u/s push (python/train_fast.py:1398-1411)
    cfg.spawn = "drop"
    cfg.seed = seed
    tr = Trainer(cfg, verbose=False)
    rew, length = [], []
    t0 = time.time()
    for _ in range(iterations):
        s = tr.train_iteration()
        rew.append((tr.global_step, float(s.get("ep_rew_mean", float("nan")))))
        length.append((tr.global_step, float(s.get("ep_len_mean", float("nan")))))
    wall = time.time() - t0
    tr.release_graphs()
    return {"ticks": tr.global_step, "wall_s": round(wall, 1), "ep_rew": rew, "ep_len": length}


def run_reference(ref, map_path: Path, iterations: int, run_dir: Path) -> dict:
    cmd = ref.reference_command(map_path, run_dir, iterations)
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "LOCAL_WORLD_SIZE",
                                                             "MASTER_ADDR", "MASTER_PORT")}
    env["PYTHONPATH"] = str(ref.REF / "python")
    t0 = time.time()
    proc = subprocess.run(cmd, cwd=str(ref.REF), env=env, capture_output=True, text=True,
                          timeout=float(os.environ.get("SURF_REF_TIMEOUT_S", 3000)))
    wall = time.time() - t0
    (run_dir / "learning_ab_reference.log").write_text(" ".join(cmd) + "\n\n" + proc.stdout + "\n" + proc.stderr)
    if proc.returncode != 0:
        return {"unavailable": f"reference run failed (rc={proc.returncode})"}
    rew, length = [], []
    with open(run_dir / "progress.csv", newline="", encoding="utf-8") as f:
        for row in csv.DictReader(f):
            t = float(row["time/total_timesteps"])
            rew.append((t, float(row["rollout/ep_rew_mean"] or "nan")))
            length.append((t, float(row["rollout/ep_len_mean"] or "nan")))
    return {"ticks": rew[-1][0] if rew else 0, "wall_s": round(wall, 1), "ep_rew": rew, "ep_len": length}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iterations", type=int, default=60)
    ap.add_argument("--seeds", type=int, default=1, help="our arm: independent seeds (the reference runs once)")
    ap.add_argument("--ours-only", action="store_true")
    ap.add_argument("--json", default=None)
    args = ap.parse_args()
    ref = _ref_module()
    work = Path(os.environ.get("SURF_AB_DIR", f"/tmp/surf_learning_ab_{os.getpid()}"))
    map_path = ref.write_bench_map(work / "map")
    out = {"bench": "learning_ab", "iterations": args.iterations, "map": map_path.name,
           "ours_config": "benchmark configuration, curiosity off (coverage reward, revisit_pen 0.25), drop spawns "
                          "400-800u (the reference's --spawn ramp)",
           "reference_command": " ".join(ref.reference_command(map_path, work / "reference", args.iterations))}
    arms = {("ours" if k == 0 else f"ours_seed{k}"): run_ours(map_path, args.iterations, k) for k in range(args.seeds)}
    if args.ours_only:
        pass
    elif (ref.REF / "python" / "train_fast.py").exists():
        (work / "reference").mkdir(parents=True, exist_ok=True)
        arms["reference"] = run_reference(ref, map_path, args.iterations, work / "reference")
    else:
        arms["reference"] = {"unavailable": "reference not installed under baseline/_ref"}
    for name, a in arms.items():
        if "ep_rew" not in a:
            out[name] = a
            continue
        r0, r1 = _quarters(a["ep_rew"], "ep_rew")
        l0, l1 = _quarters(a["ep_len"], "ep_len")
        out[name] = {"ticks": a["ticks"], "wall_s": a["wall_s"], "ep_rew_first_quarter": r0,
                     "ep_rew_last_quarter": r1, "ep_len_first_quarter": l0, "ep_len_last_quarter": l1,
                     "curve": [[int(t), round(v, 3)] for t, v in a["ep_rew"]]}
    line = json.dumps(out)
    print(line, flush=True)
    if args.json:
        Path(args.json).write_text(line)


if __name__ == "__main__":
    main()
