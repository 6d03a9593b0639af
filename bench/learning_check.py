"""Learning check: does the GPU trainer improve its objective?

Runs ``--iterations`` PPO iterations of a configuration through the public
trainer API and reports the episode return / length trend (first vs last
quarter of the iterations, over iterations that finished episodes), the
policy entropy and KL, and the wall time per iteration. Used to show that the
kernels train a policy, not only that they run fast.

    python bench/learning_check.py [--config bench|race] [--iterations 120] [--json out.json]
"""
from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", choices=["bench", "race", "eyeless"], default="bench")
    ap.add_argument("--iterations", type=int, default=120)
    ap.add_argument("--envs", type=int, default=2048)
    ap.add_argument("--json", default=None)
    args = ap.parse_args()
    import numpy as np
    import surfb200  # noqa: F401
    from surfb200.rewards.spec import RewardSpec
    from surfb200.trainer.config import TrainConfig, bench_config
    from surfb200.trainer.ppo import Trainer
    if args.config == "bench":
        cfg = bench_config(args.envs)
        cfg.ep_ticks = 1500
    elif args.config == "race":
        cfg = TrainConfig(map="race", envs=args.envs, ep_ticks=3000, spawn="pool",
                          reward=RewardSpec(mode="race", int_coef=0.25, int_view=8, int_speed=8, stall_secs=15.0))
    else:
        cfg = TrainConfig(map="ramps", envs=args.envs, vision=False, device="cpu", graphs=False, ep_ticks=600,
                          n_steps=64, reward=RewardSpec(mode="speed"))
    tr = Trainer(cfg, verbose=True)
    rows = []
    t0 = time.time()
    for i in range(args.iterations):
        s = tr.train_iteration()
        rows.append({k: s.get(k) for k in ("iteration", "global_step", "episodes", "ep_rew_mean", "ep_len_mean",
                                             "entropy", "approx_kl", "policy_loss", "value_loss", "success_rate")})
        if i % 10 == 0:
            print(json.dumps(rows[-1]), flush=True)
    wall = time.time() - t0
    ok = [r for r in rows if r["episodes"] and np.isfinite(r["ep_rew_mean"])]
    q = max(1, len(ok) // 4)
    first, last = ok[:q], ok[-q:]
    mean = lambda rs, k: float(np.mean([r[k] for r in rs])) if rs else float("nan")
    summary = {"config": args.config, "iterations": args.iterations, "ticks": tr.global_step,
               "wall_s": round(wall, 1), "ms_per_iteration": round(1e3 * wall / args.iterations, 1),
               "ep_rew_first_quarter": mean(first, "ep_rew_mean"), "ep_rew_last_quarter": mean(last, "ep_rew_mean"),
               "ep_len_first_quarter": mean(first, "ep_len_mean"), "ep_len_last_quarter": mean(last, "ep_len_mean"),
               "entropy_first": rows[0]["entropy"], "entropy_last": rows[-1]["entropy"],
               "success_last_quarter": mean(last, "success_rate")}
    print("SUMMARY " + json.dumps(summary), flush=True)
    if args.json:
        Path(args.json).write_text(json.dumps({"summary": summary, "rows": rows}))
    tr.release_graphs()


if __name__ == "__main__":
    main()
