"""GPU env step throughput: K-tick steps of N envs with random actions on
the procedural field map, one CUDA thread per env (CUDA-event timed), next
to the host batch on the same actions.

    python bench/bench_gpu_env.py [--envs 2048] [--k 3] [--decisions 100] [--map field]
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
    ap.add_argument("--envs", type=int, default=2048)
    ap.add_argument("--k", type=int, default=3)
    ap.add_argument("--decisions", type=int, default=100)
    ap.add_argument("--map", default="field")
    args = ap.parse_args()
    import numpy as np
    import torch
    import surfb200  # noqa: F401
    from surfb200.sim import mapgen
    from surfb200.sim.core import REC_COLS, TERM_COLS, SimCore, default_config
    from surfb200.sim.gpu_env import GpuEnv
    n, k = args.envs, args.k
    m = mapgen.generate(args.map, 0)
    core = SimCore.from_bytes(m.image, default_config(n, spawn_mode=2, max_episode_ticks=1500), threads=None)
    if m.spawn_pool is not None:
        core.set_spawn_pool(m.spawn_pool)
    genv = GpuEnv(core)
    dev = "cuda"
    rows = {name: torch.zeros(n, c, device=dev) for name, c in (("obs", 15), ("tobs", 15), ("rec", REC_COLS),
                                                                  ("trec", TERM_COLS))}
    genv.reset(1, obs=rows["obs"], rec=rows["rec"])
    core.reset(1)
    rng = np.random.default_rng(0)
    acts = [np.stack([rng.integers(0, 15, n), rng.integers(0, 7, n), rng.integers(0, 3, n), rng.integers(0, 3, n),
                      rng.random(n) < 0.1, rng.random(n) < 0.05, np.zeros(n), np.zeros(n)], 1).astype(np.int32)
            for _ in range(args.decisions)]
    acts_d = [torch.as_tensor(a, device=dev) for a in acts]
    for a in acts_d[:5]:
        genv.step_k(a, k, obs=rows["obs"], term_obs=rows["tobs"], rec=rows["rec"], term_rec=rows["trec"])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for a in acts_d:
        genv.step_k(a, k, obs=rows["obs"], term_obs=rows["tobs"], rec=rows["rec"], term_rec=rows["trec"])
    e1.record()
    torch.cuda.synchronize()
    gpu_ms = e0.elapsed_time(e1) / args.decisions
    t0 = time.perf_counter()
    for a in acts:
        core.step_k_numpy(a, k)
    host_ms = (time.perf_counter() - t0) * 1e3 / args.decisions
    print(json.dumps({"bench": "gpu_env_step", "envs": n, "k": k, "map": args.map,
                      "gpu_ms_per_decision": round(gpu_ms, 4), "gpu_ticks_per_s": n * k / (gpu_ms * 1e-3),
                      "host_ms_per_decision": round(host_ms, 4), "host_ticks_per_s": n * k / (host_ms * 1e-3),
                      "host_threads": core.threads if hasattr(core, "threads") else None}))
    genv.close()
    core.close()


if __name__ == "__main__":
    main()
