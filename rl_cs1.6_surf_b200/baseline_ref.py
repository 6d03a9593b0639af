"""``bench.py --impl reference``: the unmodified reference trainer on this box.

Runs the reference's own public entry point, ``python/train_fast.py`` from
the installed copy under ``baseline/_ref`` (its C core built from source by
its own ``build.sh``), on the benchmark map of this framework's bench (the
seeded procedural random field, written to disk as BSP v30, which the
reference core loads), with the benchmark's PPO shape: 2048 envs, 128
decisions x 3 ticks, 4 epochs x 8 minibatches, 128x64 depth camera on a 16u
SDF, coverage reward, ramp drop spawns 400-800u. The reference prints one
``TIMING iter=N ... total=ms`` line per iteration with ``--timing``
(python/train_fast.py:311-401); the first W iterations are warm-up and the
next K are timed. Its own per-iteration wall time is the measurement (it
synchronises the device once per iteration before reading it).

The reference has no data parallelism (docs/ddp-plan.md is a design it
never built); under torchrun each rank runs one independent reference
training on its own GPU — the reference's documented way of using several
GPUs (docs/perf-results.md:488-501) — and the aggregate is N x ticks per
iteration / the slowest rank's time.
"""
from __future__ import annotations

import json
import os
import re
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"
TICKS_PER_ITER = 2048 * 128 * 3


def _unavailable(why: str) -> None:
    print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)


def _dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def reference_command(map_path: Path, run_dir: Path, iters: int) -> list:
    return [sys.executable, str(REF / "python" / "train_fast.py"),
            "--map", str(map_path), "--envs", "2048", "--n-steps", "128", "--act-every", "3",
            "--epochs", "4", "--minibatches", "8", "--gamma", "0.9995", "--lidar-w", "128", "--lidar-h", "64",
            "--lidar-cell", "16", "--spawn", "ramp", "--drop-min", "400", "--drop-max", "800",
            "--reward", "coverage", "--timing", "--steps", str(float(iters * TICKS_PER_ITER)),
            "--record-every", "1e18", "--ckpt-every", "1e18", "--run", str(run_dir)]


def parse_timing(text: str) -> list:
    """[(iteration, total_ms)] from the reference's TIMING lines."""
    out = []
    for line in text.splitlines():
        m = re.match(r"TIMING iter=(\d+) (.*)", line.strip())
        if not m:
            continue
        fields = dict(kv.split("=", 1) for kv in m.group(2).split() if "=" in kv)
        if "total" in fields:
            out.append((int(m.group(1)), float(fields["total"])))
    return out


def run_reference_bench(args) -> None:
    rank, world, local = _dist_env()
    if not (REF / "python" / "train_fast.py").exists() or not (REF / "build" / "libsurfcore.so").exists():
        if rank == 0:
            _unavailable("reference not installed under baseline/_ref (train_fast.py or build/libsurfcore.so missing)")
        return
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=3600))
        pg = dist
    sys.path.insert(0, str(ROOT))
    import surfb200  # noqa: F401
    from surfb200.sim import mapgen
    maps = ROOT / "maps" / f"reference_rank{rank}"      # one SDF cache per rank (no shared writes)
    map_path = mapgen.cached_map("field", 0, directory=maps)
    run_dir = Path(os.environ.get("SURF_REF_RUN_DIR", f"/tmp/surf_ref_bench_r{rank}_{os.getpid()}"))
    iters = args.warmup + args.steps
    cmd = reference_command(map_path, run_dir, iters)
    env = dict(os.environ)
    env["CUDA_VISIBLE_DEVICES"] = str(local)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "LOCAL_WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT",
              "TORCHELASTIC_RUN_ID", "GROUP_RANK", "ROLE_RANK"):
        env.pop(k, None)
    env["PYTHONPATH"] = str(REF / "python")
    from bench import ClockSampler    # the same nvidia-smi sampler as this framework's arm
    sampler = ClockSampler(local)
    sampler.start()
    t0 = time.time()
    try:
        proc = subprocess.run(cmd, cwd=str(REF), env=env, capture_output=True, text=True,
                              timeout=float(os.environ.get("SURF_REF_TIMEOUT_S", 3000)))
        out, rc = proc.stdout + "\n" + proc.stderr, proc.returncode
    except subprocess.TimeoutExpired as e:
        out, rc = (e.stdout or "") if isinstance(e.stdout, str) else "", -9
    wall = time.time() - t0
    clocks = sampler.stop()
    log = Path(os.environ.get("SURF_REF_LOG", ROOT / "gpurun_out" / f"reference_rank{rank}.log"))
    try:
        log.parent.mkdir(parents=True, exist_ok=True)
        log.write_text(" ".join(cmd) + "\n\n" + out)
    except OSError:
        pass
    timings = parse_timing(out)
    timed = [ms for it, ms in timings if args.warmup < it <= args.warmup + args.steps]
    ok = rc == 0 and len(timed) == args.steps
    ms = sum(timed) if ok else float("nan")
    if pg is not None:
        import torch
        t = torch.tensor([ms if ok else float("inf")], dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
        ok = ms != float("inf")
    if rank == 0:
        if not ok:
            tail = " | ".join(l for l in out.strip().splitlines()[-3:])[:300]
            _unavailable(f"reference run failed (rc={rc}, {len(timings)} TIMING lines): {tail}")
        else:
            value = world * TICKS_PER_ITER * args.steps / (ms / 1e3)
            print(json.dumps({
                "impl": "reference", "metric": "vision-PPO env-steps/s", "value": round(value, 1), "unit": "ticks/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": round(value / 281482.0, 3),
                "dtype": "bf16", "data": "synthetic (seeded procedural BSP map, random-init weights)",
                "config": {"model": "reference Policy (conv trunk + tanh towers), train_fast.py stock path",
                           "global_batch": 2048 * world, "seq_len": 128,
                           "parallelism": f"{world} independent runs (the reference has no data parallelism)",
                           "map": "procedural random field, 512 brushes, 16u SDF", "reward": "coverage",
                           "timing": "reference's own per-iteration TIMING total (wall, one device sync)",
                           "l2": "inputs larger than L2 (rollout images)"},
                "clocks": clocks,
                "e2e": {"value": round(value, 1), "unit": "ticks/s", "note": "the reference's timing is end to end"},
                "setup_wall_s": round(wall - ms / 1e3, 1),
            }), flush=True)
    if pg is not None:
        pg.destroy_process_group()
