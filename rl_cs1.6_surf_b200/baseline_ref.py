"""``bench.py --impl reference``: the unmodified reference trainer on this box.

Runs the reference's own public entry point, ``python/train_fast.py`` from
the installed copy under ``baseline/_ref`` (its C core built from source by
its own ``build.sh``), on the benchmark map of this framework's bench (the
seeded procedural random field, a BSP v30 file that the reference core
loads), with the benchmark's PPO shape: 2048 envs, 128 decisions x 3 ticks,
4 epochs x 8 minibatches, 128x64 depth camera on a 16u SDF, ramp drop spawns
400-800u. The reference prints one ``TIMING iter=N ... total=ms`` line per
iteration with ``--timing`` (python/train_fast.py:311-401); the first W
iterations are warm-up and the next K are timed. Its own per-iteration wall
time is the measurement (it synchronises the device once per iteration
before reading it).

Process isolation: this module imports nothing of this framework. The map
file is written by a separate child process (``python surfb200.py mapgen``)
that exits before the reference starts, so neither the process that runs
this arm nor the reference trainer it launches maps any library of this
repository.

Two settings cannot be made equal and are stated in the JSON line: the
reference's network is its own trunk (train_fast.py:115-133: conv 5x5/2 16,
3x3/2 32, 3x3/2 64, 4x8 average pool, FC 512, two tanh towers of 448), not
the Nature CNN of the benchmark configuration; and its count-based curiosity
exists only inside its race reward (train_fast.py:1526-1538), so its arm runs
the coverage reward without the curiosity term.

The reference has no data parallelism (docs/ddp-plan.md is a design it
never built); under torchrun each rank runs one independent reference
training on its own GPU (the reference's documented way of using several
GPUs, docs/perf-results.md:488-501) and the aggregate is N x ticks per
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
ENVS, DECISIONS, ACT_EVERY = 2048, 128, 3
TICKS_PER_ITER = ENVS * DECISIONS * ACT_EVERY
# host <-> device bytes the reference moves per iteration, counted from its
# pinned staging tensors: per decision the pose rows (N x 6 fp32,
# train_fast.py:1731), rewards and done flags (2 x N fp32, :2099-2101) and
# the scalar observation (N x 15 fp32, :2103) go up; the sampled actions
# (N x 6 int64, :1723/:1975) come down.
REF_H2D_PER_ITER = (DECISIONS + 1) * ENVS * (6 + 2 + 15) * 4
REF_D2H_PER_ITER = DECISIONS * ENVS * 6 * 8

REFERENCE_MODEL = ("reference Policy: conv 5x5/2->16, 3x3/2->32, 3x3/2->64, avgpool 4x8, FC 512, "
                   "pi/vf tanh towers 448x448 (train_fast.py:115-133), torch.compile update, CUDA-graph rollout")
REFERENCE_REWARD = "coverage (revisit_pen 0.25); no curiosity term (the reference pays curiosity only in race mode)"


def _unavailable(why: str) -> None:
    print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)


def _dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def reference_command(map_path: Path, run_dir: Path, iters: int) -> list:
    return [sys.executable, str(REF / "python" / "train_fast.py"),
            "--map", str(map_path), "--envs", str(ENVS), "--n-steps", str(DECISIONS), "--act-every", str(ACT_EVERY),
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


def write_bench_map(directory: Path, kind: str = "field", seed: int = 0) -> Path:
    """The benchmark's procedural map on disk, written by a child process
    (``surfb200.py mapgen``) so that the caller never loads this framework."""
    name = {"ramps": "proc_ramps", "field": "proc_field", "race": "proc_race"}[kind] + f"_s{seed}"
    path = directory / f"{name}.bsp"
    if path.exists() and (directory / f"{name}.meta.json").exists():
        return path
    directory.mkdir(parents=True, exist_ok=True)
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR",
                                                             "MASTER_PORT")}
    env["CUDA_VISIBLE_DEVICES"] = ""
    subprocess.run([sys.executable, str(ROOT / "surfb200.py"), "mapgen", "--kind", kind, "--seed", str(seed),
                    "--out", str(directory)], cwd=str(ROOT), env=env, check=True, capture_output=True, timeout=600)
    if not path.exists():
        raise RuntimeError(f"map writer did not produce {path}")
    return path


def run_reference_bench(args, clock_sampler) -> None:
    """``clock_sampler(gpu_index)`` is bench.py's clock sampler (start / stop -> dict)."""
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
    map_path = write_bench_map(ROOT / "maps" / f"reference_rank{rank}")   # one SDF cache per rank
    run_dir = Path(os.environ.get("SURF_REF_RUN_DIR", f"/tmp/surf_ref_bench_r{rank}_{os.getpid()}"))
    iters = args.warmup + args.steps
    cmd = reference_command(map_path, run_dir, iters)
    env = dict(os.environ)
    env["CUDA_VISIBLE_DEVICES"] = str(local)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "LOCAL_WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT",
              "TORCHELASTIC_RUN_ID", "GROUP_RANK", "ROLE_RANK"):
        env.pop(k, None)
    env["PYTHONPATH"] = str(REF / "python")
    sampler = clock_sampler(local)
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
    log = Path(os.environ.get("SURF_REF_LOG", run_dir / f"reference_rank{rank}.log"))
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
                "config": {"model": REFERENCE_MODEL, "global_batch": ENVS * world, "seq_len": DECISIONS,
                           "parallelism": f"{world} independent runs (the reference has no data parallelism)",
                           "envs_per_gpu": ENVS, "act_every": ACT_EVERY, "epochs": 4, "minibatches": 8,
                           "map": "procedural random field, 512 brushes, 16u SDF (written by a separate process)",
                           "reward": REFERENCE_REWARD,
                           "differs_from_ours": ["network: reference trunk vs Nature CNN + proprio 256",
                                                 "reward: coverage vs coverage + curiosity 0.25"],
                           "timing": "reference's own per-iteration TIMING total (wall, one device sync)",
                           "l2": "inputs larger than L2 (rollout images)"},
                "clocks": clocks,
                "e2e": {"value": round(value, 1), "unit": "ticks/s", "h2d_bytes_per_step": REF_H2D_PER_ITER,
                        "d2h_bytes_per_step": REF_D2H_PER_ITER,
                        "note": "the reference's timing is end to end; bytes counted from its staging tensors"},
                "setup_wall_s": round(wall - ms / 1e3, 1),
            }), flush=True)
    if pg is not None:
        pg.destroy_process_group()
