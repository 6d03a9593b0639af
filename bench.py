"""Headline benchmark: end-to-end vision-PPO throughput (physics ticks / s).

One step = one PPO iteration of the benchmark configuration (per GPU: 2048
envs x 128 decisions x 3 ticks = 786,432 physics ticks of rollout, GAE, and
4 epochs x 8 minibatches of updates). Weak scaling: every rank runs 2048
envs, data parallel over NVLink. The value is the whole-job aggregate.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

For N > 1 launch with torchrun (one rank per GPU). Timing: W untimed
iterations, then exactly K iterations bracketed by a barrier and a device
synchronize on both sides, measured with CUDA events on the training stream;
the job time is the max over ranks. Rollout buffers (~4.3 GB of depth
images per GPU) exceed L2, so no flush is needed between iterations.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BASELINE_TICKS_PER_S = 281482.0          # the reference's published number, 1x RTX 5090 (docs/perf-results.md:5-6)
METRIC = "vision-PPO env-steps/s"
# trainer phases reported in the JSON line (host wall ms, and device ms of the
# rollout / update event spans): rollout = env + wait_gpu + launch overheads
PHASE_KEYS = ("rollout", "env", "wait_gpu", "rollout_gpu_ms", "respawn", "update", "update_gpu_ms", "total")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--envs", type=int, default=2048)
    ap.add_argument("--comm", choices=["p2p", "nccl"], default="p2p")
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--env-device", choices=["cpu", "cuda"], default="cpu",
                    help="cpu: C++ env threads + pinned rows (the headline); cuda: the same env rules on the GPU")
    ap.add_argument("--env-groups", type=int, default=None,
                    help="rollout env groups alternating host stepping with GPU work (default: the config's)")
    ap.add_argument("--no-async-env", action="store_true",
                    help="host env: step each group synchronously (no overlap of its launches with env stepping)")
    ap.add_argument("--no-render-order", action="store_true",
                    help="host env: render each group in env index order instead of the env step's spatial order")
    ap.add_argument("--race", action="store_true",
                    help="the race configuration (config 5: race track, geodesic potential, 2048 envs per GPU)")
    ap.add_argument("--json", default=None)
    ap.add_argument("--timing", action="store_true", help="also print each timed iteration's TIMING line to stderr")
    ap.add_argument("--no-phases", action="store_true",
                    help="skip the per-phase times (events and host clocks; on by default, reported max over ranks)")
    return ap.parse_args()


class ClockSampler:
    """SM clock, power and throttle-reason sampling of this rank's GPU during
    the timed region, every 100 ms: in-process NVML reads (the library
    nvidia-smi reports from; read-only queries), or nvidia-smi itself where
    the NVML binding is missing. An nvidia-smi process per sample costs
    0.2-0.5 s of CPU each, taken from the rank's CPU share that the host
    env steps on."""

    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []                  # (sm_mhz, sm_max_mhz, set of active reason names)
        self._stop = threading.Event()
        self._t = None

    def _nvml_reader(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self.index)
            bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                    "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                    "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                    "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
            mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))

            def read():
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                return (float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)), mx,
                        {k for k, b in bits.items() if r & b})
            read()
            return read
        except Exception:
            return None

    def _smi_read(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        out = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}", "--format=csv,noheader,nounits"],
                             capture_output=True, text=True, timeout=5).stdout.strip()
        s = [x.strip() for x in out.split(",")]
        num = lambda x: float(x) if x.replace(".", "").isdigit() else None
        return (num(s[1]), num(s[2]), {self.REASONS[i] for i in range(4) if s[4 + i].lower() == "active"})

    def start(self):
        def run():
            read = self._nvml_reader() or self._smi_read
            while not self._stop.is_set():
                try:
                    self.samples.append(read())
                except Exception:
                    pass
                self._stop.wait(0.1)
        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()

    def stop(self) -> dict:
        self._stop.set()
        if self._t:
            self._t.join(timeout=6)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(s[0] for s in self.samples if s[0] is not None)
        mx = max((s[1] for s in self.samples if s[1] is not None), default=None)
        reasons = sorted(set().union(*(s[2] for s in self.samples)))
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(self.samples)}


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def run_ours(args) -> None:
    import torch
    import surfb200  # noqa: F401
    from surfb200.trainer.config import bench_config, race_bench_config
    from surfb200.trainer.ppo import Trainer
    from surfb200.ops import _lib as L

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    comm = None
    if world > 1:
        from surfb200.parallel.dist import init_process_group, make_comm
        init_process_group()
        comm = make_comm(args.comm)
    cfg = race_bench_config(args.envs) if args.race else bench_config(args.envs)
    cfg.graphs = not args.no_graphs
    cfg.seed = 0
    cfg.timing = args.timing or not args.no_phases
    cfg.env_device = args.env_device
    if args.env_groups:
        cfg.env_groups = args.env_groups
    if args.no_async_env:
        cfg.async_env = False
    if args.no_render_order:
        cfg.render_order = False
    tr = Trainer(cfg, rank=rank, world=world, comm=comm, verbose=(rank == 0))
    for _ in range(args.warmup):
        tr.train_iteration()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    if comm is not None:
        comm.barrier()
    torch.cuda.synchronize()
    launches0 = L.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    e0.record()
    phase_sum = {}
    for _ in range(args.steps):
        stats = tr.train_iteration()
        for k, v in stats.get("timing", {}).items():
            phase_sum[k] = phase_sum.get(k, 0.0) + v
        if args.timing and rank == 0:
            from surfb200.utils.timer import PhaseClock
            print(PhaseClock.timing_line(tr.iteration, stats.get("timing", {})), file=sys.stderr, flush=True)
    e1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - w0
    if comm is not None:
        comm.barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    launches = L.launch_count() - launches0
    # per-phase ms per timed iteration, max over ranks (every rank reports the same fixed key list)
    phases = {k: phase_sum.get(k, 0.0) / args.steps for k in PHASE_KEYS} if phase_sum else {}
    per_rank = None
    if comm is not None:
        ms = comm.max_scalar(ms)
        wall = comm.max_scalar(wall)
        if phases:
            # every rank's rollout / env / update, to show which side sets the pace
            import torch.distributed as dist
            got = [None] * world
            dist.all_gather_object(got, {k: round(phases[k], 1) for k in ("rollout", "env", "update")})
            per_rank = {k: [g[k] for g in got] for k in ("rollout", "env", "update")}
        phases = {k: comm.max_scalar(v) for k, v in phases.items()}
    ticks_per_iter = cfg.envs * cfg.n_steps * cfg.act_every * world
    value = ticks_per_iter * args.steps / (ms / 1e3)
    # end-to-end through the public API: the same iterations, wall clock incl.
    # every host<->device copy of the step (env records in, actions out, stats out)
    h2d = (cfg.n_steps + 1) * cfg.envs * 64 * 4 if cfg.env_device == "cpu" else 0
    d2h = (cfg.n_steps * cfg.envs * 8 * 4 if cfg.env_device == "cpu" else 0) + 6 * 4 + 8 * 4
    e2e = ticks_per_iter * args.steps / wall
    if rank == 0:
        out = {
            "metric": METRIC, "value": round(value, 1), "unit": "ticks/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": round(value / BASELINE_TICKS_PER_S, 3), "dtype": "bf16",
            "data": "synthetic (seeded procedural BSP map, random-init weights)",
            "config": {"model": "nature-cnn-128x64+proprio256 vision PPO", "global_batch": cfg.envs * world,
                       "seq_len": cfg.n_steps, "parallelism": f"dp{world}", "envs_per_gpu": cfg.envs,
                       "act_every": cfg.act_every, "epochs": cfg.epochs, "minibatches": cfg.minibatches,
                       "map": ("procedural race track (40 chained ramps, 4 gap jumps over teleport fail nets, "
                               "finish curtain), 16u SDF and geodesic grid" if args.race else
                               "procedural random field, 512 brushes, 16u SDF 1024x1024x256"),
                       "comm": args.comm if world > 1 else "none", "cuda_graphs": cfg.graphs,
                       "env_device": cfg.env_device, "env_groups": cfg.env_groups, "async_env": cfg.async_env, "render_order": cfg.render_order, "env_threads": tr.core.threads,
                       "reward": ("race: potential on the geodesic distance to the finish, 15 s stall kill, + "
                                  "count curiosity 0.25" if args.race else
                                  "coverage (revisit_pen 0.25) + count curiosity 0.25 (256u cell x 8 yaw x 8 speed)"),
                       "differs_from_reference_arm": ["network: Nature CNN + proprio 256 vs the reference's own trunk",
                                                      "reward: curiosity 0.25 on top of coverage (the reference "
                                                      "pays curiosity only in race mode)"],
                       "l2": "inputs larger than L2 (4.3 GB rollout images per GPU)"},
            "clocks": clocks,
            "e2e": {"value": round(e2e, 1), "unit": "ticks/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "goal_field_bake_ms": round(tr.field_bake_ms, 1) if tr.field_bake_ms is not None else None,
            "phases_ms_per_step": {k: round(v, 2) for k, v in phases.items()} or None,
            "phases_ms_per_rank": per_rank,
            "last_iteration": {k: v for k, v in stats.items() if k != "timing"},
        }
        line = json.dumps(out)
        print(line, flush=True)
        if args.json:
            Path(args.json).write_text(line)
    tr.release_graphs()
    if comm is not None:
        comm.close()


def run_reference(args) -> None:
    # loaded by file path: the reference arm's process imports no module of
    # this framework's package (and so maps none of its native libraries)
    import importlib.util
    spec = importlib.util.spec_from_file_location("surf_reference_arm", ROOT / "rl_cs1.6_surf_b200" / "baseline_ref.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.run_reference_bench(args, ClockSampler)


if __name__ == "__main__":
    a = parse()
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)
