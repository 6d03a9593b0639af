"""Command line: ``python -m surfb200 <command> [options]``.

Commands (reference tools they replace in brackets):

  train             PPO training, resumable (python/train_fast.py); launch with
                    torchrun for data parallelism, one rank per GPU
  eval              evaluation episodes of a checkpoint, optional JSONL
                    recording (tools/record_ckpt.py)
  mapgen            write a seeded procedural map (.bsp + zones/spawns/meta)
  bake              build and cache a map's SDF and goal field
                    (python/surfgym/vision.py build_sdf, goalfield.py)
  export-map        mesh JSON of a map's solid geometry (tools/export_map.py)
  export-goalfield  arrow-field JSON of the race potential
                    (tools/export_goalfield.py)
  perf-report       medians / IQR of TIMING lines, A/B (tools/perf_report.py)
  gpu-health        HBM copy and bf16 GEMM against the measured peaks
                    (tools/gpu_health.py)
  render-pov        depth frames along a recorded trajectory, headless
                    (tools/render_pov.py)
  sample-traj       synthetic trajectory file (tools/make_sample_traj.py)
  compare-runs      runs side by side at step marks (tools/compare_runs.py)
  serve-metrics     JSON metrics API over a runs directory (tools/dashboard.py)
  bench-env         env step throughput per thread count (tools/bench_env.py)
  strafe-audit      air-acceleration capture of recorded episodes
                    (tools/strafe_audit.py)
  route-bound       time floors and energy budget of a recorded route
                    (tools/route_bound.py)
  tas-search        batched hill climb over one action window of a run
                    (tools/tas_search.py)
  tas-chain         window-by-window search of a whole run (tools/tas_chain.py)

Train flags mirror the reference's (--envs, --n-steps, --epochs, --lr,
--gamma, --reward, --int-coef, ...): every ``TrainConfig`` field is a flag.
A flag that is not given is restored from ``--ckpt`` when resuming, else
takes its default.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import sys
import time
from pathlib import Path
from typing import Optional, get_args, get_origin

import numpy as np

from .trainer.config import TrainConfig
from .rewards.spec import RewardSpec

# reward fields exposed under their reference flag names
_REWARD_FLAGS = {"mode": "reward", "scale": "reward-scale"}


def _flag(name: str) -> str:
    return "--" + name.replace("_", "-")


def _add_dataclass_flags(ap: argparse.ArgumentParser, cls, prefix: str = "", rename: Optional[dict] = None,
                         skip=()):
    for f in dataclasses.fields(cls):
        if f.name in skip:
            continue
        flag = "--" + (rename or {}).get(f.name, f.name.replace("_", "-"))
        dest = prefix + f.name
        t = f.type if not isinstance(f.type, str) else eval(f.type, {"Optional": Optional, "tuple": tuple})  # noqa: S307
        if get_origin(t) is not None and type(None) in get_args(t):
            t = [a for a in get_args(t) if a is not type(None)][0]
        if t is bool:
            ap.add_argument(flag, dest=dest, action=argparse.BooleanOptionalAction, default=None)
        elif t is tuple or get_origin(t) is tuple:
            ap.add_argument(flag, dest=dest, default=None, help="comma-separated list")
        elif t in (int, float, str):
            ap.add_argument(flag, dest=dest, type=t, default=None)


def _overrides(args) -> dict:
    """Explicitly given TrainConfig / RewardSpec values."""
    out, rew = {}, {}
    for f in dataclasses.fields(TrainConfig):
        if f.name == "reward":
            continue
        v = getattr(args, f.name, None)
        if v is None:
            continue
        if f.name in ("heads", "mlp"):
            parts = [p for p in str(v).split(",") if p]
            v = tuple(int(p) for p in parts) if f.name == "mlp" else tuple(parts)
        out[f.name] = v
    for f in dataclasses.fields(RewardSpec):
        v = getattr(args, "r_" + f.name, None)
        if v is not None:
            rew[f.name] = v
    return out, rew


def _train_parser(sub) -> None:
    ap = sub.add_parser("train", help="PPO training (resumable)")
    _add_dataclass_flags(ap, TrainConfig, skip=("reward",))
    _add_dataclass_flags(ap, RewardSpec, prefix="r_", rename=_REWARD_FLAGS)
    ap.add_argument("--ckpt", default=None, help="resume from a checkpoint file or run directory")
    ap.add_argument("--reset-steps", action="store_true", help="restart the step counter / schedules on resume")
    ap.add_argument("--reset-int-counts", action="store_true", help="drop the checkpoint's curiosity counts")
    ap.add_argument("--iterations", type=int, default=None, help="stop after this many iterations")
    # reference spellings of two settings (python/train_fast.py:785, 804)
    ap.add_argument("--keep-teleports", dest="teleport_fail", action="store_false", default=None,
                    help="falling into a teleport does not end the episode (same as --no-teleport-fail)")
    ap.add_argument("--free-pitch", action="store_true",
                    help="drop a resumed checkpoint's fixed gaze (fix_pitch) and re-enable the pitch head")


def _dist():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def cmd_train(args) -> int:
    import torch
    from .trainer import checkpoint as C
    from .trainer.evaluate import evaluate
    from .trainer.ppo import Trainer
    from .utils.runlog import RunLogger
    rank, world, local = _dist()
    over, rew_over = _overrides(args)
    if getattr(args, "free_pitch", False):
        over["fix_pitch"] = None                 # an explicit override: wins over the checkpoint's value
    sd = None
    restored, changed = [], []
    if args.ckpt:
        path = C.find_resume(args.ckpt)
        if path is None:
            raise SystemExit(f"no checkpoint found at {args.ckpt}")
        sd = C.load(path)
        if rew_over:
            base = RewardSpec.from_dict(sd["config"]["reward"])
            over["reward"] = dataclasses.replace(base, **rew_over)
        cfg, restored, changed = C.resolve_config(sd, over)
    else:
        if rew_over:
            over["reward"] = dataclasses.replace(TrainConfig().reward, **rew_over)
        cfg = TrainConfig(**over)
    if cfg.device == "cuda" and not torch.cuda.is_available():
        raise SystemExit("no CUDA device: pass --device cpu --no-vision for the CPU (eyeless) trainer")
    comm = None
    if cfg.device == "cuda":
        torch.cuda.set_device(local)
    if world > 1:
        from .parallel.dist import init_process_group, make_comm
        init_process_group("nccl" if cfg.device == "cuda" else "gloo")
        comm = make_comm(cfg.comm if cfg.device == "cuda" else "nccl")
    tr = Trainer(cfg, rank=rank, world=world, comm=comm, verbose=(rank == 0))
    if sd is not None:
        tr.load_state_dict(sd, reset_steps=args.reset_steps, reset_counts=args.reset_int_counts)
        if rank == 0:
            print(f"resumed from {args.ckpt} at step {tr.global_step:,}"
                  + (f"; restored {', '.join(restored)}" if restored else "")
                  + (f"; overridden {', '.join(changed)}" if changed else ""), flush=True)
    run_dir = Path(cfg.run)
    log = RunLogger(run_dir, cfg.to_dict(), enabled=(rank == 0),
                    meta={"world": world, "resumed_from": str(args.ckpt) if args.ckpt else None,
                          "restored": restored, "overridden": changed})
    cad = C.Cadence(cfg.ckpt_every, 60.0, tr.global_step)
    next_rec = (tr.global_step // cfg.record_every + 1) * cfg.record_every if cfg.record_every > 0 else float("inf")
    it0 = tr.iteration
    try:
        while tr.global_step < cfg.steps and (args.iterations is None or tr.iteration - it0 < args.iterations):
            stats = tr.train_iteration()
            stats["vf_coef"] = cfg.vf
            line = log.log(stats)
            if rank == 0:
                print(line, flush=True)
                if cfg.timing and stats.get("timing"):
                    from .utils.timer import PhaseClock
                    print(PhaseClock.timing_line(tr.iteration, stats["timing"]), flush=True)
            if tr.global_step >= next_rec:
                next_rec += cfg.record_every
                out = run_dir / "recordings" / f"eval_{tr.global_step:010d}.traj.jsonl" if rank == 0 else None
                summ = evaluate(tr, episodes=cfg.eval_eps, greedy=True, max_ticks=cfg.ep_ticks, out=out)
                log.set_eval(summ)
                if rank == 0:
                    print(f"eval: return {summ['ep_return']:.2f} speed_max {summ['speed_max']:.0f} "
                          f"success {summ['success_rate']:.2f} -> {summ.get('file')}", flush=True)
                if not cfg.eval_greedy_only:        # the stochastic recording beside the greedy one
                    sout = out.with_name(out.name.replace(".traj.jsonl", "_stoch.traj.jsonl")) if out else None
                    ss = evaluate(tr, episodes=cfg.eval_eps, greedy=False, max_ticks=cfg.ep_ticks, out=sout,
                                  seed=tr.global_step & 0x7FFFFFFF)
                    if rank == 0:
                        print(f"eval (stochastic): return {ss['ep_return']:.2f} -> {ss.get('file')}", flush=True)
            numbered = cad.numbered(tr.global_step)
            latest = cad.latest_due(time.time())
            if comm is not None:
                latest = comm.max_scalar(1.0 if latest else 0.0) > 0.5
            if numbered or latest:
                state = tr.state_dict()                     # collective under data parallelism
                if rank == 0:
                    if numbered:
                        C.save(run_dir / f"ckpt_{tr.global_step:010d}.pt", state)
                    C.save(run_dir / "ckpt_latest.pt", state)
        state = tr.state_dict()
        if rank == 0:
            C.save(run_dir / "ckpt_final.pt", state)
            C.save(run_dir / "ckpt_latest.pt", state)
        log.finish({"global_step": tr.global_step, "iterations": tr.iteration})
    finally:
        tr.release_graphs()
        if comm is not None:
            comm.close()
    return 0


def cmd_eval(args) -> int:
    import torch
    from .trainer import checkpoint as C
    from .trainer.evaluate import evaluate
    from .trainer.ppo import Trainer
    path = C.find_resume(args.ckpt)
    if path is None:
        raise SystemExit(f"no checkpoint at {args.ckpt}")
    sd = C.load(path)
    unknown = C.audit(sd)
    if unknown:
        raise SystemExit(f"refusing {path}: its configuration has settings this build does not mirror: {unknown}")
    cfg = TrainConfig.from_dict(sd["config"])
    cfg.envs = max(8, args.episodes)
    cfg.graphs = False
    if not torch.cuda.is_available():
        if cfg.vision:
            raise SystemExit("this checkpoint's policy has a depth camera: evaluating it needs a CUDA device")
        cfg.device = "cpu"
    if cfg.reward.int_coef > 0:
        cfg.reward = dataclasses.replace(cfg.reward, table_log2=min(cfg.reward.table_log2, 12))
    tr = Trainer(cfg, verbose=False)
    tr.net.load_state_dict(sd["policy"])
    out = args.out or (Path(path).parent / "recordings" / f"{Path(path).stem}.traj.jsonl")
    summ = evaluate(tr, episodes=args.episodes, greedy=not args.stochastic, max_ticks=args.max_ticks or cfg.ep_ticks,
                    out=None if args.no_record else out, seed=args.seed)
    print(json.dumps(summ))
    return 0


def cmd_mapgen(args) -> int:
    from .sim import mapgen
    m = mapgen.generate(args.kind, args.seed)
    p = m.save(args.out)
    print(f"{p} ({len(m.image):,} bytes, {m.meta.get('brushes', '?')} brushes, "
          f"{0 if m.spawn_pool is None else len(m.spawn_pool)} pool spawns)")
    return 0


def _open_map(path_or_kind: str, seed: int = 0):
    from .sim import mapgen
    from .sim.core import SimCore, default_config
    if path_or_kind in mapgen.MAP_KINDS:
        m = mapgen.generate(path_or_kind, seed)
        return SimCore.from_bytes(m.image, default_config(1), threads=1), m.name, m
    return SimCore(path_or_kind, default_config(1), threads=1), Path(path_or_kind).stem, None


def cmd_bake(args) -> int:
    import numpy as np
    import torch
    from .ops.vision import SdfVolume
    core, name, m = _open_map(args.map, args.seed)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    t0 = time.time()
    kw = {}
    if m is not None and "grid_mins" in m.meta and args.cell is None:
        kw = dict(cell=m.meta["cell"], mins=np.array(m.meta["grid_mins"]), dims=tuple(m.meta["dims"]))
    vol = SdfVolume.build(core, cell=args.cell or kw.pop("cell", 16.0), device=dev, **kw)
    p = vol.save(out / f"{name}.sdf.npz")
    print(f"sdf {vol.dims} cell {vol.cell} -> {p} ({time.time() - t0:.1f}s)")
    if args.goal:
        from .ops.geodesic import bake_goal_field
        zones = m.zones if m is not None else json.loads(Path(args.map).with_suffix(".zones.json").read_text())
        if not zones.get("end"):
            raise SystemExit("the map has no finish zone")
        t0 = time.time()
        gf = bake_goal_field(core, zones["end"], cell=args.goal_cell, device=dev)
        gp = out / f"{name}.goal.npz"
        gf.save(gp)
        print(f"goal field {gf.grid.shape} reach_max {gf.reach_max:.0f}u -> {gp} ({time.time() - t0:.1f}s)")
    return 0


def cmd_export_map(args) -> int:
    from .sim.export import export_mesh
    core, name, _ = _open_map(args.map, args.seed)
    doc = export_mesh(core, name)
    Path(args.out).write_text(json.dumps(doc, separators=(",", ":")))
    print(f"{args.out}: {len(doc['vertices']) // 3:,} vertices, {len(doc['indices']) // 3:,} triangles")
    return 0


def cmd_export_goalfield(args) -> int:
    import numpy as np
    from .rewards.spec import GoalFieldData
    from .sim.export import export_goalfield
    gf = GoalFieldData.load(args.field)
    doc = export_goalfield(gf, stride=args.stride)
    Path(args.out).write_text(json.dumps(doc, separators=(",", ":")))
    print(f"{args.out}: {len(doc['arrows'])} arrows")
    del np
    return 0


def cmd_perf_report(args) -> int:
    from .utils.perf_report import main as perf_main
    return perf_main(args)


def cmd_gpu_health(args) -> int:
    from .utils.gpu_health import main as health_main
    return health_main(args)


def cmd_render_pov(args) -> int:
    from .utils.tools import render_pov
    n = render_pov(args.traj, args.map, args.out, width=args.width, height=args.height, cell=args.cell,
                   episode=args.episode, stride=args.stride, pinhole=args.pinhole)
    print(f"{n} frames -> {args.out}")
    return 0


def cmd_sample_traj(args) -> int:
    from .utils.tools import sample_trajectory
    print(sample_trajectory(args.out))
    return 0


def cmd_compare_runs(args) -> int:
    from .utils.tools import compare_runs
    marks = tuple(float(x) for x in args.marks.split(","))
    print(compare_runs(args.runs, marks, args.col))
    return 0


def cmd_serve_metrics(args) -> int:
    from .utils.tools import serve_metrics
    print(f"serving {args.runs_dir} on http://{args.host}:{args.port}/api/runs", flush=True)
    serve_metrics(args.runs_dir, args.host, args.port)
    return 0


def cmd_bench_env(args) -> int:
    from .utils.tools import env_thread_sweep
    for r in env_thread_sweep(args.map, args.envs, args.k, args.reps):
        print(json.dumps(r))
    return 0


def _episodes_arg(args):
    from .utils import tas
    eps = tas.episodes(args.traj)
    if not eps:
        raise SystemExit(f"no episodes in {args.traj}")
    return eps


def cmd_strafe_audit(args) -> int:
    from .utils import tas
    eps = _episodes_arg(args)
    sel = [eps[args.ep - 1]] if args.ep else eps
    print(json.dumps(tas.strafe_audit_many(sel)))
    return 0


def cmd_route_bound(args) -> int:
    from .utils import tas
    eps = _episodes_arg(args)
    if args.ep is None:
        for k, e in enumerate(eps, 1):
            print(json.dumps({"episode": k, "ticks": len(e), "z_drop": float(e[0, 3] - e[:, 3].min()),
                              "peak_speed": float(np.hypot(e[:, 4], e[:, 5]).max())}))
        return 0
    e = eps[args.ep - 1]
    if args.from_drop:
        e = tas.from_drop(e)
    print(json.dumps(tas.route_bound(e, gravity=args.gravity, segments=args.segments, target=args.target)))
    return 0


def _search_env(args):
    from .sim import mapgen
    from .sim.core import SimCore, default_config
    from .sim.zones import load_zones
    from .utils import tas
    cfg = default_config(args.envs, max_episode_ticks=1_000_000, sv_maxvelocity=args.maxvel)
    if args.map in mapgen.MAP_KINDS:
        m = mapgen.generate(args.map, args.seed)
        core, zones = SimCore.from_bytes(m.image, cfg, threads=args.threads), m.zones
    else:
        core, zones = SimCore(args.map, cfg, threads=args.threads), load_zones(args.map)
    core.reset(0)
    return core, tas.make_scorer(core, zones, cell=args.cell)


def cmd_tas_search(args) -> int:
    from .utils import tas
    e = _episodes_arg(args)[args.ep - 1]
    core, score = _search_env(args)
    r = tas.tas_search(core, score, e, args.t0, args.window, args.iters, args.p_mutate, args.seed,
                       log=lambda m: print(m, flush=True))
    acts = r.pop("actions")
    if args.out:
        np.save(args.out, acts)
    print(json.dumps(r))
    core.close()
    return 0


def cmd_tas_chain(args) -> int:
    from .utils import tas
    e = _episodes_arg(args)[args.ep - 1]
    if args.from_drop:
        e = tas.from_drop(e)
    core, score = _search_env(args)
    r = tas.tas_chain(core, score, e, args.window, args.iters, args.p_mutate, args.max_windows, args.seed,
                      finish_score=getattr(score, "finish", None), log=lambda m: print(m, flush=True))
    out = Path(args.out) if args.out else Path(args.traj).with_suffix(".chained.npy")
    np.save(out, r.pop("actions"))
    print(json.dumps({**r, "actions": str(out)}))
    core.close()
    return 0


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="surfb200", description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    _train_parser(sub)
    e = sub.add_parser("eval", help="evaluation episodes / recording of a checkpoint")
    e.add_argument("--ckpt", required=True)
    e.add_argument("--episodes", type=int, default=3)
    e.add_argument("--stochastic", action="store_true", help="sample actions instead of the greedy argmax")
    e.add_argument("--max-ticks", type=int, default=None)
    e.add_argument("--out", default=None)
    e.add_argument("--no-record", action="store_true")
    e.add_argument("--seed", type=int, default=4242)
    g = sub.add_parser("mapgen", help="write a procedural map")
    g.add_argument("--kind", default="field")
    g.add_argument("--seed", type=int, default=0)
    g.add_argument("--out", default="maps")
    b = sub.add_parser("bake", help="build the SDF (and goal field) caches of a map")
    b.add_argument("--map", required=True, help="a .bsp path or a procedural kind")
    b.add_argument("--seed", type=int, default=0)
    b.add_argument("--cell", type=float, default=None)
    b.add_argument("--goal", action="store_true")
    b.add_argument("--goal-cell", type=float, default=16.0)
    b.add_argument("--out", default="maps/cache")
    x = sub.add_parser("export-map", help="mesh JSON of a map")
    x.add_argument("--map", required=True)
    x.add_argument("--seed", type=int, default=0)
    x.add_argument("--out", required=True)
    xg = sub.add_parser("export-goalfield", help="arrow JSON of a baked goal field")
    xg.add_argument("--field", required=True)
    xg.add_argument("--stride", type=int, default=8)
    xg.add_argument("--out", required=True)
    pr = sub.add_parser("perf-report", help="summarise TIMING lines")
    pr.add_argument("logs", nargs="+")
    pr.add_argument("--last", type=int, default=30)
    pr.add_argument("--vs", default=None, help="a second log to compare against")
    rp = sub.add_parser("render-pov", help="depth frames (PGM + npy) along a recorded trajectory")
    rp.add_argument("--traj", required=True)
    rp.add_argument("--map", required=True, help="a .bsp path or a procedural kind")
    rp.add_argument("--out", required=True)
    rp.add_argument("--width", type=int, default=128)
    rp.add_argument("--height", type=int, default=64)
    rp.add_argument("--cell", type=float, default=16.0)
    rp.add_argument("--episode", type=int, default=0)
    rp.add_argument("--stride", type=int, default=3)
    rp.add_argument("--pinhole", action="store_true")
    st = sub.add_parser("sample-traj", help="write a synthetic trajectory file")
    st.add_argument("--out", required=True)
    cr = sub.add_parser("compare-runs", help="runs side by side at step marks")
    cr.add_argument("runs", nargs="+")
    cr.add_argument("--marks", default="250e6,500e6,1e9")
    cr.add_argument("--col", default="rew", choices=["rew", "len", "spd", "track", "fin"])
    sm = sub.add_parser("serve-metrics", help="JSON metrics API over a runs directory")
    sm.add_argument("runs_dir")
    sm.add_argument("--host", default="127.0.0.1")
    sm.add_argument("--port", type=int, default=8008)
    be = sub.add_parser("bench-env", help="env ticks/s per worker thread count")
    be.add_argument("--map", default="field")
    be.add_argument("--envs", type=int, default=2048)
    be.add_argument("--k", type=int, default=3)
    be.add_argument("--reps", type=int, default=20)
    sa = sub.add_parser("strafe-audit", help="air-acceleration capture of recorded episodes")
    sa.add_argument("traj")
    sa.add_argument("--ep", type=int, default=None, help="1-based episode (default: all)")
    rb = sub.add_parser("route-bound", help="time floors and energy budget of a recorded route")
    rb.add_argument("traj")
    rb.add_argument("--ep", type=int, default=None, help="1-based episode (default: list them)")
    rb.add_argument("--target", type=float, default=None, help="target time, s")
    rb.add_argument("--segments", type=int, default=10)
    rb.add_argument("--gravity", type=float, default=800.0)
    rb.add_argument("--from-drop", action="store_true", help="start the clock at the opening drop")
    for name, hlp in (("tas-search", "batched hill climb over one window of a recorded run"),
                      ("tas-chain", "window-by-window search of a whole recorded run")):
        ts = sub.add_parser(name, help=hlp)
        ts.add_argument("traj")
        ts.add_argument("--map", required=True, help="a .bsp path or a procedural kind")
        ts.add_argument("--seed", type=int, default=0)
        ts.add_argument("--ep", type=int, default=1, help="1-based episode")
        ts.add_argument("--window", type=int, default=300 if name == "tas-search" else 150)
        ts.add_argument("--iters", type=int, default=40 if name == "tas-search" else 25)
        ts.add_argument("--envs", type=int, default=2048 if name == "tas-search" else 1024)
        ts.add_argument("--p-mutate", type=float, default=0.06 if name == "tas-search" else 0.05)
        ts.add_argument("--cell", type=float, default=32.0, help="goal-field voxel size")
        ts.add_argument("--maxvel", type=float, default=4000.0)
        ts.add_argument("--threads", type=int, default=None)
        ts.add_argument("--out", default=None, help=".npy file for the best action sequence")
        if name == "tas-search":
            ts.add_argument("--t0", type=int, default=0, help="tick to branch at")
        else:
            ts.add_argument("--max-windows", type=int, default=0, help="0 = the whole run")
            ts.add_argument("--from-drop", action="store_true", help="start at the opening drop")
    gh = sub.add_parser("gpu-health", help="HBM and bf16 GEMM health check")
    gh.add_argument("--seconds", type=float, default=2.0)
    gh.add_argument("--peaks", default=None)
    return ap


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    fn = {"train": cmd_train, "eval": cmd_eval, "mapgen": cmd_mapgen, "bake": cmd_bake,
          "export-map": cmd_export_map, "export-goalfield": cmd_export_goalfield, "perf-report": cmd_perf_report,
          "gpu-health": cmd_gpu_health, "render-pov": cmd_render_pov, "sample-traj": cmd_sample_traj,
          "compare-runs": cmd_compare_runs, "serve-metrics": cmd_serve_metrics, "bench-env": cmd_bench_env,
          "strafe-audit": cmd_strafe_audit, "route-bound": cmd_route_bound, "tas-search": cmd_tas_search,
          "tas-chain": cmd_tas_chain}[args.cmd]
    return int(fn(args) or 0)


if __name__ == "__main__":
    sys.exit(main())
