"""Evaluation episodes and trajectory recording (JSONL).

``evaluate`` rolls the trainer's current policy (greedy or stochastic) on a
separate env batch, one episode per env, ticking the simulator one physics
tick at a time (the policy decides every ``act_every`` ticks) so that every
tick can be recorded. ``TrajectoryWriter`` writes the reference's
trajectory format (python/surfgym/record.py:1-26), which its viewer reads:

    {"map": ..., "tick_ms": 10, "phys": {...}, "episode": k}      header
    [t, x, y, z, vx, vy, vz, yaw, buttons, onground, progress, reward,
     pitch, fwd, side]                                             one per tick
    {"end": "done|fail|trunc", "ticks": n, "best_progress": p}     trailer

A tick line holds the state at the start of the tick with the action taken
and the reward earned during it; buttons are IN_JUMP (2) | IN_DUCK (4).
"""
from __future__ import annotations

import json
import math
from pathlib import Path
from typing import Optional

import numpy as np
import torch

from ..sim.core import REC_COLS, TERM_COLS, SimCore, config_to_dict, default_config

IN_JUMP, IN_DUCK = 2, 4
DONE_BONUS_MIN = 25.0
C_OBS, C_TOBS, C_REC, C_TREC, H_COLS = 0, 16, 32, 48, 64


class TrajectoryWriter:
    def __init__(self, path, map_name: str, phys: dict, tick_ms: int = 10):
        self.path = Path(path)
        self.path.parent.mkdir(parents=True, exist_ok=True)
        self.f = open(self.path, "w", encoding="utf-8", newline="\n")
        self.base = {"map": map_name, "tick_ms": int(tick_ms), "phys": phys}

    def header(self, episode: int) -> None:
        self.f.write(json.dumps({**self.base, "episode": int(episode)}, separators=(",", ":")) + "\n")

    def tick(self, t: int, st, act, reward: float) -> None:
        buttons = (IN_JUMP if act[4] else 0) | (IN_DUCK if act[5] else 0)
        o, v = st["origin"], st["velocity"]
        line = [int(t), round(float(o[0]), 2), round(float(o[1]), 2), round(float(o[2]), 2),
                round(float(v[0]), 2), round(float(v[1]), 2), round(float(v[2]), 2), round(float(st["yaw"]), 2),
                int(buttons), int(int(st["onground"]) >= 0), round(float(st["progress"]), 2), round(float(reward), 5),
                round(float(st["pitch"]), 2), int(act[2]), int(act[3])]
        self.f.write(json.dumps(line, separators=(",", ":")) + "\n")

    def trailer(self, end: str, ticks: int, best_progress: float) -> dict:
        t = {"end": end, "ticks": int(ticks), "best_progress": round(float(best_progress), 2)}
        self.f.write(json.dumps(t, separators=(",", ":")) + "\n")
        self.f.flush()
        return t

    def close(self) -> None:
        self.f.close()


def read_trajectory(path) -> list:
    """Episodes of a trajectory file: [{"header", "ticks" (array), "trailer"}]."""
    eps = []
    cur = None
    for line in Path(path).read_text().splitlines():
        if not line.strip():
            continue
        v = json.loads(line)
        if isinstance(v, dict) and "episode" in v:
            cur = {"header": v, "ticks": [], "trailer": None}
            eps.append(cur)
        elif isinstance(v, dict):
            cur["trailer"] = v
        else:
            cur["ticks"].append(v)
    for e in eps:
        e["ticks"] = np.asarray(e["ticks"], np.float64).reshape(-1, 15)
    return eps


class _EvalFrames:
    """Frame history of an evaluation (one episode per env, all started
    together): a ring of the last ``pro + 1`` renders, composed by the same
    stacking kernel as the trainer's rollout."""

    def __init__(self, trainer, n: int):
        from ..ops.framestack import FrameStacker
        st = trainer.stacker
        self.ring = st.pro + 1
        self.stacker = FrameStacker(trainer.n_frames, st.fr, st.C0, ring=self.ring)
        dev = trainer.device
        self.frames = torch.zeros((self.ring, n, st.fr), dtype=torch.bfloat16, device=dev)
        self.age = torch.zeros(n, dtype=torch.int32, device=dev)
        self.rec = torch.zeros(n, dtype=torch.int32, device=dev)
        self.zero = torch.zeros(n, dtype=torch.float32, device=dev)
        self.out = torch.zeros((n, st.fr * st.K), dtype=torch.bfloat16, device=dev)
        self.d = 0

    def __call__(self, camera, pose: torch.Tensor) -> torch.Tensor:
        slot = self.d % self.ring
        camera.render(pose, out=self.frames[slot])
        out = self.stacker.rollout(self.frames, slot, 0, self.frames.shape[1], self.zero if self.d > 0 else None,
                                   self.age, self.rec, self.out)
        self.d += 1
        return out


class _RewardFeed:
    """The obs-reward observation during evaluation (reference
    _make_eval_reward_feed, python/train_fast.py:1478-1499): the eval env pays
    no training reward, so the race shaping term is recomputed from the goal
    field per decision, r = clip(d_prev - d, +-100 K) * scale - time_pen * K
    (zeros on the first decision), and the policy reads tanh(r / 0.1)."""

    def __init__(self, trainer, K: int):
        spec = trainer.cfg.reward
        self.field, self.K = trainer.field, K
        self.scale = spec.resolved_scale(trainer.d0)
        self.time_pen = spec.time_pen
        self.d = None

    def __call__(self, origins: np.ndarray) -> np.ndarray:
        d = np.asarray(self.field.sample(origins.astype(np.float64)), np.float64)
        prev, self.d = self.d, d
        if prev is None:
            return np.zeros(len(d), np.float32)
        delta = np.clip(prev - d, -100.0 * self.K, 100.0 * self.K)
        return (delta * self.scale - self.time_pen * self.K).astype(np.float32)


def _policy_actions(trainer, h: np.ndarray, greedy: bool, gen: Optional[torch.Generator], frames=None,
                    rew: Optional[np.ndarray] = None):
    """Action rows [n, 8] int32 for host records h [n, 64] (``frames``: the
    frame history when the policy stacks frames; ``rew``: the obs-reward feed,
    raw rewards of the previous decision)."""
    from ..models.policy import Workspace, forward_gpu
    from ..ops import rl as R
    net, layout = trainer.net, trainer.layout
    n = h.shape[0]
    if trainer.gpu:
        dev = trainer.device
        hd = torch.as_tensor(h, device=dev)
        scal = torch.zeros((n, 16), dtype=torch.bfloat16, device=dev)
        trainer._features(hd[:, C_OBS:C_OBS + 15].contiguous(), scal,
                          rew=torch.as_tensor(rew, device=dev) if rew is not None else None)
        img = None
        if trainer.cfg.vision:
            pose = hd[:, C_REC:C_REC + 6].contiguous()
            img = frames(trainer.camera, pose) if frames is not None else trainer.camera.render(pose)
        ws = getattr(trainer, "_eval_ws", None)
        if ws is None or ws.B < n:
            ws = trainer._eval_ws = Workspace(net, max(n, 8))
        out = forward_gpu(net, ws, scal, img, B=n).float().cpu()
    else:
        feats = np.zeros((n, 16), np.float32)
        feats[:, :len(trainer.feat_idx)] = h[:, [C_OBS + i for i in trainer.feat_idx]]
        if trainer.rew_col >= 0:
            feats[:, trainer.rew_col] = np.tanh((rew if rew is not None else np.zeros(n, np.float32)) / 0.1)
        with torch.no_grad():
            out = net.forward_reference(torch.from_numpy(feats), None)
    act, _ = R.sample_reference(out, layout, net.p("log_std").detach().float().cpu(), gen, greedy=greedy)
    return act.numpy()


def evaluate(trainer, episodes: int = 3, greedy: bool = True, max_ticks: int = 6000, out=None, seed: int = 4242,
             pool: Optional[np.ndarray] = None, record_all: bool = True) -> dict:
    """Roll ``episodes`` episodes (one per env) and summarise them; with
    ``out`` a trajectory file is written (every env's episode in turn, or env
    0 only when ``record_all`` is False)."""
    cfg = trainer.cfg
    n = int(episodes)
    env_cfg = default_config(n, max_episode_ticks=max_ticks, spawn_mode=2 if (pool is not None or
                                                                               trainer.spawn_pool is not None) else 0,
                             sv_maxvelocity=cfg.maxvel, sv_airaccelerate=cfg.airaccelerate,
                             pitch_rate_max_deg=0.0 if cfg.fix_pitch is not None else cfg.pitch_rate,
                             yaw_adaptive=int(cfg.yaw_adaptive))
    core = SimCore.from_bytes(trainer.map_image, env_cfg, threads=min(8, n))
    sp = pool if pool is not None else trainer.spawn_pool
    if sp is not None:
        core.set_spawn_pool(sp)
    core.set_teleport_fail(cfg.teleport_fail)
    end_zone = trainer.zones.get("end") if trainer.zones else None
    if end_zone:
        core.set_goal_box(end_zone["mins"], end_zone["maxs"])
    obs = core.reset(seed)
    h = np.zeros((n, H_COLS), np.float32)
    st = core.states_view
    h[:, C_OBS:C_OBS + 15] = obs[:, :15]
    h[:, C_REC:C_REC + 3] = st["origin"]
    h[:, C_REC + 3] = st["yaw"]
    h[:, C_REC + 4] = st["pitch"]
    h[:, C_REC + 5] = st["ducked"]
    gen = torch.Generator().manual_seed(seed)
    yaw_slot = 6 if trainer.layout.continuous_yaw else -1
    active = np.ones(n, bool)
    ticks = np.zeros(n, np.int64)
    ret = np.zeros(n)
    best = np.zeros(n)
    peak_speed = np.zeros(n)
    start = st["origin"].astype(np.float64).copy()
    fwd_max = np.zeros(n)
    path_len = np.zeros(n)
    ends = [None] * n
    rows: list = [[] for _ in range(n)]
    K = cfg.act_every
    t = 0
    frames = _EvalFrames(trainer, n) if getattr(trainer, "stacker", None) is not None else None
    feed = _RewardFeed(trainer, K) if trainer.rew_col >= 0 else None
    while active.any() and t < max_ticks:
        rew_feed = feed(h[:, C_REC:C_REC + 3]) if feed is not None else None
        act = np.ascontiguousarray(_policy_actions(trainer, h, greedy, gen, frames, rew_feed).astype(np.int32))
        for _ in range(K):
            pre = st.copy()
            hp = h.ctypes.data
            core.step_k(act.ctypes.data, 8, 1, yaw_slot=yaw_slot, fail_slot=-1, obs=(hp + 4 * C_OBS, H_COLS),
                        term_obs=(hp + 4 * C_TOBS, H_COLS), rec=(hp + 4 * C_REC, H_COLS),
                        term_rec=(hp + 4 * C_TREC, H_COLS))
            rew = h[:, C_REC + 10]
            done = h[:, C_REC + 11] != 0
            trunc = h[:, C_REC + 12] != 0
            for e in np.flatnonzero(active):
                if out is not None and (record_all or e == 0):
                    rows[e].append((int(ticks[e]), pre[e], act[e].copy(), float(rew[e])))
                ret[e] += float(rew[e])
                best[e] = max(best[e], float(pre[e]["best_progress"]), float(pre[e]["progress"]))
                peak_speed[e] = max(peak_speed[e], math.hypot(float(pre[e]["velocity"][0]), float(pre[e]["velocity"][1])))
                d = pre[e]["origin"].astype(np.float64) - start[e]
                fwd_max[e] = max(fwd_max[e], float(np.hypot(d[0], d[1])))
                ticks[e] += 1
                if done[e] or trunc[e]:
                    ends[e] = ("done" if float(rew[e]) >= DONE_BONUS_MIN or bool(core.goal_hits[e]) else "fail") \
                        if done[e] else "trunc"
                    active[e] = False
            t += 1
            if not active.any() or t >= max_ticks:
                break
    for e in np.flatnonzero(active):
        ends[e] = "trunc"
    summary = {"episodes": n, "ep_return": float(ret.mean()), "ticks_mean": float(ticks.mean()),
               "speed_max": float(peak_speed.max()), "fwd_max": float(fwd_max.max()),
               "progress": float(best.mean()), "success_rate": float(np.mean([x == "done" for x in ends])),
               "ends": ends}
    fin = [ticks[e] * 0.01 for e in range(n) if ends[e] == "done"]
    summary["finish_s"] = float(np.min(fin)) if fin else None
    if out is not None:
        phys = config_to_dict(env_cfg).get("phys", {})
        name = trainer.procmap.name if trainer.procmap is not None else Path(str(cfg.map)).stem
        w = TrajectoryWriter(out, name, phys)
        for e in range(n):
            if not (record_all or e == 0):
                continue
            w.header(e)
            for (tt, s, a, r) in rows[e]:
                w.tick(tt, s, a, r)
            w.trailer(ends[e], ticks[e], best[e])
        w.close()
        summary["file"] = str(out)
    core.close()
    return summary
