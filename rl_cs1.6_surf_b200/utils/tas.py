"""Trajectory analysis and search on the batched simulator.

Four analyses of a recorded run (the JSONL trajectory format of
``trainer.evaluate``), none of which involves a policy network:

* ``strafe_audit`` — how much of the engine's air acceleration the run
  banked. In air the wish speed is capped at 30 u/s along ``wishdir``
  (PM_AirAccelerate), and at sv_airaccelerate 100 the per-tick impulse is
  saturated, so |v_h|^2 grows by 900 - (v . wishdir)^2 when v . wishdir < 30
  and by nothing otherwise (reference: tools/strafe_audit.py:1-112).
* ``route_bound`` — lower bounds on the time of the recorded polyline: a
  rigorous floor (|v|^2 <= v0^2 + 2 g dz + 900 n, no energy lost at ramps)
  and a practical floor (perfect strafe, the recorded fractional loss at each
  contact), with per-segment and contact-quality sensitivity tables
  (reference: tools/route_bound.py:1-187).
* ``tas_search`` — a (1 + lambda) hill climb over the action window after a
  recorded tick: every env of one batch restores the recorded state and plays
  a mutation of the incumbent window; the candidate ending with the best
  score becomes the incumbent (reference: tools/tas_search.py:1-172).
* ``tas_chain`` — the same search window after window, each starting from the
  best state reached so far, which builds a whole improved run
  (reference: tools/tas_chain.py:1-128).

Scores are the geodesic distance to the finish zone when the map has one
(``ops.geodesic.bake_goal_field``), else minus the env's track progress. A
candidate whose episode ends inside the window scores +inf when it failed and
ranks by ticks when it reached the goal.
"""
from __future__ import annotations

import math
from typing import Callable, Optional

import numpy as np

# yaw-rate bins of the discrete action (degrees per tick; csrc/sim/env.cpp kYawBins)
YAW_BINS = np.array([-10.0, -7.0, -4.0, -2.0, -1.0, -0.5, -0.25, 0.0, 0.25, 0.5, 1.0, 2.0, 4.0, 7.0, 10.0])
PITCH_ZERO_BIN = 3
IN_JUMP, IN_DUCK = 2, 4
AIR_CAP = 30.0                 # PM_AirAccelerate wish-speed cap
MAX_DV2 = AIR_CAP * AIR_CAP    # largest growth of |v_h|^2 per tick
TICK = 0.01
TELEPORT_STEP = 110.0          # a position jump longer than this is a teleport, never credited as route


# ---- recordings -----------------------------------------------------------------------------------
def episodes(path) -> list:
    """Tick arrays (n, 15) of every episode of a trajectory file."""
    from ..trainer.evaluate import read_trajectory
    return [e["ticks"] for e in read_trajectory(path)]


def from_drop(ticks: np.ndarray, drop: float = 100.0) -> np.ndarray:
    """The run clock of a start-platform map: from the first tick ``drop``
    units below the first recorded height."""
    below = np.flatnonzero(ticks[:, 3] < ticks[0, 3] - drop)
    return ticks[int(below[0]):] if len(below) else ticks


def infer_actions(ticks: np.ndarray, yaw_scale: float = 1.0) -> np.ndarray:
    """(n - 1, 6) int32 action rows that reproduce a recording: fwd / side /
    buttons are recorded verbatim; the yaw bin is the one nearest the realised
    per-tick yaw change (wrapped). Pitch only aims the camera, so it is left
    at the zero bin."""
    dy = (np.diff(ticks[:, 7]) + 180.0) % 360.0 - 180.0
    bins = YAW_BINS * yaw_scale
    act = np.zeros((len(dy), 6), np.int32)
    act[:, 0] = np.abs(dy[:, None] - bins[None, :]).argmin(1)
    act[:, 1] = PITCH_ZERO_BIN
    act[:, 2] = ticks[:-1, 13].astype(np.int32)
    act[:, 3] = ticks[:-1, 14].astype(np.int32)
    btn = ticks[:-1, 8].astype(np.int32)
    act[:, 4] = (btn & IN_JUMP) != 0
    act[:, 5] = (btn & IN_DUCK) != 0
    return act


# ---- strafe audit -----------------------------------------------------------------------------------
def strafe_audit(ticks: np.ndarray) -> dict:
    """Air-acceleration capture of one episode (fractions of the 900/tick ceiling)."""
    v, yaw = ticks[:, 4:7], np.radians(ticks[:, 7])
    move = lambda b: np.where(b <= 0, -400.0, np.where(b >= 2, 400.0, 0.0))
    fm, sm = move(ticks[:, 13].astype(int)), move(ticks[:, 14].astype(int))
    # forward = (cos y, sin y), right = (sin y, -cos y)
    wx = np.cos(yaw) * fm + np.sin(yaw) * sm
    wy = np.sin(yaw) * fm - np.cos(yaw) * sm
    wn = np.hypot(wx, wy)
    has = wn > 1e-6
    ux, uy = np.where(has, wx / np.maximum(wn, 1e-9), 0.0), np.where(has, wy / np.maximum(wn, 1e-9), 0.0)
    vh = np.hypot(v[:, 0], v[:, 1])
    along = v[:, 0] * ux + v[:, 1] * uy
    angle = np.degrees(np.arccos(np.clip(along / np.maximum(vh, 1e-9), -1.0, 1.0)))
    active = has & (along < AIR_CAP)
    gain = np.where(active, MAX_DV2 - along * along, 0.0)
    n = len(ticks) - 1
    sl = slice(0, n)
    turn = np.abs((np.diff(ticks[:, 7]) + 180.0) % 360.0 - 180.0)
    return {"ticks": n, "capture": float(gain[sl].sum() / (MAX_DV2 * max(n, 1))),
            "in_window": float(active[sl].mean()) if n else 0.0,
            "median_angle_error_deg": float(np.median(np.abs(angle[sl] - 90.0))) if n else 0.0,
            "within_5deg": float(np.mean(np.abs(angle[sl] - 90.0) < 5.0)) if n else 0.0,
            "mean_speed": float(vh.mean()), "peak_speed": float(vh.max()),
            "mean_turn_deg": float(turn.mean()) if n else 0.0}


def strafe_audit_many(eps: list) -> dict:
    """Tick-weighted means over several episodes."""
    st = [strafe_audit(e) for e in eps]
    w = np.array([s["ticks"] for s in st], np.float64)
    out = {k: float(np.average([s[k] for s in st], weights=w)) for k in st[0] if k not in ("ticks", "peak_speed")}
    out.update(episodes=len(st), ticks=int(w.sum()), peak_speed=max(s["peak_speed"] for s in st))
    return out


# ---- route bounds -----------------------------------------------------------------------------------
def _route(pos: np.ndarray):
    step = np.linalg.norm(np.diff(pos, axis=0), axis=1)
    return np.where(step <= TELEPORT_STEP, step, 0.0)


def rigorous_floor(pos: np.ndarray, v0: float, gravity: float = 800.0, vmax: float = 4000.0 * math.sqrt(3.0)):
    """(seconds, route length): a particle marched along the polyline at the
    speed ceiling sqrt(v0^2 + 2 g (z0 - z) + 900 n) after n ticks."""
    step = _route(pos)
    cum = np.concatenate(([0.0], np.cumsum(step)))
    total = float(cum[-1])
    s, n, seg = 0.0, 0, 0
    while s < total and n < 1_000_000:
        while seg + 2 < len(cum) and cum[seg + 1] <= s:
            seg += 1
        span = cum[seg + 1] - cum[seg]
        f = (s - cum[seg]) / span if span > 0 else 0.0
        z = pos[seg, 2] + f * (pos[seg + 1, 2] - pos[seg, 2])
        v2 = v0 * v0 + 2.0 * gravity * (pos[0, 2] - z) + MAX_DV2 * n
        s += min(math.sqrt(max(v2, 0.0)), vmax) * TICK
        n += 1
    return n * TICK, total


def practical_floor(pos: np.ndarray, e0: float, loss_frac: np.ndarray, gravity: float = 800.0,
                    loss_cut: float = 0.0):
    """(seconds, per-step seconds): perfect strafe (specific energy +450 per
    tick of flight) with the recorded fractional kinetic-energy loss at each
    step, optionally reduced by ``loss_cut``."""
    step = np.linalg.norm(np.diff(pos, axis=0), axis=1)
    e, total = e0, 0.0
    per = np.zeros(len(step))
    for i in range(len(step)):
        kin = max(1.0, e - gravity * pos[i, 2])
        dt = step[i] / max(math.sqrt(2.0 * kin), 1.0)
        e += 0.5 * MAX_DV2 * dt / TICK
        kin = max(1.0, e - gravity * pos[i + 1, 2]) * (1.0 - loss_frac[i] * (1.0 - loss_cut))
        e = kin + gravity * pos[i + 1, 2]
        per[i] = dt
        total += dt
    return total, per


def route_bound(ticks: np.ndarray, gravity: float = 800.0, segments: int = 10, target: Optional[float] = None) -> dict:
    """Energy budget, floors, per-segment table and contact sensitivity of one episode."""
    p, v = ticks[:, 1:4], ticks[:, 4:7]
    sp2 = (v * v).sum(1)
    energy = 0.5 * sp2 + gravity * p[:, 2]
    de = np.diff(energy)
    d = np.linalg.norm(np.diff(p, axis=0), axis=1)
    cum = np.concatenate(([0.0], np.cumsum(d)))
    loss, gain = np.where(de < 0, -de, 0.0), np.where(de > 0, de, 0.0)
    kin = 0.5 * sp2[:-1]
    frac = np.divide(loss, kin, out=np.zeros_like(loss), where=kin > 1e-6)
    floor, length = rigorous_floor(p, math.sqrt(sp2[0]), gravity)
    prac, per = practical_floor(p, energy[0], frac, gravity)
    actual = len(d) * TICK
    grav = gravity * (p[0, 2] - p[-1, 2])
    rows = []
    total = cum[-1]
    for k in range(segments):
        lo, hi = k * total / segments, (k + 1) * total / segments
        m = (cum[:-1] >= lo) & (cum[:-1] < hi)
        if not m.any():
            continue
        idx = np.flatnonzero(m)
        n = len(idx)
        rows.append({"segment": k + 1, "actual_s": n * TICK, "perfect_s": float(per[m].sum()),
                     "gain_s": n * TICK - float(per[m].sum()), "ramp_loss": float(loss[m].sum()),
                     "z_drop": float(p[idx[0], 2] - p[idx[-1] + 1, 2]), "mean_speed": float(d[m].sum() / (n * TICK))})
    sens = {int(c * 100): practical_floor(p, energy[0], frac, gravity, c)[0] for c in (0.0, 0.1, 0.2, 0.3, 0.4)}
    out = {"length": float(length), "height_drop": float(p[0, 2] - p[:, 2].min()), "actual_s": actual,
           "mean_speed": float(total / max(actual, 1e-9)), "peak_speed": float(math.sqrt(sp2.max())),
           "rigorous_floor_s": floor, "practical_floor_s": prac, "gravity_supplied": float(grav),
           "strafe_supplied": float(gain.sum()), "strafe_ceiling_frac": float(gain.sum() / (0.5 * MAX_DV2 * len(de))),
           "ramp_destroyed": float(loss.sum()),
           "ramp_destroyed_frac": float(loss.sum() / max(grav + gain.sum(), 1e-9)),
           "segments": rows, "loss_cut_sensitivity_s": sens}
    if target is not None:
        out["target_s"] = float(target)
        out["route_can_host_target"] = bool(floor < target)
        out["line_can_host_target"] = bool(prac < target)
    return out


# ---- batched search -------------------------------------------------------------------------------
def make_scorer(core, zones: Optional[dict], cell: float = 32.0, device: Optional[str] = None) -> Callable:
    """score(states) -> lower is better: geodesic distance to the end zone, or
    minus the track progress when the map has no end zone. The scorer's
    ``finish`` attribute is the score inside the finish zone (None without one)."""
    if zones and zones.get("end"):
        from ..ops.geodesic import bake_goal_field
        if device is None:
            import torch
            device = "cuda" if torch.cuda.is_available() else "cpu"
        gf = bake_goal_field(core, zones["end"], cell=cell, device=device)

        def geo(st):
            return gf.sample(np.asarray(st["origin"], np.float64))
        geo.finish = 200.0
        return geo

    def progress(st):
        return -np.asarray(st["progress"], np.float64)
    progress.finish = None
    return progress


class Brancher:
    """Rolls a batch of candidate action windows, every env starting from the same state."""

    def __init__(self, core, score: Callable):
        self.core, self.score = core, score
        self.n = core.num_envs

    def run(self, state, cands: np.ndarray) -> np.ndarray:
        """cands (n, W, 6) int32 -> scores (n,) at the window end."""
        core, n = self.core, self.n
        for i in range(n):
            core.set_state(i, state)
        alive = np.ones(n, bool)
        fixed = np.full(n, np.nan)
        W = cands.shape[1]
        for t in range(W):
            _, _, done, trunc, _ = core.step(np.ascontiguousarray(cands[:, t, :]))
            ended = alive & ((done != 0) | (trunc != 0))
            if ended.any():
                goal = np.asarray(core.goal_hits, bool)[:n] & ended
                fixed[ended] = np.inf
                fixed[goal] = -1e9 + t
                alive &= ~ended
        sc = self.score(self.core.states_view)
        return np.where(np.isnan(fixed), sc, fixed)

    def final_state(self, state, actions: np.ndarray):
        """Replay one window on env 0 and return its end state."""
        core = self.core
        core.set_state(0, state)
        for t in range(len(actions)):
            core.step(np.ascontiguousarray(np.repeat(actions[t][None], self.n, axis=0)))
        return core.states_view[0].copy()


def _mutate(best: np.ndarray, n: int, p: float, rng) -> np.ndarray:
    cands = np.repeat(best[None], n, axis=0)
    m = rng.random(cands.shape[:2]) < p
    m[0] = False                                   # the incumbent is always re-evaluated
    k = int(m.sum())
    if k:
        flat = cands.reshape(-1, 6)
        idx = np.flatnonzero(m.ravel())
        flat[idx, 0] = rng.integers(0, len(YAW_BINS), k)
        flat[idx, 3] = rng.integers(0, 3, k)
    return cands


def recorded_state(core, row: np.ndarray):
    """A full simulator state carrying a recorded tick's origin, velocity, yaw and ground flag."""
    st = core.get_states()[0].copy()
    st["origin"] = row[1:4]
    st["velocity"] = row[4:7]
    st["yaw"] = row[7]
    st["pitch"] = row[12]
    st["onground"] = 0 if row[9] else -1
    return st


def tas_search(core, score: Callable, ticks: np.ndarray, t0: int, window: int = 300, iters: int = 40,
               p_mutate: float = 0.06, seed: int = 0, log: Optional[Callable] = None) -> dict:
    acts = infer_actions(ticks)
    t1 = min(t0 + window, len(acts))
    W = t1 - t0
    if W < 10:
        raise ValueError("window too short: t0 is at or past the end of the episode")
    br = Brancher(core, score)
    st0 = recorded_state(core, ticks[t0])
    base = acts[t0:t1]
    rec = core.get_states()[:1].copy()
    rec["origin"] = ticks[t1, 1:4]
    rec["progress"] = ticks[t1, 10]
    d_rec = float(score(rec)[0])
    rep = float(br.run(st0, np.repeat(base[None], br.n, axis=0))[0])
    best, best_d = base.copy(), rep
    rng = np.random.default_rng(seed)
    gens = []
    for it in range(iters):
        cands = _mutate(best, br.n, p_mutate, rng)
        d = br.run(st0, cands)
        k = int(np.argmin(d))
        if d[k] < best_d - 1.0:
            best_d, best = float(d[k]), cands[k].copy()
            gens.append((it, best_d))
            if log:
                log(f"gen {it:3d}: {best_d:,.0f} ({d_rec - best_d:+,.0f} vs recorded)")
    return {"t0": t0, "window": W, "candidates": br.n, "recorded": d_rec, "replay": rep,
            "replay_error": abs(rep - d_rec), "best": best_d, "gain": d_rec - best_d, "improvements": gens,
            "actions": best}


def tas_chain(core, score: Callable, ticks: np.ndarray, window: int = 150, iters: int = 25, p_mutate: float = 0.05,
              max_windows: int = 0, seed: int = 0, finish_score: Optional[float] = None,
              log: Optional[Callable] = None) -> dict:
    """``finish_score``: stop once a window ends below it (e.g. 200 units of
    geodesic distance: inside the finish zone)."""
    acts = infer_actions(ticks)
    br = Brancher(core, score)
    cur = recorded_state(core, ticks[0])
    n_win = len(acts) // window
    if max_windows:
        n_win = min(n_win, max_windows)
    rng = np.random.default_rng(seed)
    chained, rows = [], []
    for w in range(n_win):
        lo, hi = w * window, (w + 1) * window
        best, best_d = acts[lo:hi].copy(), None
        for it in range(iters + 1):
            cands = np.repeat(best[None], br.n, axis=0) if it == 0 else _mutate(best, br.n, p_mutate, rng)
            d = br.run(cur, cands)
            k = int(np.argmin(d))
            if best_d is None or d[k] < best_d:
                best_d, best = float(d[k]), cands[k].copy()
        cur = br.final_state(cur, best)
        chained.append(best)
        rec = core.get_states()[:1].copy()
        rec["origin"] = ticks[min(hi, len(ticks) - 1), 1:4]
        rec["progress"] = ticks[min(hi, len(ticks) - 1), 10]
        rows.append({"window": w, "chained": best_d, "recorded": float(score(rec)[0])})
        if log:
            log(f"window {w:3d} [{lo:5d}-{hi:5d}] chained {best_d:12,.1f} recorded {rows[-1]['recorded']:12,.1f}")
        if finish_score is not None and best_d < finish_score:
            break
    return {"windows": rows, "ticks": len(chained) * window,
            "actions": np.concatenate(chained, 0) if chained else np.zeros((0, 6), np.int32)}
