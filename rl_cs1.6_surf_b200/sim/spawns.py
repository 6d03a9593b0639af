"""Spawn pools: the states episodes start from.

Every pool is a ``STATE_DTYPE`` array handed to ``SimCore.set_spawn_pool``;
the env draws a uniform entry at each reset. The rules follow the reference's
pools (python/surfgym/rewards.py:754-995):

* ``map_pool``       the map's own spawn points (info_player_*), airborne;
* ``platform_pool``  game-authentic starts: stand near the edge of the start
                     platform, facing out over a surfable face; kept only if
                     holding +forward from there really reaches 120 u/s
                     (the walk-off lands on a ramp);
* ``scan_faces``     column scan of the map for surfable faces (|n.z| in
                     (0.35, 0.68) under open air);
* ``drop_pool``      exploration starts 400-800u above scanned faces with a
                     random horizontal velocity, yaw and gaze pitch
                     (structural checks only: free hull, no ledge below);
* ``ramp_pool``      on-face starts facing down-slope, kept only if they
                     slide >= 120 u/s with no input within 80 ticks.

Column scans and structural checks run as batched native traces
(``SimCore.trace_batch``); auditions step the native movement code.
"""
from __future__ import annotations

import math
from typing import Optional

import numpy as np

from .core import STATE_DTYPE, PlayerState, SimCore

SURF_NZ = (0.35, 0.68)


def _pool(rows) -> np.ndarray:
    pool = np.zeros(len(rows), STATE_DTYPE)
    for i, r in enumerate(rows):
        pool[i]["origin"] = r[0]
        pool[i]["velocity"] = r[1]
        pool[i]["yaw"] = r[2]
        pool[i]["pitch"] = r[3]
        pool[i]["onground"] = -1
    return pool


def _state(origin, velocity=(0.0, 0.0, 0.0), yaw: float = 0.0) -> PlayerState:
    st = PlayerState()
    for k in range(3):
        st.origin[k] = float(origin[k])
        st.velocity[k] = float(velocity[k])
    st.yaw = float(yaw)
    st.onground = -1
    return st


def map_pool(core: SimCore, yaw=None) -> np.ndarray:
    """The map's spawn points; ``yaw`` overrides their angles (scalar or per point)."""
    sp = core.spawns()
    if not sp:
        raise RuntimeError("map_pool: the map has no spawn points")
    yaws = [y for _, y in sp] if yaw is None else np.broadcast_to(np.asarray(yaw, np.float64), (len(sp),))
    return _pool([(o, (0.0, 0.0, 0.0), float(y), 0.0) for (o, _), y in zip(sp, yaws)])


def platform_pool(core: SimCore, edge_back: float = 35.0, probe_dirs: int = 24, max_walk: float = 700.0,
                  drop_min: float = 100.0, nz_range=SURF_NZ, audition_ticks: int = 300,
                  min_speed: float = 120.0) -> np.ndarray:
    """Edge-of-platform starts facing a ramp, auditioned by walking off."""
    rows = []
    for origin, _ in core.spawns():
        o = np.asarray(origin, np.float64)
        g = core.trace(o, o - [0.0, 0.0, 200.0], hull=0)
        if g.fraction >= 1.0 or g.startsolid:
            continue
        gx, gy, gz = (float(v) for v in g.endpos)
        angs = 2.0 * np.pi * np.arange(probe_dirs) / probe_dirs
        dirs = np.stack([np.cos(angs), np.sin(angs)], 1)
        steps = np.arange(25.0, max_walk + 1e-3, 25.0)
        # walk every direction outward in one batch: the first column whose
        # floor falls away by drop_min is the edge; a solid start is a wall
        pts = np.zeros((probe_dirs, len(steps), 3))
        pts[:, :, 0] = gx + dirs[:, 0:1] * steps
        pts[:, :, 1] = gy + dirs[:, 1:2] * steps
        pts[:, :, 2] = gz + 20.0
        end = pts.copy()
        end[:, :, 2] -= drop_min + 40.0
        tr = core.trace_batch(pts.reshape(-1, 3), end.reshape(-1, 3), hull=0).reshape(probe_dirs, len(steps), 8)
        for di in range(probe_dirs):
            edge = None
            for si in range(len(steps)):
                if tr[di, si, 7]:
                    break
                if tr[di, si, 0] >= 1.0:
                    edge = steps[si]
                    break
            if edge is None:
                continue
            dx, dy = dirs[di]
            q = np.array([gx + dx * (edge + 60.0), gy + dy * (edge + 60.0), gz + 20.0])
            tq = core.trace(q, q - [0.0, 0.0, 900.0], hull=0)
            if tq.fraction >= 1.0 or tq.startsolid or not (nz_range[0] < tq.normal[2] < nz_range[1]):
                continue
            sx, sy = gx + dx * (edge - edge_back), gy + dy * (edge - edge_back)
            ts = core.trace((sx, sy, gz + 30.0), (sx, sy, gz - 60.0), hull=0)
            if ts.fraction >= 1.0 or ts.startsolid or ts.normal[2] < 0.7:
                continue
            yaw = math.degrees(math.atan2(dy, dx)) % 360.0
            st = _state((sx, sy, float(ts.endpos[2])), yaw=yaw)
            peak = 0.0
            for _ in range(audition_ticks):
                core.pm_step_usercmd(st, yaw, 0.0, 400.0, 0.0, 0, 10)
                peak = max(peak, math.hypot(st.velocity[0], st.velocity[1]))
            if peak >= min_speed:
                rows.append(((sx, sy, float(ts.endpos[2])), (0.0, 0.0, 0.0), yaw, 0.0))
    if not rows:
        raise RuntimeError("platform_pool: no edge-facing-ramp start found")
    return _pool(rows)


def scan_faces(core: SimCore, grid: int = 48, nz_range=SURF_NZ, min_drop: float = 80.0,
               step: float = 150.0, probe: float = 600.0):
    """(points [n,3], normals [n,3]): the highest surfable face under each
    column of a grid x grid lattice, with at least ``min_drop`` of air above."""
    mins, maxs = (np.asarray(v, np.float64) for v in core.map_bounds())
    ix = np.arange(1, grid)
    gx, gy = np.meshgrid(mins[0] + (maxs[0] - mins[0]) * (ix + 0.5) / grid,
                         mins[1] + (maxs[1] - mins[1]) * (ix + 0.5) / grid, indexing="ij")
    cx, cy = gx.ravel(), gy.ravel()
    z = np.full(len(cx), maxs[2] - 200.0)
    active = np.ones(len(cx), bool)
    found_p, found_n = [], []
    while active.any():
        idx = np.flatnonzero(active & (z > mins[2] + 200.0))
        active[~(z > mins[2] + 200.0)] = False
        if len(idx) == 0:
            break
        p = np.stack([cx[idx], cy[idx], z[idx]], 1)
        free = core.trace_batch(p, p, hull=0)[:, 7] == 0
        down = p.copy()
        down[:, 2] -= probe
        tr = core.trace_batch(p, down, hull=0)
        hit = free & (tr[:, 0] < 1.0) & (tr[:, 7] == 0)
        surf = hit & (tr[:, 6] > nz_range[0]) & (tr[:, 6] < nz_range[1]) & ((p[:, 2] - tr[:, 3]) > min_drop)
        for j in np.flatnonzero(surf):
            found_p.append(tr[j, 1:4].astype(np.float64))
            found_n.append(tr[j, 4:7].astype(np.float64))
        active[idx[surf]] = False
        skip = hit & ~surf
        z[idx[skip]] = tr[skip, 3]
        z[idx] -= step
    if not found_p:
        raise RuntimeError("scan_faces: no surfable face found")
    return np.array(found_p), np.array(found_n)


def drop_pool(core: SimCore, h_range=(400.0, 800.0), speed_range=(100.0, 400.0), pitch_range=(-45.0, 15.0),
              variants: int = 6, grid: int = 48, nz_range=SURF_NZ, min_drop: float = 80.0, seed: int = 17,
              faces: Optional[tuple] = None) -> np.ndarray:
    """Drops above scanned surfable faces with a random entry state."""
    pts, _ = faces if faces is not None else scan_faces(core, grid, nz_range, min_drop)
    _, maxs = core.map_bounds()
    rng = np.random.default_rng(seed)
    cand = []
    for e in pts:
        for _ in range(variants):
            h = rng.uniform(*h_range)
            spd = rng.uniform(*speed_range)
            ang = rng.uniform(0.0, 2.0 * np.pi)
            yaw = rng.uniform(0.0, 360.0)
            pitch = rng.uniform(*pitch_range)
            oz = min(e[2] + h, maxs[2] - 64.0)
            if oz - e[2] < 0.5 * h_range[0]:
                continue                                   # a ceiling ate the drop
            cand.append(((e[0], e[1], oz), (math.cos(ang) * spd, math.sin(ang) * spd, 0.0), yaw, pitch))
    if not cand:
        raise RuntimeError("drop_pool: no candidate")
    o = np.array([c[0] for c in cand])
    free = core.trace_batch(o, o, hull=0)[:, 7] == 0
    below = o.copy()
    below[:, 2] -= 0.5 * h_range[0]
    clear = core.trace_batch(o, below, hull=0)[:, 0] >= 1.0
    water = np.array([core.point_contents(p) == -3 for p in o])
    keep = free & clear & ~water
    rows = [c for c, k in zip(cand, keep) if k]
    if not rows:
        raise RuntimeError("drop_pool: no candidate survived the structural checks")
    return _pool(rows)


def ramp_pool(core: SimCore, grid: int = 48, nz_range=SURF_NZ, height_above: float = 30.0, min_drop: float = 80.0,
              initial_speed: float = 0.0, audition_ticks: int = 80, min_speed: float = 120.0,
              faces: Optional[tuple] = None) -> np.ndarray:
    """On-face starts facing down-slope that really slide."""
    pts, nrm = faces if faces is not None else scan_faces(core, grid, nz_range, min_drop)
    rows = []
    for e, n in zip(pts, nrm):
        h = math.hypot(n[0], n[1]) or 1.0
        dx, dy = n[0] / h, n[1] / h
        yaw = math.degrees(math.atan2(dy, dx)) % 360.0
        o = (e[0], e[1], e[2] + height_above)
        v = (dx * initial_speed, dy * initial_speed, 0.0)
        st = _state(o, v, yaw)
        for _ in range(audition_ticks):
            core.pm_step_usercmd(st, yaw, 0.0, 0.0, 0.0, 0, 10)
        if math.hypot(st.velocity[0], st.velocity[1]) >= min_speed:
            rows.append((o, v, yaw, 0.0))
    if not rows:
        raise RuntimeError("ramp_pool: no candidate survived the slide audition")
    return _pool(rows)


def mixed_pool(platform: np.ndarray, drops: np.ndarray, drop_frac: float = 0.5) -> np.ndarray:
    """Platform starts replicated so that drops make up ``drop_frac`` of the
    entries (the env draws entries uniformly)."""
    f = float(np.clip(drop_frac, 0.01, 0.99))
    reps = max(1, int(round(len(drops) * (1.0 - f) / (f * max(len(platform), 1)))))
    return np.concatenate([np.concatenate([platform] * reps), drops])
