"""Reward specification, the GPU reward state and the numpy oracle.

``RewardSpec`` holds every knob (reference flags: --reward, --revisit-pen,
--time-pen, --success-bonus, --finish-k/--finish-tref, --fail-pen,
--speed-coef, --speed-equiv, --stall-secs, --int-coef/--int-view/--int-speed;
python/train_fast.py:860-966). ``GpuReward`` owns the per-env device state
and launches ``surf_reward`` once per decision; ``CpuReward`` restates the
same rules in numpy (CPU training and the kernel's oracle).
"""
from __future__ import annotations

import ctypes
import math
from ctypes import c_float, c_int, c_int64, c_uint32, c_void_p
from dataclasses import asdict, dataclass, field
from typing import Optional

import numpy as np
import torch

from ..ops import _lib
from ..ops._lib import check, ptr, stream_ptr

MODES = ("speed", "avgspeed", "forward", "path", "maxspeed", "coverage", "race", "acro", "blend")
DEFAULT_SCALE = {"speed": 0.01, "avgspeed": 0.0005, "forward": 0.01, "path": 0.01, "maxspeed": 0.05,
                 "coverage": 0.001, "race": None, "acro": 0.001, "blend": 0.01}
STATE_FLOATS = 24
REC_O, REC_YAW, REC_V, REC_TICK, REC_BASE, REC_DONE, REC_TRUNC, REC_GOAL, REC_ENDED, REC_ONGROUND = \
    0, 3, 6, 9, 10, 11, 12, 13, 14, 15


@dataclass
class RewardSpec:
    mode: str = "coverage"
    scale: Optional[float] = None          # None: the mode's default (race: 100 / d0)
    max_step: float = 50.0                  # per-tick teleport filter / race delta clip (units)
    revisit_pen: float = 0.25
    cover_cell: float = 512.0
    # race
    time_pen: float = 0.005
    success_bonus: float = 50.0
    finish_k: float = 0.0
    finish_tref: float = 120.0
    fail_pen: float = 0.0
    speed_coef: float = 0.0
    speed_equiv: float = 0.0
    stall_secs: float = 15.0
    stall_eps: float = 32.0
    # acro style (per tick)
    spin_bonus: float = 1.5
    switch_bonus: float = 2.0
    spin_rate_cap: float = 6.0
    max_spins: int = 2
    min_air: int = 30
    back_bonus: float = 0.01
    # blend: forward -> path between these global steps
    blend_start: float = 100e6
    blend_end: float = 200e6
    # curiosity
    int_coef: float = 0.0
    int_cell: float = 256.0
    int_view: int = 0
    int_speed: int = 0
    table_log2: int = 22

    def resolved_scale(self, d0: Optional[float] = None) -> float:
        if self.scale is not None:
            return float(self.scale)
        if self.mode == "race":
            return 100.0 / max(d0 or 1.0, 1.0)
        return DEFAULT_SCALE[self.mode]

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, d) -> "RewardSpec":
        return cls(**{k: v for k, v in d.items() if k in cls.__dataclass_fields__})


class RewardParams(ctypes.Structure):
    _fields_ = [("mode", c_int), ("n", c_int), ("K", c_int), ("scale", c_float), ("max_step", c_float),
                ("revisit_pen", c_float), ("cmin", c_float * 3), ("cell", c_float), ("cdim", c_int * 3),
                ("cov_words", c_int), ("field", c_void_p), ("quant", c_float), ("fmin", c_float * 3),
                ("fcell", c_float), ("valid_max", c_float), ("sentinel", c_float), ("fdim", c_int * 3),
                ("time_pen", c_float), ("success_bonus", c_float), ("finish_k", c_float), ("finish_tref", c_float),
                ("fail_pen", c_float), ("speed_coef", c_float), ("speed_equiv", c_float), ("stall_ticks", c_int),
                ("stall_eps", c_float), ("int_coef", c_float), ("int_cell", c_float), ("int_view", c_int),
                ("int_speed", c_int), ("int_min", c_float * 3), ("int_dim", c_int * 3), ("table_mask", c_uint32),
                ("gamma_boot", c_float), ("spin_bonus", c_float), ("switch_bonus", c_float),
                ("spin_rate_cap", c_float), ("back_bonus", c_float), ("gravity_tick", c_float), ("max_spins", c_int),
                ("min_air", c_int), ("blend_w", c_void_p)]


RLIB = "libsurf_rl.so"
_lib.register(RLIB, {
    "surf_reward_params_size": (c_int, []),
    "surf_reward_state_floats": (c_int, []),
    "surf_reward_init": (c_int, [ctypes.POINTER(RewardParams), c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                                 c_void_p]),
    "surf_reward": (c_int, [ctypes.POINTER(RewardParams), c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                            c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    "surf_reward_counts": (c_int, [ctypes.POINTER(RewardParams), c_void_p, c_void_p, c_void_p, c_void_p]),
    "surf_obs_features": (c_int, [c_void_p, c_int64, c_void_p, c_int, c_int, c_void_p, c_int64, c_int, c_void_p,
                                  c_int, c_void_p]),
    "surf_permutation": (c_int, [c_void_p, c_int64, c_void_p, c_void_p]),
    "surf_permutation_pool": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p]),
})


@dataclass
class GoalFieldData:
    """Geodesic distance-to-goal grid (uint16, value * quant = units)."""
    grid: np.ndarray            # [nz, ny, nx] uint16
    mins: np.ndarray
    cell: float
    quant: float
    reach_max: float

    @property
    def sentinel(self) -> float:
        return self.reach_max + 2.0 * self.cell

    @property
    def valid_max(self) -> float:
        return self.reach_max + 0.5 * self.cell

    def save(self, path) -> None:
        np.savez_compressed(path, grid=self.grid, mins=self.mins, cell=self.cell, quant=self.quant,
                            reach_max=self.reach_max)

    @classmethod
    def load(cls, path) -> "GoalFieldData":
        z = np.load(path)
        return cls(z["grid"], z["mins"].astype(np.float64), float(z["cell"]), float(z["quant"]), float(z["reach_max"]))

    def sample(self, pos: np.ndarray) -> np.ndarray:
        """Honest-corner trilinear sample (numpy), float32."""
        g = (np.atleast_2d(np.asarray(pos, np.float64)) - self.mins) / self.cell - 0.5
        i0 = np.floor(g).astype(np.int64)
        f = (g - i0).astype(np.float32)
        nz, ny, nx = self.grid.shape
        num = np.zeros(len(g), np.float32)
        den = np.zeros(len(g), np.float32)
        for dz in (0, 1):
            for dy in (0, 1):
                for dx in (0, 1):
                    ix = np.clip(i0[:, 0] + dx, 0, nx - 1)
                    iy = np.clip(i0[:, 1] + dy, 0, ny - 1)
                    iz = np.clip(i0[:, 2] + dz, 0, nz - 1)
                    v = self.grid[iz, iy, ix].astype(np.float32) * np.float32(self.quant)
                    w = ((f[:, 0] if dx else 1 - f[:, 0]) * (f[:, 1] if dy else 1 - f[:, 1])
                         * (f[:, 2] if dz else 1 - f[:, 2]) * (v < self.valid_max))
                    num += w * v
                    den += w
        return np.where(den > 1e-6, num / np.maximum(den, 1e-6), self.sentinel).astype(np.float32)


def _cell_dims(mins, maxs, cell):
    return [int(math.ceil((maxs[i] - mins[i]) / cell)) + 1 for i in range(3)]


def build_params(spec: RewardSpec, n: int, K: int, bounds, field: Optional[GoalFieldData] = None,
                 field_ptr: int = 0, d0: Optional[float] = None) -> RewardParams:
    mins, maxs = (np.asarray(b, np.float64) for b in bounds)
    p = RewardParams()
    p.mode = MODES.index(spec.mode)
    p.n, p.K = n, K
    p.scale = spec.resolved_scale(d0)
    p.max_step = spec.max_step
    p.revisit_pen = spec.revisit_pen
    cd = _cell_dims(mins, maxs, spec.cover_cell)
    for a in range(3):
        p.cmin[a] = mins[a]
        p.cdim[a] = cd[a]
    p.cell = spec.cover_cell
    p.cov_words = (cd[0] * cd[1] * cd[2] + 31) // 32
    if field is not None:
        p.field = field_ptr
        p.quant = field.quant
        for a in range(3):
            p.fmin[a] = field.mins[a]
        p.fcell = field.cell
        p.valid_max = field.valid_max
        p.sentinel = field.sentinel
        nz, ny, nx = field.grid.shape
        p.fdim[0], p.fdim[1], p.fdim[2] = nx, ny, nz
    p.time_pen, p.success_bonus = spec.time_pen, spec.success_bonus
    p.finish_k, p.finish_tref, p.fail_pen = spec.finish_k, spec.finish_tref, spec.fail_pen
    p.speed_coef, p.speed_equiv = spec.speed_coef, spec.speed_equiv
    p.stall_ticks = int(round(spec.stall_secs * 100)) if spec.mode == "race" else 0
    p.stall_eps = spec.stall_eps
    p.int_coef, p.int_cell = spec.int_coef, spec.int_cell
    p.int_view, p.int_speed = spec.int_view, spec.int_speed
    idim = _cell_dims(mins, maxs, spec.int_cell)
    for a in range(3):
        p.int_min[a] = mins[a]
        p.int_dim[a] = idim[a]
    p.table_mask = (1 << spec.table_log2) - 1
    p.spin_bonus, p.switch_bonus, p.spin_rate_cap = spec.spin_bonus, spec.switch_bonus, spec.spin_rate_cap
    p.back_bonus, p.max_spins, p.min_air = spec.back_bonus, spec.max_spins, spec.min_air
    p.gravity_tick = 800.0 * 0.01
    return p


def blend_weight(spec: RewardSpec, global_step: float) -> float:
    """Forward -> path curriculum weight (reference BlendedReward.weight)."""
    return min(1.0, max(0.0, (float(global_step) - spec.blend_start) / max(spec.blend_end - spec.blend_start, 1.0)))


class GpuReward:
    """Device-resident reward state for n envs."""

    def __init__(self, spec: RewardSpec, n: int, K: int, bounds, device, field: Optional[GoalFieldData] = None,
                 d0: Optional[float] = None):
        self.spec, self.n, self.K = spec, n, K
        dev = torch.device(device)
        self.field_t = torch.as_tensor(field.grid.astype(np.int16).view(np.int16), device=dev) if field is not None else None
        self.params = build_params(spec, n, K, bounds, field, ptr(self.field_t), d0)
        self.state = torch.zeros(n * STATE_FLOATS, dtype=torch.float32, device=dev)
        self.blend_w = torch.zeros(1, dtype=torch.float32, device=dev)
        self.params.blend_w = ptr(self.blend_w)
        self.keys = torch.zeros(n, dtype=torch.int64, device=dev)
        self.visited = torch.zeros(max(1, n * self.params.cov_words), dtype=torch.int32, device=dev)
        tsize = 1 << spec.table_log2 if spec.int_coef > 0 else 1
        self.counts = torch.zeros(tsize, dtype=torch.int32, device=dev)
        self.delta = torch.zeros(tsize, dtype=torch.int32, device=dev)       # counts added since the last merge
        self.new_key = torch.zeros(n, dtype=torch.int64, device=dev)
        self.stall = torch.zeros(n, dtype=torch.uint8, device=dev)
        self.boot = torch.zeros(n, dtype=torch.float32, device=dev)
        self.stats = torch.zeros(8, dtype=torch.float32, device=dev)
        self.lib = _lib.lib(RLIB)
        if int(self.lib.surf_reward_params_size()) != ctypes.sizeof(RewardParams) or \
                int(self.lib.surf_reward_state_floats()) != STATE_FLOATS:
            raise RuntimeError("libsurf_rl.so reward layout differs from rewards/spec.py (rebuild the library)")
        self._group_params: dict = {}

    def _params(self, lo: int, hi: int) -> RewardParams:
        if (lo, hi) == (0, self.n):
            return self.params
        key = (lo, hi)
        if key not in self._group_params:
            p = RewardParams()
            ctypes.memmove(ctypes.byref(p), ctypes.byref(self.params), ctypes.sizeof(RewardParams))
            p.n = hi - lo
            self._group_params[key] = p
        return self._group_params[key]

    def _ptrs(self, lo: int):
        w = self.params.cov_words
        return (ptr(self.state) + 4 * STATE_FLOATS * lo, ptr(self.visited) + 4 * w * lo if w else ptr(self.visited),
                ptr(self.boot) + 4 * lo, ptr(self.stall) + lo, ptr(self.new_key) + 8 * lo, ptr(self.keys) + 8 * lo)

    def set_step(self, global_step: float) -> None:
        """Schedules that live in device memory (the blend weight)."""
        if self.spec.mode == "blend":
            self.blend_w.fill_(blend_weight(self.spec, global_step))

    def init(self, rec: torch.Tensor, lo: int = 0, hi: Optional[int] = None) -> None:
        """Per-env state from the spawn records; ``rec`` holds rows lo..hi."""
        hi = self.n if hi is None else hi
        st, vis, _, _, _, keys = self._ptrs(lo)
        check(self.lib.surf_reward_init(ctypes.byref(self._params(lo, hi)), ptr(rec), rec.stride(0), st, vis, keys,
                                        stream_ptr(rec.device)), "surf_reward_init")

    def __call__(self, rec: torch.Tensor, rew_out: torch.Tensor, done_out: torch.Tensor, lo: int = 0,
                 hi: Optional[int] = None, counts: bool = True) -> None:
        """Rewards of envs lo..hi (``rec``, ``rew_out``, ``done_out`` hold those
        rows). With ``counts=False`` the curiosity increments are only staged;
        ``count_all`` applies them for every env (env groups call it once per
        decision after the last group, so every bonus of a decision reads the
        counts from before it)."""
        hi = self.n if hi is None else hi
        st, vis, boot, stall, nk, keys = self._ptrs(lo)
        check(self.lib.surf_reward(ctypes.byref(self._params(lo, hi)), ptr(rec), rec.stride(0), st, vis,
                                   ptr(self.counts), ptr(self.delta), boot, ptr(rew_out), ptr(done_out), stall, nk,
                                   keys, ptr(self.stats), 1 if counts else 0, stream_ptr(rec.device)),
              "surf_reward" if counts and self.spec.int_coef > 0 else "surf_reward_phase1")

    def count_all(self) -> None:
        if self.spec.int_coef > 0:
            check(self.lib.surf_reward_counts(ctypes.byref(self.params), ptr(self.new_key), ptr(self.counts),
                                              ptr(self.delta), stream_ptr(self.counts.device)), "surf_reward_counts")

    def pop_stats(self) -> dict:
        s = self.stats.tolist()
        self.stats.zero_()
        return _stats_dict(s)


def _stats_dict(s) -> dict:
    eps = s[0]
    return {"episodes": int(eps), "ep_rew_mean": s[1] / eps if eps else float("nan"),
            "ep_len_mean": s[2] / eps if eps else float("nan"), "success_rate": s[3] / eps if eps else float("nan"),
            "fail_rate": s[4] / eps if eps else float("nan"), "int_paid": s[6], "reward_sum": s[7]}


def _bucket(keys: np.ndarray, mask: int) -> np.ndarray:
    """SplitMix64 finaliser as the table hash (matches the kernel)."""
    with np.errstate(over="ignore"):
        z = keys.astype(np.uint64) + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return (z.astype(np.uint32) & np.uint32(mask)).astype(np.int64)


class CpuReward:
    """numpy restatement of surf_reward (same per-decision rules)."""

    def __init__(self, spec: RewardSpec, n: int, K: int, bounds, field: Optional[GoalFieldData] = None,
                 d0: Optional[float] = None):
        self.spec, self.n, self.K = spec, n, K
        self.p = build_params(spec, n, K, bounds, field, 0, d0)
        self.field = field
        self.mode = spec.mode
        ncell = int(np.prod(list(self.p.cdim)))
        self.visited = np.zeros((n, ncell), bool)
        self.counts = np.zeros(1 << spec.table_log2 if spec.int_coef > 0 else 1, np.int64)
        self.stats = np.zeros(8, np.float64)
        self.step = 0.0

    def set_step(self, global_step: float) -> None:
        self.step = float(global_step)

    def _cov_cell(self, pos):
        c = [np.clip(np.floor((pos[:, a] - self.p.cmin[a]) / self.p.cell).astype(np.int64), 0, self.p.cdim[a] - 1)
             for a in range(3)]
        return c[0] + self.p.cdim[0] * (c[1] + self.p.cdim[1] * c[2])

    def _key(self, rec):
        p = self.p
        c = [np.clip(np.floor((rec[:, a] - p.int_min[a]) / p.int_cell).astype(np.int64), 0, p.int_dim[a] - 1)
             for a in range(3)]
        key = c[0] + p.int_dim[0] * (c[1] + p.int_dim[1] * c[2])
        if p.int_view > 0:
            y = np.mod(rec[:, REC_YAW], 360.0)
            yb = np.clip(np.floor(y / 360.0 * p.int_view).astype(np.int64), 0, p.int_view - 1)
            key = key * p.int_view + yb
        if p.int_speed > 0:
            sp = np.hypot(rec[:, REC_V], rec[:, REC_V + 1])
            sb = np.clip((sp / (4000.0 / p.int_speed)).astype(np.int64), 0, p.int_speed - 1)
            key = key * p.int_speed + sb
        return key

    def init(self, rec: np.ndarray) -> None:
        n = self.n
        self.pos = rec[:, 0:3].astype(np.float32).copy()
        self.speed = np.hypot(rec[:, REC_V], rec[:, REC_V + 1]).astype(np.float32)
        self.best = self.speed.copy()
        yaw = np.radians(rec[:, REC_YAW])
        self.dir = np.stack([np.cos(yaw), np.sin(yaw)], 1).astype(np.float32)
        self.ref = rec[:, 0:2].astype(np.float32).copy()
        self.since = np.zeros(n, np.float32)
        self.ticks = np.zeros(n, np.float32)
        self.ep_ret = np.zeros(n, np.float32)
        self.ep_len = np.zeros(n, np.float32)
        if self.mode == "race":
            self.d = self.field.sample(rec[:, 0:3])
            self.best = self.d.copy()
        if self.mode in ("forward", "blend"):
            self.best[:] = 0.0
        self.yaw = rec[:, REC_YAW].astype(np.float32).copy()
        self.vel = rec[:, REC_V:REC_V + 3].astype(np.float32).copy()
        self.streak = np.zeros(n, np.float32)
        self.spin = np.zeros(n, np.float32)
        self.cell = self._cov_cell(rec[:, 0:3])
        self.visited[:] = False
        self.visited[np.arange(n), self.cell] = True
        self.key = self._key(rec) if self.spec.int_coef > 0 else None

    def __call__(self, rec: np.ndarray, boot: Optional[np.ndarray] = None):
        p, n = self.p, self.n
        ended = rec[:, REC_ENDED] != 0
        done = rec[:, REC_DONE] != 0
        goal = rec[:, REC_GOAL] != 0
        sp = np.hypot(rec[:, REC_V], rec[:, REC_V + 1]).astype(np.float32)
        dxy = rec[:, 0:2] - self.pos[:, 0:2]
        hstep = np.hypot(dxy[:, 0], dxy[:, 1]).astype(np.float32)
        tele = hstep > p.max_step * p.K
        m = self.mode
        if m == "speed":
            r = (sp - self.speed) * p.scale
        elif m == "avgspeed":
            r = sp * p.scale
        elif m == "path":
            r = np.where(tele, 0.0, hstep * p.scale)
        elif m == "maxspeed":
            r = np.maximum(sp - self.best, 0) * p.scale
            self.best = np.maximum(self.best, sp)
        elif m == "forward":
            self.ref[tele] += dxy[tele]
            proj = (rec[:, 0] - self.ref[:, 0]) * self.dir[:, 0] + (rec[:, 1] - self.ref[:, 1]) * self.dir[:, 1]
            r = np.maximum(proj - self.best, 0) * p.scale
            self.best = np.maximum(self.best, proj)
        elif m == "blend":
            self.ref[tele] += dxy[tele]
            proj = (rec[:, 0] - self.ref[:, 0]) * self.dir[:, 0] + (rec[:, 1] - self.ref[:, 1]) * self.dir[:, 1]
            fwd = np.maximum(proj - self.best, 0) * p.scale
            self.best = np.maximum(self.best, proj)
            path = np.where(tele, 0.0, hstep * p.scale)
            w = blend_weight(self.spec, self.step)
            r = (1.0 - w) * fwd + w * path
        elif m in ("coverage", "acro"):
            c = self._cov_cell(rec[:, 0:3])
            moved = c != self.cell
            seen = self.visited[np.arange(n), c]
            r = np.where(moved, np.where(seen, -p.revisit_pen, sp * p.scale), 0.0)
            self.visited[np.arange(n), c] = True
            self.cell = c
        else:  # race
            d = self.field.sample(rec[:, 0:3])
            clip = p.max_step * p.K
            delta = np.clip(self.d - d, -clip, clip)
            r = delta * p.scale - p.time_pen * p.K
            if p.speed_coef > 0:
                r = r + p.speed_coef / 1000.0 * sp
            if p.speed_equiv > 0:
                r = r + p.scale * p.speed_equiv * (sp - self.speed)
            r = np.where(ended, 0.0, r)
            r = r + np.where(goal, p.success_bonus, 0.0)
            if p.finish_k > 0:
                r = r + np.where(goal, p.finish_k * np.maximum(0.0, p.finish_tref - (self.ticks + p.K) / 100.0), 0.0)
            dead = done & ~goal
            r = r - np.where(dead, p.fail_pen, 0.0)
            if p.speed_equiv > 0:
                r = r - np.where(dead, p.scale * p.speed_equiv * self.speed, 0.0)
            self.ticks += p.K
            improved = d < self.best - p.stall_eps
            self.best = np.minimum(self.best, d)
            self.since = np.where(improved, 0.0, self.since + p.K)
            self.d = d
        r = r.astype(np.float32)
        if m == "acro":
            K = float(p.K)
            v = rec[:, REC_V:REC_V + 3].astype(np.float32)
            dv = v - self.vel
            contact = (np.abs(dv[:, 0]) + np.abs(dv[:, 1]) > 40.0 * K) | (np.abs(dv[:, 2] + p.gravity_tick * K) > 12.0 * K)
            grounded = rec[:, REC_ONGROUND] != 0
            ballistic = ~grounded & ~contact
            wrap = lambda a: np.mod(a + 180.0, 360.0) - 180.0
            dyaw = np.abs(wrap(rec[:, REC_YAW] - self.yaw))
            flight_end = (self.streak * K >= p.min_air) & (contact | grounded)
            style = np.where(flight_end, p.spin_bonus * np.minimum(self.spin, 360.0 * p.max_spins) / 360.0, 0.0)
            heading = np.degrees(np.arctan2(v[:, 1], v[:, 0]))
            back = np.abs(wrap(rec[:, REC_YAW] - heading)) >= 140.0
            style += np.where(flight_end & (sp >= 300.0) & back, p.switch_bonus, 0.0)
            style += np.where(~grounded & contact & (sp >= 500.0) & back, p.back_bonus * K, 0.0)
            self.spin = np.where(ballistic, self.spin + np.where(self.streak > 0, np.minimum(dyaw, p.spin_rate_cap * K), 0),
                                 0.0).astype(np.float32)
            self.streak = np.where(ballistic, self.streak + 1, 0).astype(np.float32)
            r = (r + np.where(ended, 0.0, style)).astype(np.float32)
            self.spin[ended] = 0
            self.streak[ended] = 0
        self.yaw = rec[:, REC_YAW].astype(np.float32).copy()
        self.vel = rec[:, REC_V:REC_V + 3].astype(np.float32).copy()
        if m != "race":
            r[ended] = 0.0
        if self.spec.int_coef > 0:
            key = self._key(rec)
            mv = (key != self.key) & ~ended
            b = _bucket(key, p.table_mask)
            bonus = np.where(mv, p.int_coef / np.sqrt(self.counts[b] + 1.0), 0.0).astype(np.float32)
            r += bonus
            np.add.at(self.counts, b[mv], 1)
            self.key = key
            self.stats[6] += bonus.sum()
        if boot is not None:
            r += boot
        r += rec[:, REC_BASE]
        self.ep_ret += r
        self.ep_len += p.K
        e = np.flatnonzero(ended)
        if len(e):
            self.stats[0] += len(e)
            self.stats[1] += self.ep_ret[e].sum()
            self.stats[2] += self.ep_len[e].sum()
            self.stats[3] += goal[e].sum()
            self.stats[4] += (done & ~goal)[e].sum()
            self.stats[5] += (~done)[e].sum()
            self.ep_ret[e] = 0
            self.ep_len[e] = 0
            self.best[e] = sp[e]
            yaw = np.radians(rec[e, REC_YAW])
            self.dir[e] = np.stack([np.cos(yaw), np.sin(yaw)], 1)
            self.ref[e] = rec[e, 0:2]
            if m in ("forward", "blend"):
                self.best[e] = 0.0
            if m == "race":
                self.best[e] = self.d[e]
                self.since[e] = 0
                self.ticks[e] = 0
            if m in ("coverage", "acro"):
                self.visited[e] = False
                c = self._cov_cell(rec[e, 0:3])
                self.visited[e, c] = True
                self.cell[e] = c
        stall = None
        if m == "race" and p.stall_ticks > 0:
            stall = self.since >= p.stall_ticks
            self.since[stall] = 0
        self.stats[7] += r.sum()
        self.pos = rec[:, 0:3].astype(np.float32).copy()
        self.speed = sp
        return r, ended.astype(np.float32), stall

    def pop_stats(self) -> dict:
        s = self.stats.tolist()
        self.stats[:] = 0
        return _stats_dict(s)
