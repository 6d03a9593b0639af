"""Python binding of the C++ simulator (``libsurfsim.so``).

API parity with the reference binding ``SurfCore`` (python/surfgym/core.py:
458-878): construction from a BSP path, ``reset``/``step`` with same-step
autoreset and terminal observations, a zero-copy structured view of the
per-env states, traces, point contents, occupancy grids, single-player
usercmd stepping, spawn pools, goal box, force-fail and map queries. Extras:

* ``SimCore.from_bytes`` loads a BSP image from memory (procedural maps),
* ``step_k`` runs K ticks of action repeat in one native call and writes the
  observation, terminal observation and per-env record rows into caller
  buffers (typically one pinned host tensor shipped to the GPU by one copy),
* a continuous yaw action may replace the yaw bin.

Every call into the library releases the GIL (ctypes foreign calls do).
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int32, c_int64, c_uint8, c_uint64, c_void_p
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Optional, Union

import numpy as np

from .._native import load

ACTION_DIM = 6
OBS_FIXED = 15
NVEC = (15, 7, 3, 3, 2, 2)            # yaw bin, pitch bin, fwd, side, jump, duck
IN_JUMP, IN_DUCK = 2, 4
CONTENTS_EMPTY, CONTENTS_SOLID, CONTENTS_WATER = -1, -2, -3

# Record columns written by step_k (csrc/sim/env.hpp RecCol / TermCol).
REC = dict(origin=slice(0, 3), yaw=3, pitch=4, ducked=5, vel=slice(6, 9), tick=9, reward=10,
           done=11, trunc=12, goal=13, ended=14, onground=15)
REC_COLS = 16
TERM = dict(origin=slice(0, 3), yaw=3, pitch=4, ducked=5, tick=6)
TERM_COLS = 8


class Physics(ctypes.Structure):
    _fields_ = [("sv_gravity", c_float), ("sv_airaccelerate", c_float), ("sv_accelerate", c_float),
                ("sv_friction", c_float), ("edgefriction", c_float), ("sv_stopspeed", c_float),
                ("sv_maxspeed", c_float), ("player_maxspeed", c_float), ("sv_maxvelocity", c_float),
                ("sv_stepsize", c_float), ("sv_bounce", c_float), ("msec", c_int32),
                ("enable_stamina", c_int32), ("enable_bhop_cap", c_int32), ("enable_duck", c_int32)]


class EnvConfig(ctypes.Structure):
    _fields_ = [("num_envs", c_int32), ("max_episode_ticks", c_int32), ("lookahead_k", c_int32),
                ("lookahead_dt", c_float), ("spawn_mode", c_int32), ("spawn_curriculum_frac", c_float),
                ("yaw_rate_max_deg", c_float), ("yaw_jitter_deg", c_float), ("kill_z", c_float),
                ("water_fail", c_int32), ("pitch_rate_max_deg", c_float), ("lidar_w", c_int32),
                ("lidar_h", c_int32), ("lidar_hfov_deg", c_float), ("lidar_vfov_deg", c_float),
                ("lidar_range", c_float), ("phys", Physics), ("yaw_adaptive", c_int32)]


class PlayerState(ctypes.Structure):
    _fields_ = [("origin", c_float * 3), ("velocity", c_float * 3), ("basevelocity", c_float * 3),
                ("yaw", c_float), ("pitch", c_float), ("fuser2", c_float), ("base_vel_flag", c_int32),
                ("onground", c_int32), ("oldbuttons", c_int32), ("ducked", c_int32), ("tick", c_int32),
                ("seg_hint", c_int32), ("progress", c_float), ("best_progress", c_float),
                ("stuck_ticks", c_int32), ("induck", c_int32), ("duck_time", c_float),
                ("waterjumptime", c_float), ("movedir", c_float * 3)]


class TraceOut(ctypes.Structure):
    _fields_ = [("endpos", c_float * 3), ("normal", c_float * 3), ("dist", c_float), ("fraction", c_float),
                ("startsolid", c_int32), ("allsolid", c_int32), ("ent", c_int32)]


# numpy view of PlayerState (byte-compatible with the reference STATE_DTYPE).
STATE_DTYPE = np.dtype([
    ("origin", np.float32, (3,)), ("velocity", np.float32, (3,)), ("basevelocity", np.float32, (3,)),
    ("yaw", np.float32), ("pitch", np.float32), ("fuser2", np.float32), ("base_vel_flag", np.int32),
    ("onground", np.int32), ("oldbuttons", np.int32), ("ducked", np.int32), ("tick", np.int32),
    ("seg_hint", np.int32), ("progress", np.float32), ("best_progress", np.float32),
    ("stuck_ticks", np.int32), ("induck", np.int32), ("duck_time", np.float32),
    ("waterjumptime", np.float32), ("movedir", np.float32, (3,)),
])
assert STATE_DTYPE.itemsize == ctypes.sizeof(PlayerState) == 108
assert ctypes.sizeof(EnvConfig) == 128 and ctypes.sizeof(Physics) == 60

PHYS_DEFAULTS = {
    "sv_gravity": 800.0, "sv_airaccelerate": 100.0, "sv_accelerate": 5.0, "sv_friction": 4.0,
    "edgefriction": 2.0, "sv_stopspeed": 75.0, "sv_maxspeed": 320.0, "player_maxspeed": 250.0,
    "sv_maxvelocity": 2000.0, "sv_stepsize": 18.0, "sv_bounce": 1.0, "msec": 10,
    "enable_stamina": 1, "enable_bhop_cap": 1, "enable_duck": 1,
}
ENV_DEFAULTS = {
    "max_episode_ticks": 6000, "lookahead_k": 8, "lookahead_dt": 0.25, "spawn_mode": 1,
    "spawn_curriculum_frac": 0.99, "yaw_rate_max_deg": 10.0, "yaw_adaptive": 0, "yaw_jitter_deg": 5.0,
    "kill_z": -1e38, "water_fail": 1, "pitch_rate_max_deg": 10.0, "lidar_w": 0, "lidar_h": 0,
    "lidar_hfov_deg": 120.0, "lidar_vfov_deg": 90.0, "lidar_range": 2000.0,
}


def default_config(num_envs: int = 1, **overrides: Any) -> EnvConfig:
    """EnvConfig with documented defaults; ``overrides`` take any EnvConfig or
    Physics field by name (unknown keys raise TypeError). The reference's
    defaults (python/surfgym/core.py:209-244) except that the CPU lidar is off
    by default: depth vision is rendered on the GPU."""
    if num_envs < 1:
        raise ValueError(f"num_envs must be >= 1, got {num_envs}")
    env = dict(ENV_DEFAULTS)
    phys = dict(PHYS_DEFAULTS)
    for k, v in overrides.items():
        if k in env:
            env[k] = v
        elif k in phys:
            phys[k] = v
        else:
            raise TypeError(f"unknown config field {k!r}; valid: {sorted(env) + sorted(phys)}")
    cfg = EnvConfig()
    cfg.num_envs = int(num_envs)
    for name, ctype in EnvConfig._fields_:
        if name in env:
            setattr(cfg, name, int(env[name]) if ctype is c_int32 else float(env[name]))
    for name, ctype in Physics._fields_:
        setattr(cfg.phys, name, int(phys[name]) if ctype is c_int32 else float(phys[name]))
    return cfg


def config_to_dict(cfg: EnvConfig) -> dict:
    out = {}
    for name, ctype in EnvConfig._fields_:
        if name == "phys":
            out[name] = {n: (int(getattr(cfg.phys, n)) if t is c_int32 else float(getattr(cfg.phys, n)))
                         for n, t in Physics._fields_}
        else:
            out[name] = int(getattr(cfg, name)) if ctype is c_int32 else float(getattr(cfg, name))
    return out


def config_from_dict(d: dict) -> EnvConfig:
    flat = {k: v for k, v in d.items() if k not in ("phys", "num_envs")}
    flat.update(d.get("phys", {}))
    return default_config(int(d.get("num_envs", 1)), **flat)


def validate_actions(actions: np.ndarray, num_envs: int) -> None:
    """Actions must be a C-contiguous int32 ndarray of shape (num_envs, 6)."""
    if not isinstance(actions, np.ndarray):
        raise TypeError(f"actions must be a numpy ndarray, got {type(actions).__name__}")
    if actions.dtype != np.int32:
        raise ValueError(f"actions dtype must be int32, got {actions.dtype}")
    if actions.shape != (num_envs, ACTION_DIM):
        raise ValueError(f"actions shape must be ({num_envs}, {ACTION_DIM}), got {actions.shape}")
    if not actions.flags["C_CONTIGUOUS"]:
        raise ValueError("actions must be C-contiguous")


_P_F = POINTER(c_float)
_P_I = POINTER(c_int32)
_P_U8 = POINTER(c_uint8)


def _bind(lib: ctypes.CDLL) -> ctypes.CDLL:
    if getattr(lib, "_surf_bound", False):
        return lib
    sig = {
        "surfsim_abi_version": (c_int32, []),
        "surfsim_create": (c_void_p, [c_char_p, POINTER(EnvConfig), c_int32, c_char_p, c_int32]),
        "surfsim_create_from_memory": (c_void_p, [c_void_p, c_int64, POINTER(EnvConfig), c_int32, c_char_p, c_int32]),
        "surfsim_destroy": (None, [c_void_p]),
        "surfsim_obs_dim": (c_int32, [c_void_p]),
        "surfsim_num_envs": (c_int32, [c_void_p]),
        "surfsim_set_waypoints": (c_int32, [c_void_p, _P_F, c_int32]),
        "surfsim_set_spawn_pool": (c_int32, [c_void_p, c_void_p, c_int32]),
        "surfsim_set_teleport_fail": (None, [c_void_p, c_int32]),
        "surfsim_set_goal_box": (None, [c_void_p, _P_F, _P_F]),
        "surfsim_goal_hits": (_P_U8, [c_void_p]),
        "surfsim_force_fail": (None, [c_void_p, _P_U8]),
        "surfsim_reset_all": (None, [c_void_p, c_uint64, _P_F]),
        "surfsim_step": (None, [c_void_p, _P_I, _P_F, _P_F, _P_U8, _P_U8, _P_F]),
        "surfsim_step_k": (None, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32,
                                  c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64]),
        "surfsim_step_k_range": (None, [c_void_p, c_int32, c_int32, c_void_p, c_int32, c_int32, c_int32, c_int32,
                                        c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64]),
        "surfsim_step_k_range_async": (None, [c_void_p, c_int32, c_int32, c_void_p, c_int32, c_int32, c_int32,
                                              c_int32, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64,
                                              c_void_p, c_int64]),
        "surfsim_step_wait": (None, [c_void_p]),
        "surfsim_env_order": (None, [c_void_p, c_int32, c_int32, c_void_p]),
        "surfsim_states_ptr": (c_void_p, [c_void_p]),
        "surfsim_get_states": (None, [c_void_p, c_void_p]),
        "surfsim_set_state": (None, [c_void_p, c_int32, c_void_p]),
        "surfsim_trace": (None, [c_void_p, _P_F, _P_F, c_int32, POINTER(TraceOut)]),
        "surfsim_trace_batch": (None, [c_void_p, c_void_p, c_int64, c_int32, c_void_p]),
        "surfsim_point_contents": (c_int32, [c_void_p, _P_F]),
        "surfsim_occupancy_grid": (None, [c_void_p, _P_F, c_float, c_int32, c_int32, c_int32, c_void_p]),
        "surfsim_pm_step_usercmd": (None, [c_void_p, c_void_p, c_float, c_float, c_float, c_float, c_int32, c_int32]),
        "surfsim_play_step": (c_int32, [c_void_p, c_void_p, c_float, c_float, c_float, c_float, c_int32, c_int32]),
        "surfsim_pm_step_single": (None, [c_void_p, c_void_p, _P_I]),
        "surfsim_num_spawns": (c_int32, [c_void_p]),
        "surfsim_get_spawn": (None, [c_void_p, c_int32, _P_F, _P_F]),
        "surfsim_map_bounds": (None, [c_void_p, _P_F, _P_F]),
        "surfsim_map_counts": (None, [c_void_p, _P_I]),
        "surfsim_export_hull0": (None, [c_void_p, c_void_p, c_void_p, c_void_p, _P_I]),
        "surfsim_export_mesh": (c_int32, [c_void_p, c_void_p, c_int32, c_void_p, c_int32, _P_I]),
        "surfsim_geodesic": (c_int64, [c_void_p, c_int32, c_int32, c_int32, c_float, c_void_p, c_void_p, c_void_p]),
        "surfsim_core_bytes": (c_int32, [c_void_p, c_void_p, c_int32]),
        "surfsim_solid_entities": (c_int32, [c_void_p, c_void_p, c_int32]),
        "surfsim_triggers": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_int32]),
        "surfsim_trigger_contains": (None, [c_void_p, c_int32, c_void_p, c_int64, c_int32, c_void_p]),
        "surfsim_compile_bsp": (c_int64, [c_void_p, c_int64, c_char_p, c_void_p, c_int64, c_char_p, c_int32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    lib._surf_bound = True
    return lib


def simlib() -> ctypes.CDLL:
    return _bind(load("libsurfsim.so"))


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(_P_F)


def _vec3(v) -> ctypes.Array:
    a = np.ascontiguousarray(np.asarray(v, np.float32).reshape(3))
    return (c_float * 3)(*a.tolist())


@dataclass
class TraceResult:
    endpos: np.ndarray
    normal: np.ndarray
    dist: float
    fraction: float
    startsolid: bool
    allsolid: bool
    ent: int


def default_threads() -> int:
    """Env worker threads: this process's share of the CPUs it may use (the
    node's ranks, LOCAL_WORLD_SIZE, split them evenly, unless the rank is
    already pinned to its share), capped at 64
    (overridable via SURF_THREADS). The calling (Python/GPU-driving) thread is
    one of them: it steps the first chunk of envs itself, and the GPU work of
    the other env group was launched before the step."""
    env = os.environ.get("SURF_THREADS")
    if env:
        return max(1, int(env))
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:   # pragma: no cover
        n = os.cpu_count() or 4
    # a rank pinned to its own CPU share (parallel.dist.pin_rank_cpus) uses all of it
    local = 1 if os.environ.get("SURF_CPUS_PINNED") == "1" else max(1, int(os.environ.get("LOCAL_WORLD_SIZE", "1")))
    return max(1, min(64, n // local))


class SimCore:
    """A batch of ``cfg.num_envs`` surf environments on one map."""

    def __init__(self, bsp: Union[str, os.PathLike, bytes], cfg: Optional[EnvConfig] = None,
                 threads: Optional[int] = None, **overrides: Any) -> None:
        self.lib = simlib()
        if cfg is None:
            cfg = default_config(**overrides)
        elif overrides:
            raise TypeError("pass either cfg or overrides, not both")
        self.cfg = cfg
        self.threads = int(threads or default_threads())
        err = ctypes.create_string_buffer(512)
        if isinstance(bsp, (bytes, bytearray)):
            self._image = bytes(bsp)
            self.bsp_path = None
            buf = ctypes.create_string_buffer(self._image, len(self._image))
            h = self.lib.surfsim_create_from_memory(ctypes.cast(buf, c_void_p), len(self._image),
                                                    ctypes.byref(cfg), self.threads, err, 512)
        else:
            self.bsp_path = str(bsp)
            self._image = None
            h = self.lib.surfsim_create(self.bsp_path.encode(), ctypes.byref(cfg), self.threads, err, 512)
        if not h:
            raise RuntimeError(f"surfsim_create failed: {err.value.decode(errors='replace')}")
        self._h = c_void_p(h)
        self.num_envs = int(self.lib.surfsim_num_envs(self._h))
        self.obs_dim = int(self.lib.surfsim_obs_dim(self._h))
        n, d = self.num_envs, self.obs_dim
        self._obs = np.zeros((n, d), np.float32)
        self._term = np.zeros((n, d), np.float32)
        self._rew = np.zeros(n, np.float32)
        self._done = np.zeros(n, np.uint8)
        self._trunc = np.zeros(n, np.uint8)
        ptr = self.lib.surfsim_states_ptr(self._h)
        self.states_view = np.ctypeslib.as_array((ctypes.c_uint8 * (n * STATE_DTYPE.itemsize)).from_address(ptr)) \
            .view(STATE_DTYPE)
        gp = self.lib.surfsim_goal_hits(self._h)
        self.goal_hits = np.ctypeslib.as_array(gp, shape=(n,))

    @classmethod
    def from_bytes(cls, image: bytes, cfg: Optional[EnvConfig] = None, threads: Optional[int] = None,
                   **overrides: Any) -> "SimCore":
        return cls(image, cfg, threads, **overrides)

    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.surfsim_destroy(self._h)
            self._h = None

    def __del__(self):   # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    # ---- episode control ----------------------------------------------------
    def reset(self, seed: int = 0) -> np.ndarray:
        self.lib.surfsim_reset_all(self._h, c_uint64(int(seed) & (2 ** 64 - 1)), _fptr(self._obs))
        return self._obs

    def step(self, actions: np.ndarray):
        """One tick for every env. Returns internal buffers (overwritten next call):
        obs, rewards, done (uint8), trunc (uint8), terminal_obs."""
        validate_actions(actions, self.num_envs)
        self.lib.surfsim_step(self._h, actions.ctypes.data_as(_P_I), _fptr(self._obs), _fptr(self._rew),
                              self._done.ctypes.data_as(_P_U8), self._trunc.ctypes.data_as(_P_U8), _fptr(self._term))
        return self._obs, self._rew, self._done, self._trunc, self._term

    def step_k(self, actions_ptr: int, action_stride: int, k: int, *, yaw_slot: int = -1, fail_slot: int = -1,
               obs: tuple = (0, 0), term_obs: tuple = (0, 0), rec: tuple = (0, 0), term_rec: tuple = (0, 0)) -> None:
        """K ticks of action repeat over raw host pointers (int addresses, e.g.
        ``tensor.data_ptr()`` of pinned tensors). Action rows are int32 of
        ``action_stride``; ``yaw_slot`` names a slot holding a continuous yaw
        (float bits in [-1, 1]) and ``fail_slot`` one holding a force-fail
        flag (-1 = unused). ``obs``/``term_obs``/``rec``/``term_rec`` are
        (pointer, row stride in floats) pairs; 0 skips one."""
        self.lib.surfsim_step_k(self._h, c_void_p(actions_ptr), int(action_stride), int(yaw_slot), int(fail_slot),
                                int(k),
                                c_void_p(obs[0] or None), int(obs[1]), c_void_p(term_obs[0] or None), int(term_obs[1]),
                                c_void_p(rec[0] or None), int(rec[1]), c_void_p(term_rec[0] or None), int(term_rec[1]))

    def step_k_range(self, lo: int, hi: int, actions_ptr: int, action_stride: int, k: int, *, yaw_slot: int = -1,
                     fail_slot: int = -1, obs: tuple = (0, 0), term_obs: tuple = (0, 0), rec: tuple = (0, 0),
                     term_rec: tuple = (0, 0)) -> None:
        """``step_k`` over envs [lo, hi) only; pointers index the whole batch."""
        self.lib.surfsim_step_k_range(self._h, int(lo), int(hi), c_void_p(actions_ptr), int(action_stride),
                                      int(yaw_slot), int(fail_slot), int(k),
                                      c_void_p(obs[0] or None), int(obs[1]), c_void_p(term_obs[0] or None),
                                      int(term_obs[1]), c_void_p(rec[0] or None), int(rec[1]),
                                      c_void_p(term_rec[0] or None), int(term_rec[1]))

    def step_k_range_async(self, lo: int, hi: int, actions_ptr: int, action_stride: int, k: int, *,
                           yaw_slot: int = -1, fail_slot: int = -1, obs: tuple = (0, 0), term_obs: tuple = (0, 0),
                           rec: tuple = (0, 0), term_rec: tuple = (0, 0)) -> None:
        """``step_k_range`` on the simulator's worker threads: returns at once,
        ``step_wait`` joins the work (the calling thread steps envs too) and
        returns when it is done. Until then the action rows and output rows of
        envs [lo, hi) belong to the simulator; every other call waits first."""
        self.lib.surfsim_step_k_range_async(self._h, int(lo), int(hi), c_void_p(actions_ptr), int(action_stride),
                                            int(yaw_slot), int(fail_slot), int(k),
                                            c_void_p(obs[0] or None), int(obs[1]), c_void_p(term_obs[0] or None),
                                            int(term_obs[1]), c_void_p(rec[0] or None), int(rec[1]),
                                            c_void_p(term_rec[0] or None), int(term_rec[1]))

    def step_wait(self) -> None:
        self.lib.surfsim_step_wait(self._h)

    def env_order(self, lo: int, hi: int, out_ptr: int) -> None:
        """Write the order the last step of envs [lo, hi) visited them in
        (int32 offsets from lo, a permutation) to the address ``out_ptr``."""
        self.lib.surfsim_env_order(self._h, int(lo), int(hi), c_void_p(out_ptr))

    def step_k_numpy(self, actions: np.ndarray, k: int, yaw: Optional[np.ndarray] = None,
                     fail: Optional[np.ndarray] = None):
        """Convenience step_k on numpy arrays: returns (obs, term_obs, rec, term_rec)."""
        n = self.num_envs
        rows = np.zeros((n, 8), np.int32)
        rows[:, :6] = np.asarray(actions, np.int32)[:, :6]
        if yaw is not None:
            rows[:, 6] = np.ascontiguousarray(yaw, np.float32).view(np.int32)
        if fail is not None:
            rows[:, 7] = np.asarray(fail, np.int32)
        obs = np.zeros((n, self.obs_dim), np.float32)
        tob = np.zeros((n, self.obs_dim), np.float32)
        rec = np.zeros((n, REC_COLS), np.float32)
        trec = np.zeros((n, TERM_COLS), np.float32)
        self.step_k(rows.ctypes.data, 8, k, yaw_slot=6 if yaw is not None else -1,
                    fail_slot=7 if fail is not None else -1, obs=(obs.ctypes.data, self.obs_dim),
                    term_obs=(tob.ctypes.data, self.obs_dim), rec=(rec.ctypes.data, REC_COLS),
                    term_rec=(trec.ctypes.data, TERM_COLS))
        return obs, tob, rec, trec

    def set_waypoints(self, xyz) -> None:
        a = np.ascontiguousarray(np.asarray(xyz, np.float32).reshape(-1, 3))
        if self.lib.surfsim_set_waypoints(self._h, _fptr(a), len(a)) != 0:
            raise ValueError("need >= 2 waypoints")

    def set_spawn_pool(self, pool: np.ndarray) -> None:
        p = np.ascontiguousarray(np.asarray(pool, STATE_DTYPE))
        if len(p) < 1 or self.lib.surfsim_set_spawn_pool(self._h, c_void_p(p.ctypes.data), len(p)) != 0:
            raise ValueError("spawn pool needs >= 1 entry")

    def set_teleport_fail(self, enable: bool = True) -> None:
        self.lib.surfsim_set_teleport_fail(self._h, 1 if enable else 0)

    def set_goal_box(self, mins=None, maxs=None) -> None:
        if mins is None or maxs is None:
            self.lib.surfsim_set_goal_box(self._h, None, None)
        else:
            self.lib.surfsim_set_goal_box(self._h, _vec3(mins), _vec3(maxs))

    def force_fail(self, mask: np.ndarray) -> None:
        m = np.ascontiguousarray(np.asarray(mask, np.uint8).reshape(self.num_envs))
        self.lib.surfsim_force_fail(self._h, m.ctypes.data_as(_P_U8))

    def get_states(self) -> np.ndarray:
        out = np.zeros(self.num_envs, STATE_DTYPE)
        self.lib.surfsim_get_states(self._h, c_void_p(out.ctypes.data))
        return out

    def set_state(self, env: int, state) -> None:
        row = np.ascontiguousarray(np.asarray(state, STATE_DTYPE).reshape(1))
        self.lib.surfsim_set_state(self._h, int(env), c_void_p(row.ctypes.data))

    # ---- geometry queries -----------------------------------------------------
    def trace(self, start, end, hull: int = 0) -> TraceResult:
        out = TraceOut()
        self.lib.surfsim_trace(self._h, _vec3(start), _vec3(end), int(hull), ctypes.byref(out))
        return TraceResult(np.array(out.endpos, np.float32), np.array(out.normal, np.float32), float(out.dist),
                           float(out.fraction), bool(out.startsolid), bool(out.allsolid), int(out.ent))

    def trace_batch(self, start: np.ndarray, end: np.ndarray, hull: int = 2) -> np.ndarray:
        """(n,3),(n,3) -> (n,8): fraction, endpos(3), normal(3), startsolid."""
        seg = np.ascontiguousarray(np.concatenate([np.asarray(start, np.float32).reshape(-1, 3),
                                                   np.asarray(end, np.float32).reshape(-1, 3)], 1))
        out = np.zeros((len(seg), 8), np.float32)
        self.lib.surfsim_trace_batch(self._h, c_void_p(seg.ctypes.data), len(seg), int(hull), c_void_p(out.ctypes.data))
        return out

    def point_contents(self, p) -> int:
        return int(self.lib.surfsim_point_contents(self._h, _vec3(p)))

    def occupancy_grid(self, mins, cell: float, nx: int, ny: int, nz: int) -> np.ndarray:
        out = np.zeros((nz, ny, nx), np.uint8)
        m = np.ascontiguousarray(np.asarray(mins, np.float32).reshape(3))
        self.lib.surfsim_occupancy_grid(self._h, _fptr(m), float(cell), nx, ny, nz, c_void_p(out.ctypes.data))
        return out

    # ---- single-player stepping --------------------------------------------------
    def pm_step_usercmd(self, st: PlayerState, yaw: float, pitch: float, fmove: float, smove: float,
                        buttons: int = 0, msec: int = 10) -> None:
        self.lib.surfsim_pm_step_usercmd(self._h, ctypes.byref(st), yaw, pitch, fmove, smove, int(buttons), int(msec))

    def play_step(self, st: PlayerState, yaw: float, pitch: float, fmove: float, smove: float,
                  buttons: int = 0, msec: int = 10) -> int:
        return int(self.lib.surfsim_play_step(self._h, ctypes.byref(st), yaw, pitch, fmove, smove, int(buttons), int(msec)))

    def pm_step_single(self, st: PlayerState, action) -> None:
        a = (c_int32 * 6)(*[int(x) for x in action])
        self.lib.surfsim_pm_step_single(self._h, ctypes.byref(st), a)

    # ---- map info ------------------------------------------------------------------
    def spawns(self):
        out = []
        for i in range(int(self.lib.surfsim_num_spawns(self._h))):
            o = (c_float * 3)()
            y = c_float()
            self.lib.surfsim_get_spawn(self._h, i, o, ctypes.byref(y))
            out.append((np.array(o, np.float32), float(y.value)))
        return out

    def map_bounds(self):
        mn, mx = (c_float * 3)(), (c_float * 3)()
        self.lib.surfsim_map_bounds(self._h, mn, mx)
        return np.array(mn, np.float64), np.array(mx, np.float64)

    def map_counts(self) -> dict:
        c = (c_int32 * 8)()
        self.lib.surfsim_map_counts(self._h, c)
        keys = ("planes", "nodes", "clipnodes", "models", "solids", "volumes", "triggers", "spawns")
        return dict(zip(keys, [int(x) for x in c]))

    def export_hull0(self):
        """(planes float32 [P,4], plane types int32 [P], nodes int32 [N,3], headnode)."""
        c = self.map_counts()
        planes = np.zeros((c["planes"], 4), np.float32)
        types = np.zeros(c["planes"], np.int32)
        nodes = np.zeros((c["nodes"], 3), np.int32)
        head = c_int32()
        self.lib.surfsim_export_hull0(self._h, c_void_p(planes.ctypes.data), c_void_p(types.ctypes.data),
                                      c_void_p(nodes.ctypes.data), ctypes.byref(head))
        return planes, types, nodes, int(head.value)

    def core_bytes(self) -> bytes:
        """The batch's per-env rule set (EnvCore, host pointers into this core)
        as raw bytes: what ``GpuEnv`` copies to the device."""
        n = self.lib.surfsim_core_bytes(self._h, None, 0)
        buf = ctypes.create_string_buffer(n)
        self.lib.surfsim_core_bytes(self._h, ctypes.cast(buf, c_void_p), n)
        return buf.raw

    def export_mesh(self):
        """(vertices float32 [V, 3], triangles int32 [T, 3]) of the solid geometry."""
        n = (c_int32 * 2)()
        self.lib.surfsim_export_mesh(self._h, None, 0, None, 0, n)
        v = np.zeros((n[0], 3), np.float32)
        t = np.zeros((n[1], 3), np.int32)
        self.lib.surfsim_export_mesh(self._h, c_void_p(v.ctypes.data), n[0], c_void_p(t.ctypes.data), n[1], n)
        return v, t

    def solid_entities(self) -> np.ndarray:
        """(n, 10) float32 rows: hull-0 head node (int32 bits), origin, absmin, absmax."""
        n = self.map_counts()["solids"]
        out = np.zeros((n, 10), np.float32)
        if n:
            self.lib.surfsim_solid_entities(self._h, c_void_p(out.ctypes.data), n)
        return out

    def triggers(self):
        n = self.map_counts()["triggers"]
        kinds = np.zeros((max(n, 1), 3), np.int32)
        bounds = np.zeros((max(n, 1), 6), np.float32)
        dmg = np.zeros(max(n, 1), np.float32)
        self.lib.surfsim_triggers(self._h, c_void_p(kinds.ctypes.data), c_void_p(bounds.ctypes.data),
                                  c_void_p(dmg.ctypes.data), n)
        names = ("teleport", "hurt", "push")
        return [dict(kind=names[kinds[i, 0]], model=int(kinds[i, 1]), has_dest=bool(kinds[i, 2]),
                     mins=bounds[i, :3].copy(), maxs=bounds[i, 3:].copy(), damage=float(dmg[i])) for i in range(n)]

    def trigger_contains(self, index: int, points: np.ndarray, usehull: int = 0) -> np.ndarray:
        p = np.ascontiguousarray(np.asarray(points, np.float32).reshape(-1, 3))
        out = np.zeros(len(p), np.uint8)
        self.lib.surfsim_trigger_contains(self._h, int(index), c_void_p(p.ctypes.data), len(p), int(usehull),
                                          c_void_p(out.ctypes.data))
        return out.astype(bool)


def compile_bsp(brushes: list, entities: str) -> bytes:
    """Compile brushes into a BSP v30 image. ``brushes``: list of
    (model, contents, planes[(nx, ny, nz, d), ...]) with solid where n.x <= d."""
    recs = []
    for model, contents, planes in brushes:
        recs += [float(model), float(contents), float(len(planes))]
        for p in planes:
            recs += [float(x) for x in p]
    arr = np.asarray(recs, np.float32)
    lib = simlib()
    err = ctypes.create_string_buffer(512)
    ent = entities.encode()
    size = lib.surfsim_compile_bsp(c_void_p(arr.ctypes.data), len(arr), ent, None, 0, err, 512)
    if size < 0:
        raise RuntimeError(err.value.decode())
    buf = ctypes.create_string_buffer(int(size))
    lib.surfsim_compile_bsp(c_void_p(arr.ctypes.data), len(arr), ent, ctypes.cast(buf, c_void_p), size, err, 512)
    return buf.raw[:size]
