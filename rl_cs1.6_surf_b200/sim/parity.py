"""Parity harness against the reference core built from source.

The reference simulator (Sorrow321/RL_CS1.6_Surf, C11) compiles to
``libsurfcore.so`` with its own ``build.sh``; ``baseline/_ref/build`` holds
that build. Its structs are layout-compatible with ours (SurfEnvConfig 128 B,
SurfState 108 B, SurfTrace 44 B — reference src/surfcore.h:66-150), so the
same config and state buffers drive both, tick for tick. The harness only
calls the reference's public C exports.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int32, c_uint8, c_uint64, c_void_p
from pathlib import Path
from typing import Optional

import numpy as np

from .core import STATE_DTYPE, EnvConfig, PlayerState, TraceOut

REPO = Path(__file__).resolve().parents[2]
REF_LIB = REPO / "baseline" / "_ref" / "build" / "libsurfcore.so"


def reference_available() -> bool:
    return REF_LIB.exists()


class RefCore:
    """Minimal binding of the reference core's exports (batch env + traces)."""

    def __init__(self, bsp_path: str, cfg: EnvConfig, lib_path: Optional[Path] = None):
        os.environ.setdefault("OMP_NUM_THREADS", "4")
        lib = ctypes.CDLL(str(lib_path or REF_LIB))
        P_F = POINTER(c_float)
        lib.surf_create.restype = c_void_p
        lib.surf_create.argtypes = [c_char_p, POINTER(EnvConfig), c_char_p, c_int32]
        lib.surf_destroy.argtypes = [c_void_p]
        lib.surf_obs_dim.restype = c_int32
        lib.surf_obs_dim.argtypes = [c_void_p]
        lib.surf_reset_all.argtypes = [c_void_p, c_uint64, P_F]
        lib.surf_step.argtypes = [c_void_p, POINTER(c_int32), P_F, P_F, POINTER(c_uint8), POINTER(c_uint8), P_F]
        lib.surf_states_ptr.restype = c_void_p
        lib.surf_states_ptr.argtypes = [c_void_p]
        lib.surf_trace.argtypes = [c_void_p, P_F, P_F, c_int32, POINTER(TraceOut)]
        lib.surf_point_contents.restype = c_int32
        lib.surf_point_contents.argtypes = [c_void_p, P_F]
        lib.surf_pm_step_usercmd.argtypes = [c_void_p, c_void_p, c_float, c_float, c_float, c_float, c_int32, c_int32]
        lib.surf_set_goal_box.argtypes = [c_void_p, P_F, P_F]
        lib.surf_set_teleport_fail.argtypes = [c_void_p, c_int32]
        lib.surf_set_spawn_pool.restype = c_int32
        lib.surf_set_spawn_pool.argtypes = [c_void_p, c_void_p, c_int32]
        lib.surf_set_waypoints.restype = c_int32
        lib.surf_set_waypoints.argtypes = [c_void_p, P_F, c_int32]
        self.lib = lib
        err = ctypes.create_string_buffer(256)
        h = lib.surf_create(str(bsp_path).encode(), ctypes.byref(cfg), err, 256)
        if not h:
            raise RuntimeError(err.value.decode())
        self.h = c_void_p(h)
        self.n = cfg.num_envs
        self.obs_dim = int(lib.surf_obs_dim(self.h))
        self.obs = np.zeros((self.n, self.obs_dim), np.float32)
        self.term = np.zeros_like(self.obs)
        self.rew = np.zeros(self.n, np.float32)
        self.done = np.zeros(self.n, np.uint8)
        self.trunc = np.zeros(self.n, np.uint8)
        ptr = lib.surf_states_ptr(self.h)
        self.states_view = np.ctypeslib.as_array(
            (ctypes.c_uint8 * (self.n * STATE_DTYPE.itemsize)).from_address(ptr)).view(STATE_DTYPE)

    def reset(self, seed: int) -> np.ndarray:
        self.lib.surf_reset_all(self.h, c_uint64(seed), self.obs.ctypes.data_as(POINTER(c_float)))
        return self.obs

    def step(self, actions: np.ndarray):
        a = np.ascontiguousarray(actions, np.int32)
        P = lambda x, t: x.ctypes.data_as(POINTER(t))
        self.lib.surf_step(self.h, P(a, c_int32), P(self.obs, c_float), P(self.rew, c_float), P(self.done, c_uint8),
                           P(self.trunc, c_uint8), P(self.term, c_float))
        return self.obs, self.rew, self.done, self.trunc, self.term

    def trace(self, start, end, hull: int) -> TraceOut:
        out = TraceOut()
        s = (c_float * 3)(*map(float, start))
        e = (c_float * 3)(*map(float, end))
        self.lib.surf_trace(self.h, s, e, hull, ctypes.byref(out))
        return out

    def point_contents(self, p) -> int:
        return int(self.lib.surf_point_contents(self.h, (c_float * 3)(*map(float, p))))

    def pm_step_usercmd(self, st: PlayerState, yaw, pitch, fmove, smove, buttons=0, msec=10) -> None:
        self.lib.surf_pm_step_usercmd(self.h, ctypes.byref(st), yaw, pitch, fmove, smove, buttons, msec)

    def set_teleport_fail(self, on: bool) -> None:
        self.lib.surf_set_teleport_fail(self.h, 1 if on else 0)

    def set_goal_box(self, mins, maxs) -> None:
        self.lib.surf_set_goal_box(self.h, (c_float * 3)(*map(float, mins)), (c_float * 3)(*map(float, maxs)))

    def set_spawn_pool(self, pool: np.ndarray) -> None:
        p = np.ascontiguousarray(pool, STATE_DTYPE)
        self.lib.surf_set_spawn_pool(self.h, c_void_p(p.ctypes.data), len(p))

    def close(self) -> None:
        if self.h:
            self.lib.surf_destroy(self.h)
            self.h = None
