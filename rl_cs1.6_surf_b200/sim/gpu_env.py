"""The env batch on the GPU (``libsurf_env.so``): one CUDA thread per env.

The simulator's per-env rules (pm_shared movement, hull traces, triggers,
spline progress, autoreset: ``EnvCore`` in csrc/sim/env_core.hpp) are
header-only code compiled for both the host batch and the device. A
``GpuEnv`` is built from a configured ``SimCore`` (map, waypoints, spawn pool,
goal box and rules copied to the device) and then steps with device action
rows in and device observation / record rows out, in the same column layout
the host batch writes into pinned memory — so the trainer's reward, camera
and policy kernels read them in place and a rollout never leaves the GPU.

Reference: the reference steps its envs on CPU threads only
(src/env.c:529-644); this is the same step moved next to the policy.
"""
from __future__ import annotations

import ctypes
from ctypes import c_int, c_int64, c_uint64, c_void_p

import numpy as np
import torch

from ..ops import _lib
from ..ops._lib import KernelError, check, ptr, stream_ptr
from .core import STATE_DTYPE, SimCore

ELIB = "libsurf_env.so"
_V, _I, _L = c_void_p, c_int, c_int64
_lib.register(ELIB, {
    "surf_genv_core_size": (_I, []),
    "surf_genv_create": (_V, [_V, _I, ctypes.POINTER(c_int)]),
    "surf_genv_destroy": (None, [_V]),
    "surf_genv_num_envs": (_I, [_V]),
    "surf_genv_set_spawn_pool": (_I, [_V, _V, _I]),
    "surf_genv_reset": (_I, [_V, c_uint64, _V, _L, _V, _L, _V]),
    "surf_genv_step_k": (_I, [_V, _I, _I, _V, _L, _I, _I, _I, _V, _L, _V, _L, _V, _L, _V, _L, _V]),
    "surf_genv_get_states": (_I, [_V, _V, _V]),
    "surf_genv_set_states": (_I, [_V, _V, _V]),
    "surf_genv_rng": (_I, [_V, _V, _I, _V]),
})

_CREATE_ERRORS = {1: "the CPU lidar is configured (the GPU env renders no lidar; use the depth camera)",
                  2: "a clip tree of this map is deeper than the device descent stack",
                  3: "EnvCore layout differs between the simulator and the GPU env libraries"}


def _rows(t):
    """(pointer, row stride in floats) of a 2-D float32 CUDA tensor (or None)."""
    if t is None:
        return None, 0
    if t.dtype != torch.float32 or t.stride(-1) != 1 or not t.is_cuda:
        raise ValueError("output rows must be float32 CUDA tensors with unit column stride")
    return ptr(t), t.stride(0)


class GpuEnv:
    """The batch of ``core`` (its config, map and current rules) on the GPU."""

    def __init__(self, core: SimCore, device="cuda"):
        self.device = torch.device(device)
        with torch.cuda.device(self.device):
            L = _lib.lib(ELIB)
            err = c_int(0)
            raw = core.core_bytes()
            buf = ctypes.create_string_buffer(raw, len(raw))
            self._h = L.surf_genv_create(ctypes.cast(buf, c_void_p), len(raw), ctypes.byref(err))
            if not self._h:
                code = err.value
                msg = _CREATE_ERRORS.get(code, f"CUDA error {code - 100}" if code >= 100 else f"code {code}")
                raise KernelError(f"GpuEnv: {msg}")
            self.L = L
            self.num_envs = int(L.surf_genv_num_envs(self._h))
            self.obs_dim = 15

    def close(self) -> None:
        if getattr(self, "_h", None):
            self.L.surf_genv_destroy(self._h)
            self._h = None

    def __del__(self):   # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    def reset(self, seed: int, obs=None, rec=None) -> None:
        """Spawn every env (the host batch's reset_all with the same seed
        gives the same spawns) and write observation / record rows."""
        po, so = _rows(obs)
        pr, sr = _rows(rec)
        check(self.L.surf_genv_reset(self._h, int(seed) & 0xFFFFFFFFFFFFFFFF, po, so, pr, sr,
                                     stream_ptr(self.device)), "surf_genv_reset")

    def step_k(self, actions: torch.Tensor, k: int, lo: int = 0, hi: int = None, yaw_slot: int = -1,
               fail_slot: int = -1, obs=None, term_obs=None, rec=None, term_rec=None) -> None:
        """K ticks of action repeat for envs [lo, hi). ``actions``: int32 CUDA
        rows (slots 0..5 the discrete action; a float bit pattern in
        ``yaw_slot`` replaces the yaw bin; non-zero ``fail_slot`` force-fails)."""
        if actions.dtype != torch.int32 or not actions.is_cuda or actions.stride(-1) != 1:
            raise ValueError("actions must be int32 CUDA rows")
        hi = self.num_envs if hi is None else hi
        args = [_rows(t) for t in (obs, term_obs, rec, term_rec)]
        flat = [x for pair in args for x in pair]
        check(self.L.surf_genv_step_k(self._h, int(lo), int(hi), ptr(actions), actions.stride(0), int(yaw_slot),
                                      int(fail_slot), int(k), *flat, stream_ptr(self.device)), "surf_genv_step_k")

    def get_states(self) -> np.ndarray:
        out = np.zeros(self.num_envs, STATE_DTYPE)
        check(self.L.surf_genv_get_states(self._h, c_void_p(out.ctypes.data), stream_ptr(self.device)),
              "surf_genv_get_states")
        return out

    def set_states(self, states: np.ndarray) -> None:
        arr = np.ascontiguousarray(np.asarray(states, STATE_DTYPE).reshape(self.num_envs))
        check(self.L.surf_genv_set_states(self._h, c_void_p(arr.ctypes.data), stream_ptr(self.device)),
              "surf_genv_set_states")

    def set_spawn_pool(self, pool: np.ndarray) -> None:
        arr = np.ascontiguousarray(np.asarray(pool, STATE_DTYPE))
        check(self.L.surf_genv_set_spawn_pool(self._h, c_void_p(arr.ctypes.data), len(arr)),
              "surf_genv_set_spawn_pool")

    def rng(self) -> np.ndarray:
        out = np.zeros(self.num_envs, np.uint64)
        check(self.L.surf_genv_rng(self._h, c_void_p(out.ctypes.data), 0, stream_ptr(self.device)), "surf_genv_rng")
        return out

    def set_rng(self, values: np.ndarray) -> None:
        arr = np.ascontiguousarray(np.asarray(values, np.uint64).reshape(self.num_envs))
        check(self.L.surf_genv_rng(self._h, c_void_p(arr.ctypes.data), 1, stream_ptr(self.device)), "surf_genv_rng")
