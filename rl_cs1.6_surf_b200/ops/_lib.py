"""ctypes bindings of the CUDA kernel libraries.

Every entry point takes raw device pointers and the CUDA stream to launch on
(the caller's current torch stream), so the kernels compose with torch
tensors and can be captured in CUDA graphs. A non-zero return value is a CUDA
error code and raises.
"""
from __future__ import annotations

import ctypes
from ctypes import c_double, c_float, c_int, c_int64, c_void_p

import torch

from .._native import load

_V = c_void_p
_I = c_int
_L = c_int64
_F = c_float
_D = c_double

_SIGS = {
    "libsurf_vision.so": {
        "surf_march": (_I, [_V, _L, _I, _I, _I, _V, _I, _I, _I, _F, _F, _F, _F, _V, _V, _F, _F, _I, _I, _V, _L, _I,
                            _I, _V, _V, _I, _V, _V]),
        "surf_brick_size": (_L, [_I, _I, _I]),
        "surf_brick_sdf": (_I, [_V, _I, _V, _I, _I, _I, _V]),
        "surf_brick_i8": (_I, [_V, _V, _I, _I, _I, _V]),
        "surf_occupancy": (_I, [_V, _V, _V, _I, _V, _I, _F, _F, _F, _F, _I, _I, _I, _I, _V, _V]),
        "surf_edt_workspace_bytes": (_L, [_I, _I, _I]),
        "surf_edt": (_I, [_V, _I, _I, _I, _F, _V, _V, _V, _V, _V]),
        "surf_surfnz_bake": (_I, [_V, _I, _V, _V, _V, _I, _V, _I, _D, _D, _D, _D, _I, _I, _I, _V, _V, _V, _V]),
    },
}


class KernelError(RuntimeError):
    pass


_bound: dict = {}


class _Bound:
    """A loaded library exposing only its registered entry points.

    ctypes would call an entry point without a signature by converting every
    Python int to a C int, silently truncating 64-bit device pointers; an
    unregistered name therefore raises instead."""

    def __init__(self, name: str, cdll: ctypes.CDLL):
        self._name = name
        self._cdll = cdll
        for fn, (res, args) in _SIGS.get(name, {}).items():
            f = getattr(cdll, fn)
            f.restype = res
            f.argtypes = args
            setattr(self, fn, f)

    def __getattr__(self, fn: str):
        if fn.startswith("surf_"):
            raise AttributeError(f"{self._name}: entry point {fn} has no registered signature")
        raise AttributeError(fn)


def lib(name: str) -> _Bound:
    if name in _bound:
        return _bound[name]
    b = _Bound(name, load(name))
    _bound[name] = b
    return b


def register(name: str, sigs: dict) -> None:
    _SIGS.setdefault(name, {}).update(sigs)
    _bound.pop(name, None)


def stream_ptr(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


# Kernel launches issued by each entry point (for launch accounting; entry
# points not listed launch exactly one kernel).
_KERNELS_PER_CALL = {"surf_reward": 2, "surf_permutation": 2, "surf_permutation_pool": 2, "surf_edt": 4, "surf_geodesic_pass": 3,
                     "surf_geodesic_init": 3, "surf_geodesic_finish": 2}
_launches = [0]


def check(code: int, what: str) -> None:
    """Raise on a non-zero CUDA status; count the entry point's launches."""
    _launches[0] += _KERNELS_PER_CALL.get(what, 1)
    if code != 0:
        raise KernelError(f"{what} failed with CUDA error {code}")


def launch_count() -> int:
    """Kernels launched through this package so far (graph replays included
    via ``add_launches``)."""
    return _launches[0]


def add_launches(n: int) -> None:
    _launches[0] += int(n)


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise KernelError(f"{what}: the CUDA kernel needs CUDA tensors (use the *_reference CPU oracle on CPU)")
