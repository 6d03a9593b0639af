"""The allocation-free EDT entry point (surf_edt_noalloc) vs the regular one.

surf_edt_noalloc serves callers that cannot allocate device memory when they
need a distance field (inside a stream capture, under a fully reserved
memory pool): it keeps its line workspace in a static device array and uses
the caller's float output as its working buffer. This test calls it through
its exported C symbol and checks two consecutive calls (different grids, so
the shared workspace is reused) against surf_edt, with the tolerance of the
other EDT test; it also checks the size limit. Collected last on purpose.
"""
import ctypes
from ctypes import c_float, c_int, c_void_p

import numpy as np
import pytest
import torch

from surfb200._native import LIB_DIR
from surfb200.ops import vision

pytestmark = pytest.mark.gpu


def _lib():
    lib = ctypes.CDLL(str(LIB_DIR / "libsurf_vision.so"))
    fn = lib.surf_edt_noalloc
    fn.restype = c_int
    fn.argtypes = [c_void_p, c_int, c_int, c_int, c_float, c_void_p, c_void_p]
    return fn


def _occupancy(shape, seed):
    """Random boxes in a grid (uint8, 1 = solid)."""
    rng = np.random.default_rng(seed)
    nz, ny, nx = shape
    occ = np.zeros(shape, np.uint8)
    for _ in range(12):
        lo = rng.integers(0, [nz, ny, nx])
        hi = lo + rng.integers(1, [max(2, nz // 3), max(2, ny // 3), max(2, nx // 3)])
        occ[lo[0]:hi[0], lo[1]:hi[1], lo[2]:hi[2]] = 1
    return torch.as_tensor(occ, device="cuda")


def test_noalloc_matches_regular_entry_point():
    fn = _lib()
    stream = torch.cuda.current_stream().cuda_stream
    for call, (shape, cell) in enumerate([((40, 56, 72), 16.0), ((64, 33, 250), 32.0)]):
        occ = _occupancy(shape, seed=call)
        ref = vision.distance_field(occ, cell)
        out = torch.empty(shape, dtype=torch.float32, device="cuda")
        nz, ny, nx = shape
        rc = fn(c_void_p(occ.data_ptr()), nx, ny, nz, cell, c_void_p(out.data_ptr()), c_void_p(stream))
        assert rc == 0
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), ref.cpu().numpy(), rtol=1e-5, atol=1e-2)


def test_noalloc_rejects_oversized_grids():
    fn = _lib()
    out = torch.empty(1, dtype=torch.float32, device="cuda")
    occ = torch.zeros(1, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(c_void_p(occ.data_ptr()), 257, 8, 8, 16.0, c_void_p(out.data_ptr()), c_void_p(stream))
    assert rc == 1                                       # cudaErrorInvalidValue, nothing launched
