"""The allocation-free EDT entry point (surf_edt_noalloc) vs the regular one.

surf_edt_noalloc (declared in csrc/kernels/sdf_noalloc.h) is for callers
that must not allocate GPU memory, such as a plugin inside a host program that
reserved the whole device for its own pool, or a real-time loop that forbids
cudaMalloc after start-up. It keeps its scratch in a static device array and
uses the caller's float output as its working buffer. These tests call it
through its exported C symbol and check two consecutive calls (different
grids, so the shared scratch is reused) against surf_edt, with the tolerance
of the other EDT test; they also check that bad arguments are rejected
without a launch. The file is collected last on purpose, and passes alone in
a fresh process as well as after the other tests.
"""
import ctypes
import re
from ctypes import c_float, c_int, c_void_p
from pathlib import Path

import numpy as np
import pytest
import torch

from surfb200 import _native
from surfb200.ops import vision

pytestmark = pytest.mark.gpu

HEADER = Path(__file__).resolve().parents[1] / "csrc" / "kernels" / "sdf_noalloc.h"
INVALID_VALUE = 1                                        # cudaErrorInvalidValue


def _lib():
    _native.load("libsurf_vision.so")                    # builds the library first if it is stale
    lib = ctypes.CDLL(str(_native.LIB_DIR / "libsurf_vision.so"))
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


def test_header_declares_the_called_signature():
    text = HEADER.read_text()
    proto = re.search(r"int surf_edt_noalloc\(([^)]*)\);", text)
    assert proto, "sdf_noalloc.h must declare surf_edt_noalloc"
    types = [a.rsplit(" ", 1)[0].replace(" *", "*").strip() for a in proto.group(1).split(",")]
    assert types == ["const uint8_t*", "int", "int", "int", "float", "float*", "void*"]
    assert "no counterpart in the reference" in text


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


def test_noalloc_rejects_bad_arguments():
    fn = _lib()
    out = torch.full((4,), -7.0, dtype=torch.float32, device="cuda")
    occ = torch.zeros(4, dtype=torch.uint8, device="cuda")
    stream = c_void_p(torch.cuda.current_stream().cuda_stream)
    o, p = c_void_p(occ.data_ptr()), c_void_p(out.data_ptr())
    assert fn(o, 257, 8, 8, 16.0, p, stream) == INVALID_VALUE       # beyond the 256-voxel line limit
    assert fn(o, 8, 8, 300, 16.0, p, stream) == INVALID_VALUE
    assert fn(o, 0, 2, 2, 16.0, p, stream) == INVALID_VALUE         # empty axis
    assert fn(o, 2, -1, 2, 16.0, p, stream) == INVALID_VALUE
    assert fn(None, 2, 2, 1, 16.0, p, stream) == INVALID_VALUE      # null input
    assert fn(o, 2, 2, 1, 16.0, None, stream) == INVALID_VALUE      # null output
    torch.cuda.synchronize()
    assert torch.all(out == -7.0)                                   # nothing was launched
