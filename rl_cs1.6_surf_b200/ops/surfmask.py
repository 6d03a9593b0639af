"""Surface slope mask: the depth camera's optional second channel.

A depth pixel cannot say whether it sees floor, surf ramp or wall. The mask
stores, per voxel of the vision grid, |n_z| * 127 (int8) of the solid face
the voxel holds: 127 flat floor, ~38-89 the rideable ramp band, 0 wall or no
surface. The march kernel re-derives the voxel it stopped in and writes
``byte / 127`` next to the depth value, so a 2-channel frame is pixel-major
(depth, slope) — channel fastest, the layout the first convolution reads.

Reference: python/surfgym/surfmask.py:1-40 (semantics), :112-179 (the
two-pass rasterization: margin claims, then exact claims on top, largest area
wins inside a pass). Differences, by design:

* the bake is one CUDA kernel (``surf_surfnz_bake``, csrc/kernels/sdf.cu):
  the two ordered passes become a single 64-bit ``atomicMax`` whose key orders
  claims by (exact, area, triangle index) — the same winner;
* the triangles are this framework's hull-0 solid-leaf polyhedra
  (``SimCore.export_mesh``), i.e. the geometry physics collides with, so the
  reference's "invisible solid brush renders as wall" limit does not apply.
  Those polyhedra include faces between two solid cells; the kernel drops a
  face whose outward side is solid at all its probe points.

``surfnz_reference`` is the float64 numpy oracle of the claim rule (it
mirrors the kernel's operation order, so results match bit for bit).
"""
from __future__ import annotations

from typing import Optional, Tuple

import numpy as np
import torch

from . import _lib
from ._lib import check, ptr, require_cuda, stream_ptr

VLIB = "libsurf_vision.so"
WALKABLE = 89                 # round(0.7 * 127): the physics walks on n_z >= 0.7


def solid_triangles(core) -> np.ndarray:
    """(T, 3, 3) float32 triangles of the map's solid geometry (outward winding)."""
    v, t = core.export_mesh()
    if len(t) == 0:
        return np.zeros((0, 3, 3), np.float32)
    return np.ascontiguousarray(v[t].astype(np.float32))


def bake(tris: np.ndarray, mins, cell: float, dims, core=None, device="cuda",
         linear: bool = True) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Bake the mask on the GPU -> (bricked int8 [brick_size], linear int8 [nz, ny, nx] or None).

    ``core`` given: its hull-0 tree and solid entities drive the internal-face
    filter (faces buried between solid cells claim nothing)."""
    dev = torch.device(device)
    require_cuda(torch.empty(0, device=dev), "surfmask.bake")
    nx, ny, nz = (int(d) for d in dims)
    L = _lib.lib(VLIB)
    tris_t = torch.as_tensor(np.ascontiguousarray(tris, np.float32).reshape(-1, 9), device=dev)
    keys = torch.empty(nx * ny * nz, dtype=torch.int64, device=dev)
    brk = torch.empty(int(L.surf_brick_size(nx, ny, nz)), dtype=torch.int8, device=dev)
    lin = torch.empty((nz, ny, nx), dtype=torch.int8, device=dev) if linear else None
    keep = []
    tree = (None, None, None, 0, None, 0)
    if core is not None:
        planes, types, nodes, head = core.export_hull0()
        ents = core.solid_entities()
        P = torch.as_tensor(planes, device=dev)
        T = torch.as_tensor(types, device=dev)
        N = torch.as_tensor(nodes, device=dev)
        E = torch.as_tensor(ents if len(ents) else np.zeros((1, 10), np.float32), device=dev)
        keep = [P, T, N, E]
        tree = (ptr(P), ptr(T), ptr(N), int(head), ptr(E), len(ents))
    m = np.asarray(mins, np.float64)
    check(L.surf_surfnz_bake(ptr(tris_t), tris_t.shape[0], *tree, float(m[0]), float(m[1]), float(m[2]), float(cell),
                             nx, ny, nz, ptr(keys), ptr(lin), ptr(brk), stream_ptr(dev)), "surf_surfnz_bake")
    del keep
    return brk, lin


def for_volume(core, volume, device=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """The mask on exactly ``volume``'s grid (same mins, cell and dims, so one
    voxel index reads both)."""
    dev = volume.bricked.device if device is None else torch.device(device)
    return bake(solid_triangles(core), volume.mins, volume.cell, volume.dims, core=core, device=dev)


def surfnz_reference(tris: np.ndarray, mins, cell: float, dims, keep: Optional[np.ndarray] = None) -> np.ndarray:
    """CPU oracle of the claim rule -> int8 [nz, ny, nx] (``keep``: optional
    per-triangle mask, e.g. the internal-face filter's decisions)."""
    nx, ny, nz = (int(d) for d in dims)
    key = np.zeros((nz, ny, nx), np.uint64)
    tris = np.asarray(tris, np.float32).astype(np.float64).reshape(-1, 3, 3)
    mn = np.asarray(mins, np.float64)
    dim = np.array([nx, ny, nz])
    cell = float(cell)
    for ti, tr in enumerate(tris):
        if keep is not None and not keep[ti]:
            continue
        a, b, c = tr
        u, w = b - a, c - a
        cr = np.array([u[1] * w[2] - u[2] * w[1], u[2] * w[0] - u[0] * w[2], u[0] * w[1] - u[1] * w[0]])
        area2 = np.sqrt((cr[0] * cr[0] + cr[1] * cr[1]) + cr[2] * cr[2])
        if not area2 > 1e-9:
            continue
        n = cr / area2
        val = int(np.rint(abs(n[2]) * 127.0))
        tight = (0.5 * cell) * ((abs(n[0]) + abs(n[1])) + abs(n[2]))
        margin = tight + 0.5 * cell
        pd = (n[0] * a[0] + n[1] * a[1]) + n[2] * a[2]
        lo = np.clip(np.floor((tr.min(0) - cell - mn) / cell), 0, dim).astype(np.int64)
        hi = np.clip(np.floor((tr.max(0) + cell - mn) / cell) + 1.0, 0, dim).astype(np.int64)
        if np.any(hi - lo <= 0):
            continue
        ax = [((np.arange(lo[k], hi[k]) + 0.5) * cell + mn[k]) * n[k] for k in range(3)]
        dist = (ax[2][:, None, None] + ax[1][None, :, None]) + ax[0][None, None, :] - pd
        ad = np.abs(dist)
        base = (np.uint64(np.float32(area2).view(np.uint32)) << np.uint64(31)) | \
               (np.uint64(ti & 0xFFFFFF) << np.uint64(7)) | np.uint64(val)
        k = np.where(ad <= tight, base | np.uint64(1 << 63), base)
        k = np.where(ad <= margin, k, np.uint64(0))
        blk = key[lo[2]:hi[2], lo[1]:hi[1], lo[0]:hi[0]]
        np.maximum(blk, k, out=blk)
    return np.where(key != 0, (key & np.uint64(127)).astype(np.int8), np.int8(0)).astype(np.int8)


def internal_faces_reference(core, tris: np.ndarray) -> np.ndarray:
    """Host restatement of the kernel's internal-face filter -> bool keep per
    triangle (world hull only: for maps without solid brush entities)."""
    tris = np.asarray(tris, np.float32).astype(np.float64).reshape(-1, 3, 3)
    keep = np.zeros(len(tris), bool)
    for i, (a, b, c) in enumerate(tris):
        cr = np.cross(b - a, c - a)
        ar = np.linalg.norm(cr)
        if not ar > 1e-9:
            continue
        n = cr / ar
        g = (a + b + c) / 3.0
        for p in (g, 0.5 * (g + a), 0.5 * (g + b), 0.5 * (g + c)):
            q = (p + 0.25 * n).astype(np.float32)
            if core.point_contents(q) not in (-2, -6):
                keep[i] = True
                break
    return keep


def histogram(grid: np.ndarray) -> dict:
    """Share of surfaced voxels per slope class (the reference bake's report)."""
    g = np.asarray(grid)
    surf = g[g > 0].astype(np.float32) / 127.0
    edges = [0.0, 0.1, 0.3, 0.7, 0.95, 1.01]
    names = ["wall", "steep", "surfable", "walkable", "flat"]
    counts = np.histogram(surf, bins=edges)[0] if surf.size else np.zeros(5, int)
    return {"surfaced": int(surf.size), "voxels": int(g.size), **{n: int(c) for n, c in zip(names, counts)}}
