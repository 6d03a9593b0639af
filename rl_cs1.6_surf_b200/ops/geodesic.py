"""Geodesic distance-to-goal bake (csrc/kernels/geodesic.cu) and its oracle.

Reference behaviour: python/surfgym/goalfield.py:158-298 — multi-source
26-connected shortest paths from the free voxels of the goal zone (grown by
max(0.75 cell, 20u)) over the slab occupancy grid, solid and unreachable
voxels holding a sentinel, stored as uint16 at cell/8 units.
"""
from __future__ import annotations

import math
from ctypes import c_float, c_int, c_int64, c_void_p
from typing import Optional

import numpy as np
import torch

from . import _lib
from ._lib import check, ptr, stream_ptr
from ..rewards.spec import GoalFieldData

VLIB = "libsurf_vision.so"
_lib.register(VLIB, {
    "surf_geodesic_tiles": (c_int64, [c_int, c_int, c_int]),
    "surf_geodesic_init": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_float,
                                   c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "surf_geodesic_pass": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                   c_float, c_void_p, c_void_p]),
    "surf_geodesic_finish": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_float, c_float, c_void_p, c_void_p]),
})


def seed_box(zone, mins, cell: float, dims):
    """Voxel index box (inclusive) of the goal zone grown by max(0.75 cell, 20)."""
    grow = max(0.75 * cell, 20.0)
    zmin = np.asarray(zone["mins"], np.float64) - grow
    zmax = np.asarray(zone["maxs"], np.float64) + grow
    lo = np.maximum(np.floor((zmin - mins) / cell - 0.5), 0).astype(int)
    hi = np.minimum(np.ceil((zmax - mins) / cell - 0.5), np.asarray(dims) - 1).astype(int)
    return lo, hi


def geodesic(occ: torch.Tensor, cell: float, lo, hi, max_passes: int = 100000,
             stats: Optional[dict] = None) -> torch.Tensor:
    """Distances (float [nz, ny, nx], +3e38 where unreachable) on the GPU.
    ``stats`` (optional dict) receives the number of worklist passes."""
    _lib.require_cuda(occ, "geodesic")
    nz, ny, nx = occ.shape
    L = _lib.lib(VLIB)
    dev = occ.device
    tiles = int(L.surf_geodesic_tiles(nx, ny, nz))
    dist = torch.empty((nz, ny, nx), dtype=torch.float32, device=dev)
    flags = torch.zeros(tiles, dtype=torch.uint8, device=dev)
    work = torch.zeros(2 * tiles, dtype=torch.int64, device=dev)
    counts = torch.zeros(2, dtype=torch.int32, device=dev)
    n_seed = torch.zeros(1, dtype=torch.int32, device=dev)
    changed = torch.zeros(1, dtype=torch.int32, device=dev)
    s = stream_ptr(dev)
    occ = occ.contiguous()
    check(L.surf_geodesic_init(ptr(dist), ptr(occ), ptr(flags), ptr(work), ptr(counts), nx, ny, nz, float(cell),
                               int(lo[0]), int(lo[1]), int(lo[2]), int(hi[0]), int(hi[1]), int(hi[2]), ptr(n_seed), s),
          "surf_geodesic_init")
    if int(n_seed.item()) == 0:
        raise RuntimeError("goal zone contains no free voxel")
    cur = 0
    passes = 0
    for _ in range(max_passes):
        changed.zero_()
        check(L.surf_geodesic_pass(ptr(dist), ptr(occ), ptr(flags), ptr(work), ptr(counts), cur, nx, ny, nz,
                                   float(cell), ptr(changed), s), "surf_geodesic_pass")
        cur = 1 - cur
        passes += 1
        if not int(changed.item()):
            break
    if stats is not None:
        stats["passes"] = passes
    return dist


def geodesic_reference(occ: np.ndarray, cell: float, lo, hi, max_sweeps: int = 100000) -> np.ndarray:
    """numpy Bellman-Ford with 26 shifted relaxations per sweep (the oracle)."""
    nz, ny, nx = occ.shape
    inf = np.float32(3.0e38)
    d = np.full((nz, ny, nx), inf, np.float32)
    solid = occ != 0
    d[lo[2]:hi[2] + 1, lo[1]:hi[1] + 1, lo[0]:hi[0] + 1] = 0
    d[solid] = inf
    offs = [(oz, oy, ox) for oz in (-1, 0, 1) for oy in (-1, 0, 1) for ox in (-1, 0, 1) if (oz, oy, ox) != (0, 0, 0)]
    w = {1: np.float32(cell), 2: np.float32(cell) * np.float32(1.41421356), 3: np.float32(cell) * np.float32(1.73205081)}
    for _ in range(max_sweeps):
        pad = np.pad(d, 1, constant_values=inf)
        new = d.copy()
        for oz, oy, ox in offs:
            m = abs(oz) + abs(oy) + abs(ox)
            src = pad[1 + oz:1 + oz + nz, 1 + oy:1 + oy + ny, 1 + ox:1 + ox + nx]
            np.minimum(new, src + w[m], out=new)
        new[solid] = inf
        if np.array_equal(new, d):
            break
        d = new
    return d


def geodesic_cpu(occ: np.ndarray, cell: float, lo, hi) -> np.ndarray:
    """Host geodesic (native Dijkstra, csrc/sim/geodesic.cpp): the same fixed
    point as the GPU relaxation and ``geodesic_reference``, one settle per voxel."""
    from ctypes import c_int32, c_void_p
    from ..sim.core import simlib
    occ = np.ascontiguousarray(occ, np.uint8)
    nz, ny, nx = occ.shape
    out = np.empty((nz, ny, nx), np.float32)
    lo3 = (c_int32 * 3)(*[int(v) for v in lo])
    hi3 = (c_int32 * 3)(*[int(v) for v in hi])
    r = simlib().surfsim_geodesic(c_void_p(occ.ctypes.data), nx, ny, nz, float(cell), lo3, hi3,
                                  c_void_p(out.ctypes.data))
    if r < 0:
        raise ValueError("grid too large for the host geodesic (32-bit voxel indices)")
    return out


def kill_voxel_mask(core, mins, cell: float, dims):
    """[(z0, y0, x0, mask bool [dz, dy, dx])] of the voxel centres that lie
    inside a kill volume (a teleport with a destination, or a hurt trigger of
    at least 90 damage: the map's fail nets). Each trigger's AABB (grown by
    1u) is only the broad phase; the centres are classified through the
    trigger's own hull-1 clip tree, the simulator's kill test, because kill
    triggers are often thin curtains inside large boxes (reference
    --race-kill-aware, python/surfgym/goalfield.py:159-219)."""
    nx, ny, nz = dims
    mins = np.asarray(mins, np.float64)
    out = []
    for i, trg in enumerate(core.triggers()):
        kill = (trg["kind"] == "teleport" and trg["has_dest"]) or (trg["kind"] == "hurt" and trg["damage"] >= 90.0)
        if not kill:
            continue
        bmn = np.asarray(trg["mins"], np.float64) - 1.0
        bmx = np.asarray(trg["maxs"], np.float64) + 1.0
        lo = np.maximum(np.floor((bmn - mins) / cell - 0.5), 0).astype(int)
        hi = np.minimum(np.ceil((bmx - mins) / cell - 0.5) + 1, [nx, ny, nz]).astype(int)
        if (hi <= lo).any():
            continue
        axes = [mins[a] + (np.arange(lo[a], hi[a]) + 0.5) * cell for a in range(3)]
        zz, yy, xx = np.meshgrid(axes[2], axes[1], axes[0], indexing="ij")
        pts = np.stack([xx.ravel(), yy.ravel(), zz.ravel()], 1)
        inside = core.trigger_contains(i, pts, usehull=1).reshape(zz.shape)
        if inside.any():
            out.append((int(lo[2]), int(lo[1]), int(lo[0]), inside))
    return out


def euclid_goal_field(zone, mins, cell: float, dims, device="cpu") -> GoalFieldData:
    """Straight-line distance from every voxel centre to the goal AABB, in the
    goal field's uint16 format (reference EuclidField / --race-dist euclid,
    python/surfgym/goalfield.py:110-138): no geometry, no bake, every voxel
    valid; a wall between agent and goal is invisible to this potential."""
    nx, ny, nz = dims
    dev = torch.device(device)
    lo_b = torch.as_tensor(np.asarray(zone["mins"], np.float64), device=dev)
    hi_b = torch.as_tensor(np.asarray(zone["maxs"], np.float64), device=dev)
    m = torch.as_tensor(np.asarray(mins, np.float64), device=dev)
    ax = [m[a] + (torch.arange(n, device=dev, dtype=torch.float64) + 0.5) * cell for a, n in enumerate((nx, ny, nz))]
    dx = (ax[0] - ax[0].clamp(lo_b[0], hi_b[0])).view(1, 1, nx)
    dy = (ax[1] - ax[1].clamp(lo_b[1], hi_b[1])).view(1, ny, 1)
    dz = (ax[2] - ax[2].clamp(lo_b[2], hi_b[2])).view(nz, 1, 1)
    dist = torch.sqrt(dx * dx + dy * dy + dz * dz).float()
    reach_max = float(dist.max())
    quant = cell / 8.0
    while (reach_max + 2.0 * cell) / quant > 65535:       # stay inside uint16 on very large maps
        quant *= 2.0
    grid = torch.round(dist / quant).clamp(0, 65535).to(torch.int32).cpu().numpy().astype(np.uint16)
    return GoalFieldData(grid, np.asarray(mins, np.float64), float(cell), float(quant), reach_max)


def bake_goal_field(core, zone, cell: float = 16.0, device="cuda", mins=None, dims=None,
                    kill_aware: bool = False) -> GoalFieldData:
    """Occupancy + geodesic + uint16 quantisation (GPU kernels; native host
    code on CPU). ``kill_aware``: kill volumes are walls of the goal graph
    only (``kill_voxel_mask``), so the shaping routes around fail nets;
    physics and vision are unchanged."""
    from .vision import grid_dims, occupancy, occupancy_reference
    if mins is None or dims is None:
        mn, mx = core.map_bounds()
        mins, nx, ny, nz = grid_dims(mn, mx, cell)
        dims = (nx, ny, nz)
    lo, hi = seed_box(zone, mins, cell, dims)
    dev = torch.device(device)
    kills = kill_voxel_mask(core, mins, cell, dims) if kill_aware else []
    if dev.type == "cuda":
        occ = occupancy(core, mins, cell, dims, slab=True, device=dev)
        for z0, y0, x0, m in kills:
            sub = occ[z0:z0 + m.shape[0], y0:y0 + m.shape[1], x0:x0 + m.shape[2]]
            sub |= torch.as_tensor(m.astype(np.uint8), device=dev)
        dist = geodesic(occ, cell, lo, hi)
        L = _lib.lib(VLIB)
        mx_bits = torch.zeros(1, dtype=torch.int32, device=dev)
        nz, ny, nx = dist.shape
        check(L.surf_geodesic_finish(ptr(dist), nx, ny, nz, ptr(mx_bits), 0.0, 0.0, None, stream_ptr(dev)),
              "surf_geodesic_finish")
        reach_max = float(np.array([mx_bits.item()], np.int32).view(np.float32)[0])
        quant = cell / 8.0
        sentinel = reach_max + 2.0 * cell
        if sentinel / quant > 65535:
            raise RuntimeError("goal field exceeds the uint16 range at cell/8 quantisation; use a larger cell")
        q = torch.empty((nz, ny, nx), dtype=torch.int16, device=dev)
        check(L.surf_geodesic_finish(ptr(dist), nx, ny, nz, None, quant, sentinel, ptr(q), stream_ptr(dev)),
              "surf_geodesic_finish")
        grid = q.cpu().numpy().view(np.uint16)
    else:
        occ = occupancy_reference(core, mins, cell, dims, slab=True)
        for z0, y0, x0, m in kills:
            occ[z0:z0 + m.shape[0], y0:y0 + m.shape[1], x0:x0 + m.shape[2]] |= m.astype(np.uint8)
        dist = geodesic_cpu(occ, cell, lo, hi)
        fin = dist < 1e30
        reach_max = float(dist[fin].max())
        quant = cell / 8.0
        sentinel = reach_max + 2.0 * cell
        grid = np.where(fin, np.rint(dist / quant), np.rint(sentinel / quant)).clip(0, 65535).astype(np.uint16)
    return GoalFieldData(grid, np.asarray(mins, np.float64), float(cell), float(quant), float(reach_max))
