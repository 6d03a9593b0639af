"""Data exports for external viewers: map mesh JSON and goal-field arrows.

The reference writes the render faces of a BSP as mesh JSON
(tools/export_map.py) and the race potential as an arrow field
(tools/export_goalfield.py) for its browser viewer. Maps written by this
framework carry collision hulls only, so the mesh comes from the hull-0 tree
(solid-leaf polyhedra, ``SimCore.export_mesh``). The browser viewer itself is
graphics and not part of this framework; these files are its data.
"""
from __future__ import annotations

import numpy as np


def export_mesh(core, name: str) -> dict:
    v, t = core.export_mesh()
    mn, mx = core.map_bounds()
    return {"map": name, "source": "hull0 solid leaves", "bounds": [mn.tolist(), mx.tolist()],
            "vertices": np.round(v.astype(np.float64), 2).ravel().tolist(), "indices": t.ravel().tolist()}


def descent_directions(gf, points: np.ndarray, h: float = None) -> np.ndarray:
    """Unit horizontal direction of steepest geodesic descent at points (central differences)."""
    h = gf.cell if h is None else h
    p = np.atleast_2d(np.asarray(points, np.float64))
    gx = gf.sample(p + [h, 0, 0]) - gf.sample(p - [h, 0, 0])
    gy = gf.sample(p + [0, h, 0]) - gf.sample(p - [0, h, 0])
    g = -np.stack([gx, gy], 1)
    n = np.linalg.norm(g, axis=1, keepdims=True)
    return np.where(n > 1e-6, g / np.maximum(n, 1e-6), 0.0)


def export_goalfield(gf, stride: int = 8) -> dict:
    """Arrows [x, y, z, dx, dy, distance] at every ``stride``-th reachable voxel."""
    nz, ny, nx = gf.grid.shape
    zz, yy, xx = np.meshgrid(np.arange(0, nz, stride), np.arange(0, ny, stride), np.arange(0, nx, stride),
                             indexing="ij")
    q = gf.grid[zz, yy, xx].astype(np.float64) * gf.quant
    keep = q < gf.valid_max
    pts = np.stack([xx[keep], yy[keep], zz[keep]], 1) * gf.cell + gf.mins + 0.5 * gf.cell
    d = descent_directions(gf, pts)
    arrows = np.concatenate([pts, d, q[keep][:, None]], 1)
    return {"mins": gf.mins.tolist(), "cell": gf.cell, "stride": stride, "reach_max": gf.reach_max,
            "arrows": np.round(arrows, 2).tolist()}
