"""GPU depth vision: occupancy bake, distance field, SDF sphere-trace camera.

Reference behaviour: python/surfgym/vision.py (``map_occupancy``,
``slab_occupancy``, ``build_sdf``, ``GpuLidar``). Here every stage runs on
the GPU through hand-written kernels (csrc/kernels/sdf.cu, march.cu); each
stage has a CPU oracle (``*_reference``) written from the same rules that
the tests compare the kernels against.

Camera convention (shared with the simulator's CPU lidar): row 0 looks up
(+vfov/2), column 0 looks left (+hfov/2), positive pitch = up, eye height 17
standing / 12 ducked; the encoded depth is min(t, near)/near plus a bounded
far tail 0.25*(1 - exp(-(t - near)/2500)); ``near == range`` gives the linear
t/range code.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import _lib
from ._lib import check, ptr, require_cuda, stream_ptr

VLIB = "libsurf_vision.so"
# timing studies only: extra surf_march flag bits (4 = 64-bit voxel addressing for any grid size)
MARCH_DIAG_FLAGS = 0
LAYOUT_NHW, LAYOUT_S2D4 = 0, 1


def grid_dims(mins, maxs, cell: float, pad_cells: int = 4):
    """The vision grid over map bounds padded by ``pad_cells`` voxels per side:
    (mins float64 (3,), nx, ny, nz). One definition shared by every grid the
    camera indexes (occupancy, distance, surfability)."""
    mn = np.asarray(mins, np.float64) - pad_cells * cell
    ext = np.asarray(maxs, np.float64) + pad_cells * cell - mn
    nx, ny, nz = (int(math.ceil(e / cell)) for e in ext)
    return mn, nx, ny, nz


def pick_cell(mins, maxs, budget_voxels: float = 700e6) -> float:
    """Smallest power-of-two voxel size from 16u whose grid fits the budget."""
    cell = 16.0
    while cell < 256.0:
        _, nx, ny, nz = grid_dims(mins, maxs, cell)
        if nx * ny * nz <= budget_voxels:
            break
        cell *= 2.0
    return cell


# ---- occupancy -------------------------------------------------------------------
_SLAB_OFFSETS = [(a, k) for a in range(3) for k in (-2, -1, 1, 2)]


def occupancy_reference(core, mins, cell: float, dims, slab: bool = True) -> np.ndarray:
    """CPU oracle: the simulator's own point-contents test at voxel centres,
    OR-ed over the quarter-cell shifted lattices when ``slab``."""
    nx, ny, nz = dims
    occ = core.occupancy_grid(np.asarray(mins, np.float32), cell, nx, ny, nz)
    if slab:
        for axis, k in _SLAB_OFFSETS:
            off = np.zeros(3)
            off[axis] = k * cell / 4.0
            occ |= core.occupancy_grid(np.asarray(mins, np.float64) + off, cell, nx, ny, nz)
    return occ


def occupancy(core, mins, cell: float, dims, slab: bool = True, device="cuda") -> torch.Tensor:
    """Occupancy grid (uint8 [nz, ny, nx]) computed by walking the map's
    hull-0 clip tree on the GPU."""
    nx, ny, nz = dims
    planes, types, nodes, head = core.export_hull0()
    dev = torch.device(device)
    P = torch.as_tensor(planes, device=dev)
    T = torch.as_tensor(types, device=dev)
    N = torch.as_tensor(nodes, device=dev)
    ents = core.solid_entities()
    E = torch.as_tensor(ents if len(ents) else np.zeros((1, 10), np.float32), device=dev)
    out = torch.empty((nz, ny, nx), dtype=torch.uint8, device=dev)
    m = np.asarray(mins, np.float64)
    check(_lib.lib(VLIB).surf_occupancy(ptr(P), ptr(T), ptr(N), int(head), ptr(E), len(ents), float(m[0]),
                                        float(m[1]), float(m[2]), float(cell), nx, ny, nz, 1 if slab else 0,
                                        ptr(out), stream_ptr(dev)), "surf_occupancy")
    return out


# ---- distance field ---------------------------------------------------------------
def distance_reference(occ: np.ndarray, cell: float) -> np.ndarray:
    """CPU oracle: scipy's exact EDT of the free space, outside = solid."""
    from scipy.ndimage import distance_transform_edt
    padded = np.pad(occ, 1, constant_values=1)
    return distance_transform_edt(padded == 0, sampling=cell)[1:-1, 1:-1, 1:-1].astype(np.float32)


def distance_field(occ: torch.Tensor, cell: float, dtype=torch.float32) -> torch.Tensor:
    """Exact Euclidean distance (map units) from free voxel centres to the
    nearest solid voxel centre (GPU, separable lower-envelope transform)."""
    require_cuda(occ, "distance_field")
    nz, ny, nx = occ.shape
    L = _lib.lib(VLIB)
    dev = occ.device
    d2 = torch.empty((nz, ny, nx), dtype=torch.float32, device=dev)
    ws = torch.empty(int(L.surf_edt_workspace_bytes(nx, ny, nz)), dtype=torch.uint8, device=dev)
    out = torch.empty((nz, ny, nx), dtype=dtype, device=dev)
    f32 = out if dtype == torch.float32 else None
    f16 = out if dtype == torch.float16 else None
    check(L.surf_edt(ptr(occ.contiguous()), nx, ny, nz, float(cell), ptr(d2), ptr(ws), ptr(f32), ptr(f16),
                     stream_ptr(dev)), "surf_edt")
    return out


def brick(grid: torch.Tensor) -> torch.Tensor:
    """Linear [nz, ny, nx] float/half grid -> 4x4x4-bricked fp16 (flat)."""
    require_cuda(grid, "brick")
    nz, ny, nx = grid.shape
    L = _lib.lib(VLIB)
    out = torch.empty(int(L.surf_brick_size(nx, ny, nz)), dtype=torch.float16, device=grid.device)
    src_dtype = 1 if grid.dtype == torch.float16 else 0
    g = grid.contiguous() if grid.dtype in (torch.float16, torch.float32) else grid.float().contiguous()
    check(L.surf_brick_sdf(ptr(g), src_dtype, ptr(out), nx, ny, nz, stream_ptr(grid.device)), "surf_brick_sdf")
    return out


@dataclass
class SdfVolume:
    """A distance field ready for the camera: bricked fp16 on the device plus
    its geometry; ``linear`` keeps the row-major copy for oracles/caches."""
    bricked: torch.Tensor
    linear: torch.Tensor
    mins: np.ndarray
    cell: float
    dims: tuple               # (nx, ny, nz)
    padded: bool = True       # the grid keeps >= 1 free voxel layer around all geometry

    @classmethod
    def from_linear(cls, dist: torch.Tensor, mins, cell: float) -> "SdfVolume":
        nz, ny, nx = dist.shape
        lin16 = dist.to(torch.float16)
        return cls(brick(lin16), lin16, np.asarray(mins, np.float64), float(cell), (nx, ny, nz))

    @classmethod
    def build(cls, core, cell: float = 16.0, mins=None, dims=None, device="cuda", slab: bool = True) -> "SdfVolume":
        """Bake the distance field of ``core``'s map on the GPU."""
        if mins is None or dims is None:
            mn, mx = core.map_bounds()
            mins, nx, ny, nz = grid_dims(mn, mx, cell)
            dims = (nx, ny, nz)
        occ = occupancy(core, mins, cell, dims, slab=slab, device=device)
        dist = distance_field(occ, cell, torch.float16)
        return cls.from_linear(dist, mins, cell)

    def save(self, path) -> None:
        np.savez_compressed(path, sdf=self.linear.cpu().numpy(), mins=self.mins, cell=np.float32(self.cell))

    @classmethod
    def load(cls, path, device="cuda") -> "SdfVolume":
        z = np.load(path)
        return cls.from_linear(torch.as_tensor(z["sdf"], device=device), z["mins"], float(z["cell"]))


# ---- camera -------------------------------------------------------------------------
class DepthCamera:
    """Batched depth renderer over an SdfVolume (the GpuLidar equivalent).

    ``render(pose)`` takes an (N, >=6) float32 CUDA tensor whose rows hold
    x, y, z, yaw_deg, pitch_deg, ducked (any row stride; e.g. a view into the
    env step record) and returns (N, H*W) depth in ``dtype``, in NHW order or
    the 4x4 space-to-depth order the CNN's first conv reads
    (``layout=LAYOUT_S2D4``: pixel (r, c) -> ((r/4)*(W/4) + c/4)*16 + (r%4)*4 + c%4).
    """

    def __init__(self, volume: SdfVolume, width: int = 128, height: int = 64, hfov_deg: float = 120.0,
                 vfov_deg: float = 90.0, range_units: float = 2000.0, near_range: Optional[float] = None,
                 max_steps: int = 64, pinhole: bool = False, layout: int = LAYOUT_NHW,
                 dtype: torch.dtype = torch.float32, surf_nz: Optional[torch.Tensor] = None):
        self.vol = volume
        self.W, self.H = int(width), int(height)
        self.hfov, self.vfov = float(hfov_deg), float(vfov_deg)
        self.range = float(range_units)
        self.near = float(near_range) if near_range else self.range
        self.max_steps = int(max_steps)
        self.pinhole = bool(pinhole)
        self.layout = int(layout)
        self.dtype = dtype
        self.channels = 2 if surf_nz is not None else 1
        self.surf_nz = surf_nz
        dev = volume.bricked.device
        self.col_off, self.row_off = [torch.as_tensor(a, dtype=torch.float32, device=dev) for a in self.offsets()]

    def offsets(self):
        """Per-column and per-row offsets: angles (rad) for the equiangular
        camera, tangent-plane coordinates for the pinhole camera."""
        W, H = self.W, self.H
        if not self.pinhole:
            d2r = math.pi / 180.0
            col = self.hfov * (0.5 - (np.arange(W) + 0.5) / W) * d2r
            row = self.vfov * (0.5 - (np.arange(H) + 0.5) / H) * d2r
            return col.astype(np.float32), row.astype(np.float32)
        tu = math.tan(math.radians(0.5 * self.hfov))
        tv = math.tan(math.radians(0.5 * self.vfov))
        col = tu * (2.0 * np.arange(W) / max(W - 1, 1) - 1.0) if W > 1 else np.zeros(1)
        row = tv * (1.0 - 2.0 * np.arange(H) / max(H - 1, 1)) if H > 1 else np.zeros(1)
        return col.astype(np.float32), row.astype(np.float32)

    @property
    def frame(self) -> int:
        return self.H * self.W * self.channels

    def render(self, pose: torch.Tensor, out: Optional[torch.Tensor] = None, steps: Optional[torch.Tensor] = None,
               stream: Optional[int] = None, env_order: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Depth images of every pose row into ``out`` rows. ``env_order``
        (int32 [n], a permutation of the rows) is the order the kernel renders
        them in -- spatial neighbours in a row share cached SDF bricks; the
        images are the same in any order."""
        require_cuda(pose, "DepthCamera.render")
        if pose.dtype != torch.float32 or pose.stride(-1) != 1 or pose.shape[-1] < 6:
            raise ValueError("pose must be float32 rows (x, y, z, yaw, pitch, ducked, ...) with unit column stride")
        n = pose.shape[0]
        if env_order is not None and (env_order.dtype != torch.int32 or env_order.numel() != n
                                      or not env_order.is_contiguous()):
            raise ValueError("env_order must be a contiguous int32 permutation of the pose rows")
        if out is None:
            out = torch.empty((n, self.frame), dtype=self.dtype, device=pose.device)
        if out.dtype not in (torch.float32, torch.bfloat16) or out.stride(-1) != 1 or out.shape[-1] < self.frame:
            raise ValueError("out must be float32/bfloat16 rows of at least H*W*C elements")
        v = self.vol
        check(_lib.lib(VLIB).surf_march(
            ptr(pose), pose.stride(0), n, self.H, self.W, ptr(v.bricked), v.dims[0], v.dims[1], v.dims[2],
            float(v.mins[0]), float(v.mins[1]), float(v.mins[2]), float(v.cell), ptr(self.col_off),
            ptr(self.row_off), self.range, self.near, self.max_steps, 1 if self.pinhole else 0, ptr(out),
            out.stride(0), 1 if out.dtype == torch.bfloat16 else 0, self.layout, ptr(self.surf_nz), ptr(steps),
            (1 if self.vol.padded else 0) | MARCH_DIAG_FLAGS, ptr(env_order),
            stream if stream is not None else stream_ptr(pose.device)),
            "surf_march")
        return out

    def reference(self, pose: np.ndarray, return_steps: bool = False, surf_nz: Optional[np.ndarray] = None):
        """CPU oracle (float32 numpy, same rules) -> (N, H, W) encoded depth
        ((N, H, W, 2) with the linear slope grid ``surf_nz``)."""
        return march_reference(self.vol.linear.float().cpu().numpy(), self.vol.mins, self.vol.cell, pose,
                               *self.offsets(), self.range, self.near, self.max_steps, self.pinhole,
                               return_steps=return_steps, surf_nz=surf_nz)


def march_reference(sdf: np.ndarray, mins, cell: float, pose: np.ndarray, col_off, row_off, rng: float, near: float,
                    max_steps: int, pinhole: bool = False, return_steps: bool = False,
                    surf_nz: Optional[np.ndarray] = None):
    """Lock-step numpy restatement of the sphere trace (the kernel's oracle).
    With ``surf_nz`` (linear int8 [nz, ny, nx]) the depth comes back as
    (N, H, W, 2): depth and the slope byte / 127 of the voxel the ray stopped in."""
    f = np.float32
    pose = np.asarray(pose, f)
    n = pose.shape[0]
    H, W = len(row_off), len(col_off)
    nz, ny, nx = sdf.shape
    ex = pose[:, 0].reshape(n, 1, 1)
    ey = pose[:, 1].reshape(n, 1, 1)
    ez = (pose[:, 2] + np.where(pose[:, 5] != 0, f(12), f(17))).reshape(n, 1, 1).astype(f)
    d2r = f(0.017453292519943295)
    yaw = (pose[:, 3] * d2r).reshape(n, 1, 1).astype(f)
    pit = (pose[:, 4] * d2r).reshape(n, 1, 1).astype(f)
    co = np.asarray(col_off, f).reshape(1, 1, W)
    ro = np.asarray(row_off, f).reshape(1, H, 1)
    if pinhole:
        cy, sy, cp, sp = np.cos(yaw), np.sin(yaw), np.cos(pit), np.sin(pit)
        dx = cp * cy + co * sy - ro * sp * cy
        dy = cp * sy - co * cy - ro * sp * sy
        dz = sp + ro * cp + 0 * co
        inv = f(1) / np.sqrt(dx * dx + dy * dy + dz * dz)
        dx, dy, dz = dx * inv, dy * inv, dz * inv
    else:
        yw = (yaw + co).astype(f)
        pt = (pit + ro).astype(f)
        cp = np.cos(pt)
        dx = (cp * np.cos(yw)).astype(f)
        dy = (cp * np.sin(yw)).astype(f)
        dz = np.broadcast_to(np.sin(pt), dx.shape).astype(f)
    dx, dy, dz = (np.broadcast_to(a, (n, H, W)).astype(f) for a in (dx, dy, dz))
    t = np.zeros((n, H, W), f)
    alive = np.ones((n, H, W), bool)
    steps = np.zeros((n, H, W), np.int32)
    inv_cell = f(1.0 / cell)
    mn = np.asarray(mins, f)
    hit_eps, min_step = f(0.6 * cell), f(0.3 * cell)

    def vox(p, m, k):
        return np.clip((p - m) * inv_cell, 0, k - 1).astype(np.int64)

    for _ in range(max_steps):
        if not alive.any():
            break
        ix = vox(ex + dx * t, mn[0], nx)
        iy = vox(ey + dy * t, mn[1], ny)
        iz = vox(ez + dz * t, mn[2], nz)
        d = sdf[iz, iy, ix].astype(f)
        alive &= (d > hit_eps) & (t < rng)
        t = np.where(alive, t + np.maximum(d * f(0.9), min_step), t).astype(f)
        steps += alive
    t = np.minimum(t, f(rng))
    enc = (np.minimum(t, f(near)) / f(near) + f(0.25) * (f(1) - np.exp(-np.maximum(t - f(near), 0) / f(2500)))).astype(f)
    if surf_nz is not None:
        ix = vox(ex + dx * t, mn[0], nx)
        iy = vox(ey + dy * t, mn[1], ny)
        iz = vox(ez + dz * t, mn[2], nz)
        enc = np.stack([enc, surf_nz[iz, iy, ix].astype(f) * f(1.0 / 127.0)], -1)
    return (enc, steps) if return_steps else enc


def to_s2d4(img: torch.Tensor, H: int, W: int) -> torch.Tensor:
    """(N, H*W) NHW -> (N, H*W) in the 4x4 space-to-depth order."""
    n = img.shape[0]
    x = img.reshape(n, H // 4, 4, W // 4, 4).permute(0, 1, 3, 2, 4)
    return x.reshape(n, H * W)


def from_s2d4(img: torch.Tensor, H: int, W: int) -> torch.Tensor:
    n = img.shape[0]
    x = img.reshape(n, H // 4, W // 4, 4, 4).permute(0, 1, 3, 2, 4)
    return x.reshape(n, H * W)
