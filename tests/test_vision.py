"""Depth-vision kernels vs their CPU oracles (GPU).

Reference test strategy: tests/python/test_lidar_march.py (kernel vs an
oracle march, pose non-vacuity, batch-size independence) and
test_pinhole.py (camera geometry). Oracles here are the numpy restatement of
the march, the simulator's point-contents occupancy and scipy's EDT.
"""
import numpy as np
import pytest
import torch

from surfb200.ops import vision
from surfb200.sim.core import SimCore, default_config

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def field(field_map):
    m, path = field_map
    core = SimCore(str(path), default_config(1), threads=4)
    return m, core


def small_grid(core, cell=64.0):
    mn, mx = core.map_bounds()
    mins, nx, ny, nz = vision.grid_dims(mn, mx, cell)
    return mins, (nx, ny, nz)


def test_occupancy_matches_simulator(field):
    m, core = field
    mins, dims = small_grid(core)
    ref = vision.occupancy_reference(core, mins, 64.0, dims, slab=True)
    gpu = vision.occupancy(core, mins, 64.0, dims, slab=True).cpu().numpy()
    assert ref.sum() > 1000
    assert (ref != gpu).mean() < 1e-4      # float rounding of shifted sample points only


def test_edt_matches_scipy(field):
    m, core = field
    mins, dims = small_grid(core)
    occ = vision.occupancy(core, mins, 64.0, dims, slab=False)
    ref = vision.distance_reference(occ.cpu().numpy(), 64.0)
    gpu = vision.distance_field(occ, 64.0).cpu().numpy()
    np.testing.assert_allclose(gpu, ref, rtol=1e-5, atol=1e-2)


def poses_from_pool(m, n, seed=0):
    rng = np.random.default_rng(seed)
    rows = m.spawn_pool[rng.integers(0, len(m.spawn_pool), n)]
    pose = np.zeros((n, 8), np.float32)
    pose[:, 0:3] = rows["origin"]
    pose[:, 3] = rng.uniform(0, 360, n)
    pose[:, 4] = rng.uniform(-70, 30, n)
    pose[:, 5] = rng.integers(0, 2, n)
    return pose


@pytest.mark.parametrize("pinhole", [False, True])
def test_march_matches_oracle(field, pinhole):
    m, core = field
    vol = vision.SdfVolume.build(core, cell=32.0)
    cam = vision.DepthCamera(vol, 64, 32, range_units=6000.0, near_range=2000.0, pinhole=pinhole)
    pose = poses_from_pool(m, 16)
    out = cam.render(torch.as_tensor(pose, device="cuda")).reshape(16, 32, 64).cpu().numpy()
    ref = cam.reference(pose)
    err = np.abs(out - ref)
    assert np.median(err) < 1e-6
    assert (err > 1e-3).mean() < 0.01      # a voxel-boundary tie may step differently
    assert out.std() > 0.05                # non-vacuous: the images have structure


def test_layouts_and_dtypes(field):
    m, core = field
    vol = vision.SdfVolume.build(core, cell=32.0)
    pose = torch.as_tensor(poses_from_pool(m, 8, 1), device="cuda")
    base = vision.DepthCamera(vol, 128, 64).render(pose)
    s2d = vision.DepthCamera(vol, 128, 64, layout=vision.LAYOUT_S2D4, dtype=torch.bfloat16).render(pose)
    torch.testing.assert_close(vision.to_s2d4(base, 64, 128).to(torch.bfloat16), s2d)
    torch.testing.assert_close(vision.from_s2d4(s2d.float(), 64, 128), base, atol=1e-2, rtol=1e-2)
    # strided pose rows (a view into a wider record) and a row-strided output
    wide = torch.zeros((8, 16), device="cuda")
    wide[:, :6] = pose[:, :6]
    buf = torch.zeros((8, 128 * 64 + 100), device="cuda")
    vision.DepthCamera(vol, 128, 64).render(wide, out=buf)
    torch.testing.assert_close(buf[:, :128 * 64], base)
    # batch-size independence
    one = vision.DepthCamera(vol, 128, 64).render(pose[3:4].contiguous())
    torch.testing.assert_close(one[0], base[3])


def test_render_order_changes_nothing(field):
    """env_order (the host env's spatial order) only changes which env a run
    of blocks renders: every image is bit-identical to the plain launch."""
    m, core = field
    vol = vision.SdfVolume.build(core, cell=32.0)
    pose = torch.as_tensor(poses_from_pool(m, 64, 2), device="cuda")
    cam = vision.DepthCamera(vol, 128, 64, layout=vision.LAYOUT_S2D4, dtype=torch.bfloat16)
    base = cam.render(pose)
    order = torch.randperm(64, device="cuda").to(torch.int32)
    got = cam.render(pose, env_order=order)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), base.view(torch.int16))
    with pytest.raises(ValueError):
        cam.render(pose, env_order=order[:10])


def test_depth_accuracy_vs_exact_traces(field):
    """Median error vs exact point-hull traces stays within a voxel (16u)."""
    m, core = field
    vol = vision.SdfVolume.build(core, cell=16.0)
    rng_units = 2000.0
    cam = vision.DepthCamera(vol, 32, 16, range_units=rng_units)
    pose = poses_from_pool(m, 64, 2)
    depth = cam.render(torch.as_tensor(pose, device="cuda")).reshape(64, 16, 32).cpu().numpy() * rng_units
    col, row = cam.offsets()
    eye = pose[:, :3] + np.where(pose[:, 5:6] != 0, [0, 0, 12.0], [0, 0, 17.0])
    yaw = np.radians(pose[:, 3])[:, None, None] + col[None, None, :]
    pit = np.radians(pose[:, 4])[:, None, None] + row[None, :, None]
    d = np.stack([np.cos(pit) * np.cos(yaw), np.cos(pit) * np.sin(yaw), np.sin(pit) + 0 * yaw], -1)
    start = np.broadcast_to(eye[:, None, None, :], d.shape).reshape(-1, 3)
    res = core.trace_batch(start, start + d.reshape(-1, 3) * rng_units, hull=2)
    exact = np.where(res[:, 7] > 0, 0.0, res[:, 0] * rng_units).reshape(depth.shape)
    hit = exact < rng_units * 0.98
    err = np.abs(depth - exact)[hit]
    assert hit.mean() > 0.05
    assert np.median(err) < 16.0
