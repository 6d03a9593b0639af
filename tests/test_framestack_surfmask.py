"""Frame stacking and the surface slope mask: CPU rules and GPU kernels.

Reference test strategy: tests/python/test_framestack.py (rollout ring vs
update gather equality, spawn collapse, wrap, flag-off identity) and
tests/python/test_surfmask.py (tiny synthetic triangles, channel-fastest
layout, real-map agreement). Oracles: ``framestack.stack_reference`` (torch)
and ``surfmask.surfnz_reference`` (float64 numpy, same operation order as
the kernel).
"""
import numpy as np
import pytest
import torch

from surfb200.models.policy import NetConfig, PolicyNet
from surfb200.ops import framestack as FS
from surfb200.ops import surfmask as SM


# ---- CPU: stacking rules ----------------------------------------------------------------
def test_frame_offsets():
    assert FS.frame_offsets(0) == (0,)
    assert FS.frame_offsets(1) == (0,)
    assert FS.frame_offsets(2) == (0, 1)
    assert FS.frame_offsets(5) == (0, 1, 2, 4, 8)
    with pytest.raises(ValueError):
        FS.frame_offsets(6)


def test_stack_reference_collapses_at_spawn_and_clamps():
    S, N, P = 12, 3, 8
    frames = torch.arange(S, dtype=torch.float32)[:, None, None].expand(S, N, P).clone()   # value = slot
    # env 0 age 0 (just spawned), env 1 age 2, env 2 age 9 (capped by the offsets)
    out = FS.stack_reference(frames, 4, [0, 1, 2], [10, 10, 10], [0, 2, 9]).view(3, P, 4)
    assert out[0, 0].tolist() == [10, 10, 10, 10]
    assert out[1, 0].tolist() == [10, 9, 8, 8]
    assert out[2, 0].tolist() == [10, 9, 8, 6]
    # a ring wraps the slot index
    ring = FS.stack_reference(frames[:9], 5, [2], [1], [8], ring=9).view(1, P, 5)
    assert ring[0, 0].tolist() == [1, 0, 8, 6, 2]


def test_interleave_is_pixel_major_frame_outer():
    a = torch.tensor([[1., 2., 3., 4.]])          # 2 pixels x (depth, slope)
    b = torch.tensor([[5., 6., 7., 8.]])
    assert FS.interleave([a, b], channels=2).tolist() == [[1, 2, 5, 6, 3, 4, 7, 8]]
    assert FS.interleave([a, b], channels=1).tolist() == [[1, 5, 2, 6, 3, 7, 4, 8]]


def test_policy_reference_accepts_stacked_channels():
    cfg = NetConfig(img_c=4)
    net = PolicyNet(cfg, "cpu", seed=0)
    assert net.p("conv1.w").shape == (32, 8 * 8 * 4)
    img = torch.rand(3, 64 * 128 * 4)
    out = net.forward_reference(torch.zeros(3, 16), img)
    assert out.shape == (3, cfg.out_pad) and torch.isfinite(out).all()
    # channel c of the NHWC row is input plane c: a stack of identical frames
    # through summed-per-channel weights equals one frame
    one = PolicyNet(NetConfig(), "cpu", seed=0)
    p = {n: one.p(n) for n, *_ in one.specs}
    q = {n: net.p(n).clone() for n, *_ in net.specs}
    for n in q:
        if n != "conv1.w":
            q[n] = p[n]
    q["conv1.w"] = (p["conv1.w"] / 4).repeat_interleave(4, dim=1)
    x = torch.rand(2, 64 * 128)
    a = one.forward_reference(torch.zeros(2, 16), x, p)
    b = net.forward_reference(torch.zeros(2, 16), x.repeat_interleave(4, dim=1), q)
    torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-5)


def test_config_keys_are_run_defining():
    from surfb200.trainer import checkpoint as C
    from surfb200.trainer.config import RUN_DEFINING, TrainConfig
    cfg = TrainConfig()
    assert cfg.surf_mask is False and cfg.frame_stack == 0
    for k in ("surf_mask", "frame_stack"):
        assert k in RUN_DEFINING and k in C.SHAPE_KEYS


# ---- CPU: slope-mask claim rules -------------------------------------------------------------
def _quad(z0, x0, x1, y0, y1, slope_dz=0.0):
    """Two triangles of a quad over [x0, x1] x [y0, y1] rising slope_dz along x."""
    a = [x0, y0, z0]
    b = [x1, y0, z0 + slope_dz]
    c = [x1, y1, z0 + slope_dz]
    d = [x0, y1, z0]
    return [[a, b, c], [a, c, d]]


def test_surfnz_reference_floor_ramp_wall():
    cell, dims, mins = 16.0, (16, 16, 16), (0.0, 0.0, 0.0)
    floor = np.array(_quad(64.0, 0, 256, 0, 128), np.float32)
    g = SM.surfnz_reference(floor, mins, cell, dims)
    # layers 3 and 4 (centres 56 and 72) are 8 units from z = 64: exact claims;
    # layers 2 and 5 are 24 away, beyond even the margin (16)
    assert set(np.unique(g[4, :8, :])) == {127} and g[3, 2, 2] == 127
    assert g[2, 2, 2] == 0 and g[5, 2, 2] == 0
    ramp = np.array(_quad(64.0, 0, 128, 160, 256, slope_dz=128.0), np.float32)   # 45 degrees
    g = SM.surfnz_reference(ramp, mins, cell, dims)
    assert int(np.rint(np.sqrt(0.5) * 127)) in set(np.unique(g))
    wall = np.array([[[0, 0, 0], [0, 256, 0], [0, 256, 256]]], np.float32)        # x = 0 plane
    g = SM.surfnz_reference(wall, mins, cell, dims)
    assert g.max() == 0                                      # a wall claims with value 0


def test_surfnz_reference_exact_beats_margin_then_area():
    cell, dims, mins = 16.0, (8, 8, 8), (0.0, 0.0, 0.0)
    small_floor = _quad(40.0, 32, 64, 32, 64)               # passes through the z = 2 layer (32..48)
    big_wall = [[[50.0, -500, -500], [50.0, 500, -500], [50.0, 500, 500]]]          # x = 50: exact in x-layer 3
    g = SM.surfnz_reference(np.array(small_floor + big_wall, np.float32), mins, cell, dims)
    # voxel (x=2, y=2, z=2): floor exact (|dz| = 0), wall only within margin (|dx| = 10 > 8) -> floor
    assert g[2, 2, 2] == 127
    # voxel (x=3, y=2, z=2): both exact -> the larger (wall) wins
    assert g[2, 2, 3] == 0


def test_surfnz_histogram():
    h = SM.histogram(np.array([0, 127, 60, 20, 5], np.int8))
    assert h["surfaced"] == 4 and h["flat"] == 1 and h["surfable"] == 1 and h["steep"] == 1 and h["wall"] == 1


# ---- GPU ------------------------------------------------------------------------------------------
@pytest.fixture(scope="module")
def field(field_map):
    from surfb200.sim.core import SimCore, default_config
    m, path = field_map
    return m, SimCore(str(path), default_config(1), threads=4)


@pytest.mark.gpu
def test_surfnz_bake_matches_reference_soup():
    rng = np.random.default_rng(0)
    tris = rng.uniform(0, 512, size=(60, 3, 3)).astype(np.float32)
    tris[:10] = rng.uniform(0, 64, size=(10, 3, 3))         # small ones compete with big ones
    mins, cell, dims = (-16.0, -16.0, -16.0), 16.0, (36, 34, 33)
    brk, lin = SM.bake(tris, mins, cell, dims, device="cuda")
    ref = SM.surfnz_reference(tris, mins, cell, dims)
    np.testing.assert_array_equal(lin.cpu().numpy(), ref)
    assert (ref > 0).mean() > 0.05
    # the bricked copy holds the same bytes at BrickGrid.index
    nz_, ny_, nx_ = ref.shape
    bx, by = (nx_ + 3) // 4, (ny_ + 3) // 4
    z, y, x = np.meshgrid(np.arange(nz_), np.arange(ny_), np.arange(nx_), indexing="ij")
    idx = (((z >> 2) * by + (y >> 2)) * bx + (x >> 2)) * 64 + (((z & 3) << 4) | ((y & 3) << 2) | (x & 3))
    np.testing.assert_array_equal(brk.cpu().numpy()[idx], ref)


@pytest.mark.gpu
def test_surfnz_bake_on_map_with_internal_face_filter(field):
    from surfb200.ops import vision
    m, core = field
    tris = SM.solid_triangles(core)
    assert len(tris) > 100
    mn, mx = core.map_bounds()
    mins, nx, ny, nz = vision.grid_dims(mn, mx, 32.0)
    keep = SM.internal_faces_reference(core, tris)
    assert 0 < keep.sum() < len(keep)                        # the solid-leaf mesh has buried faces
    _, lin = SM.bake(tris, mins, 32.0, (nx, ny, nz), core=core, device="cuda")
    ref = SM.surfnz_reference(tris, mins, 32.0, (nx, ny, nz), keep=keep)
    assert (lin.cpu().numpy() != ref).mean() < 1e-3        # probe points on a plane may classify differently
    h = SM.histogram(ref)
    assert h["flat"] > 0 and h["surfaced"] > 1000


@pytest.mark.gpu
def test_march_slope_channel(field):
    from surfb200.ops import vision
    from test_vision import poses_from_pool
    m, core = field
    vol = vision.SdfVolume.build(core, cell=32.0)
    brk, lin = SM.for_volume(core, vol)
    pose = poses_from_pool(m, 16, 3)
    pt = torch.as_tensor(pose, device="cuda")
    cam1 = vision.DepthCamera(vol, 64, 32, range_units=6000.0, near_range=2000.0)
    cam2 = vision.DepthCamera(vol, 64, 32, range_units=6000.0, near_range=2000.0, surf_nz=brk)
    assert cam2.frame == 2 * 64 * 32
    two = cam2.render(pt).reshape(16, 32, 64, 2)
    torch.testing.assert_close(two[..., 0], cam1.render(pt).reshape(16, 32, 64), rtol=0, atol=0)
    ref = cam2.reference(pose, surf_nz=lin.cpu().numpy())
    err = np.abs(two.cpu().numpy()[..., 1] - ref[..., 1])
    assert (err > 1e-6).mean() < 0.01
    s = two[..., 1]
    assert (s > 0).float().mean() > 0.3                     # most rays end on a claimed surface
    assert len(torch.unique((s * 127).round())) > 3         # floors, walls and slopes
    # bf16 output row layout is the same pixel-major pairs
    b16 = vision.DepthCamera(vol, 64, 32, range_units=6000.0, near_range=2000.0, surf_nz=brk,
                             dtype=torch.bfloat16).render(pt)
    torch.testing.assert_close(b16.float(), two.reshape(16, -1), atol=1e-2, rtol=1e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("K,C0", [(2, 1), (4, 1), (5, 1), (3, 2), (1, 2)])
def test_frame_stack_kernel_modes(K, C0):
    torch.manual_seed(K * 10 + C0)
    st = FS.FrameStacker(K, 64 * C0 * 4, C0)
    N, T, fr = 40, 12, st.fr
    S = st.pro + T + 1
    frames = torch.randn(S, N, fr + 8, device="cuda").to(torch.bfloat16)       # rows wider than a frame
    # mode 0: advance ages from done flags, compose decision t = 5 for envs [8, 40)
    lo, hi, t = 8, 40, 5
    age_cur = torch.randint(0, 9, (N,), dtype=torch.int32, device="cuda")
    done = (torch.rand(hi - lo, device="cuda") < 0.3).float()
    rec = torch.zeros(hi - lo, dtype=torch.int32, device="cuda")
    out = torch.zeros(hi - lo, fr * K, dtype=torch.bfloat16, device="cuda")
    a0 = age_cur.clone()
    st.rollout(frames, st.pro + t, lo, hi, done, age_cur, rec, out)
    want_age = torch.where(done > 0, 0, torch.clamp(a0[lo:hi] + 1, max=st.pro)).int()
    assert torch.equal(rec, want_age) and torch.equal(age_cur[lo:hi], want_age) and torch.equal(age_cur[:lo], a0[:lo])
    ref = FS.stack_reference(frames.cpu(), K, range(lo, hi), [st.pro + t] * (hi - lo), want_age.cpu(), fr=fr,
                             channels=C0)
    assert torch.equal(out.cpu(), ref)
    # done = None keeps the ages
    st.rollout(frames, st.pro + t, lo, hi, None, age_cur, rec, out)
    assert torch.equal(rec, want_age)
    # mode 1: terminal frames one past slot pro + t
    envs = torch.tensor([9, 3, 30], dtype=torch.int64, device="cuda")
    cur = torch.randn(3, fr, device="cuda").to(torch.bfloat16)
    out1 = torch.zeros(3, fr * K, dtype=torch.bfloat16, device="cuda")
    st.terminal(frames, st.pro + t, envs, cur, age_cur, out1)
    a1 = torch.clamp(age_cur[envs] + 1, max=st.pro).cpu()
    ref1 = FS.stack_reference(frames.cpu(), K, envs.cpu(), [st.pro + t + 1] * 3, a1, cur=cur.cpu(), fr=fr,
                              channels=C0)
    assert torch.equal(out1.cpu(), ref1)
    # mode 2: minibatch gather from recorded ages
    ages = torch.randint(0, st.pro + 1, (T * N,), dtype=torch.int32, device="cuda")
    idx = torch.randperm(T * N, device="cuda")[:100]
    out2 = torch.zeros(100, fr * K, dtype=torch.bfloat16, device="cuda")
    st.gather(frames, idx, ages, out2)
    tt, nn = (idx // N).cpu(), (idx % N).cpu()
    ref2 = FS.stack_reference(frames.cpu(), K, nn, st.pro + tt, ages.cpu()[idx.cpu()], fr=fr, channels=C0)
    assert torch.equal(out2.cpu(), ref2)


def test_space_to_depth_network_is_the_same_convolution():
    """conv1 (8x8, stride 4) on the H x W image == conv1 (2x2, stride 1) on the
    4x4 space-to-depth image with the weights in (kh', kw', r, c) order."""
    from surfb200.models.policy import space_to_depth_config
    from surfb200.ops.vision import to_s2d4
    base = NetConfig()
    s2d = space_to_depth_config(base)
    assert (s2d.img_h, s2d.img_w, s2d.img_c) == (16, 32, 16) and s2d.conv[0] == (2, 1, 32)
    assert [g["OH"] for g in s2d.conv_shapes()] == [g["OH"] for g in base.conv_shapes()]
    a, b = PolicyNet(base, "cpu", seed=0), PolicyNet(s2d, "cpu", seed=1)
    assert a.numel == b.numel
    pa = {n: a.p(n) for n, *_ in a.specs}
    pb = dict(pa)
    w = pa["conv1.w"].view(32, 2, 4, 2, 4)                      # co, kh', r, kw', c
    pb["conv1.w"] = w.permute(0, 1, 3, 2, 4).reshape(32, 64)     # co, kh', kw', r, c
    img = torch.rand(3, 64 * 128)
    ya = a.forward_reference(torch.zeros(3, 16), img, pa)
    yb = b.forward_reference(torch.zeros(3, 16), to_s2d4(img, 64, 128), pb)
    torch.testing.assert_close(ya, yb, rtol=1e-4, atol=1e-5)
    from surfb200.trainer.config import TrainConfig
    assert TrainConfig().vision_s2d and not TrainConfig.from_dict({"map": "field"}).vision_s2d
