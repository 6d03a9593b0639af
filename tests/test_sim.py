"""Simulator tests: binding layout, analytic physics gates, step_k semantics,
and tick-for-tick parity with the reference core built from source.

Reference test strategy: tests/test_physics.c, tests/test_trace.c and
python/tests/test_binding.py (analytic gates + layout checks); the parity
test replaces "trust the transcription" with a bit-exact comparison.
"""
import ctypes
import math

import numpy as np
import pytest

from surfb200.sim import mapgen
from surfb200.sim.core import (NVEC, REC, REC_COLS, STATE_DTYPE, EnvConfig, Physics, PlayerState, SimCore, default_config,
                               validate_actions)
from surfb200.sim.parity import RefCore, reference_available


def random_actions(rng, n):
    return np.stack([rng.integers(0, k, n) for k in NVEC], 1).astype(np.int32)


def test_layouts():
    assert ctypes.sizeof(Physics) == 60
    assert ctypes.sizeof(EnvConfig) == 128
    assert ctypes.sizeof(PlayerState) == STATE_DTYPE.itemsize == 108
    cfg = default_config(4, sv_gravity=790, lidar_w=8, lidar_h=4)
    assert cfg.num_envs == 4 and cfg.phys.sv_gravity == 790 and cfg.lidar_w == 8
    with pytest.raises(TypeError):
        default_config(1, not_a_field=1)


def test_validate_actions():
    validate_actions(np.zeros((3, 6), np.int32), 3)
    with pytest.raises(ValueError):
        validate_actions(np.zeros((3, 6), np.int64), 3)
    with pytest.raises(ValueError):
        validate_actions(np.zeros((2, 6), np.int32), 3)


def test_procedural_maps_compile(field_map, ramps_map):
    m, path = field_map
    core = SimCore(str(path), default_config(1), threads=1)
    c = core.map_counts()
    assert c["clipnodes"] < 32768 and c["nodes"] < 32768
    assert m.meta["n_brushes"] == 512
    mn, mx = core.map_bounds()
    assert mx[2] - mn[2] > 3000
    # spawn pool: every entry is free for the standing hull
    for row in m.spawn_pool[:64]:
        assert not core.trace(row["origin"], row["origin"], hull=0).startsolid


def test_ramp_faces_are_surfable(ramps_map):
    """Down-traces onto the generated ramps hit faces with 0 < n_z < 0.7."""
    m, path = ramps_map
    core = SimCore(str(path), default_config(1), threads=1)
    for r in m.ramps:
        p = r.face_point(0.0, 1.0, 0.5) + np.array([0, 0, 200.0])
        tr = core.trace(p, p - np.array([0, 0, 400.0]), hull=2)
        assert tr.fraction < 1.0
        assert 0.5 < tr.normal[2] < 0.7, tr.normal


def _drop(core, origin, ticks, **kw):
    st = PlayerState()
    st.origin[:] = origin
    st.onground = -1
    out = []
    for _ in range(ticks):
        core.pm_step_usercmd(st, kw.get("yaw", 0.0), 0.0, kw.get("fmove", 0.0), kw.get("smove", 0.0),
                             kw.get("buttons", 0), 10)
        out.append((np.array(st.origin), np.array(st.velocity), st.onground))
    return st, out


def test_gravity_and_landing(ramps_map):
    """Free fall follows v_z = -800 t (split half-gravity), then lands and stops."""
    m, path = ramps_map
    core = SimCore(str(path), default_config(1), threads=1)
    st, traj = _drop(core, (0.0, 0.0, 2200.0), 10)
    # after n ticks in air: v_z = -8 * n (800 u/s^2 * 10 ms)
    assert traj[4][1][2] == pytest.approx(-40.0, abs=1e-3)
    # a spot over the open floor (kill net disabled in pm-only stepping)
    mn, mx = core.map_bounds()
    p = (mx[0] - 100.0, mx[1] - 300.0, 200.0)
    st, traj = _drop(core, p, 200)
    assert traj[-1][2] != -1                      # on ground
    assert abs(traj[-1][1][2]) < 1e-6
    assert traj[-1][0][2] == pytest.approx(36.0, abs=0.05)   # hull half-height above z=0


def test_jump_apex(ramps_map):
    m, path = ramps_map
    core = SimCore(str(path), default_config(1, enable_stamina=0), threads=1)
    mn, mx = core.map_bounds()
    p = (mx[0] - 100.0, mx[1] - 300.0, 40.0)
    st, _ = _drop(core, p, 50)
    z0 = st.origin[2]
    apex = z0
    for i in range(80):
        core.pm_step_usercmd(st, 0.0, 0.0, 0.0, 0.0, 2 if i == 0 else 0, 10)
        apex = max(apex, st.origin[2])
    # v0 = sqrt(2*800*45) -> apex ~45u (discrete integration lands within a unit)
    assert 44.0 < apex - z0 < 46.5


def test_ramp_slide_gains_speed(ramps_map):
    """No input on a surf ramp: never grounded (n_z < 0.7), speed increases."""
    m, path = ramps_map
    core = SimCore(str(path), default_config(1), threads=1)
    r = m.ramps[0]
    p = r.face_point(0.0, 1.0, 0.3) + np.array([0, 0, 60.0])
    st, traj = _drop(core, p, 120)
    speeds = [float(np.hypot(v[0], v[1])) for _, v, _ in traj]
    assert all(g == -1 for _, _, g in traj)
    assert speeds[-1] > 150.0 and speeds[-1] > speeds[40]


def test_air_strafe_accelerates(ramps_map):
    """Air strafing with the view turning at the optimal rate gains speed."""
    m, path = ramps_map
    core = SimCore(str(path), default_config(1), threads=1)
    st = PlayerState()
    st.origin[:] = (0.0, 0.0, 2300.0)
    st.velocity[:] = (300.0, 0.0, 0.0)
    st.onground = -1
    yaw = 0.0
    for _ in range(30):
        v = math.hypot(st.velocity[0], st.velocity[1])
        yaw += math.degrees(math.atan(30.0 / v))
        core.pm_step_usercmd(st, yaw, 0.0, 0.0, -400.0, 0, 10)
    assert math.hypot(st.velocity[0], st.velocity[1]) > 330.0


def test_step_k_equals_sequential_steps(field_map):
    m, path = field_map
    n = 64
    cfg = default_config(n, max_episode_ticks=90, spawn_mode=2)
    a = SimCore(str(path), cfg, threads=2)
    b = SimCore(str(path), cfg, threads=2)
    for c in (a, b):
        c.set_spawn_pool(m.spawn_pool)
        c.set_teleport_fail(True)
        c.reset(5)
    rng = np.random.default_rng(0)
    for _ in range(40):
        act = random_actions(rng, n)
        obs_k, _, rec, _ = a.step_k_numpy(act, 3)
        rsum = np.zeros(n, np.float32)
        ended = np.zeros(n, bool)
        for _ in range(3):
            o, r, d, t, _ = b.step(act)
            rsum += r
            ended |= (d | t).astype(bool)
        assert a.states_view.tobytes() == b.states_view.tobytes()
        np.testing.assert_array_equal(obs_k, o)
        np.testing.assert_array_equal(rec[:, REC["ended"]] > 0, ended)
        np.testing.assert_allclose(rec[:, REC["reward"]], rsum, rtol=0, atol=1e-6)


def test_async_group_steps_match_sync(field_map):
    """Two env groups stepped with step_k_range_async / step_wait (the
    rollout's overlap of one group's stepping with the other's launches) give
    the same states and rows as synchronous step_k_range calls."""
    m, path = field_map
    n, K = 96, 3
    cfg = default_config(n, max_episode_ticks=120, spawn_mode=2)
    a = SimCore(str(path), cfg, threads=3)
    b = SimCore(str(path), cfg, threads=3)
    for c in (a, b):
        c.set_spawn_pool(m.spawn_pool)
        c.set_teleport_fail(True)
        c.reset(9)
    rows = [np.zeros((n, 8), np.int32) for _ in range(2)]
    outs = [(np.zeros((n, c.obs_dim), np.float32), np.zeros((n, REC_COLS), np.float32)) for c in (a, b)]
    rng = np.random.default_rng(4)
    groups = [(0, 40), (40, n)]
    for _ in range(30):
        act = random_actions(rng, n)
        for r in rows:
            r[:, :6] = act
        for (lo, hi) in groups:
            for c, r, (obs, rec), run in ((a, rows[0], outs[0], "async"), (b, rows[1], outs[1], "sync")):
                kw = dict(obs=(obs.ctypes.data, c.obs_dim), rec=(rec.ctypes.data, REC_COLS))
                if run == "async":
                    c.step_k_range_async(lo, hi, r.ctypes.data, 8, K, **kw)
                else:
                    c.step_k_range(lo, hi, r.ctypes.data, 8, K, **kw)
        a.step_wait()
        assert a.states_view.tobytes() == b.states_view.tobytes()
        np.testing.assert_array_equal(outs[0][0], outs[1][0])
        np.testing.assert_array_equal(outs[0][1], outs[1][1])


def test_env_order_is_a_permutation(field_map):
    """The visiting order the host env exports for a range (the render order
    of its depth images): the identity before the range's first step, a
    permutation of the range's offsets after it."""
    m, path = field_map
    n = 96
    core = SimCore(str(path), default_config(n, spawn_mode=2), threads=2)
    core.set_spawn_pool(m.spawn_pool)
    core.reset(3)
    out = np.full(n, -1, np.int32)
    core.env_order(16, 80, out[16:].ctypes.data)
    np.testing.assert_array_equal(out[16:80], np.arange(64))
    rows = np.zeros((n, 8), np.int32)
    rows[:, :6] = random_actions(np.random.default_rng(1), n)
    core.step_k_range(16, 80, rows.ctypes.data, 8, 3)
    core.env_order(16, 80, out[16:].ctypes.data)
    assert sorted(out[16:80].tolist()) == list(range(64))
    assert (out[:16] == -1).all() and (out[80:] == -1).all()


def test_continuous_yaw(field_map):
    m, path = field_map
    core = SimCore(str(path), default_config(4, spawn_mode=2, yaw_jitter_deg=0.0), threads=1)
    core.set_spawn_pool(m.spawn_pool[:1])
    core.reset(0)
    y0 = core.states_view["yaw"].copy()
    act = np.zeros((4, 6), np.int32)
    act[:, 1] = 3
    act[:, 2:4] = 1
    yaw = np.array([1.0, -1.0, 0.5, 3.0], np.float32)          # last one is clamped to 1
    core.step_k_numpy(act, 2, yaw=yaw)
    d = (core.states_view["yaw"] - y0 + 540.0) % 360.0 - 180.0
    np.testing.assert_allclose(d, [20.0, -20.0, 10.0, 20.0], atol=1e-3)


needs_ref = pytest.mark.skipif(not reference_available(), reason="reference core not built in baseline/_ref")


@needs_ref
@pytest.mark.parametrize("kind", ["ramps", "field", "race"])
def test_parity_with_reference_core(kind, maps_dir):
    m = mapgen.generate(kind, 0)
    path = str(m.save(maps_dir))
    n = 128
    cfg = default_config(n, max_episode_ticks=300, spawn_mode=2, yaw_jitter_deg=8.0)
    a = SimCore(path, cfg, threads=2)
    b = RefCore(path, cfg)
    for c in (a, b):
        c.set_spawn_pool(m.spawn_pool)
        c.set_teleport_fail(True)
    if m.zones.get("end"):
        z = m.zones["end"]
        a.set_goal_box(z["mins"], z["maxs"])
        b.set_goal_box(z["mins"], z["maxs"])
    np.testing.assert_array_equal(a.reset(11), b.reset(11))
    rng = np.random.default_rng(3)
    for _ in range(600):
        act = random_actions(rng, n)
        ra, rb = a.step(act), b.step(act)
        assert a.states_view.tobytes() == b.states_view.tobytes()
        for x, y in zip(ra, rb):
            np.testing.assert_array_equal(x, y)
    mn, mx = a.map_bounds()
    for _ in range(500):
        s = rng.uniform(mn, mx)
        e = s + rng.normal(0, 400, 3)
        for hull in (0, 1, 2):
            x, y = a.trace(s, e, hull), b.trace(s, e, hull)
            assert x.fraction == y.fraction and x.startsolid == bool(y.startsolid)
            np.testing.assert_array_equal(x.endpos, np.array(y.endpos, np.float32))
        assert a.point_contents(s) == b.point_contents(s)


@needs_ref
def test_parity_real_map(ski_map):
    """The reference's own community map (BSP v30 from the hlcsg toolchain)."""
    n = 128
    cfg = default_config(n, max_episode_ticks=700, spawn_mode=0, yaw_jitter_deg=8.0, lidar_w=8, lidar_h=4)
    a = SimCore(str(ski_map), cfg, threads=2)
    b = RefCore(str(ski_map), cfg)
    np.testing.assert_array_equal(a.reset(123), b.reset(123))
    rng = np.random.default_rng(0)
    for _ in range(400):
        act = random_actions(rng, n)
        ra, rb = a.step(act), b.step(act)
        assert a.states_view.tobytes() == b.states_view.tobytes()
        for x, y in zip(ra, rb):
            np.testing.assert_array_equal(x, y)


def test_native_gates_executable():
    """The C++ acceptance gates (load, traces, physics, single-thread throughput)."""
    import subprocess
    from surfb200 import _build
    _build.build(only=["surfsim_gates"], verbose=False)
    r = subprocess.run([str(_build.LIB / "surfsim_gates")], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "OK: 0 failed" in r.stdout
