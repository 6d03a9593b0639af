"""Trainer features on the CPU (eyeless) path: train stride, ez-greedy bursts,
fixed gaze, configuration checks and their checkpoint round trip.

Reference behaviour: --train-stride (python/train_fast.py:2162-2168), --ez-eps /
--ez-mu / --ez-max (:748-761, :1952-1971, burst rows out of the PPO pool
:2170-2177), --fix-pitch / --free-pitch (:784-785, :1320-1323, :1394),
--keep-teleports (:804), --eval-greedy-only (:852), checkpoint restore of
each (:1009-1211).
"""
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def _cfg(**kw):
    from surfb200.rewards.spec import RewardSpec
    from surfb200.trainer.config import TrainConfig
    base = dict(map="ramps", envs=16, n_steps=12, epochs=1, minibatches=4, vision=False, device="cpu", graphs=False,
                ep_ticks=300, reward=RewardSpec(mode="speed"), threads=2)
    base.update(kw)
    return TrainConfig(**base)


def test_train_pool_reference_rule():
    from surfb200.ops import rl as R
    T, n = 10, 3
    pool = R.train_pool_reference(None, T, n, 3, 1)
    t = pool // n
    assert set(t.tolist()) == {1, 4, 7} and len(pool) == 3 * n
    ez = torch.zeros(T, n, dtype=torch.uint8)
    ez[4, 1] = 1
    pool = R.train_pool_reference(ez, T, n, 3, 1)
    assert 4 * n + 1 not in pool.tolist() and len(pool) == 3 * n - 1
    assert torch.equal(pool, torch.sort(pool).values)              # row order kept


def test_ez_greedy_reference_bursts():
    from surfb200.models.policy import HeadLayout
    from surfb200.ops import rl as R
    layout = HeadLayout()
    n = 4096
    ez = R.EzGreedy(n, eps=0.05, mu=2.0, max_len=7, device="cpu")
    g = torch.Generator().manual_seed(0)
    lens, starts = [], 0
    prev_act = None
    for step in range(60):
        before = ez.left.clone()
        act = torch.full((n, 8), -1, dtype=torch.int32)
        flags = ez.apply_reference(act, layout, g).bool()
        assert torch.all(act[flags, 0] >= 0) and torch.all(act[flags, 0] < 15)
        assert torch.all(act[~flags, 0] == -1)                     # on-policy rows untouched
        cont = before > 0
        assert torch.all(flags[cont])                              # a running burst keeps going ...
        if prev_act is not None:
            assert torch.equal(act[cont, :6], prev_act[cont, :6])  # ... with the same action row
        fresh = flags & ~cont
        lens += (ez.left[fresh] + 1).tolist()                      # the drawn length of each new burst
        starts += int(fresh.sum())
        prev_act = act.clone()
    assert min(lens) >= 1 and max(lens) <= 7
    frac = float(np.mean(np.array(lens) == 1))
    assert 0.4 < frac < 0.6                                        # zeta(2): P(len = 1) = P(u > 1/2) = 1/2
    assert abs(starts / (60 * n) - 0.05 * 0.75) < 0.015           # starts only where no burst runs


def test_trainer_stride_and_ez_cpu():
    from surfb200.trainer.ppo import Trainer
    tr = Trainer(_cfg(train_stride=3, ez_eps=0.1, ez_max=5), verbose=False)
    for _ in range(3):
        s = tr.train_iteration()
        assert np.isfinite(s["policy_loss"])
        # 12 decisions / stride 3 = 4 of them, minus burst rows: at most 4 * 16 rows = one minibatch of 48
        assert tr.last_minibatches <= 1
    assert int(tr.b_ez.sum()) > 0
    tr2 = Trainer(_cfg(train_stride=2), verbose=False)
    tr2.train_iteration()
    assert tr2.last_minibatches == 2                               # 6 x 16 = 96 rows / 48 per minibatch


def test_fixed_pitch_holds_the_view():
    from surfb200.trainer.ppo import C_REC, Trainer
    tr = Trainer(_cfg(fix_pitch=-12.0), verbose=False)
    for _ in range(2):
        tr.train_iteration()
    pitch = tr.core.states_view["pitch"]
    assert np.all(pitch == np.float32(-12.0))
    assert np.all(tr.hrec.numpy()[:, C_REC + 4] == np.float32(-12.0))


@pytest.mark.parametrize("bad,msg", [(dict(train_stride=0), "train_stride"), (dict(ez_eps=0.2, ez_mu=1.0), "ez_mu"),
                                     (dict(reward_per_decision=False), "per decision"),
                                     (dict(obs_reward=True), "race"), (dict(fix_pitch=45.0), "view clamp")])
def test_config_rejects_unsupported(bad, msg):
    with pytest.raises(ValueError, match=msg):
        _cfg(**bad).validate()


def test_cli_flags_round_trip(tmp_path):
    run = tmp_path / "run"
    base = [sys.executable, str(ROOT / "surfb200.py"), "train"]
    common = ["--map", "ramps", "--envs", "16", "--n-steps", "8", "--epochs", "1", "--minibatches", "2",
              "--no-vision", "--device", "cpu", "--no-graphs", "--ep-ticks", "100", "--reward", "speed",
              "--run", str(run), "--ckpt-every", "500", "--threads", "2"]
    r = subprocess.run(base + common + ["--iterations", "1", "--train-stride", "2", "--ez-eps", "0.05",
                                        "--fix-pitch", "-8", "--keep-teleports", "--eval-greedy-only"],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    from surfb200.trainer import checkpoint as C
    cfg = C.load(run / "ckpt_final.pt")["config"]
    assert cfg["train_stride"] == 2 and cfg["ez_eps"] == 0.05 and cfg["fix_pitch"] == -8.0
    assert cfg["teleport_fail"] is False and cfg["eval_greedy_only"] is True
    r = subprocess.run(base + ["--ckpt", str(run), "--iterations", "1"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "fix_pitch" in r.stdout and "train_stride" in r.stdout          # restored from the checkpoint
    r = subprocess.run(base + ["--ckpt", str(run), "--iterations", "1", "--free-pitch"], capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "overridden fix_pitch" in r.stdout
    assert C.load(run / "ckpt_final.pt")["config"]["fix_pitch"] is None


def _ramps_core():
    from surfb200.sim import mapgen
    from surfb200.sim.core import SimCore, default_config
    m = mapgen.generate("ramps", 0)
    return SimCore.from_bytes(m.image, default_config(1), threads=2)


def test_kill_aware_goal_graph_cpu():
    """Kill volumes become walls of the goal graph only: masked voxels are
    unreachable, every masked centre is inside the trigger's hull-1 tree, and
    paths elsewhere can only get longer."""
    from surfb200.ops.geodesic import bake_goal_field, kill_voxel_mask
    from surfb200.ops.vision import grid_dims
    core = _ramps_core()
    cell = 64.0
    mn, mx = core.map_bounds()
    mins, nx, ny, nz = grid_dims(mn, mx, cell)
    kills = kill_voxel_mask(core, mins, cell, (nx, ny, nz))
    assert len(kills) == 1
    z0, y0, x0, m = kills[0]
    zi, yi, xi = np.nonzero(m)
    pts = np.stack([mins[0] + (x0 + xi + 0.5) * cell, mins[1] + (y0 + yi + 0.5) * cell,
                    mins[2] + (z0 + zi + 0.5) * cell], 1)
    assert core.trigger_contains(0, pts, usehull=1).all()
    assert pts[:, 2].max() < 65 + 36 + cell                        # the floor net, grown by the player hull only
    zone = {"mins": [-200.0, -200.0, 1200.0], "maxs": [200.0, 200.0, 1300.0]}
    plain = bake_goal_field(core, zone, cell=cell, device="cpu")
    masked = bake_goal_field(core, zone, cell=cell, device="cpu", kill_aware=True)
    gp = plain.grid.astype(np.int64)
    gm = masked.grid.astype(np.int64)
    killed = np.zeros_like(gp, bool)
    killed[z0:z0 + m.shape[0], y0:y0 + m.shape[1], x0:x0 + m.shape[2]] = m
    sent_m = int(round(masked.sentinel / masked.quant))
    assert np.all(gm[killed] == sent_m)
    assert (gp[killed] < int(round(plain.sentinel / plain.quant))).sum() > 1000    # reachable in the plain graph
    both = ~killed & (gp * plain.quant < plain.valid_max) & (gm * masked.quant < masked.valid_max)
    assert np.all(gm[both] * masked.quant >= gp[both] * plain.quant - 1e-3)


def test_euclid_goal_field_cpu():
    from surfb200.ops.geodesic import euclid_goal_field
    zone = {"mins": [100.0, -50.0, 0.0], "maxs": [300.0, 50.0, 40.0]}
    mins, cell, dims = np.array([-1024.0, -1024.0, -512.0]), 16.0, (128, 128, 64)
    f = euclid_goal_field(zone, mins, cell, dims)
    rng = np.random.default_rng(0)
    p = mins + rng.random((2000, 3)) * (np.array(dims) - 1) * cell + 0.5 * cell
    q = np.clip(p, zone["mins"], zone["maxs"])
    exact = np.linalg.norm(p - q, axis=1)
    far = exact > 3 * cell
    got = f.sample(p)
    assert np.all(np.abs(got[far] - exact[far]) < 0.06 * cell + f.quant)
    assert float(got[exact == 0].max(initial=0.0)) < cell
    assert f.grid.dtype == np.uint16 and f.reach_max > 0
