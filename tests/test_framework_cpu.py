"""CPU tests of the framework plumbing: spawn pools, scripted policies,
adapters, mesh export, checkpoints / resume rules, run logs, the CLI."""
import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def field_core():
    from surfb200.sim import mapgen
    from surfb200.sim.core import SimCore, default_config
    m = mapgen.generate("field", 0)
    c = SimCore.from_bytes(m.image, default_config(4), threads=2)
    yield c
    c.close()


def test_spawn_pools(field_core):
    from surfb200.sim import spawns
    p = spawns.platform_pool(field_core)
    assert len(p) >= 1
    faces = spawns.scan_faces(field_core)
    assert len(faces[0]) > 100
    assert np.all((faces[1][:, 2] > 0.35) & (faces[1][:, 2] < 0.68))
    d = spawns.drop_pool(field_core, faces=faces)
    speed = np.hypot(d["velocity"][:, 0], d["velocity"][:, 1])
    assert len(d) > 100 and speed.min() >= 99.9 and speed.max() <= 400.1
    # every drop start is free for the player hull
    tr = field_core.trace_batch(d["origin"], d["origin"], hull=0)
    assert not tr[:, 7].any()
    r = spawns.ramp_pool(field_core, faces=faces)
    assert len(r) > 10
    mixed = spawns.mixed_pool(p, d, 0.5)
    assert abs((len(mixed) - len(d)) / len(mixed) - 0.5) < 0.1
    assert len(spawns.map_pool(field_core)) == len(field_core.spawns())


def test_scripted_strafer_gains_speed_in_air():
    """Air-strafe sync on a ramp: horizontal speed grows (air acceleration works)."""
    from surfb200.sim import mapgen
    from surfb200.sim.core import SimCore, default_config
    from surfb200.sim.policies import RandomPolicy, ScriptedStrafer
    m = mapgen.generate("ramps", 0)
    core = SimCore.from_bytes(m.image, default_config(8, spawn_mode=2, max_episode_ticks=5000), threads=2)
    core.set_spawn_pool(m.spawn_pool[:8])
    core.reset(3)
    pol = ScriptedStrafer(core, period_ticks=60)
    v0 = np.hypot(core.states_view["velocity"][:, 0], core.states_view["velocity"][:, 1]).copy()
    peak = v0.copy()
    for _ in range(300):
        core.step(pol.act(None))
        v = np.hypot(core.states_view["velocity"][:, 0], core.states_view["velocity"][:, 1])
        peak = np.maximum(peak, v)
    assert (peak > v0 + 100).mean() >= 0.5
    a = RandomPolicy(0).act(np.zeros((5, 15)))
    assert a.shape == (5, 6) and (a < np.array([15, 7, 3, 3, 2, 2])).all()
    core.close()


def test_next_step_autoreset_shim():
    from surfb200.sim import mapgen
    from surfb200.sim.adapters import NextStepAutoreset
    from surfb200.sim.core import SimCore, default_config
    m = mapgen.generate("ramps", 0)
    core = SimCore.from_bytes(m.image, default_config(4, max_episode_ticks=20), threads=1)
    shim = NextStepAutoreset(core)
    shim.reset(0)
    act = np.tile(np.array([7, 3, 1, 1, 0, 0], np.int32), (4, 1))
    saw_end = False
    for t in range(45):
        obs, rew, done, trunc = shim.step(act)
        ended = done | trunc
        if ended.any():
            saw_end = True
            obs2, rew2, done2, trunc2 = shim.step(act)
            assert not (done2[ended] | trunc2[ended]).any()
            assert np.all(rew2[ended] == 0.0)
    assert saw_end
    core.close()


def test_mesh_export(tmp_path):
    from surfb200.sim import mapgen
    from surfb200.sim.core import SimCore, default_config
    from surfb200.sim.export import export_mesh
    m = mapgen.generate("ramps", 0)
    core = SimCore.from_bytes(m.image, default_config(1), threads=1)
    doc = export_mesh(core, m.name)
    v = np.asarray(doc["vertices"]).reshape(-1, 3)
    t = np.asarray(doc["indices"]).reshape(-1, 3)
    assert len(t) > 50 and t.max() < len(v)
    # every triangle's centroid lies on solid geometry's boundary: nudging it
    # along the outward normal leaves the solid
    p0, p1, p2 = v[t[:, 0]], v[t[:, 1]], v[t[:, 2]]
    n = np.cross(p1 - p0, p2 - p0)
    area = np.linalg.norm(n, axis=1)
    ok = area > 1.0
    n = n[ok] / area[ok, None]
    c = (p0 + p1 + p2)[ok] / 3
    outside = np.array([core.point_contents(x) for x in c + 2.0 * n])
    inside = np.array([core.point_contents(x) for x in c - 2.0 * n])
    assert (inside == -2).mean() > 0.95
    assert (outside != -2).mean() > 0.6        # coplanar faces between adjacent solid cells face solid


def test_checkpoint_resolve_rules(tmp_path):
    from surfb200.trainer import checkpoint as C
    from surfb200.trainer.config import TrainConfig
    cfg = TrainConfig(envs=32, hidden=128, lr=1e-3)
    sd = {"format": C.FORMAT, "config": cfg.to_dict(), "policy": {"flat": torch.zeros(3)}}
    p = C.save(tmp_path / "ckpt_0000000001.pt", sd)
    sd2 = C.load(p)
    new, restored, changed = C.resolve_config(sd2, {"lr": 5e-4})
    assert new.hidden == 128 and new.lr == 5e-4 and "lr" in changed and "hidden" in restored
    with pytest.raises(C.CheckpointError):
        C.resolve_config(sd2, {"hidden": 256})
    bad = dict(sd2, config=dict(sd2["config"], mystery_flag=1))
    assert C.audit(bad) == ["mystery_flag"]
    assert C.find_resume(tmp_path) == p
    cad = C.Cadence(100, 60.0, start_step=250)
    assert not cad.numbered(299) and cad.numbered(300) and not cad.numbered(350) and cad.numbered(401)


def test_runlog_csv_migration(tmp_path):
    from surfb200.utils.runlog import CSV_COLS, RunLogger
    (tmp_path / "progress.csv").write_text(",".join(CSV_COLS[:8]) + "\n1,2,3,4,5,6,7,8\n")
    log = RunLogger(tmp_path, {"a": 1})
    log.log({"global_step": 10, "iteration": 1, "policy_loss": 0.1, "value_loss": 0.2, "entropy": 1.0})
    rows = (tmp_path / "progress.csv").read_text().splitlines()
    assert rows[0].split(",") == list(CSV_COLS) and len(rows) == 3
    assert len(rows[1].split(",")) == len(CSV_COLS)
    log.finish({"x": 1})
    doc = json.loads((tmp_path / "run.json").read_text())
    assert doc["config"] == {"a": 1} and "finished" in doc


def test_perf_report_parses_timing(tmp_path):
    from surfb200.utils.perf_report import parse, summarise
    p = tmp_path / "log.txt"
    p.write_text("\n".join(f"TIMING iter={i} rollout={100 + i}.0 update=50.0 total={150 + i}.0" for i in range(40)))
    s = summarise(parse(p), last=30)
    assert s["update"]["median"] == 50.0 and s["total"]["n"] == 30


def test_cli_train_resume_eval(tmp_path):
    run = tmp_path / "run"
    base = [sys.executable, str(ROOT / "surfb200.py")]
    common = ["--map", "ramps", "--envs", "16", "--n-steps", "8", "--epochs", "1", "--minibatches", "2",
              "--no-vision", "--device", "cpu", "--no-graphs", "--ep-ticks", "100", "--reward", "speed",
              "--run", str(run), "--ckpt-every", "500", "--threads", "2"]
    r = subprocess.run(base + ["train"] + common + ["--iterations", "2"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    assert (run / "ckpt_final.pt").exists() and (run / "progress.csv").exists()
    r = subprocess.run(base + ["train", "--ckpt", str(run), "--iterations", "1", "--lr", "1e-4"], capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "resumed from" in r.stdout and "overridden lr" in r.stdout
    from surfb200.trainer import checkpoint as C
    sd = C.load(run / "ckpt_final.pt")
    assert sd["global_step"] == 3 * 16 * 8 * 3 and sd["config"]["lr"] == 1e-4
    r = subprocess.run(base + ["eval", "--ckpt", str(run / "ckpt_final.pt"), "--episodes", "2", "--max-ticks", "90",
                               "--out", str(tmp_path / "t.jsonl")], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    from surfb200.trainer.evaluate import read_trajectory
    eps = read_trajectory(tmp_path / "t.jsonl")
    assert len(eps) == 2 and eps[0]["header"]["tick_ms"] == 10 and eps[0]["trailer"]["end"] in ("done", "fail", "trunc")
    assert eps[0]["ticks"].shape[1] == 15 and eps[0]["trailer"]["ticks"] == len(eps[0]["ticks"])


def test_respawn_reservoir_rules():
    from surfb200.sim.core import STATE_DTYPE
    from surfb200.trainer.respawn import RespawnReservoir
    n = 4
    r = RespawnReservoir(n, reservoir=1000, margin_ticks=300, snap_every=100, map_id="m")
    st = np.zeros(n, STATE_DTYPE)
    for t in range(10):                    # 10 decisions of 100 ticks: snapshots at ticks 100..1000
        st["origin"][:, 0] = t
        ended = np.zeros(n, bool)
        if t == 9:
            ended[0] = True                # env 0 ends at tick 1000: snapshots at <= 700 are harvestable
        r.observe(st, ended, ticks=100, step_index=t)
    assert r.commit() == 7 and r.size == 7
    assert set(r.store["origin"][:7, 0].tolist()) == set(range(7))
    pool = r.build_pool(np.zeros(3, STATE_DTYPE), pool_size=100, fresh_frac=0.1)
    assert len(pool) == 100
    sd = r.state_dict()
    r2 = RespawnReservoir(n, map_id="other")
    assert not r2.load_state_dict(sd) and r2.size == 0
    r3 = RespawnReservoir(n, map_id="m")
    assert r3.load_state_dict(sd) and r3.size == 7


def test_respawn_binned_sampling_flattens_bins():
    from surfb200.sim.core import STATE_DTYPE
    from surfb200.trainer.respawn import RespawnReservoir
    r = RespawnReservoir(1, reservoir=5000, dist_fn=lambda o: o[:, 0], dist_max=1000.0, dist_valid_max=1000.0,
                         bins=10)
    rows = np.zeros(1900, STATE_DTYPE)
    rows["origin"][:1000, 0] = np.random.default_rng(0).uniform(0, 100, 1000)    # crowded first bin
    rows["origin"][1000:, 0] = np.random.default_rng(1).uniform(100, 1000, 900)  # sparser frontier bins
    r.new_rows = [(0, i, rows[i]) for i in range(len(rows))]
    r.commit()
    pick = r.binned_pick(2000)
    d = r.d[pick]
    first = (d < 100).mean()
    assert 0.08 < first < 0.2                 # ~1/10 of draws instead of 10/19
    counts = np.bincount(np.clip((d // 100).astype(int), 0, 9), minlength=10)
    per_bin_pop = np.bincount(np.clip((r.d[:r.size] // 100).astype(int), 0, 9), minlength=10)
    assert np.all(counts <= 4 * per_bin_pop + 1)


def test_even_shares_under_caps():
    from surfb200.trainer.respawn import even_shares_under_caps as fill
    assert fill(10, np.array([100, 100, 100])).tolist() == [4, 3, 3]
    out = fill(10, np.array([1, 100, 2]))
    assert out.tolist() == [1, 7, 2]                      # capped groups keep their cap, the rest takes the demand
    assert fill(1000, np.array([3, 4])).tolist() == [3, 4]    # demand over every cap: all caps
    assert fill(0, np.array([5])).tolist() == [0]
    rng = np.random.default_rng(0)
    for _ in range(200):
        caps = rng.integers(1, 50, rng.integers(1, 12))
        n = int(rng.integers(0, 400))
        a = fill(n, caps)
        assert np.all(a <= caps) and int(a.sum()) == min(n, int(caps.sum()))
        # evenness: a group more than one draw below the largest share is at its cap
        assert np.all((a >= a.max() - 1) | (a == caps))


def test_trainer_respawn_cpu():
    from surfb200.rewards.spec import RewardSpec
    from surfb200.trainer.config import TrainConfig
    from surfb200.trainer.ppo import Trainer
    cfg = TrainConfig(map="ramps", envs=16, n_steps=32, epochs=1, minibatches=2, vision=False, device="cpu",
                      graphs=False, ep_ticks=150, reward=RewardSpec(mode="speed"), respawn_frac=0.5,
                      respawn_margin=0.3, threads=2)
    tr = Trainer(cfg, verbose=False)
    for _ in range(3):
        tr.train_iteration()
    assert tr.respawn.size > 0
    sd = tr.state_dict()
    assert sd["respawn"]["states"] is not None


def test_zone_detection_on_race_map(tmp_path):
    from surfb200.sim import mapgen, zones
    m = mapgen.generate("race", 0)
    z = zones.detect_zones(m.image)
    assert z["end"] is not None
    want = m.zones["end"]
    assert np.allclose(z["end"]["mins"], want["mins"], atol=2) and np.allclose(z["end"]["maxs"], want["maxs"], atol=2)
    kills = zones.kill_zones(m.image)
    assert len(kills) >= 1 and all(k["class"] == "trigger_teleport" for k in kills)
    ents = zones.entities(m.image)
    assert ents[0]["classname"] == "worldspawn"
    p = tmp_path / "r.bsp"
    p.write_bytes(m.image)
    doc = zones.load_zones(p)
    assert doc["source"] == "auto" and zones.zones_path(p).exists()
    manual = {"map": "r", "source": "manual", "start": None, "end": {"mins": [0, 0, 0], "maxs": [1, 1, 1]}}
    zones.zones_path(p).write_text(json.dumps(manual))
    assert zones.load_zones(p)["end"]["maxs"] == [1, 1, 1]


def test_rnd_bonus_and_training_cpu():
    from surfb200.trainer.rnd import RND
    r = RND(15, device="cpu", warmup=2, seed=0)
    x = torch.randn(512, 15)
    assert float(r.bonus(x).abs().sum()) == 0.0          # warm-up pays nothing
    r.bonus(x)
    b0 = r.bonus(x)
    assert float(b0.mean()) > 0 and float(b0.max()) <= 5.0
    loss0 = float(r.train_step(x))
    for _ in range(200):
        loss = float(r.train_step(x))
    assert loss < 0.5 * loss0                             # the predictor fits what it sees
    fresh = torch.randn(512, 15) * 3 + 5
    assert float(r.bonus(fresh).mean()) > float(r.bonus(x).mean())   # novel inputs pay more
    sd = r.state_dict()
    r2 = RND(15, device="cpu", warmup=2, seed=1)
    r2.load_state_dict(sd)
    assert torch.allclose(r2.bonus(x), r.bonus(x), atol=1e-6)
    # the target half never moves; the predictor half does
    t0 = RND(15, device="cpu", warmup=2, seed=0).nets.weights[0][0]
    assert torch.equal(r.nets.weights[0][0].detach(), t0.detach())
    assert not torch.equal(r.nets.weights[0][1].detach(), RND(15, device="cpu", seed=0).nets.weights[0][1].detach())


def test_trainer_cpu_with_rnd_and_blend():
    from surfb200.rewards.spec import RewardSpec
    from surfb200.trainer.config import TrainConfig
    from surfb200.trainer.ppo import Trainer
    cfg = TrainConfig(map="ramps", envs=16, n_steps=8, epochs=1, minibatches=2, vision=False, device="cpu",
                      graphs=False, ep_ticks=150, reward=RewardSpec(mode="blend", blend_start=0, blend_end=1000),
                      rnd_coef=0.1, threads=2)
    tr = Trainer(cfg, verbose=False)
    for _ in range(2):
        s = tr.train_iteration()
    assert np.isfinite(s["policy_loss"])
    # the RND state (networks, optimizer, statistics) rides in the checkpoint
    sd = tr.state_dict()
    assert sd["rnd"] is not None
    tr2 = Trainer(cfg, verbose=False)
    tr2.load_state_dict(sd)
    for a, b in zip(tr.rnd.nets.parameters(), tr2.rnd.nets.parameters()):
        assert torch.equal(a.detach(), b.detach())
    assert torch.equal(tr.rnd.inputs.m2, tr2.rnd.inputs.m2) and float(tr2.rnd.calls) == float(tr.rnd.calls)
    assert tr2.rnd.opt.state_dict()["state"].keys() == tr.rnd.opt.state_dict()["state"].keys()


def test_operator_tools(tmp_path):
    import threading
    import urllib.request
    from surfb200.trainer.evaluate import read_trajectory
    from surfb200.utils import tools
    from surfb200.utils.runlog import RunLogger
    p = tools.sample_trajectory(tmp_path / "s.traj.jsonl", episodes=2, ticks=50)
    eps = read_trajectory(p)
    assert len(eps) == 2 and eps[1]["ticks"].shape == (50, 15) and eps[0]["trailer"]["end"] == "done"
    for name, k in (("a", 1.0), ("b", 2.0)):
        log = RunLogger(tmp_path / "runs" / name, {"x": 1})
        for i in range(10):
            log.log({"global_step": (i + 1) * 1e6, "ep_rew_mean": k * i, "iteration": i})
    table = tools.compare_runs([tmp_path / "runs" / "a", tmp_path / "runs" / "b"], marks=(5e6,))
    assert "a" in table and "b" in table
    srv = tools.serve_metrics(tmp_path / "runs", port=0, once=True)
    th = threading.Thread(target=srv.handle_request, daemon=True)
    th.start()
    port = srv.server_address[1]
    runs = json.loads(urllib.request.urlopen(f"http://127.0.0.1:{port}/api/runs", timeout=10).read())
    assert [r["run"] for r in runs] == ["a", "b"]
    th.join(5)
    th = threading.Thread(target=srv.handle_request, daemon=True)
    th.start()
    m = json.loads(urllib.request.urlopen(f"http://127.0.0.1:{port}/api/metrics?run=b", timeout=10).read())
    assert len(m["rows"]) == 10
    th.join(5)
    srv.server_close()
    sweep = tools.env_thread_sweep("ramps", envs=64, k=3, reps=2, threads=[1, 2])
    assert len(sweep) == 2 and all(r["ticks_per_s"] > 0 for r in sweep)


def test_native_geodesic_matches_relaxation_oracle():
    """Host Dijkstra (csrc/sim/geodesic.cpp) reaches the Bellman-Ford fixed point bit for bit."""
    from surfb200.ops.geodesic import geodesic_cpu, geodesic_reference
    rng = np.random.default_rng(1)
    occ = (rng.random((10, 30, 44)) < 0.3).astype(np.uint8)
    occ[:, 15, 3:40] = 1
    occ[1:4, 1:4, 1:4] = 0
    for cell in (16.0, 37.5):
        ref = geodesic_reference(occ, cell, (1, 1, 1), (3, 3, 3))
        got = geodesic_cpu(occ, cell, (1, 1, 1), (3, 3, 3))
        assert np.array_equal(ref, got)
    assert (ref < 1e30).sum() > 1000


def _strafer_recording(tmp_path, ticks=240):
    """A ramp-map episode of the scripted strafer, written as a trajectory file."""
    from surfb200.sim import mapgen
    from surfb200.sim.core import SimCore, default_config
    from surfb200.sim.policies import ScriptedStrafer
    from surfb200.trainer.evaluate import TrajectoryWriter
    m = mapgen.generate("ramps", 0)
    core = SimCore.from_bytes(m.image, default_config(1, spawn_mode=2, max_episode_ticks=5000), threads=1)
    core.set_spawn_pool(m.spawn_pool[:1])
    core.reset(3)
    pol = ScriptedStrafer(core, period_ticks=60)
    w = TrajectoryWriter(tmp_path / "s.traj.jsonl", m.name, {})
    w.header(0)
    for t in range(ticks):
        st = core.states_view[0].copy()
        a = pol.act(None)
        _, rew, done, trunc, _ = core.step(a)
        w.tick(t, st, a[0], float(rew[0]))
        if done[0] or trunc[0]:
            break
    w.trailer("trunc", t + 1, 0.0)
    w.close()
    core.close()
    return m, tmp_path / "s.traj.jsonl"


def test_strafe_audit_and_route_bound(tmp_path):
    from surfb200.utils import tas
    _, path = _strafer_recording(tmp_path)
    e = tas.episodes(path)[0]
    a = tas.strafe_audit(e)
    assert a["ticks"] == len(e) - 1 and -1.0 <= a["capture"] <= 1.0 and a["mean_speed"] > 0
    assert 0.0 <= a["in_window"] <= 1.0
    many = tas.strafe_audit_many([e, e])
    assert many["episodes"] == 2 and abs(many["capture"] - a["capture"]) < 1e-9
    r = tas.route_bound(e, segments=4, target=1.0)
    assert r["rigorous_floor_s"] <= r["actual_s"] + 0.05
    s = [r["loss_cut_sensitivity_s"][c] for c in (0, 10, 20, 30, 40)]
    assert all(b <= a_ + 1e-9 for a_, b in zip(s, s[1:]))       # less contact loss is never slower
    assert len(r["segments"]) >= 1 and r["route_can_host_target"] in (True, False)
    # inferred actions reproduce the recorded fwd / side / yaw bins
    act = tas.infer_actions(e)
    assert act.shape == (len(e) - 1, 6) and (act[:, 0] < 15).all()


def test_tas_search_and_chain_replay_the_recording(tmp_path):
    from surfb200.sim.core import SimCore, default_config
    from surfb200.utils import tas
    m, path = _strafer_recording(tmp_path)
    e = tas.episodes(path)[0]
    core = SimCore.from_bytes(m.image, default_config(16, max_episode_ticks=1_000_000), threads=2)
    core.reset(0)
    score = lambda st: -np.asarray(st["origin"], np.float64)[:, 0]     # progress along +x
    r = tas.tas_search(core, score, e, t0=20, window=40, iters=3, p_mutate=0.1, seed=1)
    assert r["window"] == 40 and r["replay_error"] < 5.0        # restore + inferred actions track the recording
    assert r["best"] <= r["replay"] and r["actions"].shape == (40, 6)
    c = tas.tas_chain(core, score, e, window=40, iters=2, max_windows=2, seed=1)
    assert len(c["windows"]) == 2 and c["actions"].shape == (80, 6)
    core.close()


def test_phase_clock_nvtx_ranges_balance(monkeypatch):
    """SURF_NVTX=1 turns every timed block into an NVTX range (push at the
    start, pop at the end), with timing off too."""
    import torch
    from surfb200.utils.timer import PhaseClock
    calls = []
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda name: calls.append(("push", name)))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: calls.append(("pop", None)))
    monkeypatch.setenv("SURF_NVTX", "1")
    clock = PhaseClock(False, True)
    with clock.phase("update"):
        with clock.gpu("update_gpu"):
            pass
    assert calls == [("push", "update"), ("push", "update_gpu"), ("pop", None), ("pop", None)]
    monkeypatch.setenv("SURF_NVTX", "0")
    calls.clear()
    clock = PhaseClock(True, False)
    clock.new_iteration()
    with clock.phase("env"):
        pass
    with clock.phase("env"):
        pass
    got = clock.collect()
    assert calls == [] and set(got) == {"env", "total"} and got["total"] >= got["env"] >= 0.0
    line = PhaseClock.timing_line(3, {"env": 1.25, "total": 2.0})
    assert line == "TIMING iter=3 env=1.2 total=2.0"
