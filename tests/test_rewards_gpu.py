"""surf_reward (GPU) against the numpy oracle CpuReward, every mode, on
random record sequences with teleports, episode ends and flights; plus the
env-group addressing (two half-batch calls == one full call)."""
import numpy as np
import pytest
import torch

from surfb200.rewards.spec import CpuReward, GoalFieldData, GpuReward, RewardSpec

pytestmark = pytest.mark.gpu

BOUNDS = (np.array([-4096.0, -4096.0, 0.0]), np.array([4096.0, 4096.0, 2048.0]))


def _records(n, T, seed):
    rng = np.random.default_rng(seed)
    rec = np.zeros((T + 1, n, 16), np.float32)
    pos = rng.uniform([-3000, -3000, 100], [3000, 3000, 1500], (n, 3))
    vel = rng.normal(0, 400, (n, 3))
    yaw = rng.uniform(0, 360, n)
    for t in range(T + 1):
        vel += rng.normal(0, 60, (n, 3))
        vel[:, 2] -= 24
        catch = rng.random(n) < 0.05
        vel[catch] *= 0.3                                 # ramp catches: big velocity changes
        pos += vel * 0.03
        tele = rng.random(n) < 0.01
        pos[tele] += rng.uniform(-3000, 3000, (tele.sum(), 3))
        pos = np.clip(pos, BOUNDS[0] + 10, BOUNDS[1] - 10)
        yaw = (yaw + rng.normal(0, 25, n)) % 360
        rec[t, :, 0:3] = pos
        rec[t, :, 3] = yaw
        rec[t, :, 6:9] = vel
        rec[t, :, 9] = t * 3
        rec[t, :, 10] = rng.normal(0, 0.01, n) * (rng.random(n) < 0.2)
        ended = rng.random(n) < 0.03 if t > 0 else np.zeros(n, bool)
        done = ended & (rng.random(n) < 0.7)
        rec[t, :, 11] = done
        rec[t, :, 12] = ended & ~done
        rec[t, :, 13] = done & (rng.random(n) < 0.3)
        rec[t, :, 14] = ended
        rec[t, :, 15] = rng.random(n) < 0.2
    return rec


def _field():
    nz, ny, nx = 16, 64, 64
    z, y, x = np.meshgrid(np.arange(nz), np.arange(ny), np.arange(nx), indexing="ij")
    d = (np.hypot(x - 10.0, y - 50.0) * 128.0 + z * 10.0)
    grid = np.rint(d / 16.0).astype(np.uint16)
    return GoalFieldData(grid, BOUNDS[0].copy(), 128.0, 16.0, float(d.max()))


@pytest.mark.parametrize("mode", ["speed", "avgspeed", "forward", "path", "maxspeed", "coverage", "acro", "blend",
                                  "race"])
@pytest.mark.parametrize("curiosity", [False, True])
def test_gpu_reward_matches_oracle(mode, curiosity):
    n, T, K = 512, 40, 3
    spec = RewardSpec(mode=mode, int_coef=0.25 if curiosity else 0.0, int_view=8, int_speed=8, table_log2=16,
                      blend_start=0.0, blend_end=10.0)
    field = _field() if mode == "race" else None
    d0 = 4000.0 if mode == "race" else None
    rec = _records(n, T, seed=hash(mode) % 1000)
    cpu = CpuReward(spec, n, K, BOUNDS, field, d0)
    gpu = GpuReward(spec, n, K, BOUNDS, "cuda", field, d0)
    cpu.set_step(4.0)
    gpu.set_step(4.0)
    cpu.init(rec[0].copy())
    gpu.init(torch.as_tensor(rec[0], device="cuda"))
    rew_g = torch.zeros(n, device="cuda")
    done_g = torch.zeros(n, device="cuda")
    for t in range(1, T + 1):
        r_c, d_c, _ = cpu(rec[t].copy())
        gpu(torch.as_tensor(rec[t], device="cuda"), rew_g, done_g)
        np.testing.assert_allclose(rew_g.cpu().numpy(), r_c, rtol=2e-4, atol=2e-4, err_msg=f"{mode} t={t}")
        np.testing.assert_array_equal(done_g.cpu().numpy(), d_c)
    sg, sc = gpu.pop_stats(), cpu.pop_stats()
    assert sg["episodes"] == sc["episodes"]
    if curiosity:
        assert np.array_equal(gpu.counts.cpu().numpy().astype(np.int64)[:len(cpu.counts)], cpu.counts)


def test_group_calls_equal_full_call():
    n, T, K = 256, 10, 3
    spec = RewardSpec(mode="coverage", int_coef=0.25, int_view=8, int_speed=8, table_log2=16)
    rec = _records(n, T, seed=5)
    a = GpuReward(spec, n, K, BOUNDS, "cuda")
    b = GpuReward(spec, n, K, BOUNDS, "cuda")
    a.init(torch.as_tensor(rec[0], device="cuda"))
    b.init(torch.as_tensor(rec[0], device="cuda"))
    ra, da = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    rb, db = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    h = n // 2
    for t in range(1, T + 1):
        r = torch.as_tensor(rec[t], device="cuda")
        a(r, ra, da)
        b(r[:h], rb[:h], db[:h], 0, h, counts=False)
        b(r[h:], rb[h:], db[h:], h, n, counts=False)
        b.count_all()
        torch.testing.assert_close(ra, rb)
        torch.testing.assert_close(da, db)
    assert torch.equal(a.counts, b.counts)
