"""The stable-baselines3 VecEnv adapter (sim/adapters.py:SurfVecEnv) on a
real simulator batch, with gymnasium's spaces and SB3's VecEnv base class
replaced by minimal stand-ins (neither package is installed here). The
stand-ins reproduce the parts of the SB3 contract the adapter relies on:
VecEnv.__init__(num_envs, observation_space, action_space) and step() =
step_async() + step_wait(). Checked: shapes and dtypes, same-step autoreset
with ``terminal_observation`` and ``TimeLimit.truncated`` in the infos (the
reference's SurfVecEnv contract, python/surfgym/vec_env.py:80-95), the custom reward
hook, seed / get_attr / env_is_wrapped."""
import importlib
import sys
import types

import numpy as np
import pytest


class _Box:
    def __init__(self, low, high, shape, dtype):
        self.low, self.high, self.shape, self.dtype = low, high, shape, dtype


class _MultiDiscrete:
    def __init__(self, nvec):
        self.nvec = np.asarray(nvec)


class _VecEnv:
    def __init__(self, num_envs, observation_space, action_space):
        self.num_envs = num_envs
        self.observation_space = observation_space
        self.action_space = action_space

    def step(self, actions):
        self.step_async(actions)
        return self.step_wait()


@pytest.fixture
def sb3_stubs(monkeypatch):
    gym = types.ModuleType("gymnasium")
    gym.spaces = types.SimpleNamespace(Box=_Box, MultiDiscrete=_MultiDiscrete)
    vec_env = types.ModuleType("stable_baselines3.common.vec_env")
    vec_env.VecEnv = _VecEnv
    common = types.ModuleType("stable_baselines3.common")
    common.vec_env = vec_env
    sb3 = types.ModuleType("stable_baselines3")
    sb3.common = common
    for name, mod in (("gymnasium", gym), ("stable_baselines3", sb3), ("stable_baselines3.common", common),
                      ("stable_baselines3.common.vec_env", vec_env)):
        monkeypatch.setitem(sys.modules, name, mod)
    import surfb200.sim.adapters as ad
    ad = importlib.reload(ad)              # the adapter classes are built on first use, against the stubs
    yield ad
    importlib.reload(ad)


def _core(n, ticks):
    from surfb200.sim import mapgen
    from surfb200.sim.core import SimCore, default_config
    m = mapgen.generate("ramps", 0)
    return SimCore.from_bytes(m.image, default_config(n, max_episode_ticks=ticks), threads=1)


def test_vecenv_contract(sb3_stubs):
    from surfb200.sim.core import NVEC
    core = _core(4, 20)
    env = sb3_stubs.SurfVecEnv(core, seed=3, own_core=True)
    assert isinstance(env, _VecEnv) and env.num_envs == 4
    assert env.observation_space.shape == (core.obs_dim,)
    assert list(env.action_space.nvec) == list(NVEC)
    obs = env.reset()
    assert obs.shape == (4, core.obs_dim) and obs.dtype == np.float32
    act = np.tile(np.array([7, 3, 1, 1, 0, 0], np.int32), (4, 1))
    saw_trunc = False
    for _ in range(45):
        obs, rew, dones, infos = env.step(act)
        assert obs.shape == (4, core.obs_dim) and rew.shape == (4,) and dones.dtype == bool and len(infos) == 4
        for i in np.flatnonzero(dones):
            term = infos[i]["terminal_observation"]
            assert term.shape == (core.obs_dim,)
            saw_trunc |= bool(infos[i].get("TimeLimit.truncated", False))
        for i in np.flatnonzero(~dones):
            assert "terminal_observation" not in infos[i]
    assert saw_trunc                       # the 20-tick limit truncates every episode
    assert env.seed(11) == [11] * 4
    assert env.get_attr("num_envs", [0, 2]) == [4, 4]
    assert env.env_is_wrapped(object) == [False] * 4
    with pytest.raises(NotImplementedError):
        env.env_method("anything")
    env.close()


def test_vecenv_reward_hook(sb3_stubs):
    core = _core(2, 100)
    seen = []

    def reward_fn(prev, obs, term, rew, done, trunc, c):
        seen.append((prev.shape, obs.shape))
        return np.full(c.num_envs, 0.5, np.float32)

    env = sb3_stubs.SurfVecEnv(core, reward_fn=reward_fn, own_core=True)
    env.reset()
    _, rew, _, _ = env.step(np.zeros((2, 6), np.int32))
    assert np.all(rew == 0.5) and seen == [((2, core.obs_dim), (2, core.obs_dim))]
    env.close()
