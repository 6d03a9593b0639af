"""Adapters to the common RL environment interfaces.

The simulator autoresets in the same step (an ended env's ``obs`` row is
already the next episode's first observation; ``terminal_obs`` holds the real
last one). That is exactly the stable-baselines3 VecEnv contract, so
``SurfVecEnv`` passes it through with ``infos[i]["terminal_observation"]``.
gymnasium's vector API instead autoresets on the *next* step; the
``NextStepAutoreset`` shim converts: an ended env returns its terminal
observation now and its already-started new episode's first observation on
the following step (whose reward is 0 and flags false); the action given on
that following step is applied to the new episode's first tick.

gymnasium / stable-baselines3 are imported only when an adapter class is
first used (``from surfb200.sim.adapters import SurfVecEnv``); the module and
the shim work without either. Reference: python/surfgym/vec_env.py:35-130,
gym_env.py:51-194.
"""
from __future__ import annotations

from typing import Any, Optional

import numpy as np

from .core import NVEC

__all__ = ["NextStepAutoreset", "SurfVecEnv", "SurfGymEnv", "SurfGymVecEnv"]


class NextStepAutoreset:
    """Same-step -> next-step autoreset conversion over a SimCore batch."""

    def __init__(self, core) -> None:
        self.core = core
        self.pending: Optional[np.ndarray] = None   # envs whose new-episode obs is due next step
        self.next_obs: Optional[np.ndarray] = None

    def reset(self, seed: int = 0) -> np.ndarray:
        self.pending = None
        return self.core.reset(seed).copy()

    def step(self, actions: np.ndarray):
        obs, rew, done, trunc, term = self.core.step(np.ascontiguousarray(actions, np.int32))
        obs, rew = obs.copy(), rew.copy()
        done, trunc = done.astype(bool), trunc.astype(bool)
        if self.pending is not None and self.pending.any():
            # these envs restarted last step: report the start observation now;
            # this step's transition already belongs to the new episode
            obs[self.pending] = self.next_obs[self.pending]
            rew[self.pending] = 0.0
            done[self.pending] = False
            trunc[self.pending] = False
        ended = done | trunc
        if ended.any():
            self.next_obs = obs.copy()
            obs[ended] = term[ended]
        self.pending = ended
        return obs, rew, done, trunc


def _build() -> dict:
    import gymnasium as gym

    class SurfGymEnv(gym.Env):
        """One environment (a one-env SimCore), gymnasium API."""
        metadata = {"render_modes": []}

        def __init__(self, core) -> None:
            if core.num_envs != 1:
                raise ValueError("SurfGymEnv wraps a one-env core")
            self.core = core
            self.observation_space = gym.spaces.Box(-np.inf, np.inf, (core.obs_dim,), np.float32)
            self.action_space = gym.spaces.MultiDiscrete(list(NVEC))
            self._seed = 0

        def reset(self, *, seed: Optional[int] = None, options=None):
            if seed is not None:
                self._seed = int(seed)
            obs = self.core.reset(self._seed)[0].copy()
            self._seed += 1
            return obs, {}

        def step(self, action):
            obs, rew, done, trunc, term = self.core.step(np.asarray(action, np.int32).reshape(1, -1))
            ended = bool(done[0] or trunc[0])
            o = (term[0] if ended else obs[0]).copy()
            return o, float(rew[0]), bool(done[0]), bool(trunc[0]), {}

    class SurfGymVecEnv(gym.vector.VectorEnv):
        """The whole batch, gymnasium vector API (next-step autoreset)."""

        def __init__(self, core) -> None:
            self.core = core
            self.num_envs = core.num_envs
            self.single_observation_space = gym.spaces.Box(-np.inf, np.inf, (core.obs_dim,), np.float32)
            self.single_action_space = gym.spaces.MultiDiscrete(list(NVEC))
            self.observation_space = gym.vector.utils.batch_space(self.single_observation_space, self.num_envs)
            self.action_space = gym.vector.utils.batch_space(self.single_action_space, self.num_envs)
            self.shim = NextStepAutoreset(core)

        def reset(self, *, seed: Optional[int] = None, options=None):
            return self.shim.reset(0 if seed is None else int(seed)), {}

        def step(self, actions):
            obs, rew, done, trunc = self.shim.step(actions)
            return obs, rew, done, trunc, {}

    return {"SurfGymEnv": SurfGymEnv, "SurfGymVecEnv": SurfGymVecEnv}


def _build_sb3() -> dict:
    import gymnasium as gym
    from stable_baselines3.common.vec_env import VecEnv

    class SurfVecEnv(VecEnv):
        """stable-baselines3 VecEnv over a SimCore batch (same-step autoreset)."""

        def __init__(self, core, seed: int = 0, own_core: bool = False, reward_fn=None) -> None:
            self.core, self.reward_fn, self._seed, self._own = core, reward_fn, int(seed), own_core
            self._prev = None
            self._act = None
            super().__init__(core.num_envs, gym.spaces.Box(-np.inf, np.inf, (core.obs_dim,), np.float32),
                             gym.spaces.MultiDiscrete(list(NVEC)))

        def reset(self):
            obs = self.core.reset(self._seed).copy()
            self._prev = obs.copy()
            return obs

        def step_async(self, actions) -> None:
            self._act = np.ascontiguousarray(actions, np.int32)

        def step_wait(self):
            obs, rew, done, trunc, term = self.core.step(self._act)
            ended = (done | trunc).astype(bool)
            if self.reward_fn is not None:
                rew = np.asarray(self.reward_fn(self._prev, obs, term, rew, done, trunc, self.core), np.float32)
            self._prev = obs.copy()
            infos: list[dict[str, Any]] = [{} for _ in range(self.num_envs)]
            for i in np.flatnonzero(ended):
                infos[i]["terminal_observation"] = term[i].copy()
                if trunc[i] and not done[i]:
                    infos[i]["TimeLimit.truncated"] = True
            return obs.copy(), rew.copy(), ended, infos

        def close(self) -> None:
            if self._own:
                self.core.close()

        def seed(self, seed=None):
            if seed is not None:
                self._seed = int(seed)
            return [self._seed] * self.num_envs

        def get_attr(self, name, indices=None):
            target = self.core if hasattr(self.core, name) else self
            return [getattr(target, name)] * len(self._idx(indices))

        def set_attr(self, name, value, indices=None) -> None:
            setattr(self, name, value)

        def env_method(self, *a, **k):
            raise NotImplementedError("the batch has no per-env Python objects")

        def env_is_wrapped(self, wrapper_class, indices=None):
            return [False] * len(self._idx(indices))

        def _idx(self, indices):
            if indices is None:
                return list(range(self.num_envs))
            return [indices] if isinstance(indices, int) else list(indices)

    return {"SurfVecEnv": SurfVecEnv}


def __getattr__(name: str):
    if name in ("SurfGymEnv", "SurfGymVecEnv"):
        globals().update(_build())
        return globals()[name]
    if name == "SurfVecEnv":
        globals().update(_build_sb3())
        return globals()[name]
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
