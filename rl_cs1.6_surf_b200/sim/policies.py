"""Non-learning policies over the multi-discrete action rows.

``ScriptedStrafer`` is the movement port's pulse check (reference
python/surfgym/policies.py:25-107): one sine cycle of yaw turning per
``period_ticks``, the strafe key matched to the turn direction (turning left
= positive yaw delta = moveleft, side bin 0). Air-strafing that gains speed on
a ramp shows that air acceleration behaves. ``RandomPolicy`` draws uniform
actions over the action vector sizes (15, 7, 3, 3, 2, 2).

Both return int32 rows [N, 6]: yaw bin, pitch bin, forward, side, jump, duck.
"""
from __future__ import annotations

from typing import Optional

import numpy as np

from .core import ACTION_DIM, NVEC

# turn per tick of each yaw bin at yaw_rate_max_deg = 10 (scaled by the config's rate)
YAW_BINS = np.array([-10.0, -7.0, -4.0, -2.0, -1.0, -0.5, -0.25, 0.0, 0.25, 0.5, 1.0, 2.0, 4.0, 7.0, 10.0])
SIDE_LEFT, SIDE_NONE, SIDE_RIGHT = 0, 1, 2
FWD_NONE = 1
PITCH_LEVEL = 3


class ScriptedStrafer:
    def __init__(self, core, period_ticks: int = 100, side_hold: int = 1) -> None:
        if period_ticks < 2:
            raise ValueError("period_ticks must be >= 2")
        self.n = int(core.num_envs)
        self.period = int(period_ticks)
        self.side_hold = int(side_hold)
        self.rate = float(core.cfg.yaw_rate_max_deg)
        self.bins = YAW_BINS * (self.rate / 10.0)
        self.rows = np.zeros((self.n, ACTION_DIM), np.int32)
        self.rows[:, 1] = PITCH_LEVEL
        self.rows[:, 2] = FWD_NONE
        self.reset()

    def reset(self) -> None:
        self.t = 0
        self.side = SIDE_LEFT
        self.still = 0

    def act(self, obs=None) -> np.ndarray:
        want = self.rate * np.sin(2.0 * np.pi * self.t / self.period)
        self.t += 1
        b = int(np.argmin(np.abs(self.bins - want)))
        turn = self.bins[b]
        if turn != 0.0:
            self.side = SIDE_LEFT if turn > 0.0 else SIDE_RIGHT
            self.still = 0
            side = self.side
        else:
            self.still += 1
            side = self.side if self.still <= self.side_hold else SIDE_NONE
        self.rows[:, 0] = b
        self.rows[:, 3] = side
        return self.rows


class RandomPolicy:
    def __init__(self, seed: Optional[int] = 0) -> None:
        self.rng = np.random.default_rng(seed)
        self.nvec = np.asarray(NVEC, np.int32)

    def act(self, obs) -> np.ndarray:
        n = int(np.asarray(obs).shape[0])
        return self.rng.integers(0, self.nvec, size=(n, ACTION_DIM), dtype=np.int32)
