"""Reward library: one spec, a GPU implementation and a numpy oracle.

Modes (reference: python/surfgym/rewards.py): ``speed``, ``avgspeed``,
``forward``, ``path``, ``maxspeed``, ``coverage`` (coverage-gated speed),
``race`` (geodesic potential shaping with success/fail/stall rules); any mode
can add count-based curiosity over hashed (cell x gaze sector x speed bin)
keys. See csrc/kernels/reward.cu for the exact rules.
"""
from .spec import MODES, RewardSpec  # noqa: F401
