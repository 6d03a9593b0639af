"""Self-describing checkpoints and the resume rules.

A checkpoint is one ``torch.save`` dict (reference layout,
python/train_fast.py:1822-1835): ``policy`` (flat fp32 master weights + the
network configuration), ``optimizer`` (Adam m / v / hyper-parameters, the
full arrays even when the optimizer state is sharded across ranks),
``global_step`` (physics ticks, all ranks), ``iteration``, ``config`` (the
complete ``TrainConfig``), ``int_counts`` (curiosity table, uint32) and
``respawn`` (reservoir rows). ``format`` names the schema version.

Resume (reference restore logic, train_fast.py:1009-1306): a bare
``--ckpt`` restores every run-defining setting from the checkpoint; a flag
given on the command line wins, except for the settings that change the
network's tensor shapes (sensor geometry, heads, widths), which are refused
because the weights could not be loaded.

Files: ``ckpt_<global_step:010d>.pt`` at the ``ckpt_every`` cadence,
``ckpt_latest.pt`` at least every 60 s (crash recovery) and
``ckpt_final.pt`` at the end, each written to a temporary name and renamed
so that a reader never sees a torn file.
"""
from __future__ import annotations

import os
from pathlib import Path
from typing import Iterable, Optional

import torch

from .config import RUN_DEFINING, TrainConfig

FORMAT = "surfb200-ckpt-1"

# keys whose change alters parameter shapes: never overridden on resume
SHAPE_KEYS = ("vision", "lidar_w", "lidar_h", "vision_s2d", "surf_mask", "frame_stack", "heads", "continuous_yaw", "gps", "hidden",
              "fc", "proprio", "mlp")


class CheckpointError(RuntimeError):
    pass


def save(path, state: dict) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + ".tmp")
    torch.save(state, tmp)
    os.replace(tmp, path)
    return path


def load(path) -> dict:
    sd = torch.load(Path(path), map_location="cpu", weights_only=False)
    fmt = sd.get("format")
    if fmt != FORMAT:
        raise CheckpointError(f"{path}: unknown checkpoint format {fmt!r} (expected {FORMAT})")
    return sd


def audit(sd: dict) -> list:
    """Keys of the stored configuration this build does not know (a
    recording or resume from such a checkpoint would silently drop them)."""
    known = set(TrainConfig.__dataclass_fields__)
    return sorted(k for k in sd.get("config", {}) if k not in known)


def resolve_config(sd: dict, overrides: dict) -> tuple:
    """(TrainConfig, restored keys, overridden keys) for a resume.

    ``overrides`` holds only the flags the user gave explicitly."""
    unknown = audit(sd)
    if unknown:
        raise CheckpointError(f"checkpoint config has settings this build does not mirror: {unknown}")
    stored = sd["config"]
    cfg = TrainConfig.from_dict(stored)
    restored, changed = [], []
    for k in RUN_DEFINING:
        if k in overrides and k in stored:
            new, old = overrides[k], stored[k]
            if k == "reward":
                new = new.to_dict() if hasattr(new, "to_dict") else new
            if _norm(new) != _norm(old):
                if k in SHAPE_KEYS:
                    raise CheckpointError(f"--{k.replace('_', '-')} {new!r} conflicts with the checkpoint's {old!r}: "
                                          f"it changes the network's shapes")
                changed.append(k)
        elif k in stored:
            restored.append(k)
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg, restored, changed


def _norm(v):
    if isinstance(v, (list, tuple)):
        return [_norm(x) for x in v]
    if isinstance(v, dict):
        return {k: _norm(x) for k, x in v.items()}
    return v


class Cadence:
    """When to write numbered / latest checkpoints (identical on every rank:
    the time-based latest checkpoint is decided by rank 0 and shared)."""

    def __init__(self, every_steps: float, latest_s: float = 60.0, start_step: int = 0):
        self.every = float(every_steps)
        self.latest_s = float(latest_s)
        self.next_step = (start_step // self.every + 1) * self.every if self.every > 0 else float("inf")
        self.last_latest = None

    def numbered(self, step: int) -> bool:
        if step >= self.next_step:
            while self.next_step <= step:
                self.next_step += self.every
            return True
        return False

    def latest_due(self, now: float) -> bool:
        if self.last_latest is None:
            self.last_latest = now
            return False
        if now - self.last_latest >= self.latest_s:
            self.last_latest = now
            return True
        return False


def checkpoint_files(run_dir) -> list:
    return sorted(Path(run_dir).glob("ckpt_*.pt"))


def find_resume(path) -> Optional[Path]:
    """A checkpoint path, or a run directory (its ckpt_latest / newest file)."""
    p = Path(path)
    if p.is_file():
        return p
    if p.is_dir():
        for name in ("ckpt_latest.pt", "ckpt_final.pt"):
            if (p / name).exists():
                return p / name
        files = [f for f in checkpoint_files(p) if f.name[5:15].isdigit()]
        return files[-1] if files else None
    return None


def iter_state_tensors(sd: dict) -> Iterable:
    yield sd["policy"]["flat"]
    for k in ("m", "v"):
        if k in sd.get("optimizer", {}):
            yield sd["optimizer"][k]
