"""Random Network Distillation novelty on the 15 scalar observations.

Behaviour of the reference (python/surfgym/rnd.py:70-140): a frozen random
target MLP f and a trained predictor f' (15 -> 128 -> 128 -> 64, ReLU,
orthogonal init); bonus = mean squared difference of their outputs on
RMS-normalised inputs (clipped to +-5), divided by the running RMS of the
bonus itself and clipped to [0, 5]; the first ``warmup`` calls pay nothing.

Unlike the reference, every running statistic lives in device tensors and
``bonus`` performs no host synchronisation, so it runs inside the rollout's
CUDA graphs. The predictor trains eagerly once per iteration. RND is off by
default (the reference screened it negative); ``--rnd-coef`` enables it.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn


def _mlp(i: int, h: int, o: int) -> nn.Sequential:
    m = nn.Sequential(nn.Linear(i, h), nn.ReLU(), nn.Linear(h, h), nn.ReLU(), nn.Linear(h, o))
    for layer in m:
        if isinstance(layer, nn.Linear):
            nn.init.orthogonal_(layer.weight, math.sqrt(2))
            nn.init.zeros_(layer.bias)
    return m


class _Moments:
    """Running mean / variance over batches (parallel-variance merge), device tensors."""

    def __init__(self, dim, device):
        self.mean = torch.zeros(dim, device=device)
        self.var = torch.ones(dim, device=device)
        self.count = torch.full((), 1e-4, device=device)

    def update(self, x: torch.Tensor) -> None:
        bm = x.mean(0)
        bv = x.var(0, unbiased=False)
        bc = float(x.shape[0])                  # a Python number: no host-device copy (graph-capturable)
        delta = bm - self.mean
        tot = self.count + bc
        self.mean.add_(delta * bc / tot)
        self.var.copy_((self.var * self.count + bv * bc + delta.pow(2) * self.count * bc / tot) / tot)
        self.count.copy_(tot)


class RND:
    def __init__(self, in_dim: int = 15, feat: int = 64, hidden: int = 128, lr: float = 1e-4, warmup: int = 50,
                 device="cuda", seed: int = 0):
        self.device = torch.device(device)
        with torch.random.fork_rng(devices=[]):
            torch.manual_seed(seed)
            self.target = _mlp(in_dim, hidden, feat).to(self.device)
            self.pred = _mlp(in_dim, hidden, feat).to(self.device)
        for p in self.target.parameters():
            p.requires_grad_(False)
        self.opt = torch.optim.Adam(self.pred.parameters(), lr=lr)
        self.obs = _Moments(in_dim, self.device)
        self.bon = _Moments((), self.device)
        self.calls = torch.zeros((), device=self.device)
        self.warmup = int(warmup)

    def _norm(self, x: torch.Tensor) -> torch.Tensor:
        return ((x - self.obs.mean) / torch.sqrt(self.obs.var + 1e-8)).clamp(-5.0, 5.0)

    @torch.no_grad()
    def bonus(self, x: torch.Tensor) -> torch.Tensor:
        x = x.float()
        self.obs.update(x)
        self.calls.add_(1.0)
        xn = self._norm(x)
        err = (self.target(xn) - self.pred(xn)).pow(2).mean(1)
        self.bon.update(err)
        out = (err / torch.sqrt(self.bon.var + 1e-8)).clamp(0.0, 5.0)
        return out * (self.calls > self.warmup).float()

    def train_step(self, x: torch.Tensor) -> torch.Tensor:
        xn = self._norm(x.float().detach())
        loss = (self.target(xn) - self.pred(xn)).pow(2).mean()
        self.opt.zero_grad(set_to_none=True)
        loss.backward()
        self.opt.step()
        return loss.detach()

    def state_dict(self) -> dict:
        return {"target": self.target.state_dict(), "pred": self.pred.state_dict(), "opt": self.opt.state_dict(),
                "obs": [self.obs.mean.cpu(), self.obs.var.cpu(), self.obs.count.cpu()],
                "bon": [self.bon.mean.cpu(), self.bon.var.cpu(), self.bon.count.cpu()], "calls": self.calls.cpu()}

    def load_state_dict(self, sd: dict) -> None:
        self.target.load_state_dict(sd["target"])
        self.pred.load_state_dict(sd["pred"])
        self.opt.load_state_dict(sd["opt"])
        for m, vals in ((self.obs, sd["obs"]), (self.bon, sd["bon"])):
            m.mean.copy_(vals[0])
            m.var.copy_(vals[1])
            m.count.copy_(vals[2])
        self.calls.copy_(sd["calls"])
