"""Random Network Distillation novelty on the 15 scalar observations.

Behaviour of the reference (python/surfgym/rnd.py:70-140), the method of
Burda et al., "Exploration by Random Network Distillation" (2018): a frozen
random target network f and a trained predictor f' of the same shape
(15 -> 128 -> 128 -> 64, ReLU, orthogonal init with gain sqrt 2, zero
biases); bonus = mean squared difference of their outputs on running-RMS
normalised inputs (clipped to +-5), divided by the running RMS of the bonus
itself and clipped to [0, 5]; the first ``warmup`` calls pay nothing.

Design here: the two networks are one ``TwinMLP`` whose weights are stacked
on a leading axis of size 2 (index 0 = frozen target, 1 = predictor), so a
bonus evaluates both with one batched matmul per layer; only the predictor
slices receive gradients. Every running statistic is a device tensor kept as
(count, mean, M2) and merged batch by batch with the pairwise update of Chan,
Golub and LeVeque ("Updating formulae and a pairwise algorithm for computing
sample variances", 1979), so ``bonus`` makes no host synchronisation and
runs inside the rollout's CUDA graphs. RND is off by default (the reference
screened it negative); ``--rnd-coef`` enables it. Its full state (both
networks, the predictor's optimizer, all statistics) is checkpointed.
"""
from __future__ import annotations

import math

import torch


class TwinMLP(torch.nn.Module):
    """Target and predictor MLPs with stacked weights: ``forward(x)`` returns
    [2, B, out] (target, predictor)."""

    def __init__(self, dims=(15, 128, 128, 64), generator: torch.Generator = None):
        super().__init__()
        self.weights = torch.nn.ParameterList()
        self.biases = torch.nn.ParameterList()
        for fan_in, fan_out in zip(dims[:-1], dims[1:]):
            w = torch.empty(2, fan_in, fan_out)
            for k in range(2):
                blk = torch.empty(fan_out, fan_in)
                torch.nn.init.orthogonal_(blk, gain=math.sqrt(2.0), generator=generator)
                w[k] = blk.t()
            self.weights.append(torch.nn.Parameter(w))
            self.biases.append(torch.nn.Parameter(torch.zeros(2, 1, fan_out)))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = x.unsqueeze(0).expand(2, -1, -1)
        last = len(self.weights) - 1
        for i, (w, b) in enumerate(zip(self.weights, self.biases)):
            h = torch.baddbmm(b, h, w)
            if i < last:
                h = torch.relu(h)
        return h

    def predictor_parameters(self):
        return list(self.weights) + list(self.biases)


class RunningMoments:
    """Mean and population variance of everything seen so far, per feature."""

    def __init__(self, shape, device):
        self.n = torch.full((), 1e-4, device=device)           # a tiny prior count: var starts at 1
        self.mean = torch.zeros(shape, device=device)
        self.m2 = torch.full(shape, 1e-4, device=device)        # sum of squared deviations (= var * n)

    @property
    def var(self) -> torch.Tensor:
        return self.m2 / self.n

    def merge(self, x: torch.Tensor) -> None:
        nb = float(x.shape[0])                  # a Python number: no device-to-host copy
        mb = x.mean(0)
        m2b = (x - mb).pow(2).sum(0)
        n = self.n + nb
        delta = mb - self.mean
        self.m2.add_(m2b + delta.pow(2) * (self.n * nb / n))
        self.mean.add_(delta * (nb / n))
        self.n.copy_(n)

    def tensors(self) -> list:
        return [self.n, self.mean, self.m2]


class RND:
    def __init__(self, in_dim: int = 15, feat: int = 64, hidden: int = 128, lr: float = 1e-4, warmup: int = 50,
                 device="cuda", seed: int = 0):
        self.device = torch.device(device)
        gen = torch.Generator().manual_seed(seed)
        self.nets = TwinMLP((in_dim, hidden, hidden, feat), gen).to(self.device)
        self.opt = torch.optim.Adam(self.nets.predictor_parameters(), lr=lr)
        self.inputs = RunningMoments((in_dim,), self.device)
        self.errors = RunningMoments((), self.device)
        self.calls = torch.zeros((), device=self.device)
        self.warmup = int(warmup)

    def _whiten(self, x: torch.Tensor) -> torch.Tensor:
        return ((x - self.inputs.mean) * torch.rsqrt(self.inputs.var + 1e-8)).clamp(-5.0, 5.0)

    def _sq_error(self, xn: torch.Tensor) -> torch.Tensor:
        tp = self.nets(xn)
        return (tp[0].detach() - tp[1]).pow(2).mean(-1)

    @torch.no_grad()
    def bonus(self, x: torch.Tensor) -> torch.Tensor:
        """Per-row novelty of a batch; updates the running statistics."""
        x = x.float()
        self.inputs.merge(x)
        self.calls.add_(1.0)
        err = self._sq_error(self._whiten(x))
        self.errors.merge(err)
        scaled = (err * torch.rsqrt(self.errors.var + 1e-8)).clamp(0.0, 5.0)
        return scaled * (self.calls > self.warmup).to(scaled.dtype)

    def train_step(self, x: torch.Tensor) -> torch.Tensor:
        """One predictor update on a batch of observations; returns the loss."""
        loss = self._sq_error(self._whiten(x.float().detach())).mean()
        self.opt.zero_grad(set_to_none=True)
        loss.backward()
        # the target half of every stacked tensor stays frozen
        for p in self.nets.predictor_parameters():
            if p.grad is not None:
                p.grad[0].zero_()
        self.opt.step()
        return loss.detach()

    def state_dict(self) -> dict:
        return {"nets": {k: v.detach().cpu() for k, v in self.nets.state_dict().items()},
                "opt": self.opt.state_dict(),
                "inputs": [t.cpu() for t in self.inputs.tensors()],
                "errors": [t.cpu() for t in self.errors.tensors()], "calls": self.calls.cpu()}

    def load_state_dict(self, sd: dict) -> None:
        self.nets.load_state_dict({k: v.to(self.device) for k, v in sd["nets"].items()})
        self.opt.load_state_dict(sd["opt"])
        for mom, vals in ((self.inputs, sd["inputs"]), (self.errors, sd["errors"])):
            for dst, src in zip(mom.tensors(), vals):
                dst.copy_(src.to(self.device))
        self.calls.copy_(sd["calls"].to(self.device))
