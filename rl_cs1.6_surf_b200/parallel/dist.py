"""Data-parallel plumbing (one process per GPU, torch.distributed).

Reference design (the reference never built it): docs/ddp-plan.md — flat
gradient all-reduce after backward and before the clip (:404-434), global
advantage moments per epoch (:78-166), curiosity count deltas all-reduced
(:174-225), parameter broadcast at start (:355-380), rank-distinct seeds
(:333-353).

``NcclComm`` is the library baseline: torch.distributed collectives (NCCL on
GPUs, gloo on CPU) followed by the single-GPU fused clip + Adam.
``make_comm("p2p")`` returns the product path, ``P2PComm``
(parallel/p2p.py): fused NVLink kernels that reduce-scatter the gradient,
clip by the global norm, run Adam on the owned shard and push the updated
parameters to every peer.
"""
from __future__ import annotations

import datetime
import os
from typing import Optional

import torch
import torch.distributed as dist


def init_process_group(backend: Optional[str] = None, timeout_s: float = 120.0) -> None:
    """Join the job's process group (env:// rendezvous; 127.0.0.1 default)."""
    if dist.is_initialized():
        return
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29533")
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    kw = {}
    if backend == "nccl":
        kw["device_id"] = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)


def make_comm(kind: str = "p2p"):
    if kind == "nccl" or not torch.cuda.is_available():
        return NcclComm()
    from .p2p import P2PComm
    return P2PComm()


class NcclComm:
    """Collectives through torch.distributed (the baseline)."""

    def __init__(self):
        self.rank = dist.get_rank()
        self.world = dist.get_world_size()

    def barrier(self) -> None:
        dist.barrier()

    def broadcast_params(self, net) -> None:
        dist.broadcast(net.flat, 0)
        net.sync_bf16()

    def allreduce_moments(self, moments: torch.Tensor) -> None:
        dist.all_reduce(moments)

    def step(self, net, opt) -> None:
        """Sum the gradient over ranks (the loss is already normalised by the
        global minibatch), then clip + Adam locally (identical on every rank)."""
        dist.all_reduce(net.grad)
        opt.step()

    def merge_counts(self, reward) -> None:
        """Apply the other ranks' curiosity count increments of this iteration."""
        if reward.spec.int_coef <= 0 or not torch.is_tensor(reward.counts):
            return
        mine = reward.delta.clone()
        dist.all_reduce(reward.delta)
        reward.counts.add_(reward.delta - mine)
        reward.delta.zero_()

    def max_scalar(self, x: float) -> float:
        t = torch.tensor([float(x)], dtype=torch.float64,
                         device="cuda" if dist.get_backend() == "nccl" else "cpu")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def checksum(self, net) -> tuple:
        """(min, max) over ranks of the parameter sum: equal iff replicas agree."""
        s = net.flat.double().sum().reshape(1)
        lo, hi = s.clone(), s.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        return float(lo.item()), float(hi.item())

    def close(self) -> None:
        if dist.is_initialized():
            dist.destroy_process_group()
