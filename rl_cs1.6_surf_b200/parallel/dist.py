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


def physical_cores(cpus) -> list:
    """``cpus`` grouped by physical core (hyperthread siblings together),
    from /sys topology; one group per CPU where it cannot be read."""
    cpus = sorted(cpus)
    key = {}
    for c in cpus:
        try:
            base = f"/sys/devices/system/cpu/cpu{c}/topology/"
            with open(base + "physical_package_id") as f:
                pkg = int(f.read())
            with open(base + "core_id") as f:
                core = int(f.read())
            key[c] = (pkg, core)
        except (OSError, ValueError):
            key[c] = ("cpu", c)
    groups = {}
    for c in cpus:
        groups.setdefault(key[c], []).append(c)
    return sorted(groups.values(), key=lambda g: g[0])


def rank_cpu_share(cpus, local_rank: int, local_world: int) -> list:
    """This local rank's disjoint share of ``cpus``: whole physical cores,
    contiguous blocks, the remainder spread over the first ranks."""
    cores = physical_cores(cpus)
    if local_world <= 1 or len(cores) < local_world:
        return sorted(cpus)
    per, extra = divmod(len(cores), local_world)
    start = local_rank * per + min(local_rank, extra)
    mine = cores[start:start + per + (1 if local_rank < extra else 0)]
    return sorted(c for g in mine for c in g)


def pin_rank_cpus() -> Optional[list]:
    """Pin this process (and the env threads it starts later) to its rank's
    disjoint share of the node's CPUs, so the ranks' simulator pools do not
    compete for cores (process CPU affinity only). Off with SURF_NO_PIN=1 or
    with one rank per node. Returns the CPUs pinned to, or None."""
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", "1"))
    if local_world <= 1 or os.environ.get("SURF_NO_PIN") == "1" or not hasattr(os, "sched_setaffinity"):
        return None
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    share = rank_cpu_share(os.sched_getaffinity(0), local_rank, local_world)
    os.sched_setaffinity(0, share)
    os.environ["SURF_CPUS_PINNED"] = "1"          # default_threads(): the affinity is this rank's share
    return share


def init_process_group(backend: Optional[str] = None, timeout_s: float = 120.0) -> None:
    """Join the job's process group (env:// rendezvous; 127.0.0.1 default)
    and pin this rank to its share of the node's CPUs."""
    if dist.is_initialized():
        return
    pin_rank_cpus()
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
