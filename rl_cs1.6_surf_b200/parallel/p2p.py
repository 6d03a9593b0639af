"""Data-parallel collectives as fused NVLink peer-memory kernels (csrc/comm/p2p.cu).

``P2PComm`` is the product path of the data-parallel trainer (one process per
GPU on one node). At set-up every rank exports CUDA IPC handles of the
buffers the kernels touch (gradient, fp32 master weights, bf16 weights, the
curiosity-count increments and a 48 KB sync block); the handles travel once
over the process group, after which no library collective runs on the hot
path:

* ``bucket`` — the gradient range that is final before the backward ends
  (the tower and FC weights, ~93% of the parameters) is published in bf16
  and reduce-scattered over peer loads on a side stream while the
  convolutions' backward runs (``PolicyNet.overlap_range``);
* ``step``  — reduce-scatter of the rest of the gradient (bf16 over NVLink,
  fp32 sums), global-norm clip over both parts, Adam on the owned shard,
  push of the updated shard to every peer (one cooperative kernel with
  in-kernel grid barriers, graph-capturable; replaces all-reduce + clip +
  Adam);
* ``allreduce_moments`` — per-minibatch advantage moments (one block);
* ``merge_counts`` — curiosity count increments summed into every rank's
  table, then cleared.

The optimizer state is sharded: each rank updates ``m``/``v`` only on its own
shard (ZeRO-1 style); ``full_optimizer_state`` reassembles them for
checkpoints. Every device-side wait is bounded (``timeout_s``); a wait that
runs out records an error code in the sync block, later collective kernels
return immediately, and ``check()`` raises on the host.

Reference design: docs/ddp-plan.md:404-434 (gradient sum before the clip),
:133-147 (global moments), :174-225 (count deltas), :355-380 (broadcast +
checksum). The reference never built it.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_double, c_int, c_int64, c_void_p
from typing import Optional

import torch
import torch.distributed as dist

from ..ops import _lib
from ..ops._lib import check, ptr, stream_ptr
from .dist import NcclComm

CLIB = "libsurf_comm.so"
_lib.register(CLIB, {
    "surf_p2p_sync_words": (c_int, []),
    "surf_p2p_max_world": (c_int, []),
    "surf_p2p_max_moments": (c_int, []),
    "surf_ipc_handle": (c_int, [c_void_p, c_void_p, ctypes.POINTER(c_int64)]),
    "surf_ipc_open": (c_int, [c_void_p, c_int64, ctypes.POINTER(c_void_p)]),
    "surf_ipc_close_all": (c_int, []),
    "surf_p2p_create": (c_void_p, [c_int, c_int, ctypes.POINTER(c_void_p), c_double]),
    "surf_p2p_destroy": (None, [c_void_p]),
    "surf_p2p_set_grad": (c_int, [c_void_p, c_int64, ctypes.POINTER(c_void_p), ctypes.POINTER(c_void_p),
                                  ctypes.POINTER(c_void_p), c_void_p, c_void_p, c_void_p, c_int64]),
    "surf_p2p_shard": (c_int64, [c_void_p]),
    "surf_p2p_set_grad16": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "surf_p2p_set_buckets": (c_int, [c_void_p, c_int, ctypes.POINTER(c_int64), ctypes.POINTER(c_int64)]),
    "surf_p2p_bucket": (c_int, [c_void_p, c_int, c_void_p]),
    "surf_p2p_set_counts": (c_int, [c_void_p, c_int64, c_void_p, ctypes.POINTER(c_void_p)]),
    "surf_p2p_grad_step": (c_int, [c_void_p, c_void_p]),
    "surf_p2p_moments": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "surf_p2p_merge_counts": (c_int, [c_void_p, c_void_p]),
    "surf_p2p_prof_words": (c_int, []),
})


# sync-block words (csrc/comm/p2p.cu)
W_SEQ_GRAD, W_SEQ_MOM, W_SEQ_CNT, W_ERR, W_ERR_TARGET, W_PROF = 0, 1, 2, 3, 4, 112
_STAGES = {1: "gradient barrier", 2: "norm exchange", 3: "parameter push", 4: "moments", 5: "count barrier",
           6: "count drain", 7: "in-kernel grid barrier"}


class P2PError(RuntimeError):
    pass


def describe_error(code: int, target: int) -> str:
    stage = _STAGES.get((code >> 8) & 0xF, "unknown stage")
    if (code >> 8) & 0xF == 7:
        return f"peer-memory collective timed out at an {stage} (call #{target})"
    return f"peer-memory collective timed out in the {stage} waiting for rank {code & 0xFF} (call #{target})"


def _ptr_array(ptrs) -> ctypes.Array:
    return (c_void_p * len(ptrs))(*[c_void_p(int(p)) for p in ptrs])


class P2PComm(NcclComm):
    """Fused peer-memory collectives (requires every rank on one node)."""

    def __init__(self, timeout_s: Optional[float] = None):
        super().__init__()
        L = _lib.lib(CLIB)
        if self.world > int(L.surf_p2p_max_world()):
            raise ValueError(f"P2PComm supports at most {L.surf_p2p_max_world()} ranks")
        local_world = int(os.environ.get("LOCAL_WORLD_SIZE", self.world))
        if local_world != self.world:
            raise ValueError("P2PComm needs every rank on one node (NVLink peers); use the nccl comm instead")
        self.timeout_s = float(timeout_s if timeout_s is not None else os.environ.get("SURF_P2P_TIMEOUT_S", 60.0))
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.sync = torch.zeros(int(L.surf_p2p_sync_words()), dtype=torch.int64, device=self.device)
        torch.cuda.synchronize()
        self.sync_peers = self.share(self.sync)
        self.plan = L.surf_p2p_create(self.rank, self.world, _ptr_array(self.sync_peers), self.timeout_s)
        if not self.plan:
            raise P2PError("surf_p2p_create failed")
        self.shard = 0
        self.push32_from = 0
        self._opt = None
        self._counts = False
        self.grad16 = None
        self.nbuckets = 0
        self._bucketed = set()

    # ---- set-up -------------------------------------------------------------------------
    def share(self, t: torch.Tensor) -> list:
        """Device addresses of every rank's copy of ``t`` (this rank's local)."""
        L = _lib.lib(CLIB)
        handle = (ctypes.c_char * 64)()
        off = c_int64(0)
        rc = L.surf_ipc_handle(c_void_p(t.data_ptr()), handle, ctypes.byref(off))
        if rc:
            raise P2PError(f"surf_ipc_handle failed ({rc})")
        mine = (bytes(handle), int(off.value), int(t.numel() * t.element_size()))
        allh = [None] * self.world
        dist.all_gather_object(allh, mine)
        out = []
        for q, (h, o, nbytes) in enumerate(allh):
            if nbytes != mine[2]:
                raise P2PError(f"rank {q} shares {nbytes} bytes where rank {self.rank} shares {mine[2]}")
            if q == self.rank:
                out.append(t.data_ptr())
                continue
            p = c_void_p()
            hb = (ctypes.c_char * 64).from_buffer_copy(h)
            rc = L.surf_ipc_open(hb, o, ctypes.byref(p))
            if rc:
                raise P2PError(f"surf_ipc_open of rank {q}'s buffer failed ({rc})")
            out.append(int(p.value))
        return out

    def attach(self, net, opt, reward=None) -> None:
        """Register the trainer's buffers (collective: every rank calls it)."""
        L = _lib.lib(CLIB)
        g = self.share(net.grad)
        p = self.share(net.flat)
        p16 = self.share(net.flat16)
        self.push32_from = int(getattr(net, "fp32_from", 0))
        check(L.surf_p2p_set_grad(self.plan, net.numel, _ptr_array(g), _ptr_array(p), _ptr_array(p16), ptr(opt.m),
                                  ptr(opt.v), ptr(opt.hyper), self.push32_from), "surf_p2p_set_grad")
        self.shard = int(L.surf_p2p_shard(self.plan))
        # the bf16 copy of the gradient that the peers read
        self.grad16 = torch.zeros(net.numel, dtype=torch.bfloat16, device=self.device)
        check(L.surf_p2p_set_grad16(self.plan, _ptr_array(self.share(self.grad16))), "surf_p2p_set_grad16")
        # one overlapped bucket: the range whose gradient is final before the
        # convolutions' backward (SURF_P2P_OVERLAP=0: none, everything in the step)
        rng = net.overlap_range() if hasattr(net, "overlap_range") else None
        if os.environ.get("SURF_P2P_OVERLAP", "1") == "0":
            rng = None
        flags = [None] * self.world
        dist.all_gather_object(flags, rng)
        if any(f != rng for f in flags):
            raise P2PError("ranks disagree on the overlapped gradient bucket")
        if rng is not None:
            lo, hi = (c_int64 * 1)(rng[0]), (c_int64 * 1)(rng[1])
            check(L.surf_p2p_set_buckets(self.plan, 1, lo, hi), "surf_p2p_set_buckets")
            self.nbuckets = 1
        self._opt = opt
        use_counts = reward is not None and reward.spec.int_coef > 0 and torch.is_tensor(reward.counts)
        flags = [None] * self.world
        dist.all_gather_object(flags, bool(use_counts))
        if any(flags) != all(flags):
            raise P2PError("ranks disagree on curiosity counts")
        if use_counts:
            d = self.share(reward.delta)
            check(L.surf_p2p_set_counts(self.plan, reward.delta.numel(), ptr(reward.counts), _ptr_array(d)),
                  "surf_p2p_set_counts")
            self._counts = True
        torch.cuda.synchronize()
        dist.barrier()

    # ---- collectives --------------------------------------------------------------------
    def allreduce_moments(self, moments: torch.Tensor) -> None:
        L = _lib.lib(CLIB)
        if not moments.is_cuda or moments.dtype != torch.float64 or not moments.is_contiguous():
            return super().allreduce_moments(moments)
        n = moments.numel()
        if n > int(L.surf_p2p_max_moments()):
            return super().allreduce_moments(moments)
        check(L.surf_p2p_moments(self.plan, ptr(moments), n, stream_ptr(moments.device)), "surf_p2p_moments")

    def bucket(self, b: int = 0) -> None:
        """Bucket b's gradient is final in the current stream's order: publish,
        release and reduce it there (launch on a side stream to overlap)."""
        check(_lib.lib(CLIB).surf_p2p_bucket(self.plan, int(b), stream_ptr(self.device)), "surf_p2p_bucket")
        self._bucketed.add(int(b))

    def step(self, net, opt) -> None:
        if self._opt is None:
            raise P2PError("P2PComm.step before attach()")
        # a bucket nobody launched during the backward is reduced here, in order
        for b in range(self.nbuckets):
            if b not in self._bucketed:
                self.bucket(b)
        self._bucketed.clear()
        check(_lib.lib(CLIB).surf_p2p_grad_step(self.plan, stream_ptr(net.flat.device)), "surf_p2p_grad_step")

    def merge_counts(self, reward) -> None:
        if not self._counts:
            return super().merge_counts(reward)
        check(_lib.lib(CLIB).surf_p2p_merge_counts(self.plan, stream_ptr(reward.delta.device)),
              "surf_p2p_merge_counts")

    def check(self) -> None:
        """Raise if a device-side wait of this rank ran out of time."""
        code, target = (int(x) for x in self.sync[W_ERR:W_ERR_TARGET + 1].tolist())
        if code:
            raise P2PError(f"rank {self.rank}: {describe_error(code, target)}")

    def phase_times_us(self) -> dict:
        """Phase durations of this rank's last gradient step (device clock)."""
        t = [int(x) for x in self.sync[W_PROF:W_PROF + 6].tolist()]
        names = ("barrier_in", "reduce_scatter", "norm_exchange", "adam_push", "done_wait")
        return {k: (t[i + 1] - t[i]) / 1e3 for i, k in enumerate(names)}

    def sequence(self) -> tuple:
        return tuple(int(x) for x in self.sync[:3].tolist())

    def shard_range(self, n: int) -> tuple:
        lo = min(n, self.rank * self.shard)
        return lo, min(n, lo + self.shard)

    def _gather_shards(self, t: torch.Tensor) -> torch.Tensor:
        n = t.numel()
        full = torch.zeros_like(t)
        lo, hi = self.shard_range(n)
        full[lo:hi] = t[lo:hi]
        dist.all_reduce(full)
        return full

    def full_params(self, net) -> torch.Tensor:
        """The complete fp32 master weights (collective): each rank keeps only
        its shard of the weight matrices current in fp32."""
        full = self._gather_shards(net.flat)
        if self.push32_from:
            full[self.push32_from:] = net.flat[self.push32_from:]
        return full

    def checksum(self, net) -> tuple:
        """(min, max) over ranks of the sum of the replicated parameters (bf16
        copy + fp32 tail): equal iff the replicas agree."""
        s = net.flat16.double().sum() + net.flat[self.push32_from:].double().sum()
        lo, hi = s.reshape(1).clone(), s.reshape(1).clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        return float(lo.item()), float(hi.item())

    def full_optimizer_state(self, opt) -> dict:
        """m and v of every shard on every rank (collective)."""
        return {name: self._gather_shards(getattr(opt, name)) for name in ("m", "v")}

    def close(self) -> None:
        if self.plan:
            torch.cuda.synchronize()
            if dist.is_initialized():
                dist.barrier()
            L = _lib.lib(CLIB)
            L.surf_p2p_destroy(self.plan)
            self.plan = None
            L.surf_ipc_close_all()
        super().close()
