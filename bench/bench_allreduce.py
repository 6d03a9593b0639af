"""Fused data-parallel optimizer step over NVLink vs the NCCL baseline.

    torchrun --nproc-per-node N bench/bench_allreduce.py [--iters 20]

The parameters are the flagship vision policy's (2,076,224 in its flat
layout). Per rank and step, the fused path (csrc/comm/p2p.cu) publishes a
bf16 copy of the gradient, reduce-scatters it over peer loads (fp32 sums),
clips by the global norm, runs Adam on the owned shard and pushes the new
bf16 (and fp32-tail) parameters to every peer; the baseline is
``torch.distributed.all_reduce`` (NCCL, fp32) of the gradient followed by the
single-GPU fused clip + Adam kernels. Everything runs inside CUDA graphs (10
steps per graph, launch overhead excluded), timed with CUDA events, max over
ranks. Three fused figures:

* ``fused_p2p_us``: the whole step, no overlap (SURF_P2P_OVERLAP=0 layout:
  one kernel reduces everything);
* ``bucket_then_step_us``: the overlapped layout's two parts run back to
  back (the tower / FC bucket, ~93% of the parameters, then the step kernel
  for the rest);
* ``exposed_us``: what the overlapped layout adds to a stand-in backward of
  ``--backward-ms`` (bf16 GEMMs on the main stream) when the bucket runs on a
  side stream during it, as in the trainer: T(backward + bucket + step) -
  T(backward alone).

NVLink roofline of the fused step: every rank receives (W-1)/W of the
gradient in bf16 (2 B/param, its shard from each peer) plus (W-1)/W of the
new bf16 parameters (2 B/param, pushed by the peers; the fp32 tail of
biases is negligible), and sends the same, so T_roof = 4 B x n x (W-1)/W /
770 GB/s (measured peer bandwidth per direction).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

LINK_GBS = 770.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20, help="graph replays of 10 steps each")
    ap.add_argument("--backward-ms", type=float, default=2.0, help="stand-in backward for the overlap figure")
    args = ap.parse_args()
    import torch
    import torch.distributed as dist
    import surfb200  # noqa: F401
    from surfb200.models.policy import NetConfig, PolicyNet, space_to_depth_config
    from surfb200.ops import rl as R
    from surfb200.parallel.dist import init_process_group
    from surfb200.parallel.p2p import P2PComm
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    init_process_group("nccl", timeout_s=120)
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    cfg = space_to_depth_config(NetConfig(vision=True))

    def make():
        net = PolicyNet(cfg, dev, seed=0)
        return net, R.Adam(net, lr=1e-4)

    net_a, opt_a = make()                 # overlapped layout (one bucket)
    comm = P2PComm(timeout_s=30)
    comm.attach(net_a, opt_a, None)
    assert comm.nbuckets == 1
    os.environ["SURF_P2P_OVERLAP"] = "0"
    net_b, opt_b = make()                 # one kernel for everything
    comm_b = P2PComm(timeout_s=30)
    comm_b.attach(net_b, opt_b, None)
    os.environ.pop("SURF_P2P_OVERLAP")
    ref, ropt = make()
    n = net_a.numel
    g_src = torch.randn(n, device=dev) * 1e-3
    side = torch.cuda.Stream()
    a = torch.randn(8192, 8192, device=dev, dtype=torch.bfloat16)
    per_mm_ms = 2 * 8192 ** 3 / 1.2e15 * 1e3
    n_mm = max(1, int(round(args.backward_ms / per_mm_ms)))

    def backward_standin():
        for _ in range(n_mm):
            torch.mm(a, a)

    def copy_only():
        net_a.grad.copy_(g_src)

    def fused_one_kernel():
        net_b.grad.copy_(g_src)
        comm_b.step(net_b, opt_b)

    def bucket_only():
        net_a.grad.copy_(g_src)
        comm.bucket(0)
        comm.step(net_a, opt_a)

    def overlapped():
        net_a.grad.copy_(g_src)
        main = torch.cuda.current_stream()
        side.wait_stream(main)
        with torch.cuda.stream(side):
            comm.bucket(0)
        backward_standin()
        main.wait_stream(side)
        comm.step(net_a, opt_a)

    def standin_only():
        net_a.grad.copy_(g_src)
        backward_standin()

    def baseline():
        ref.grad.copy_(g_src)
        dist.all_reduce(ref.grad)
        ropt.step()

    def timed(fn) -> float:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(10):
                fn()
        torch.cuda.synchronize()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (10 * args.iters)
        t = torch.tensor([us], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        del g
        torch.cuda.synchronize()
        return float(t.item())

    r = {name: timed(fn) for name, fn in (("copy", copy_only), ("fused", fused_one_kernel), ("bucket", bucket_only),
                                          ("nccl", baseline), ("standin", standin_only), ("overlap", overlapped))}
    comm.check()
    comm_b.check()
    phases = comm_b.phase_times_us()
    pt = [None] * world
    dist.all_gather_object(pt, phases)
    copy_us = r["copy"]
    fused_us = r["fused"] - copy_us
    nccl_us = r["nccl"] - copy_us
    split_us = r["bucket"] - copy_us
    exposed_us = r["overlap"] - r["standin"]
    bytes_dir = 4.0 * n * (world - 1) / world
    roof_us = bytes_dir / (LINK_GBS * 1e9) * 1e6
    if rank == 0:
        print(json.dumps({"bench": "dp_optimizer_step", "n_params": n, "world": world, "grad_dtype": "bf16",
                          "fused_p2p_us": round(fused_us, 2), "nccl_allreduce_adam_us": round(nccl_us, 2),
                          "speedup_vs_nccl": round(nccl_us / fused_us, 3) if fused_us > 0 else None,
                          "bucket_then_step_us": round(split_us, 2),
                          "exposed_us": round(exposed_us, 2), "standin_backward_us": round(r["standin"] - copy_us, 1),
                          "nvlink_bytes_per_direction": int(bytes_dir), "roofline_us": round(roof_us, 2),
                          "frac_of_roofline": round(roof_us / fused_us, 3) if fused_us > 0 else None,
                          "link_gbs_measured": LINK_GBS, "grad_copy_us_subtracted": round(copy_us, 2),
                          "last_step_phases_us": [{k: round(v, 2) for k, v in p.items()} for p in pt]}), flush=True)
    # comm_b first (its plan only: the peer mappings are shared), then comm
    # (mappings, process group)
    torch.cuda.synchronize()
    dist.barrier()
    from surfb200.ops import _lib
    from surfb200.parallel.p2p import CLIB
    _lib.lib(CLIB).surf_p2p_destroy(comm_b.plan)
    comm_b.plan = None
    comm.close()


if __name__ == "__main__":
    main()
