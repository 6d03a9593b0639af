"""Fused data-parallel optimizer step over NVLink vs the NCCL baseline.

    torchrun --nproc-per-node N bench/bench_allreduce.py [--n 2076129] [--iters 200]

Per rank and step: the fused path (csrc/comm/p2p.cu) reduce-scatters the fp32
gradient over peer loads, clips by the global norm, runs Adam on the owned
shard and pushes the new fp32 + bf16 parameters to every peer; the baseline
is ``torch.distributed.all_reduce`` (NCCL) of the gradient followed by the
single-GPU fused clip + Adam kernels. Both are captured in CUDA graphs (10
steps per graph) so launch overhead is excluded, timed with CUDA events and
reported as the max over ranks.

NVLink roofline of the fused step: every rank receives (W-1)/W of the
gradient (4 B/param, its shard from each peer) plus (W-1)/W of the new
parameters (6 B/param, pushed by the peers), and sends the same amount, so
T_roof = 10 B x n x (W-1)/W / 770 GB/s (measured peer bandwidth per
direction); the achieved fraction is T_roof / T_measured.
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
    ap.add_argument("--n", type=int, default=2_076_129)
    ap.add_argument("--iters", type=int, default=20, help="graph replays of 10 steps each")
    args = ap.parse_args()
    import torch
    import torch.distributed as dist
    import surfb200  # noqa: F401
    from surfb200.ops import rl as R
    from surfb200.parallel.dist import init_process_group
    from surfb200.parallel.p2p import P2PComm
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    init_process_group("nccl", timeout_s=120)
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    n = args.n

    class Net:
        pass

    def make():
        net = Net()
        net.numel = n
        net.flat = torch.randn(n, device=dev, generator=torch.Generator(device=dev).manual_seed(0))
        net.grad = torch.zeros(n, device=dev)
        net.flat16 = net.flat.to(torch.bfloat16)
        return net

    net = make()
    opt = R.Adam(net, lr=1e-4)
    comm = P2PComm(timeout_s=30)
    comm.attach(net, opt, None)
    g_src = torch.randn(n, device=dev) * 1e-3

    def fused():
        net.grad.copy_(g_src)
        comm.step(net, opt)

    ref = make()
    ropt = R.Adam(ref, lr=1e-4)

    def baseline():
        ref.grad.copy_(g_src)
        dist.all_reduce(ref.grad)
        ropt.step()

    def copy_only():
        net.grad.copy_(g_src)

    results = {}
    for name, fn in (("copy", copy_only), ("fused_p2p", fused), ("nccl_allreduce_adam", baseline)):
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
        results[name] = float(t.item())
        del g
        torch.cuda.synchronize()
    comm.check()
    phases = comm.phase_times_us()
    pt = [None] * world
    dist.all_gather_object(pt, phases)
    copy_us = results.pop("copy")
    fused_us = results["fused_p2p"] - copy_us
    nccl_us = results["nccl_allreduce_adam"] - copy_us
    bytes_dir = 10.0 * n * (world - 1) / world
    roof_us = bytes_dir / (LINK_GBS * 1e9) * 1e6
    if rank == 0:
        print(json.dumps({"bench": "dp_optimizer_step", "n_params": n, "world": world,
                          "fused_p2p_us": round(fused_us, 2), "nccl_allreduce_adam_us": round(nccl_us, 2),
                          "speedup_vs_nccl": round(nccl_us / fused_us, 3) if fused_us > 0 else None,
                          "nvlink_bytes_per_direction": int(bytes_dir), "roofline_us": round(roof_us, 2),
                          "frac_of_roofline": round(roof_us / fused_us, 3) if fused_us > 0 else None,
                          "link_gbs_measured": LINK_GBS, "grad_copy_us_subtracted": round(copy_us, 2),
                          "last_step_phases_us": [{k: round(v, 2) for k, v in p.items()} for p in pt]}), flush=True)
    comm.close()


if __name__ == "__main__":
    main()
