"""Rank bodies for the multi-process tests (spawned by torch.multiprocessing).

Each worker joins a process group on 127.0.0.1, does its part and reports
``(rank, ok, message)`` through a queue; the test process asserts on the
reports. Nothing here waits without a bound: process groups get short
timeouts and the spawning test joins with a deadline.
"""
from __future__ import annotations

import datetime
import os
import sys
import traceback
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def _env(rank: int, world: int, port: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), LOCAL_WORLD_SIZE=str(world), SURF_THREADS="2")


def _report(q, rank, fn):
    try:
        msg = fn()
        q.put((rank, True, msg or ""))
    except BaseException as e:   # noqa: BLE001 — reported to the parent
        q.put((rank, False, f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))


# ---- CPU (gloo) ----------------------------------------------------------------------------
def gloo_train(rank: int, world: int, port: int, q) -> None:
    """Two CPU ranks train the eyeless policy one iteration; replicas must agree."""
    _env(rank, world, port)

    def body():
        import torch
        import surfb200  # noqa: F401
        from surfb200.parallel.dist import NcclComm, init_process_group
        from surfb200.rewards.spec import RewardSpec
        from surfb200.trainer.config import TrainConfig
        from surfb200.trainer.ppo import Trainer
        init_process_group("gloo", timeout_s=60)
        comm = NcclComm()
        cfg = TrainConfig(map="ramps", envs=16, n_steps=8, epochs=2, minibatches=2, vision=False, device="cpu",
                          graphs=False, ep_ticks=120, reward=RewardSpec(mode="speed"))
        tr = Trainer(cfg, rank=rank, world=world, comm=comm, verbose=False)
        flat0 = tr.net.flat.clone()
        lo0, hi0 = comm.checksum(tr.net)
        s = tr.train_iteration()
        lo, hi = comm.checksum(tr.net)
        moved = not torch.equal(flat0, tr.net.flat)
        # envs differ per rank (rank-distinct reset seeds)
        spread = comm.max_scalar(float(tr.hrec[:, 32].sum()))
        comm.close()
        assert lo0 == hi0, ("initial broadcast", lo0, hi0)
        assert lo == hi, ("replicas diverged", lo, hi)
        assert moved
        assert s["global_step"] == world * 16 * 8 * cfg.act_every
        return f"checksum {lo:.6f} spread {spread:.1f}"

    _report(q, rank, body)


def gloo_dead_rank(rank: int, world: int, port: int, q) -> None:
    """Rank 1 fails before the first collective; rank 0 must get an error
    (not hang) from its next collective."""
    _env(rank, world, port)

    def body():
        import torch
        import torch.distributed as dist
        import surfb200  # noqa: F401
        from surfb200.parallel.dist import NcclComm, init_process_group
        # a generous timeout for the rendezvous (a cold start imports slowly),
        # a short one for the collective that must notice the dead peer
        init_process_group("gloo", timeout_s=120)
        comm = NcclComm()
        short = dist.new_group(ranks=list(range(world)), timeout=datetime.timedelta(seconds=5))
        dist.barrier()
        if rank == 1:
            os._exit(3)                        # the rank dies between steps
        t = torch.ones(8)
        try:
            dist.all_reduce(t, group=short)
        except Exception as e:                 # noqa: BLE001
            return f"detected: {type(e).__name__}"
        raise AssertionError("all_reduce with a dead peer returned normally")

    _report(q, rank, body)


def gloo_stalled_rank(rank: int, world: int, port: int, q) -> None:
    """Rank 1 stalls (alive, but never reaches the collective) for longer
    than the process group's timeout; rank 0's collective must end with an
    error instead of waiting for it."""
    _env(rank, world, port)

    def body():
        import time
        import torch
        import torch.distributed as dist
        import surfb200  # noqa: F401
        from surfb200.parallel.dist import init_process_group
        init_process_group("gloo", timeout_s=120)       # rendezvous: cold starts import slowly
        short = dist.new_group(ranks=list(range(world)), timeout=datetime.timedelta(seconds=3))
        dist.barrier()
        if rank == 1:
            time.sleep(10)                     # stalled between steps
            return "stalled"
        t = torch.ones(8)
        t0 = time.time()
        try:
            dist.all_reduce(t, group=short)
        except Exception as e:                 # noqa: BLE001
            return f"detected after {time.time() - t0:.1f} s: {type(e).__name__}"
        raise AssertionError("all_reduce with a stalled peer returned normally")

    _report(q, rank, body)


def gloo_corrupt_replica(rank: int, world: int, port: int, q) -> None:
    """Two CPU ranks train with a replica check every iteration; after the
    first iteration rank 1's parameters are corrupted, and the check of the
    second iteration raises ReplicaDivergence on both ranks."""
    _env(rank, world, port)

    def body():
        import surfb200  # noqa: F401
        from surfb200.parallel.dist import NcclComm, init_process_group
        from surfb200.rewards.spec import RewardSpec
        from surfb200.trainer.config import TrainConfig
        from surfb200.trainer.ppo import ReplicaDivergence, Trainer
        init_process_group("gloo", timeout_s=60)
        comm = NcclComm()
        cfg = TrainConfig(map="ramps", envs=8, n_steps=4, epochs=1, minibatches=1, vision=False, device="cpu",
                          graphs=False, ep_ticks=120, reward=RewardSpec(mode="speed"), replica_check_every=1)
        tr = Trainer(cfg, rank=rank, world=world, comm=comm, verbose=False)
        tr.train_iteration()                   # replicas agree: no error
        if rank == 1:
            tr.net.flat[7] += 1e-3             # a flipped parameter on one rank
        try:
            tr.train_iteration()
        except ReplicaDivergence as e:
            comm.close()
            return f"detected: {e}"
        raise AssertionError("diverged replicas were not detected")

    _report(q, rank, body)


# ---- GPU (NCCL + peer memory) ----------------------------------------------------------------
def p2p_collectives(rank: int, world: int, port: int, q) -> None:
    """Peer-memory gradient step / moments / count merge vs plain torch."""
    _env(rank, world, port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"

    def body():
        import torch
        import torch.distributed as dist
        import ctypes

        import surfb200  # noqa: F401
        from surfb200.ops import _lib
        from surfb200.parallel.dist import init_process_group
        from surfb200.parallel.p2p import CLIB, P2PComm
        torch.cuda.set_device(rank)
        init_process_group("nccl", timeout_s=60)
        dev = torch.device("cuda", rank)
        comm = P2PComm(timeout_s=10.0)

        class Net:
            pass

        class Opt:
            pass

        class Spec:
            int_coef = 0.25

        class Rew:
            pass

        n = 1_000_000                    # a multiple of 8: 16-byte bf16 groups
        gen = torch.Generator().manual_seed(0)
        net = Net()
        net.numel = n
        net.fp32_from = 600_000          # weights below: fp32 master sharded, bf16 replicated
        net.flat = torch.randn(n, generator=gen).to(dev)
        net.grad = torch.zeros(n, device=dev)
        net.flat16 = net.flat.to(torch.bfloat16)
        opt = Opt()
        opt.m = torch.zeros(n, device=dev)
        opt.v = torch.zeros(n, device=dev)
        lr, b1, b2, eps, max_norm = 1e-3, 0.9, 0.999, 1e-5, 0.5
        opt.hyper = torch.tensor([lr, b1, b2, eps, max_norm, 0.0], device=dev)
        rew = Rew()
        rew.spec = Spec()
        cn = (1 << 16) + 3
        rew.counts = torch.randint(0, 50, (cn,), generator=gen, dtype=torch.int32).to(dev)
        rew.delta = torch.zeros(cn, dtype=torch.int32, device=dev)
        comm.attach(net, opt, rew)

        # plain-torch reference of the same data-parallel step (full m, v)
        p_ref = net.flat.clone()
        m_ref = torch.zeros(n, device=dev)
        v_ref = torch.zeros(n, device=dev)
        owner = torch.arange(n, device=dev) // comm.shard
        graph = None
        L = _lib.lib(CLIB)
        side = torch.cuda.Stream()
        for step in range(1, 9):
            if step == 5:
                # from here on the range [200_000, 600_000) is an overlapped
                # bucket, launched on a side stream like the trainer does
                lo, hi = (ctypes.c_int64 * 1)(200_000), (ctypes.c_int64 * 1)(600_000)
                assert L.surf_p2p_set_buckets(comm.plan, 1, lo, hi) == 0
                comm.nbuckets = 1
                graph = None
            g_local = torch.randn(n, generator=torch.Generator().manual_seed(100 * step + rank)).to(dev) * 0.01
            allg = [torch.empty_like(g_local) for _ in range(world)]
            dist.all_gather(allg, g_local)
            # the kernels' sum: rank order, fp32, each element's owner adds its
            # own term in fp32 and the peers' through their bf16 copies
            gsum = torch.zeros(n, device=dev)
            for q in range(world):
                gsum += torch.where(owner == q, allg[q], allg[q].to(torch.bfloat16).float())
            norm = float(gsum.double().norm())
            coef = min(1.0, max_norm / (norm + 1e-6))
            gc = gsum * coef
            m_ref.mul_(b1).add_(gc, alpha=1 - b1)
            v_ref.mul_(b2).addcmul_(gc, gc, value=1 - b2)
            bc1, bc2 = 1 - b1 ** step, 1 - b2 ** step
            p_ref.addcdiv_(m_ref, v_ref.sqrt() / bc2 ** 0.5 + eps, value=-lr / bc1)

            net.grad.copy_(g_local)
            torch.cuda.synchronize()

            def fused_step():
                if comm.nbuckets:
                    main = torch.cuda.current_stream()
                    side.wait_stream(main)
                    with torch.cuda.stream(side):
                        comm.bucket(0)
                    main.wait_stream(side)
                comm.step(net, opt)

            if step in (1, 2, 5, 6):
                fused_step()                               # eager launches
            else:
                if graph is None:                          # the trainer replays the step inside CUDA graphs
                    s = torch.cuda.Stream()
                    s.wait_stream(torch.cuda.current_stream())
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph, stream=s):
                        fused_step()
                    torch.cuda.synchronize()
                graph.replay()
            torch.cuda.synchronize()
            comm.check()
            lo, hi = comm.shard_range(n)
            own = torch.zeros(n, dtype=torch.bool, device=dev)
            own[lo:hi] = True
            own[net.fp32_from:] = True               # the fp32 tail is replicated
            err = float(((net.flat - p_ref).abs() / (p_ref.abs() + 1e-3))[own].max())
            assert err < 1e-4, ("params", step, err)
            e16 = float(((net.flat16.float() - p_ref).abs() / (p_ref.abs() + 1e-3)).max())
            assert e16 < 1e-2, ("bf16 params", step, e16)
            assert torch.equal(net.flat16[own], net.flat[own].to(torch.bfloat16)), "bf16 copy out of sync"
            assert not net.grad.any(), "gradient not cleared"
            assert int(opt.hyper[5].item()) == step
        c_lo, c_hi = comm.checksum(net)
        assert c_lo == c_hi, ("replicas differ", c_lo, c_hi)
        full = comm.full_params(net)
        assert float(((full - p_ref).abs() / (p_ref.abs() + 1e-3)).max()) < 1e-4
        full = comm.full_optimizer_state(opt)
        assert float((full["m"] - m_ref).abs().max()) < 1e-6

        # moments: ordered sum, identical on every rank
        mom = torch.tensor([rank + 0.5 + i for i in range(16)], dtype=torch.float64, device=dev)
        for _ in range(3):                                 # repeated calls reuse the parity slots
            mm = mom.clone()
            comm.allreduce_moments(mm)
            torch.cuda.synchronize()
            want = sum(torch.tensor([r + 0.5 + i for i in range(16)], dtype=torch.float64) for r in range(world))
            assert torch.equal(mm.cpu(), want), (mm, want)

        # count merge: counts += every other rank's increments; own increments cleared
        for rnd in range(2):
            d = torch.randint(0, 3, (cn,), generator=torch.Generator().manual_seed(7 * rnd + rank),
                              dtype=torch.int32).to(dev)
            alld = [torch.empty_like(d) for _ in range(world)]
            dist.all_gather(alld, d)
            want = rew.counts + d + sum(alld) - d          # own increments were already added locally
            rew.counts.add_(d)
            rew.delta.copy_(d)
            torch.cuda.synchronize()
            comm.merge_counts(rew)
            torch.cuda.synchronize()
            comm.check()
            assert torch.equal(rew.counts, want)
            assert not rew.delta.any()
        del graph
        comm.close()
        return f"ok err<1e-4 n={n}"

    _report(q, rank, body)


def run_spawn(fn, world: int, timeout_s: float = 240.0):
    """Spawn ``world`` ranks of ``fn`` and collect their reports (bounded)."""
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    reports = {}
    import queue as _q
    import time
    deadline = time.time() + timeout_s
    while len(reports) < world and time.time() < deadline:
        try:
            r, ok, msg = q.get(timeout=1.0)
            reports[r] = (ok, msg)
        except _q.Empty:
            if all(not p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=max(1.0, deadline - time.time()))
        if p.is_alive():
            p.kill()
            p.join(5)
    return reports, [p.exitcode for p in procs]
