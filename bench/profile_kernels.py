"""Small, self-contained launches of each hot kernel, for ncu captures.

    python bench/profile_kernels.py --only march|conv1_fwd|conv2_dgrad|fc_wgrad|col2im|im2col|conv1_ifwd|
                                           conv1_iwgrad|conv2_ifwd|
                                           conv2_iwgrad|conv2_idgrad|conv3_ifwd|conv3_iwgrad|conv3_idgrad|sample|gae|
                                           ppo_loss|reward|adam|p2p1|edt|geodesic|geodesic_race|surfnz|framestack [--reps 2]

Each case builds its inputs (a few GB on the device at most, larger than L2
where the kernel streams memory), warms up once, then launches the kernel
``--reps`` times and prints the CUDA-event time per launch. Pair it with
``ncu --set full --clock-control none -k regex:<kernel> -s 1 -c 1``.
Shapes: the benchmark's 2048 envs x 128 x 64 rays, 2048-row sampling,
128 x 2048 GAE, 32,768-row loss; the convolution cases use 4,096 images
(operands still larger than L2) to keep the captures small.
"""
from __future__ import annotations

import argparse
import json
import sys
from ctypes import c_void_p
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def _time(fn, reps):
    import torch
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", required=True)
    ap.add_argument("--reps", type=int, default=2)
    ap.add_argument("--dbg", type=int, default=0, help="convolution kernel diagnostics (timing studies): "
                    "1 skip epilogue stores, 2 skip MMAs, 4 stream B per k-block instead of keeping it resident, "
                    "8 no saved-activation prefetch in the derivative epilogues")
    ap.add_argument("--trace", action="store_true", help="convolution cases: add CTA 0's pipeline timeline "
                    "(first 256 k-blocks / tiles of the last launch, microseconds) to the output")
    ap.add_argument("--wgrad-splits", type=int, default=0, help="weight-gradient cases: K splits (0: the default)")
    ap.add_argument("--march-flags", type=int, default=0, help="march case: extra kernel flag bits (timing studies)")
    ap.add_argument("--sort-poses", type=int, default=0, help="march case: order the envs by position cells of this "
                    "many units (0: random order) -- the L2 reuse of neighbouring cameras")
    ap.add_argument("--no-pairs", action="store_true", help="16-channel convolution inputs: one 32-byte tap per "
                    "box row instead of two-position windows")
    args = ap.parse_args()
    import numpy as np
    import torch
    import surfb200  # noqa: F401
    from surfb200.models.policy import HeadLayout, NetConfig, PolicyNet
    from surfb200.ops import gemm as G
    from surfb200.ops import rl as R
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(0)
    k = args.only
    info = {"case": k}

    if k == "march":
        from surfb200.ops import vision
        from surfb200.sim import mapgen
        from surfb200.sim.core import SimCore, default_config
        sys.path.insert(0, str(ROOT / "bench"))
        from bench_march import free_space_poses
        m = mapgen.generate("field", 0)
        core = SimCore.from_bytes(m.image, default_config(1), threads=4)
        vol = vision.SdfVolume.build(core, cell=m.meta["cell"], mins=np.array(m.meta["grid_mins"]),
                                     dims=tuple(m.meta["dims"]))
        vision.MARCH_DIAG_FLAGS = args.march_flags
        cam = vision.DepthCamera(vol, 128, 64, range_units=2000.0, max_steps=64, dtype=torch.bfloat16)
        pose = free_space_poses(vol, 2048, 1)
        if args.sort_poses:
            # Morton order of (x, y) cells: consecutive envs (blocks) are neighbours
            c = ((pose[:, :2] - pose[:, :2].min(0).values) / args.sort_poses).long().cpu().numpy()
            code = np.zeros(len(c), np.int64)
            for b in range(16):
                code |= ((c[:, 0] >> b) & 1) << (2 * b) | ((c[:, 1] >> b) & 1) << (2 * b + 1)
            pose = pose[torch.as_tensor(np.argsort(code), device=pose.device)].contiguous()
        out = torch.empty((2048, 128 * 64), dtype=torch.bfloat16, device=dev)
        info["ms"] = _time(lambda: cam.render(pose, out=out), args.reps)
        info["rays"] = 2048 * 128 * 64
    elif k in ("conv1_fwd", "conv2_dgrad", "fc_wgrad", "col2im", "im2col"):
        # B = 4096 images: every operand still exceeds L2, the device holds ~1 GB
        layout = HeadLayout(("yaw", "pitch", "fwd", "side", "jump", "duck"), False)
        net = PolicyNet(NetConfig(heads=layout), dev)
        B = 4096
        sh = net.cfg.conv_shapes()
        rnd = lambda *shape: (torch.randn(*shape, device=dev, generator=gen) * 0.1).to(torch.bfloat16)
        if k == "conv1_fwd":
            g = sh[0]
            rows = B * g["OH"] * g["OW"]
            col, y = rnd(rows, 64), torch.empty(rows, g["CO"], dtype=torch.bfloat16, device=dev)
            fn = lambda: G.gemm(col, net.w16("conv1.w"), out=y, bias=net.p("conv1.b"), act="relu")
            info["flops"] = 2.0 * rows * g["CO"] * 64
        elif k == "conv2_dgrad":
            g = sh[1]
            rows = B * g["OH"] * g["OW"]
            dy, dcol = rnd(rows, g["CO"]), torch.empty(rows, g["k"] ** 2 * g["C"], dtype=torch.bfloat16, device=dev)
            fn = lambda: G.gemm(dy, net.w16("conv2.w"), b_mn=True, out=dcol)
            info["flops"] = 2.0 * rows * g["CO"] * g["k"] ** 2 * g["C"]
        elif k == "fc_wgrad":
            df, feat = rnd(B, net.cfg.fc), rnd(B, net.cfg.flat_conv)
            fn = lambda: G.gemm(df, feat, a_mn=True, b_mn=True, out=net.g("fc.w"), accumulate=True, splits=4, bn=256,
                                K=B)
            info["flops"] = 2.0 * B * net.cfg.fc * net.cfg.flat_conv
        elif k == "col2im":
            g = sh[1]
            rows = B * g["OH"] * g["OW"]
            dcol = rnd(rows, g["k"] ** 2 * g["C"])
            x_act = torch.relu(rnd(B, g["H"], g["W"], g["C"]).float()).to(torch.bfloat16)
            dx = torch.empty(B, g["H"], g["W"], g["C"], dtype=torch.bfloat16, device=dev)
            fn = lambda: G.col2im(dcol, x_act, B, g["H"], g["W"], g["C"], g["k"], g["s"], out=dx)
            info["bytes"] = 2.0 * (rows * g["k"] ** 2 * g["C"] + 2 * B * g["H"] * g["W"] * g["C"])
        else:
            g = sh[1]
            rows = B * g["OH"] * g["OW"]
            x = rnd(B * g["H"] * g["W"], g["C"])
            col = torch.empty(rows, g["k"] ** 2 * g["C"], dtype=torch.bfloat16, device=dev)
            fn = lambda: G.im2col(x, B, g["H"], g["W"], g["C"], g["k"], g["s"], out=col)
            info["bytes"] = 2.0 * (rows * g["k"] ** 2 * g["C"] + B * g["H"] * g["W"] * g["C"])
        info["ms"] = _time(fn, args.reps)
    elif k in ("conv1_ifwd", "conv1_iwgrad", "conv2_ifwd", "conv2_iwgrad", "conv2_idgrad", "conv3_ifwd", "conv3_iwgrad",
               "conv3_idgrad"):
        # implicit-GEMM convolutions (4-D TMA boxes over the NHWC activations),
        # 4,096 images as above
        from surfb200.ops import conv as CV
        CV.DEBUG = args.dbg
        CV.PAIR_WINDOWS = not args.no_pairs
        info["dbg"] = args.dbg
        info["pairs"] = CV.PAIR_WINDOWS
        if args.trace:
            CV.TRACE = torch.zeros(5 * G.TRACE_N, dtype=torch.int64, device=dev)
        layout = HeadLayout(("yaw", "pitch", "fwd", "side", "jump", "duck"), False)
        from surfb200.models.policy import space_to_depth_config
        net = PolicyNet(space_to_depth_config(NetConfig(heads=layout)), dev)    # the trainer's network
        B = 4096
        li = int(k[4]) - 1
        g = net.cfg.conv_shapes()[li]
        sh = CV.ConvShape(B, g["H"], g["W"], g["C"], g["k"], g["s"], g["CO"])
        rows_in, rows = B * g["H"] * g["W"], B * g["OH"] * g["OW"]
        rnd = lambda *shape: (torch.randn(*shape, device=dev, generator=gen) * 0.1).to(torch.bfloat16)
        slack = CV.SLACK_BYTES // 2
        xb = torch.relu(rnd(rows_in * g["C"] + slack).float()).to(torch.bfloat16)
        x = xb[:rows_in * g["C"]].view(rows_in, g["C"])
        w = net.w16(f"conv{li + 1}.w")
        flops = 2.0 * rows * g["CO"] * g["k"] ** 2 * g["C"]
        if k.endswith("ifwd"):
            y = torch.empty(rows, g["CO"], dtype=torch.bfloat16, device=dev)
            fn = lambda: CV.conv_forward(x, sh, w, net.p(f"conv{li + 1}.b"), y)
        elif k.endswith("iwgrad"):
            dy = rnd(rows, g["CO"])
            gw = torch.zeros(g["CO"], g["k"] ** 2 * g["C"], device=dev)
            fn = lambda: CV.conv_weight_grad(dy, x, sh, gw, splits=args.wgrad_splits)
        else:
            dyb = rnd(rows * g["CO"] + slack)
            dy = dyb[:rows * g["CO"]].view(rows, g["CO"])
            wt = CV.weight_classes(w, sh)
            dx = torch.empty(rows_in, g["C"], dtype=torch.bfloat16, device=dev)
            fn = lambda: CV.conv_input_grad(dy, sh, wt, dx, x)
        info["flops"] = flops
        info["ms"] = _time(fn, args.reps)
        info["tflops"] = flops / (info["ms"] * 1e-3) / 1e12
        if args.trace:
            tr = CV.TRACE.view(5, G.TRACE_N).cpu().numpy().astype(np.float64)
            t0 = tr[0, 0]
            us = lambda row: [round((x - t0) / 1e3, 3) if x > 0 else None for x in row]
            info["trace_us"] = {"issue": us(tr[0]), "landed": us(tr[1]), "committed": us(tr[2]),
                                "acc_ready": us(tr[3]), "tile_done": us(tr[4])}
    elif k in ("sample", "ppo_loss", "gae"):
        layout = HeadLayout(("yaw", "pitch", "fwd", "side", "jump", "duck"), False)
        heads = R.HeadArgs(layout, dev)
        log_std = torch.zeros(1, device=dev)
        if k == "sample":
            n = 2048
            logits = torch.randn(n, 64, device=dev, generator=gen)
            act = torch.zeros(n, 8, dtype=torch.int32, device=dev)
            logp = torch.zeros(n, device=dev)
            fn = lambda: R.sample_heads(logits, heads, log_std, act, logp, 1234, 0)
        elif k == "gae":
            T, n = 128, 2048
            rew, val, done = (torch.randn(T, n, device=dev, generator=gen) for _ in range(3))
            done = (done > 1.5).float()
            last = torch.randn(n, device=dev, generator=gen)
            adv, ret = torch.zeros(T, n, device=dev), torch.zeros(T, n, device=dev)
            mom = torch.zeros(2, dtype=torch.float64, device=dev)
            fn = lambda: R.gae(rew, val, done, last, 0.9985, 0.95, adv, ret, mom)
        else:
            B = 32768
            out = torch.randn(B, 64, device=dev, generator=gen)
            act = torch.zeros(B, 8, dtype=torch.int32, device=dev)
            old = torch.zeros(B, device=dev)
            adv, ret = torch.randn(B, device=dev, generator=gen), torch.randn(B, device=dev, generator=gen)
            idx = torch.arange(B, device=dev)
            mom = torch.tensor([float(adv.sum()), float((adv * adv).sum())], dtype=torch.float64, device=dev)
            coef = torch.tensor([0.2, 0.5, 0.005], device=dev)
            dout = torch.zeros(B, 64, device=dev)
            dls = torch.zeros(1, device=dev)
            stats = torch.zeros(6, device=dev)
            fn = lambda: R.ppo_loss(out, layout.value_col, act, old, adv, ret, idx, mom, heads, log_std, coef, float(B),
                                    dout, dls, stats)
        info["ms"] = _time(fn, args.reps)
    elif k == "reward":
        from surfb200.rewards.spec import GpuReward, RewardSpec
        n = 2048
        rew = GpuReward(RewardSpec(mode="coverage", int_coef=0.25, int_view=8, int_speed=8), n, 3,
                        (np.array([-8192.0, -8192, 0]), np.array([8192.0, 8192, 4096])), dev)
        rec = torch.zeros(n, 16, device=dev)
        rec[:, :3] = torch.rand(n, 3, device=dev, generator=gen) * 8000
        rec[:, 6:9] = torch.randn(n, 3, device=dev, generator=gen) * 300
        rew.init(rec)
        r_out, d_out = torch.zeros(n, device=dev), torch.zeros(n, device=dev)
        info["ms"] = _time(lambda: rew(rec, r_out, d_out), args.reps)
    elif k in ("adam", "p2p1"):
        net = PolicyNet(NetConfig(), dev)
        net.grad.normal_(generator=gen)
        opt = R.Adam(net)
        if k == "adam":
            info["ms"] = _time(opt.step, args.reps)
        else:
            from surfb200.ops import _lib
            from surfb200.parallel import p2p as P
            L = _lib.lib(P.CLIB)
            sync = torch.zeros(int(L.surf_p2p_sync_words()), dtype=torch.int64, device=dev)
            arr = lambda *ps: (c_void_p * len(ps))(*[c_void_p(int(p)) for p in ps])
            plan = L.surf_p2p_create(0, 1, arr(sync.data_ptr()), 5.0)
            L.surf_p2p_set_grad(plan, net.numel, arr(net.grad.data_ptr()), arr(net.flat.data_ptr()),
                                arr(net.flat16.data_ptr()), opt.m.data_ptr(), opt.v.data_ptr(), opt.hyper.data_ptr(),
                                net.fp32_from)
            stream = c_void_p(torch.cuda.current_stream().cuda_stream)
            info["ms"] = _time(lambda: L.surf_p2p_grad_step(plan, stream), args.reps)
            t = [int(x) for x in sync[P.W_PROF:P.W_PROF + 6].tolist()]
            info["phases_us"] = {name: (t[i + 1] - t[i]) / 1e3 for i, name in enumerate(
                ("barrier_in", "reduce_scatter", "norm_exchange", "adam_push", "done_wait"))}
            L.surf_p2p_destroy(plan)
        info["params"] = net.numel
    elif k == "edt":
        from surfb200.ops import vision
        occ = (torch.rand(256, 512, 512, device=dev, generator=gen) > 0.999).to(torch.uint8)
        info["ms"] = _time(lambda: vision.distance_field(occ, 16.0), args.reps)
        info["voxels"] = occ.numel()
    elif k == "framestack":
        # the update's minibatch gather of 4-frame stacks: 16,384 rows of 4 x 8,192 bf16
        from surfb200.ops.framestack import FrameStacker
        st = FrameStacker(4, 128 * 64)
        T, N, mb = 32, 2048, 16384
        frames = (torch.randn(st.pro + T + 1, N, st.fr, device=dev, generator=gen)).to(torch.bfloat16)
        ages = torch.randint(0, st.pro + 1, (T * N,), dtype=torch.int32, device=dev, generator=gen)
        idx = torch.randperm(T * N, device=dev, generator=gen)[:mb]
        out = torch.empty(mb, st.width, dtype=torch.bfloat16, device=dev)
        info["ms"] = _time(lambda: st.gather(frames, idx, ages, out), args.reps)
        info["bytes"] = 2.0 * 2 * mb * st.width
    elif k == "surfnz":
        from surfb200.ops import surfmask, vision
        from surfb200.sim import mapgen
        from surfb200.sim.core import SimCore, default_config
        m = mapgen.generate("field", 0)
        core = SimCore.from_bytes(m.image, default_config(1), threads=4)
        tris = surfmask.solid_triangles(core)
        mn, mx = core.map_bounds()
        mins, nx, ny, nz = vision.grid_dims(mn, mx, 16.0)
        info["ms"] = _time(lambda: surfmask.bake(tris, mins, 16.0, (nx, ny, nz), core=core, linear=False), 1)
        info["triangles"] = len(tris)
        info["voxels"] = nx * ny * nz
    elif k == "geodesic_race":
        # the race track's free-voxel grid at 16u (config 5), seeded at its finish zone
        from surfb200.ops.geodesic import geodesic, seed_box
        from surfb200.ops.vision import grid_dims, occupancy
        from surfb200.sim import mapgen
        from surfb200.sim.core import SimCore, default_config
        m = mapgen.generate("race", 0)
        core = SimCore.from_bytes(m.image, default_config(1), threads=4)
        mn, mx = core.map_bounds()
        mins, nx, ny, nz = grid_dims(mn, mx, 16.0)
        occ = occupancy(core, mins, 16.0, (nx, ny, nz), slab=True, device=dev)
        lo, hi = seed_box(m.zones["end"], mins, 16.0, (nx, ny, nz))
        st = {}
        info["ms"] = _time(lambda: geodesic(occ, 16.0, lo, hi, stats=st), args.reps)
        info["voxels"] = nx * ny * nz
        info["dims"] = [nx, ny, nz]
        info["passes"] = st.get("passes")
    elif k == "geodesic":
        from surfb200.ops.geodesic import geodesic
        occ = torch.zeros(128, 256, 256, dtype=torch.uint8, device=dev)
        occ[:, 100:110, 20:230] = 1
        info["ms"] = _time(lambda: geodesic(occ, 16.0, (5, 5, 5), (10, 10, 10)), 1)
        info["voxels"] = occ.numel()
    else:
        raise SystemExit(f"unknown case {k}")
    print(json.dumps(info))


if __name__ == "__main__":
    main()
