"""What does more capacity cost? One PPO minibatch step (forward, fused loss,
backward, clip + Adam) through the trainer's kernels, across capacity axes:
network width (fc / hidden / conv channels), depth image resolution, stacked
frames and the surface-mask channel (reference: tools/bench_capacity.py:1-25).

    python bench/bench_capacity.py [--rows 16384] [--variants base,hidden1024,stack4]

Each variant reports the CUDA-event time of one step (median of --iters after
--warmup) and the parameter count. Frame stacking needs no extra rollout
storage (the stack is gathered from the per-decision frames), so its cost here
is the whole story.
"""
from __future__ import annotations

import argparse
import json
import statistics
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

# name -> (lidar_w, lidar_h, fc, hidden, conv channel multiplier, image channels per pixel)
VARIANTS = {
    "base": (128, 64, 512, 512, 1, 1),
    "hidden1024": (128, 64, 512, 1024, 1, 1),
    "hidden2048": (128, 64, 512, 2048, 1, 1),
    "fc1024": (128, 64, 1024, 512, 1, 1),
    "conv2x": (128, 64, 512, 512, 2, 1),
    "surfmask": (128, 64, 512, 512, 1, 2),
    "stack2": (128, 64, 512, 512, 1, 2),
    "stack4": (128, 64, 512, 512, 1, 4),
    "lidar256x128": (256, 128, 512, 512, 1, 1),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=16384)
    ap.add_argument("--variants", default=",".join(VARIANTS))
    ap.add_argument("--iters", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--json", default=None)
    args = ap.parse_args()
    import torch
    import surfb200  # noqa: F401
    from surfb200.models.policy import (HeadLayout, NetConfig, PolicyNet, Workspace, backward_gpu, forward_gpu,
                                        space_to_depth_config)
    from surfb200.ops import gemm as G
    from surfb200.ops import rl as R
    dev = torch.device("cuda")
    B = args.rows
    layout = HeadLayout(("yaw", "pitch", "fwd", "side", "jump", "duck"), False)
    heads = R.HeadArgs(layout, dev)
    g = torch.Generator(device=dev).manual_seed(0)
    out_rows = []
    for name in args.variants.split(","):
        w, h, fc, hidden, cm, ch = VARIANTS[name]
        conv = ((8, 4, 32 * cm), (4, 2, 64 * cm), (3, 1, 64 * cm))
        ncfg = space_to_depth_config(NetConfig(img_h=h, img_w=w, img_c=ch, conv=conv, fc=fc, hidden=hidden,
                                               heads=layout))
        net = PolicyNet(ncfg, dev)
        ws = Workspace(net, B)
        opt = R.Adam(net)
        img = torch.rand(B, w * h * ch, device=dev, generator=g).to(torch.bfloat16)
        scal = torch.randn(B, 16, device=dev, generator=g).to(torch.bfloat16)
        act = torch.zeros(B, 8, dtype=torch.int32, device=dev)
        old = torch.zeros(B, device=dev)
        adv = torch.randn(B, device=dev, generator=g)
        ret = torch.randn(B, device=dev, generator=g)
        idx = torch.arange(B, device=dev)
        mom = torch.tensor([float(adv.sum()), float((adv * adv).sum())], dtype=torch.float64, device=dev)
        coef = torch.tensor([0.2, 0.5, 0.005], device=dev)
        stats = torch.zeros(6, device=dev)

        def step():
            out = forward_gpu(net, ws, scal, img)
            R.ppo_loss(out, layout.value_col, act, old, adv, ret, idx, mom, heads, net.p("log_std"), coef, float(B),
                       ws.dout16, net.g("log_std"), stats)
            backward_gpu(net, ws, scal)
            opt.step()

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        times = []
        for _ in range(args.iters):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            step()
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        ms = statistics.median(times)
        row = {"variant": name, "rows": B, "ms_per_minibatch": round(ms, 3), "params": net.numel,
               "implicit_convs": sum(ws.implicit), "lidar": f"{w}x{h}", "fc": fc, "hidden": hidden,
               "conv_mult": cm, "image_channels": ch}
        print(json.dumps(row), flush=True)
        out_rows.append(row)
        del net, ws, opt, img
        torch.cuda.empty_cache()
    if args.json:
        Path(args.json).write_text(json.dumps(out_rows, indent=1))


if __name__ == "__main__":
    main()
