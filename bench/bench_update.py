"""Per-op device times of one PPO minibatch update (forward, loss, backward, Adam).

The reference's isolated minibatch bench is tools/bench_update.py; this one
runs the framework's own kernels eagerly at the benchmark minibatch (32,768
rows = 2048 envs x 128 decisions / 8 minibatches), wraps every entry point of
ops.gemm / ops.rl in CUDA-event pairs on the launching stream, and prints the
time of each call after warm-up, with the FLOPs of the GEMMs and the achieved
TFLOP/s.

    python bench/bench_update.py [--rows 32768] [--iters 5] [--json out.json] [--verify]

``--verify`` is the numerics gate (reference: tools/bench_update.py:207-243,
compiled vs eager): one minibatch through the tensor-core kernels (forward,
fused PPO loss, backward) against the same minibatch in float32 autograd
(``PolicyNet.forward_reference`` + ``ppo_loss_reference``) over identical
bf16-rounded weights and inputs. It passes when the loss agrees within 1e-3
relative and the flat gradient's cosine similarity is at least 0.99.
"""
from __future__ import annotations

import argparse
import collections
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=32768)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--json", default=None)
    ap.add_argument("--explicit", action="store_true", help="im2col + GEMM for every convolution (A/B baseline)")
    ap.add_argument("--no-shift", action="store_true",
                    help="4-D implicit GEMMs instead of the stacked shifted-grid trunk (A/B baseline)")
    ap.add_argument("--nhw", action="store_true", help="64 x 128 NHW image with the 8x8 stride-4 first layer")
    ap.add_argument("--verify", action="store_true", help="numerics gate: kernels vs float32 autograd, then exit")
    args = ap.parse_args()
    import torch
    import surfb200  # noqa: F401
    from surfb200.models.policy import (HeadLayout, NetConfig, PolicyNet, Workspace, backward_gpu, forward_gpu,
                                        space_to_depth_config)
    from surfb200.ops import conv as CV
    from surfb200.ops import gemm as G
    from surfb200.ops import rl as R

    dev = torch.device("cuda")
    layout = HeadLayout(("yaw", "pitch", "fwd", "side", "jump", "duck"), False)
    ncfg = NetConfig(vision=True, img_h=64, img_w=128, n_scalar=10, scalar_pad=16, heads=layout)
    if not args.nhw:                     # the trainer's layout: 4x4 space-to-depth image, conv1 as 2x2 stride 1
        ncfg = space_to_depth_config(ncfg)
    net = PolicyNet(ncfg, dev)
    B = args.rows
    net.implicit_conv = not args.explicit
    net.shift_conv = not (args.no_shift or args.explicit)
    ws = Workspace(net, B)
    opt = R.Adam(net)
    heads = R.HeadArgs(layout, dev)
    g = torch.Generator(device=dev).manual_seed(0)
    img = torch.rand(B, 64 * 128, device=dev, generator=g).to(torch.bfloat16)
    scal = torch.randn(B, 16, device=dev, generator=g).to(torch.bfloat16)
    act = torch.zeros(B, 8, dtype=torch.int32, device=dev)
    old_logp = torch.zeros(B, device=dev)
    adv = torch.randn(B, device=dev, generator=g)
    ret = torch.randn(B, device=dev, generator=g)
    idx = torch.arange(B, device=dev)
    mom = torch.tensor([float(adv.sum()), float((adv * adv).sum())], dtype=torch.float64, device=dev)
    coef = torch.tensor([0.2, 0.5, 0.005], device=dev)
    stats = torch.zeros(6, device=dev)

    if args.verify:
        res = verify(net, ws, layout, heads, scal, img, adv, ret, coef)
        print(json.dumps(res))
        if args.json:
            Path(args.json).write_text(json.dumps(res, indent=1))
        sys.exit(0 if res["pass"] else 1)

    records = []
    active = [False]

    def wrap(mod, name):
        fn = getattr(mod, name)

        def inner(*a, **k):
            if not active[0]:
                return fn(*a, **k)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            r = fn(*a, **k)
            e1.record()
            desc = ""
            if name == "gemm":
                A, Bm = a[0], a[1]
                M = k.get("M") or (A.shape[1] if k.get("a_mn") else A.shape[0])
                Kd = k.get("K") or (A.shape[0] if k.get("a_mn") else A.shape[1])
                N = (Bm.shape[1] if k.get("b_mn") else Bm.shape[0])
                desc = f"{M}x{N}x{Kd}{' mnA' if k.get('a_mn') else ''}{' mnB' if k.get('b_mn') else ''}"
                flops = 2.0 * M * N * Kd
            elif name in TRUNK_FLOPS:
                flops = float(TRUNK_FLOPS[name]) * B
            else:
                flops = 0.0
            records.append((name, desc, flops, e0, e1))
            return r
        setattr(mod, name, inner)

    for n in ("gemm", "im2col", "col2im", "colsum", "gather_rows", "to_bf16"):
        wrap(G, n)
    for n in ("ppo_loss",):
        wrap(R, n)
    for n in ("conv_forward", "conv_weight_grad", "conv_input_grad", "weight_classes"):
        wrap(CV, n)
    # the stacked shifted-grid trunk: useful FLOPs per image of each product
    c1, c2, c3 = 2 * 465 * 32 * 64, 2 * 84 * 64 * 512, 2 * 48 * 64 * 576
    TRUNK_FLOPS = {"conv1_forward": c1, "conv2_forward": c2, "conv3_forward": c3, "conv3_input_grad": c3,
                   "conv2_input_grad": c2, "conv3_weight_grad": c3, "conv2_weight_grad": c2, "conv1_weight_grad": c1}
    if net.uses_shift_trunk():
        for n in ("refresh", *TRUNK_FLOPS):
            wrap(net.trunk, n)


    def step():
        out = forward_gpu(net, ws, scal, img)
        R.ppo_loss(out, layout.value_col, act, old_logp, adv, ret, idx, mom, heads, net.p("log_std"), coef, float(B),
                   ws.dout16, net.g("log_std"), stats)
        backward_gpu(net, ws, scal)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        opt.step()
        e1.record()
        if active[0]:                                   # as the wrapped ops: timed steps only
            records.append(("adam", f"{net.numel}", 0.0, e0, e1))

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    active[0] = True
    t0.record()
    for _ in range(args.iters):
        step()
    t1.record()
    torch.cuda.synchronize()
    per_iter = len(records) // args.iters
    agg = collections.OrderedDict()
    for i, (name, desc, flops, e0, e1) in enumerate(records):
        key = (i % per_iter, name, desc)
        ms = e0.elapsed_time(e1)
        a = agg.setdefault(key, [0.0, flops])
        a[0] += ms / args.iters
    total = sum(v[0] for v in agg.values())
    rows = []
    print(f"{'#':>3} {'op':<12} {'shape':<28} {'ms':>8} {'%':>6} {'TFLOP/s':>8}")
    for (i, name, desc), (ms, flops) in agg.items():
        tf = flops / (ms * 1e-3) / 1e12 if flops and ms > 0 else 0.0
        rows.append({"i": i, "op": name, "shape": desc, "ms": round(ms, 4), "tflops": round(tf, 1)})
        print(f"{i:>3} {name:<12} {desc:<28} {ms:8.3f} {100 * ms / total:6.1f} {tf:8.1f}")
    wall = t0.elapsed_time(t1) / args.iters
    print(f"sum of ops {total:.3f} ms; minibatch step (events around the whole step, incl. gaps) {wall:.3f} ms")
    if args.json:
        Path(args.json).write_text(json.dumps({"rows": B, "ops": rows, "sum_ms": total, "step_ms": wall}, indent=1))


def verify(net, ws, layout, heads, scal, img, adv, ret, coef, loss_tol: float = 1e-3, cos_min: float = 0.99) -> dict:
    """One minibatch on the kernels vs float32 autograd (see the module docstring)."""
    import torch
    from surfb200.models.policy import backward_gpu, forward_gpu
    from surfb200.ops import rl as R
    from surfb200.ops.gemm import check_error_flag
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    dev = net.flat.device
    B = scal.shape[0]
    net.flat.copy_(net.flat.to(torch.bfloat16).float())      # both paths see the same (bf16) weights
    net.sync_bf16()
    # actions and old log-probs drawn from the policy itself, perturbed so that
    # the ratio spreads past the clip range on part of the rows
    out = forward_gpu(net, ws, scal, img)
    act = torch.zeros(B, 8, dtype=torch.int32, device=dev)
    logp = torch.zeros(B, device=dev)
    R.sample_heads(out, heads, net.p("log_std"), act, logp, seed=7, counter=0)
    old_logp = logp + 0.3 * torch.randn(B, device=dev)
    idx = torch.arange(B, device=dev)
    mom = torch.stack([adv.double().sum(), (adv.double() ** 2).sum()])
    stats = torch.zeros(6, device=dev)
    net.grad.zero_()
    out = forward_gpu(net, ws, scal, img)
    R.ppo_loss(out, layout.value_col, act, old_logp, adv, ret, idx, mom, heads, net.p("log_std"), coef, float(B),
               ws.dout16, net.g("log_std"), stats)
    backward_gpu(net, ws, scal)
    torch.cuda.synchronize()
    check_error_flag(dev)
    clip, vf, ent = (float(x) for x in coef.tolist())
    st = stats.double().cpu()
    loss_gpu = float((st[0] + vf * st[1] - ent * st[2]) / B)
    grad_gpu = net.grad.clone()

    params = net.autograd_params()
    ref_out = net.forward_reference(scal.float(), img.float(), params)
    loss, pg, vl, H = R.ppo_loss_reference(ref_out, layout.value_col, act, old_logp, adv, ret, layout,
                                           params["log_std"], clip, vf, ent,
                                           moments=(float(mom[0]), float(mom[1]), float(B)))
    loss.backward()
    grad_ref = torch.zeros_like(grad_gpu)
    for name, t in params.items():
        if t.grad is not None:
            net.view(name, grad_ref).copy_(t.grad)
    rel = abs(loss_gpu - float(loss)) / max(abs(float(loss)), 1e-12)
    cos = float(torch.nn.functional.cosine_similarity(grad_gpu.double(), grad_ref.double(), dim=0))
    grad_rel = float((grad_gpu - grad_ref).norm() / grad_ref.norm().clamp_min(1e-30))
    per_layer = {}
    for name, *_ in net.specs:
        a, b = net.view(name, grad_gpu).flatten(), net.view(name, grad_ref).flatten()
        if float(b.norm()) > 0:
            per_layer[name] = round(float(torch.nn.functional.cosine_similarity(a.double(), b.double(), dim=0)), 5)
    net.grad.zero_()
    return {"verify": "minibatch kernels vs float32 autograd", "rows": B, "loss_gpu": loss_gpu, "loss_fp32": float(loss),
            "loss_rel_err": rel, "grad_cos": cos, "grad_rel_err": grad_rel, "layer_cos": per_layer,
            "thresholds": {"loss_rel_err": loss_tol, "grad_cos": cos_min},
            "pass": bool(rel <= loss_tol and cos >= cos_min)}


if __name__ == "__main__":
    main()
