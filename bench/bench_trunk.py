"""Per-op device times of the vision trunk's convolutions: the stacked
shifted-grid kernels (ops/conv_shift.py, padded-grid layouts) against the
4-D-box implicit GEMMs (ops/conv.py, dense layouts), same batch, CUDA
events, median of --reps after a warm-up. Inputs are larger than L2 at the
default batch.

    python bench/bench_trunk.py [--batch 32768] [--reps 5] [--json out.json]
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=32768)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--json", default=None)
    ap.add_argument("--only", default=None, help="comma list of ops")
    ap.add_argument("--trace", action="store_true", help="CTA 0's pipeline timeline of the shifted kernels")
    ap.add_argument("--dbg", type=int, default=0, help="kernel diagnostics: 1 skip epilogue stores, 2 skip MMAs")
    args = ap.parse_args()
    import torch
    import surfb200  # noqa: F401
    from surfb200.ops import conv as CV
    from surfb200.ops import conv_shift as S
    dev = torch.device("cuda")
    B = args.batch
    g = torch.Generator(device=dev).manual_seed(0)
    rnd = lambda *sh: (torch.randn(*sh, device=dev, generator=g) * 0.1).to(torch.bfloat16)
    w1, w2, w3 = rnd(32, 64), rnd(64, 512), rnd(64, 576)
    flat = torch.cat([w1.view(-1), torch.zeros(64, dtype=torch.bfloat16, device=dev), w2.view(-1), w3.view(-1)])
    T = S.Trunk(dev, [0, 32 * 64 + 64, 32 * 64 + 64 + 64 * 512])
    T.refresh(flat)
    b1, b2, b3 = (torch.zeros(n, device=dev) for n in (32, 64, 64))
    sh1, sh2, sh3 = (CV.ConvShape(B, 16, 32, 16, 2, 1, 32), CV.ConvShape(B, 15, 31, 32, 4, 2, 64),
                     CV.ConvShape(B, 6, 14, 64, 3, 1, 64))
    wc3, wc2 = CV.weight_classes(w3, sh3), CV.weight_classes(w2, sh2)
    gw1, gw2, gw3 = torch.zeros(32, 64, device=dev), torch.zeros(64, 512, device=dev), torch.zeros(64, 576, device=dev)
    img = rnd(B * 512 + 64, 16)[:B * 512]
    # shifted-grid layouts (padded grids)
    y1 = rnd(B * 512, 32)
    y2, dy2, dy3 = rnd(B * 128, 64), rnd(B * 128, 64), rnd(B * 128, 64)
    y3 = torch.empty(B * 48, 64, dtype=torch.bfloat16, device=dev)
    dy1 = torch.empty(B * 512, 32, dtype=torch.bfloat16, device=dev)
    # 4-D-box implicit GEMM operands (dense layouts with slack rows)
    x1 = rnd(B * 465 * 32 + 64, 1)[:B * 465 * 32].view(-1, 32)
    x2 = rnd(B * 84 * 64 + 64, 1)[:B * 84 * 64].view(-1, 64)
    o1, o2, o3 = (torch.empty(B * n, c, dtype=torch.bfloat16, device=dev) for n, c in ((465, 32), (84, 64), (48, 64)))
    d1 = rnd(B * 465 * 32 + 64, 1)[:B * 465 * 32].view(-1, 32)
    d2 = rnd(B * 84 * 64 + 64, 1)[:B * 84 * 64].view(-1, 64)
    d3 = rnd(B * 48 * 64 + 64, 1)[:B * 48 * 64].view(-1, 64)
    ops = {
        "conv1_fwd": (lambda: T.conv1_forward(img, b1, y1, B), lambda: CV.conv_forward(img, sh1, w1, b1, o1)),
        "conv2_fwd": (lambda: T.conv2_forward(y1, b2, y2, B), lambda: CV.conv_forward(x1, sh2, w2, b2, o2)),
        "conv3_fwd": (lambda: T.conv3_forward(y2, b3, y3, B), lambda: CV.conv_forward(x2, sh3, w3, b3, o3)),
        "conv3_dgrad": (lambda: T.conv3_input_grad(dy3, y2, dy2, B), lambda: CV.conv_input_grad(d3, sh3, wc3, o2, x2)),
        "conv2_dgrad": (lambda: T.conv2_input_grad(dy2, y1, dy1, B), lambda: CV.conv_input_grad(d2, sh2, wc2, o1, x1)),
        "conv3_wgrad": (lambda: T.conv3_weight_grad(dy3, y2, gw3, B), lambda: CV.conv_weight_grad(d3, x2, sh3, gw3)),
        "conv2_wgrad": (lambda: T.conv2_weight_grad(dy2, y1, gw2, B), lambda: CV.conv_weight_grad(d2, x1, sh2, gw2)),
        "conv1_wgrad": (lambda: T.conv1_weight_grad(dy1, img, gw1, B), lambda: CV.conv_weight_grad(d1, img, sh1, gw1)),
    }
    flop = {"conv1_fwd": 2 * 465 * 32 * 64, "conv2_fwd": 2 * 84 * 64 * 512, "conv3_fwd": 2 * 48 * 64 * 576}
    flop.update({"conv3_dgrad": flop["conv3_fwd"], "conv2_dgrad": flop["conv2_fwd"], "conv1_wgrad": flop["conv1_fwd"],
                 "conv2_wgrad": flop["conv2_fwd"], "conv3_wgrad": flop["conv3_fwd"]})

    def timed(fn):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(args.reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return sorted(ts)[len(ts) // 2]

    import numpy as np
    from surfb200.ops import gemm as G
    res = {}
    tot = [0.0, 0.0]
    for name, (new, old) in ops.items():
        if args.only and name not in args.only.split(","):
            continue
        to = timed(old)
        CV.DEBUG = args.dbg
        if args.trace:
            CV.TRACE = torch.zeros(8 * G.TRACE_N, dtype=torch.int64, device=dev)
        tn = timed(new)
        if args.trace:
            tr = CV.TRACE.view(8, G.TRACE_N).cpu().numpy().astype(np.float64)
            CV.TRACE = None
            t0 = tr[0, 0]
            rows = [[(x - t0) / 1e3 for x in r if x > 0] for r in tr]
            iss, land, com, acc, done, pre, ld0, cend = rows
            n = min(len(iss), len(land), len(com))
            print(f"  trace {name}: units {len(iss)}; issue gaps {np.median(np.diff(iss[4:])) if len(iss) > 5 else 0:.3f} us, "
                  f"issue->landed {np.median(np.array(land[:n]) - np.array(iss[:n])):.3f} us, "
                  f"landed->committed {np.median(np.array(com[:n]) - np.array(land[:n])):.3f} us, "
                  f"landed gaps {np.median(np.diff(land[4:])) if len(land) > 5 else 0:.3f} us; "
                  f"tiles {len(acc)}, acc gaps {np.median(np.diff(acc)) if len(acc) > 2 else 0:.3f} us, "
                  f"epilogue {np.median(np.array(done[:len(acc)]) - np.array(acc[:len(done)])) if acc else 0:.3f} us",
                  flush=True)
            if pre and ld0 and cend:
                m = min(len(pre), len(acc), len(ld0), len(cend), len(done))
                P, A, L0, E, D = (np.array(x[:m]) for x in (pre, acc, ld0, cend, done))
                print(f"    epilogue split: prev done->pre-pass {np.median(P[1:] - D[:-1]) if m > 1 else 0:.3f} us, "
                      f"pre->acc ready {np.median(A - P):.3f} us, acc->first TMEM load {np.median(L0 - A):.3f} us, "
                      f"chunks {np.median(E - L0):.3f} us, copy-out {np.median(D - E):.3f} us", flush=True)
        CV.DEBUG = 0
        tot[0] += tn
        tot[1] += to
        tf = flop[name] * B / (tn * 1e-3) / 1e12
        res[name] = {"shifted_ms": round(tn, 4), "boxes_ms": round(to, 4), "speedup": round(to / tn, 2),
                     "useful_tflops": round(tf, 1)}
        print(f"{name:12s} shifted {tn:7.3f} ms ({tf:6.1f} TFLOP/s useful)   4-D boxes {to:7.3f} ms   x{to / tn:5.2f}",
              flush=True)
    print(f"{'total':12s} shifted {tot[0]:7.3f} ms   4-D boxes {tot[1]:7.3f} ms   x{tot[1] / tot[0]:5.2f}")
    out = {"batch": B, "ops": res, "total_shifted_ms": tot[0], "total_boxes_ms": tot[1]}
    if args.json:
        Path(args.json).write_text(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
