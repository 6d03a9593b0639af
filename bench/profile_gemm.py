"""Run one GEMM case a few times (for ncu captures of a single launch).

    python bench/profile_gemm.py --case conv1 --batch 4096 --iters 3
"""
import argparse
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import surfb200  # noqa: E402,F401
from surfb200.ops import gemm as G  # noqa: E402

CASES = {   # name -> (M per batch row, N, K, a_mn, b_mn)
    "conv1": (465, 32, 64, False, False),
    "conv2": (84, 64, 512, False, False),
    "fc": (1, 512, 3072, False, False),
    "fc_dgrad": (1, 3072, 512, False, True),
}

ap = argparse.ArgumentParser()
ap.add_argument("--case", default="conv1")
ap.add_argument("--batch", type=int, default=4096)
ap.add_argument("--iters", type=int, default=3)
ap.add_argument("--debug", type=int, default=0)
ap.add_argument("--time", action="store_true")
a = ap.parse_args()
mr, N, K, a_mn, b_mn = CASES[a.case]
M = mr * a.batch
A = torch.randn((K, M) if a_mn else (M, K), device="cuda").to(torch.bfloat16)
B = torch.randn((K, N) if b_mn else (N, K), device="cuda").to(torch.bfloat16)
out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
for _ in range(a.iters):
    G.gemm(A, B, a_mn=a_mn, b_mn=b_mn, out=out, debug=a.debug)
torch.cuda.synchronize()
G.check_error_flag("cuda")
if a.time:
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        G.gemm(A, B, a_mn=a_mn, b_mn=b_mn, out=out, debug=a.debug)
    e1.record()
    torch.cuda.synchronize()
    print(f"{a.case} debug={a.debug} M={M} N={N} K={K}: {e0.elapsed_time(e1) / 10 * 1000:.1f} us")
else:
    print("ok", a.case, M, N, K)
