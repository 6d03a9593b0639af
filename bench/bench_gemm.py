"""Tensor-core GEMM microbenchmark: the hand-written tcgen05 kernel vs cuBLAS
(torch.matmul) on a square problem and on the policy network's layer shapes.
Device-timed with CUDA events after warm-up; operands larger than L2.

    python bench/bench_gemm.py [--json out.json]
"""
import argparse
import json
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import surfb200  # noqa: E402,F401
from surfb200.ops import gemm as G  # noqa: E402


def timeit(fn, iters=20, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    for a, b in ev:
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    ms = sorted(a.elapsed_time(b) for a, b in ev)
    return ms[len(ms) // 2]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", default=None)
    ap.add_argument("--batch", type=int, default=32768)
    args = ap.parse_args()
    Bt = args.batch
    # (name, M, N, K, a_mn, b_mn, bn)
    cases = [
        ("square_8192", 8192, 8192, 8192, False, False, 256),
        ("conv1_fwd", Bt * 465, 32, 64, False, False, 32),
        ("conv2_fwd", Bt * 84, 64, 512, False, False, 64),
        ("conv3_fwd", Bt * 48, 64, 576, False, False, 64),
        ("fc_fwd", Bt, 512, 3072, False, False, 256),
        ("tower_fwd", Bt, 512, 768, False, False, 256),
        ("fc_dgrad", Bt, 3072, 512, False, True, 256),
        ("fc_wgrad", 512, 3072, Bt, True, True, 256),
        ("conv3_wgrad_t", 576, 64, Bt * 48, True, True, 64),
    ]
    res = []
    for name, M, N, K, a_mn, b_mn, bn in cases:
        A = torch.randn((K, M) if a_mn else (M, K), device="cuda").to(torch.bfloat16)
        B = torch.randn((K, N) if b_mn else (N, K), device="cuda").to(torch.bfloat16)
        acc = K > 100000
        out = torch.zeros(M, N, device="cuda") if acc else torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        splits = max(1, 148 // (((M + 127) // 128) * ((N + bn - 1) // bn))) if acc else 1
        ms = timeit(lambda: G.gemm(A, B, a_mn=a_mn, b_mn=b_mn, out=out, accumulate=acc, splits=splits, bn=bn))
        G.check_error_flag("cuda")
        a_ = A.t() if a_mn else A
        b_ = B if b_mn else B.t()
        ms_ref = timeit(lambda: torch.matmul(a_, b_))
        tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
        tf_ref = 2.0 * M * N * K / (ms_ref * 1e-3) / 1e12
        byts = (M * K + N * K) * 2 + M * N * (4 if acc else 2)
        r = dict(case=name, M=M, N=N, K=K, splits=splits, ms=ms, tflops=tf, gbs=byts / (ms * 1e-3) / 1e9,
                 cublas_ms=ms_ref, cublas_tflops=tf_ref)
        print(json.dumps(r), flush=True)
        res.append(r)
        del A, B, out
        torch.cuda.empty_cache()
    if args.json:
        Path(args.json).write_text(json.dumps(res, indent=2))


if __name__ == "__main__":
    main()
