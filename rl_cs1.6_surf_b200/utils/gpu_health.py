"""Box health gate: HBM copy bandwidth and sustained bf16 GEMM throughput
against the pool's measured peaks (reference tools/gpu_health.py:29-107).

Copy: a device-to-device copy of 2 GiB, timed with CUDA events. GEMM: an
8192^3 bf16 matmul (library GEMM: this is a box check, not a framework hot
path) looped for ``--seconds``. Prints both with their fraction of the
measured peaks (MEASURED_PEAKS.json at the repository root when present) and
flags a GPU that is already busy (another process holding memory).
"""
from __future__ import annotations

import json
import time
from pathlib import Path


def main(args) -> int:
    import torch
    if not torch.cuda.is_available():
        print(json.dumps({"ok": False, "reason": "no CUDA device"}))
        return 1
    dev = torch.device("cuda")
    free, total = torch.cuda.mem_get_info(dev)
    busy = (total - free) > 4 * 2 ** 30
    n = 2 ** 30
    a = torch.empty(n, dtype=torch.uint8, device=dev)
    b = torch.empty_like(a)
    a.fill_(1)
    for _ in range(3):
        b.copy_(a)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    reps = 20
    for _ in range(reps):
        b.copy_(a)
    e1.record()
    torch.cuda.synchronize()
    gbs = 2 * n * reps / (e0.elapsed_time(e1) * 1e-3) / 1e9
    del a, b
    m = 8192
    x = torch.randn(m, m, device=dev, dtype=torch.bfloat16)
    y = torch.randn(m, m, device=dev, dtype=torch.bfloat16)
    for _ in range(3):
        x @ y
    torch.cuda.synchronize()
    iters, t0 = 0, time.time()
    e0.record()
    while time.time() - t0 < args.seconds:
        for _ in range(10):
            x @ y
        iters += 10
        torch.cuda.synchronize()
    e1.record()
    torch.cuda.synchronize()
    tflops = 2 * m ** 3 * iters / (e0.elapsed_time(e1) * 1e-3) / 1e12
    peaks_path = Path(args.peaks) if args.peaks else Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    peaks = json.loads(peaks_path.read_text()) if peaks_path.exists() else {"hbm_gbs": 6650.0,
                                                                           "bf16_tflops_sustained": 1400.0}
    hbm_frac = gbs / float(peaks.get("hbm_gbs", 6650.0))
    mm_frac = tflops / float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops", 1400.0)))
    ok = hbm_frac > 0.8 and mm_frac > 0.7 and not busy
    print(json.dumps({"ok": ok, "device": torch.cuda.get_device_name(dev), "hbm_copy_gbs": round(gbs, 1),
                      "hbm_frac_of_measured": round(hbm_frac, 3), "bf16_gemm_tflops": round(tflops, 1),
                      "gemm_frac_of_measured_sustained": round(mm_frac, 3), "busy": busy,
                      "used_gib_before": round((total - free) / 2 ** 30, 2)}))
    return 0 if ok else 2
