"""Same-box A/B of the SDF depth march: the reference's Triton kernel vs march.cu.

Both arms march the same rays through the same grid on the same GPU:

1. the benchmark map (seeded 512-brush procedural field) is written by a
   child process;
2. ``bench/ref_march_arm.py`` runs in a process with only the reference on
   its path: the reference core loads the map, the reference builds its own
   16u fp16 distance field, draws the poses and times its stock
   ``GpuLidar.render`` (python/surfgym/vision.py:553-594); it saves the grid,
   the poses and its depth images;
3. this process bricks that same fp16 grid (``SdfVolume.from_linear``), renders
   the same pose sets with ``DepthCamera`` (fp32 NHW output, the reference's
   output format; and the trainer's bf16 space-to-depth format) and compares
   its depth with the reference's, pixel for pixel.

Timing for both arms: CUDA events around each render, warm-up renders first,
four pose sets cycled so consecutive renders do not share a warm L2 footprint
(the grid is 512 MB, over 4x the L2), median of ``--iters``. Same
``max_steps`` (64, the trainer's and the reference's), same ranges (2000u,
the trainer's camera, and the map diagonal, the microbenchmark's full-map
range), same near/far depth code.

    python bench/bench_march_ab.py [--envs 2048] [--iters 20] [--json out.json]
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"


def write_map(directory: Path) -> Path:
    import importlib.util
    spec = importlib.util.spec_from_file_location("surf_reference_arm", ROOT / "rl_cs1.6_surf_b200" / "baseline_ref.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.write_bench_map(directory)


def run_reference(map_path: Path, out: Path, args) -> dict:
    env = dict(os.environ)
    env["PYTHONPATH"] = str(REF / "python")
    cmd = [sys.executable, str(ROOT / "bench" / "ref_march_arm.py"), "--map", str(map_path), "--out", str(out),
           "--envs", str(args.envs), "--iters", str(args.iters), "--warmup", str(args.warmup),
           "--max-steps", str(args.max_steps), "--near", str(args.near), "--ranges", args.ranges,
           "--seed", str(args.seed)]
    p = subprocess.run(cmd, cwd=str(REF), env=env, capture_output=True, text=True, timeout=args.timeout)
    if p.returncode != 0:
        raise RuntimeError(f"reference arm failed rc={p.returncode}: {(p.stdout + p.stderr)[-1500:]}")
    line = [l for l in p.stdout.splitlines() if l.startswith("{")][-1]
    return json.loads(line)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--envs", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--max-steps", type=int, default=64)
    ap.add_argument("--near", type=float, default=2000.0)
    ap.add_argument("--ranges", default="2000,diag")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--timeout", type=float, default=1800.0)
    ap.add_argument("--maps", default=str(ROOT / "maps" / "march_ab"))
    ap.add_argument("--json", default=None)
    args = ap.parse_args()

    if not (REF / "python" / "surfgym" / "vision.py").exists():
        print(json.dumps({"metric": "sdf_rays_per_s A/B", "unavailable": "reference not installed under baseline/_ref"}))
        return
    t0 = time.time()
    map_path = write_map(Path(args.maps))
    with tempfile.TemporaryDirectory() as td:
        npz = Path(td) / "ab.npz"
        ref = run_reference(map_path, npz, args)
        z = dict(np.load(npz))
    ref_s = time.time() - t0

    import torch
    sys.path.insert(0, str(ROOT))
    import surfb200  # noqa: F401
    from surfb200.ops import vision
    dev = torch.device("cuda")
    vol = vision.SdfVolume.from_linear(torch.as_tensor(z["sdf"], device=dev), z["mins"], float(z["cell"]))
    sets = [torch.as_tensor(s, device=dev) for s in z["poses"]]
    n, H, W = args.envs, 64, 128
    rays = n * H * W
    per_range = []
    for ri, rg in enumerate(z["ranges"].tolist()):
        row = {"range": rg}
        for name, dtype, layout in (("fp32_nhw", torch.float32, vision.LAYOUT_NHW),
                                    ("bf16_s2d", torch.bfloat16, vision.LAYOUT_S2D4)):
            cam = vision.DepthCamera(vol, W, H, range_units=rg, near_range=args.near, max_steps=args.max_steps,
                                     dtype=dtype, layout=layout)
            out = torch.empty((n, cam.frame), dtype=dtype, device=dev)
            for i in range(args.warmup):
                cam.render(sets[i % len(sets)], out=out)
            torch.cuda.synchronize()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(args.iters)]
            for i in range(args.iters):
                ev[i][0].record()
                cam.render(sets[i % len(sets)], out=out)
                ev[i][1].record()
            torch.cuda.synchronize()
            ms = sorted(a.elapsed_time(b) for a, b in ev)
            med = ms[len(ms) // 2]
            row[name] = {"ms_per_render": med, "ms_min": ms[0], "rays_per_s": rays / (med * 1e-3)}
            if name == "fp32_nhw":
                steps = torch.empty((n, H, W), dtype=torch.uint8, device=dev)
                mine = cam.render(sets[0], out=out, steps=steps).reshape(n, H, W).cpu().numpy()
                theirs = z[f"depth_r{ri}"].reshape(n, H, W)
                diff = np.abs(mine.astype(np.float64) - theirs.astype(np.float64))
                # encoded depth -> units inside the near range (code = t / near there)
                row["agreement"] = {"exact_frac": float((diff == 0).mean()), "within_1e-6": float((diff <= 1e-6).mean()),
                                    "within_1e-3": float((diff <= 1e-3).mean()), "max_abs": float(diff.max()),
                                    "p99_abs_units": float(np.quantile(diff, 0.99) * args.near)}
                st = steps.float()
                row["steps"] = {"mean": float(st.mean()), "p50": float(st.median()),
                                "exhausted_frac": float((st >= args.max_steps).float().mean())}
        ref_row = ref["per_range"][ri]
        row["reference"] = {"ms_per_render": ref_row["ms_per_render"], "ms_min": ref_row["ms_min"],
                            "rays_per_s": ref_row["rays_per_s"]}
        row["speedup_fp32_nhw"] = ref_row["ms_per_render"] / row["fp32_nhw"]["ms_per_render"]
        row["speedup_bf16_s2d"] = ref_row["ms_per_render"] / row["bf16_s2d"]["ms_per_render"]
        per_range.append(row)
    result = {"metric": "sdf_rays_per_s A/B (same box, same grid, same poses)", "unit": "rays/s",
              "value": per_range[-1]["fp32_nhw"]["rays_per_s"],
              "reference_value": per_range[-1]["reference"]["rays_per_s"],
              "envs": n, "image": [H, W], "rays": rays, "grid": ref["grid"], "cell": ref["cell"],
              "max_steps": args.max_steps, "near": args.near, "per_range": per_range,
              "reference_kernel": ref["kernel"], "reference_sdf_build_s": ref["sdf_build_s"],
              "reference_arm_wall_s": round(ref_s, 1), "gpu": torch.cuda.get_device_name(),
              "timing": "CUDA events per render, median of iters, 4 pose sets cycled (grid 512 MB > L2)"}
    print(json.dumps(result), flush=True)
    if args.json:
        Path(args.json).write_text(json.dumps(result, indent=2))


if __name__ == "__main__":
    main()
