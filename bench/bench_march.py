"""SDF sphere-trace microbenchmark (the SDF rays/s headline).

Configuration: a seeded 512-brush procedural map whose 16u fp16 distance field
is exactly 1024 x 1024 x 256 voxels; 2048 envs x 128 x 64 equiangular rays;
eyes uniform in free space (>= 48u from geometry), yaw uniform, pitch uniform
in [-70, +30] degrees; full-map range with per-ray early exit; near-linear /
far-compressed depth code. Reports device-timed rays/s (CUDA events, inputs
larger than L2), the per-ray step census, and the median depth error against
exact point-hull traces of the simulator, at the trainer's 2000u range and at
the full-map range (the headline).

    python bench/bench_march.py [--envs 2048] [--iters 20] [--json out.json]
"""
from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path

import numpy as np
import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import surfb200  # noqa: E402,F401
from surfb200.ops import vision  # noqa: E402
from surfb200.sim import mapgen  # noqa: E402
from surfb200.sim.core import SimCore, default_config  # noqa: E402



def _warp_efficiency(st, H: int, W: int):
    if H % 2 or W % 16:
        return None
    w = st.reshape(st.shape[0], H // 2, 2, W // 16, 16).permute(0, 1, 3, 2, 4).reshape(-1, 32)
    return float(w.mean(1).sum() / w.amax(1).clamp(min=1).sum())

def free_space_poses(vol: vision.SdfVolume, n: int, seed: int, clearance: float = 48.0) -> torch.Tensor:
    g = torch.Generator(device="cuda").manual_seed(seed)
    nx, ny, nz = vol.dims
    out = torch.zeros((n, 8), device="cuda")
    filled = 0
    lin = vol.linear
    while filled < n:
        m = 4 * (n - filled)
        idx = torch.stack([torch.randint(0, k, (m,), device="cuda", generator=g) for k in (nx, ny, nz)], 1)
        ok = lin[idx[:, 2], idx[:, 1], idx[:, 0]].float() > clearance
        idx = idx[ok][: n - filled]
        k = idx.shape[0]
        jitter = torch.rand((k, 3), device="cuda", generator=g)
        pos = torch.as_tensor(vol.mins, dtype=torch.float32, device="cuda") + (idx.float() + jitter) * vol.cell
        out[filled:filled + k, 0:3] = pos
        out[filled:filled + k, 2] -= 17.0                        # rows hold origins; eye = origin + 17
        filled += k
    out[:, 3] = torch.rand(n, device="cuda", generator=g) * 360.0
    out[:, 4] = torch.rand(n, device="cuda", generator=g) * 100.0 - 70.0
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--envs", type=int, default=2048)
    ap.add_argument("--width", type=int, default=128)
    ap.add_argument("--height", type=int, default=64)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--max-steps", type=int, default=64)
    ap.add_argument("--near", type=float, default=2000.0)
    ap.add_argument("--trainer-range", type=float, default=2000.0, help="the trainer's camera range (lidar_range)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--check-rays", type=int, default=20000)
    ap.add_argument("--json", default=None)
    args = ap.parse_args()

    t0 = time.time()
    m = mapgen.generate("field", args.seed, spawns=16)
    core = SimCore.from_bytes(m.image, default_config(1), threads=None)
    cell = m.meta["cell"]
    dims = tuple(m.meta["dims"])
    torch.cuda.synchronize()
    tb = time.time()
    vol = vision.SdfVolume.build(core, cell=cell, mins=np.array(m.meta["grid_mins"]), dims=dims)
    torch.cuda.synchronize()
    bake_s = time.time() - tb
    diag = float(np.linalg.norm(np.array(dims) * cell))
    # several pose sets, cycled, so consecutive renders do not reuse a warm L2 footprint
    sets = [free_space_poses(vol, args.envs, args.seed + 17 * i) for i in range(4)]
    rays = args.envs * args.width * args.height
    pose = sets[0].cpu().numpy()
    rng = np.random.default_rng(0)
    n_chk = min(args.check_rays, rays)
    sel = rng.integers(0, rays, n_chk)
    e, r, c = sel // (args.width * args.height), (sel // args.width) % args.height, sel % args.width

    def measure(range_units: float) -> dict:
        cam = vision.DepthCamera(vol, args.width, args.height, range_units=range_units, near_range=args.near,
                                 max_steps=args.max_steps, dtype=torch.bfloat16, layout=vision.LAYOUT_S2D4)
        out = torch.empty((args.envs, cam.frame), dtype=torch.bfloat16, device="cuda")
        for i in range(args.warmup):
            cam.render(sets[i % 4], out=out)
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.iters)]
        for i in range(args.iters):
            ev[i][0].record()
            cam.render(sets[i % 4], out=out)
            ev[i][1].record()
        torch.cuda.synchronize()
        ms = sorted(a.elapsed_time(b) for a, b in ev)
        med = ms[len(ms) // 2]
        steps = torch.empty((args.envs, args.height, args.width), dtype=torch.uint8, device="cuda")
        cam.render(sets[0], out=out, steps=steps)
        st = steps.float()
        # accuracy: exact point-hull traces of a sample of rays of set 0, hits within the range
        lin_cam = vision.DepthCamera(vol, args.width, args.height, range_units=range_units, near_range=range_units,
                                     max_steps=args.max_steps)
        dep = lin_cam.render(sets[0]).reshape(args.envs, args.height, args.width).cpu().numpy() * range_units
        col, row = lin_cam.offsets()
        eye = pose[e, :3] + np.where(pose[e, 5:6] != 0, [0, 0, 12.0], [0, 0, 17.0])
        yaw = np.radians(pose[e, 3]) + col[c]
        pit = np.radians(pose[e, 4]) + row[r]
        d = np.stack([np.cos(pit) * np.cos(yaw), np.cos(pit) * np.sin(yaw), np.sin(pit)], 1)
        res = core.trace_batch(eye, eye + d * diag, hull=2)
        exact = res[:, 0] * diag
        hit = (res[:, 0] < 0.999) & (res[:, 7] == 0) & (exact < range_units)
        err = np.abs(dep[e, r, c] - exact)[hit]
        return {"range": range_units, "rays_per_s": rays / (med * 1e-3), "ms_per_render": med, "ms_min": ms[0],
                "mean_steps": float(st.mean()), "p50_steps": float(st.median()),
                "p99_steps": float(torch.quantile(st.flatten()[::97], 0.99)),
                "exhausted_frac": float((st >= args.max_steps).float().mean()),
                # SIMD efficiency of the 16 x 2 pixel warps: mean steps / longest ray's steps per warp
                "warp_step_efficiency": _warp_efficiency(st, args.height, args.width),
                "median_abs_err_units": float(np.median(err)) if err.size else None,
                "checked_hits": int(hit.sum())}

    # the trainer's range (TrainConfig.lidar_range) and the whole map (the headline)
    per_range = [measure(args.trainer_range), measure(diag)]
    full = per_range[-1]
    result = {
        "metric": "sdf_rays_per_s", "value": full["rays_per_s"], "unit": "rays/s", "ms_per_render": full["ms_per_render"],
        "ms_min": full["ms_min"], "rays": rays, "envs": args.envs, "image": [args.height, args.width],
        "grid": list(dims), "cell": cell, "sdf_bytes": int(vol.bricked.numel() * 2), "range": diag,
        "max_steps": args.max_steps, "mean_steps": full["mean_steps"], "p50_steps": full["p50_steps"],
        "p99_steps": full["p99_steps"], "exhausted_frac": full["exhausted_frac"],
        "warp_step_efficiency": full["warp_step_efficiency"],
        "median_abs_err_units": full["median_abs_err_units"], "checked_hits": full["checked_hits"],
        "per_range": per_range,
        "bake_s": bake_s, "setup_s": time.time() - t0, "gpu": torch.cuda.get_device_name(),
    }
    print(json.dumps(result))
    if args.json:
        Path(args.json).write_text(json.dumps(result, indent=2))


if __name__ == "__main__":
    main()
