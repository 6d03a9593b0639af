"""Reference arm of the depth-march A/B: the reference's own ``GpuLidar``.

Runs in a process of its own with only the reference on ``sys.path``
(``PYTHONPATH=baseline/_ref/python``); it imports nothing of this framework.
It loads the benchmark map with the reference core (``surfgym.SurfCore``),
builds the reference's 16u distance field through its stock path
(``GpuLidar.__init__`` -> ``build_sdf``: C-core occupancy on the slab
lattice, scipy EDT, fp16 for grids over 100M voxels; python/surfgym/vision.py:409-440),
draws the benchmark poses, and times ``GpuLidar.render`` (the stock Triton
``_march_kernel`` launch, python/surfgym/vision.py:553-594) with CUDA events.

Everything the other arm needs to march the same rays is written to one
``.npz``: the reference's own fp16 grid, its origin and cell, the pose sets,
and the reference's depth output of pose set 0 for every range.

Poses (the SDF microbenchmark's definition): eyes uniform over free voxels
at least ``--clearance`` units from geometry, jittered inside the voxel;
yaw uniform in [0, 360); pitch uniform in [-70, +30] degrees; standing.

    PYTHONPATH=baseline/_ref/python python bench/ref_march_arm.py --map M.bsp --out ab.npz
"""
from __future__ import annotations

import argparse
import json
import time

import numpy as np
import torch


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--map", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--envs", type=int, default=2048)
    ap.add_argument("--width", type=int, default=128)
    ap.add_argument("--height", type=int, default=64)
    ap.add_argument("--ranges", default="2000,diag", help="comma list of ray ranges (units); 'diag' = map diagonal")
    ap.add_argument("--near", type=float, default=2000.0)
    ap.add_argument("--max-steps", type=int, default=64)
    ap.add_argument("--cell", type=float, default=16.0)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--sets", type=int, default=4)
    ap.add_argument("--clearance", type=float, default=48.0)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args()

    from surfgym import SurfCore, default_config
    from surfgym import vision as rv

    dev = torch.device("cuda")
    t0 = time.time()
    core = SurfCore(args.map, default_config(num_envs=1))
    lid0 = rv.GpuLidar(core, args.width, args.height, range_units=2000.0, cell=args.cell,
                       max_steps=args.max_steps, near_range=args.near, device="cuda")
    build_s = time.time() - t0
    nz, ny, nx = lid0.nz, lid0.ny, lid0.nx
    sdf16 = lid0.sdf_flat.reshape(nz, ny, nx)
    mins = np.asarray(lid0.mins_f, np.float64)
    cell = lid0.cell
    diag = float(np.linalg.norm(np.array([nx, ny, nz], np.float64) * cell))

    rng = np.random.default_rng(args.seed)
    flat = sdf16.reshape(-1)
    sets = []
    for _ in range(args.sets):
        rows = np.zeros((args.envs, 8), np.float32)
        filled = 0
        while filled < args.envs:
            m = 4 * (args.envs - filled)
            idx = np.stack([rng.integers(0, k, m) for k in (nx, ny, nz)], 1)
            lin = torch.as_tensor(idx[:, 2] * ny * nx + idx[:, 1] * nx + idx[:, 0], device=dev)
            ok = (flat[lin].float() > args.clearance).cpu().numpy()
            idx = idx[ok][: args.envs - filled]
            k = idx.shape[0]
            pos = mins + (idx + rng.random((k, 3))) * cell
            rows[filled:filled + k, 0:3] = pos
            rows[filled:filled + k, 2] -= 17.0          # rows hold player origins; the eye is 17 up
            filled += k
        rows[:, 3] = rng.random(args.envs) * 360.0
        rows[:, 4] = rng.random(args.envs) * 100.0 - 70.0
        sets.append(rows)

    ranges = [diag if r.strip() == "diag" else float(r) for r in args.ranges.split(",")]
    dsets = [torch.as_tensor(s, device=dev) for s in sets]
    result = {"impl": "reference", "kernel": "surfgym.vision._march_kernel (Triton, stock GpuLidar.render)",
              "envs": args.envs, "image": [args.height, args.width], "rays": args.envs * args.width * args.height,
              "grid": [nx, ny, nz], "cell": cell, "max_steps": args.max_steps, "near": args.near,
              "sdf_build_s": round(build_s, 1), "gpu": torch.cuda.get_device_name(), "per_range": []}
    outs = {}
    for ri, rg in enumerate(ranges):
        lid = rv.GpuLidar.__new__(rv.GpuLidar)        # the same object with another range: no second SDF build
        lid.__dict__.update(lid0.__dict__)
        lid.range = float(rg)
        lid.near = float(args.near) if args.near else lid.range

        def render(ps):
            return lid.render(ps[:, 0:3], ps[:, 3], ps[:, 4], ps[:, 5])

        for i in range(args.warmup):
            render(dsets[i % len(dsets)])
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.iters)]
        for i in range(args.iters):
            ev[i][0].record()
            render(dsets[i % len(dsets)])
            ev[i][1].record()
        torch.cuda.synchronize()
        ms = sorted(a.elapsed_time(b) for a, b in ev)
        med = ms[len(ms) // 2]
        outs[f"depth_r{ri}"] = render(dsets[0]).cpu().numpy().astype(np.float32)
        result["per_range"].append({"range": rg, "ms_per_render": med, "ms_min": ms[0],
                                    "rays_per_s": result["rays"] / (med * 1e-3)})
    np.savez(args.out, sdf=sdf16.cpu().numpy(), mins=mins, cell=np.float32(cell), poses=np.stack(sets),
             ranges=np.asarray(ranges, np.float64), near=np.float32(args.near), **outs)
    print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
