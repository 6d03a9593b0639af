"""Small operator tools (reference tools/*.py equivalents, headless).

* ``render_pov``     depth frames of a recorded trajectory through the same
                     GPU depth camera the policy sees, written as 16-bit PGM
                     images plus one ``.npy`` stack (tools/render_pov.py
                     encodes an mp4 with cv2/ffmpeg; here the frames are the
                     product, encoding is left to the user).
* ``sample_trajectory`` a synthetic circular-flight trajectory file in the
                     viewer format (tools/make_sample_traj.py).
* ``compare_runs``   several runs' progress.csv side by side at fixed step
                     marks (tools/compare_runs.py).
* ``serve_metrics``  a JSON metrics API over a runs directory: /api/runs,
                     /api/metrics?run=NAME (the data endpoints of
                     tools/dashboard.py; its browser pages are graphics and not
                     part of this framework).
* ``env_thread_sweep`` env ticks/s of one batched K-tick step per worker
                     thread count (tools/bench_env.py).
"""
from __future__ import annotations

import csv
import json
import math
import time
from pathlib import Path
from typing import Optional

import numpy as np


# ---- POV frames -----------------------------------------------------------------------------------
def render_pov(traj_path, map_src, out_dir, width: int = 128, height: int = 64, cell: float = 16.0,
               episode: int = 0, stride: int = 3, pinhole: bool = False) -> int:
    """Render the depth view along one recorded episode; returns the frame count."""
    import torch
    from ..ops.vision import DepthCamera, SdfVolume
    from ..sim import mapgen
    from ..sim.core import SimCore, default_config
    from ..trainer.evaluate import read_trajectory
    if str(map_src) in mapgen.MAP_KINDS:
        m = mapgen.generate(str(map_src), 0)
        core = SimCore.from_bytes(m.image, default_config(1), threads=1)
        kw = dict(cell=m.meta["cell"], mins=np.array(m.meta["grid_mins"]), dims=tuple(m.meta["dims"])) \
            if "grid_mins" in m.meta else dict(cell=cell)
    else:
        core = SimCore(str(map_src), default_config(1), threads=1)
        kw = dict(cell=cell)
    vol = SdfVolume.build(core, device="cuda", **kw)
    cam = DepthCamera(vol, width, height, pinhole=pinhole, dtype=torch.float32)
    ep = read_trajectory(traj_path)[episode]["ticks"][::stride]
    pose = torch.zeros((len(ep), 8), dtype=torch.float32, device="cuda")
    pose[:, 0:3] = torch.as_tensor(ep[:, 1:4], dtype=torch.float32)
    pose[:, 3] = torch.as_tensor(ep[:, 7], dtype=torch.float32)
    pose[:, 4] = torch.as_tensor(ep[:, 12], dtype=torch.float32)
    frames = cam.render(pose).view(len(ep), height, width).clamp(0, 1.25).cpu().numpy()
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    np.save(out / "frames.npy", frames.astype(np.float16))
    img = (np.clip(frames / 1.25, 0, 1) * 65535).astype(">u2")
    for i, f in enumerate(img):
        with open(out / f"frame_{i:05d}.pgm", "wb") as fh:
            fh.write(f"P5\n{width} {height}\n65535\n".encode())
            fh.write(f.tobytes())
    core.close()
    return len(img)


# ---- synthetic trajectory -------------------------------------------------------------------------
def sample_trajectory(path, center=(0.0, 0.0, 512.0), radius: float = 1500.0, episodes: int = 2,
                      ticks: int = 600, map_name: str = "sample") -> Path:
    from ..sim.core import PHYS_DEFAULTS
    from ..trainer.evaluate import TrajectoryWriter
    w = TrajectoryWriter(path, map_name, dict(PHYS_DEFAULTS))
    cx, cy, cz = center
    for e in range(episodes):
        w.header(e)
        omega = 2 * math.pi / ticks * (1 if e % 2 == 0 else -1)
        for t in range(ticks):
            a = omega * t
            st = {"origin": (cx + radius * math.cos(a), cy + radius * math.sin(a), cz + 100 * math.sin(3 * a)),
                  "velocity": (-radius * omega * 100 * math.sin(a), radius * omega * 100 * math.cos(a), 0.0),
                  "yaw": math.degrees(a + math.copysign(math.pi / 2, omega)) % 360, "onground": -1,
                  "progress": float(t), "pitch": 0.0}
            w.tick(t, st, (7, 3, 1, 1, 0, 0), 0.0)
        w.trailer("done", ticks, float(ticks))
    w.close()
    return Path(path)


# ---- run comparison --------------------------------------------------------------------------------
COLS = {"rew": "rollout/ep_rew_mean", "len": "rollout/ep_len_mean", "spd": "eval/speed_max",
        "track": "race/eval_progress", "fin": "race/eval_finish_s"}


def read_progress(run_dir) -> dict:
    p = Path(run_dir) / "progress.csv"
    with open(p, newline="") as f:
        rows = list(csv.DictReader(f))
    out = {"step": np.array([float(r["time/total_timesteps"]) for r in rows])}
    for k, c in COLS.items():
        out[k] = np.array([float(r[c]) if r.get(c) not in (None, "") else np.nan for r in rows])
    return out


def compare_runs(run_dirs, marks=(250e6, 500e6, 1e9), col: str = "rew") -> str:
    lines = [f"{'run':<24}" + "".join(f"{m / 1e6:>12.0f}M" for m in marks)]
    for d in run_dirs:
        p = read_progress(d)
        vals = []
        for m in marks:
            i = np.searchsorted(p["step"], m)
            lo, hi = max(0, i - 2), min(len(p["step"]), i + 3)
            v = p[col][lo:hi]
            v = v[np.isfinite(v)]
            vals.append(f"{v.mean():>13.3f}" if len(v) and i < len(p["step"]) else f"{'-':>13}")
        lines.append(f"{Path(d).name:<24}" + "".join(vals))
    return "\n".join(lines)


# ---- metrics API -----------------------------------------------------------------------------------
def serve_metrics(runs_dir, host: str = "127.0.0.1", port: int = 8008, once: bool = False):
    """Serve /api/runs and /api/metrics?run=NAME (JSON) from a runs directory."""
    from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
    from urllib.parse import parse_qs, urlparse
    root = Path(runs_dir)

    class H(BaseHTTPRequestHandler):
        def _json(self, obj, code=200):
            body = json.dumps(obj).encode()
            self.send_response(code)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(body)))
            self.end_headers()
            self.wfile.write(body)

        def do_GET(self):            # noqa: N802
            u = urlparse(self.path)
            if u.path == "/api/runs":
                runs = []
                for d in sorted(p for p in root.iterdir() if (p / "progress.csv").exists()):
                    meta = json.loads((d / "run.json").read_text()) if (d / "run.json").exists() else {}
                    runs.append({"run": d.name, "started": meta.get("started"), "finished": meta.get("finished"),
                                 "recordings": sorted(x.name for x in (d / "recordings").glob("*.jsonl"))
                                 if (d / "recordings").exists() else []})
                return self._json(runs)
            if u.path == "/api/metrics":
                name = parse_qs(u.query).get("run", [""])[0]
                d = root / name
                if not name or "/" in name or not (d / "progress.csv").exists():
                    return self._json({"error": "unknown run"}, 404)
                with open(d / "progress.csv", newline="") as f:
                    rows = list(csv.DictReader(f))
                return self._json({"run": name, "columns": list(rows[0].keys()) if rows else [], "rows": rows})
            return self._json({"error": "not found"}, 404)

        def log_message(self, *a):
            pass

    srv = ThreadingHTTPServer((host, port), H)
    if once:
        return srv
    try:
        srv.serve_forever()
    finally:
        srv.server_close()
    return None


# ---- env thread sweep ------------------------------------------------------------------------------
def env_thread_sweep(kind: str = "field", envs: int = 2048, k: int = 3, reps: int = 20,
                     threads: Optional[list] = None) -> list:
    import os
    from ..sim import mapgen
    from ..sim.core import SimCore, default_config
    m = mapgen.generate(kind, 0)
    threads = threads or sorted({1, 2, 4, 8, 16, max(1, (os.cpu_count() or 2) - 1)})
    out = []
    for th in threads:
        core = SimCore.from_bytes(m.image, default_config(envs, spawn_mode=2), threads=th)
        core.set_spawn_pool(m.spawn_pool)
        core.reset(1)
        rows = np.tile(np.array([7, 3, 2, 1, 0, 0, 0, 0], np.int32), (envs, 1))
        core.step_k(rows.ctypes.data, 8, k)
        t0 = time.perf_counter()
        for _ in range(reps):
            core.step_k(rows.ctypes.data, 8, k)
        dt = time.perf_counter() - t0
        out.append({"threads": th, "ms_per_call": 1e3 * dt / reps, "ticks_per_s": envs * k * reps / dt})
        core.close()
    return out
