"""Seeded procedural surf maps, compiled to BSP v30.

The reference trains on hand-built community maps; this generator makes
reproducible maps of a chosen shape so that benchmarks and tests need no
downloaded assets. Every map is a set of convex brushes compiled by the
native writer (csrc/sim/bspwrite.cpp) into a file that both this framework's
simulator and the reference core load (the parity tests use exactly that).

Map families (one per benchmark configuration):

* ``ramps_map``         eight wedge surf ramps over a floor-level teleport
                        kill volume (eyeless CPU PPO);
* ``random_field_map``  512 seeded random boxes and wedge ramps in a
                        16k x 16k x 4k volume whose 16u vision grid is exactly
                        1024 x 1024 x 256 (SDF microbench, vision PPO);
* ``race_track_map``    a descending serpentine of chained ramps with
                        gap-jump transfers over teleport fail-nets and a 1u
                        finish curtain (race objective).

A surf ramp is a triangular prism: two faces tilted ``angle`` degrees from
horizontal (normal z = cos(angle) < 0.7, i.e. too steep to stand on) meeting
at a ridge, end caps and a flat bottom.
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional

import numpy as np

from .core import CONTENTS_SOLID, STATE_DTYPE, SimCore, compile_bsp, default_config

Plane = tuple  # (nx, ny, nz, d): solid where n.x <= d


def box_planes(lo, hi) -> list:
    lo = [float(v) for v in lo]
    hi = [float(v) for v in hi]
    return [(1, 0, 0, hi[0]), (-1, 0, 0, -lo[0]), (0, 1, 0, hi[1]), (0, -1, 0, -lo[1]),
            (0, 0, 1, hi[2]), (0, 0, -1, -lo[2])]


@dataclass
class Ramp:
    cx: float
    cy: float
    z0: float            # bottom
    yaw: float           # degrees, direction of the ridge
    length: float
    width: float         # base width
    angle: float         # face tilt from horizontal, degrees

    @property
    def height(self) -> float:
        return 0.5 * self.width * math.tan(math.radians(self.angle))

    def axes(self):
        y = math.radians(self.yaw)
        u = np.array([math.cos(y), math.sin(y)])
        w = np.array([-math.sin(y), math.cos(y)])
        return u, w

    def planes(self) -> list:
        u, w = self.axes()
        c = np.array([self.cx, self.cy])
        a = math.radians(self.angle)
        sa, ca = math.sin(a), math.cos(a)
        hw = 0.5 * self.width
        out = []
        for side in (1.0, -1.0):
            n = (side * w[0] * sa, side * w[1] * sa, ca)
            edge = c + side * hw * w
            d = n[0] * edge[0] + n[1] * edge[1] + n[2] * self.z0
            out.append((n[0], n[1], n[2], d))
        out.append((0.0, 0.0, -1.0, -self.z0))
        for side in (1.0, -1.0):
            n = (side * u[0], side * u[1], 0.0)
            d = side * float(u @ c) + 0.5 * self.length
            out.append((n[0], n[1], n[2], d))
        return out

    def face_point(self, s: float, side: float, f: float) -> np.ndarray:
        """Point on a sloped face: s along the ridge from the centre, side +-1,
        f in [0,1] from ridge (0) to base edge (1)."""
        u, w = self.axes()
        xy = np.array([self.cx, self.cy]) + s * u + side * f * 0.5 * self.width * w
        return np.array([xy[0], xy[1], self.z0 + self.height * (1.0 - f)])

    def face_normal(self, side: float) -> np.ndarray:
        _, w = self.axes()
        a = math.radians(self.angle)
        return np.array([side * w[0] * math.sin(a), side * w[1] * math.sin(a), math.cos(a)])


@dataclass
class ProcMap:
    name: str
    image: bytes
    zones: dict
    meta: dict
    ramps: list = field(default_factory=list)
    spawn_pool: Optional[np.ndarray] = None

    def save(self, directory) -> Path:
        d = Path(directory)
        d.mkdir(parents=True, exist_ok=True)
        p = d / f"{self.name}.bsp"
        p.write_bytes(self.image)
        doc = {"map": self.name, "source": "procedural", **self.zones}
        (d / f"{self.name}.zones.json").write_text(json.dumps(doc, indent=2))
        if self.spawn_pool is not None:
            np.save(d / f"{self.name}.spawns.npy", self.spawn_pool)
        (d / f"{self.name}.meta.json").write_text(json.dumps(self.meta, indent=2))
        return p


class MapBuilder:
    """Collects brushes and entities, then compiles a BSP image."""

    def __init__(self) -> None:
        self.brushes: list = []           # (model, contents, planes)
        self.entities: list = [{"classname": "worldspawn", "wad": "", "mapversion": "220"}]
        self.nmodels = 1

    def world(self, planes, contents: int = CONTENTS_SOLID) -> None:
        self.brushes.append((0, contents, planes))

    def brush_entity(self, classname: str, brushes: list, **kv) -> int:
        m = self.nmodels
        self.nmodels += 1
        for planes in brushes:
            self.brushes.append((m, CONTENTS_SOLID, planes))
        ent = {"classname": classname, "model": f"*{m}"}
        ent.update({k: str(v) for k, v in kv.items()})
        self.entities.append(ent)
        return m

    def point(self, classname: str, origin, **kv) -> None:
        ent = {"classname": classname, "origin": " ".join(f"{float(v):g}" for v in origin)}
        ent.update({k: str(v) for k, v in kv.items()})
        self.entities.append(ent)

    def entity_text(self) -> str:
        out = []
        for e in self.entities:
            out.append("{\n" + "".join(f'"{k}" "{v}"\n' for k, v in e.items()) + "}\n")
        return "".join(out)

    def compile(self) -> bytes:
        return compile_bsp(self.brushes, self.entity_text())


def _kill_net(b: MapBuilder, lo, hi, dest) -> None:
    """A teleport volume whose destination resolves (so the env treats it as a
    benign teleport that the teleport-fail rule turns into a death)."""
    b.brush_entity("trigger_teleport", [box_planes(lo, hi)], target="failnet_dest")
    b.point("info_teleport_destination", dest, targetname="failnet_dest", angle="0")


def _probe_core(image: bytes) -> SimCore:
    return SimCore.from_bytes(image, default_config(1), threads=1)


def drop_spawns(core: SimCore, ramps: list, rng: np.random.Generator, count: int,
                height=(400.0, 800.0), speed=(100.0, 400.0), pitch=(-45.0, 15.0),
                zmax: Optional[float] = None) -> np.ndarray:
    """Spawn states dropped ``height`` above random points of ramp faces with a
    random horizontal velocity, yaw and view pitch (the reference's drop pool
    rules, python/surfgym/rewards.py:843-909), placed by construction from the
    known ramp geometry instead of a grid scan; every candidate must be free
    for the standing hull and have open air below it."""
    rows = []
    tries = 0
    while len(rows) < count and tries < 50 * count:
        tries += 1
        r = ramps[int(rng.integers(len(ramps)))]
        s = rng.uniform(-0.45, 0.45) * r.length
        side = 1.0 if rng.random() < 0.5 else -1.0
        p = r.face_point(s, side, rng.uniform(0.15, 0.85))
        h = rng.uniform(*height)
        o = p + np.array([0, 0, h])
        if zmax is not None and o[2] > zmax - 64:
            continue
        if core.trace(o, o, hull=0).startsolid:
            continue
        below = core.trace(o, o - np.array([0, 0, 0.5 * height[0]]), hull=0)
        if below.fraction < 1.0:
            continue
        ang = rng.uniform(0, 2 * math.pi)
        spd = rng.uniform(*speed)
        rows.append((o, (math.cos(ang) * spd, math.sin(ang) * spd, 0.0), rng.uniform(0, 360), rng.uniform(*pitch)))
    if not rows:
        raise RuntimeError("drop_spawns: no valid spawn found")
    pool = np.zeros(len(rows), STATE_DTYPE)
    for i, (o, v, yaw, pt) in enumerate(rows):
        pool[i]["origin"] = o
        pool[i]["velocity"] = v
        pool[i]["yaw"] = yaw
        pool[i]["pitch"] = pt
        pool[i]["onground"] = -1
    return pool


def ramps_map(seed: int = 0, n_ramps: int = 8, length: float = 2000.0, width: float = 512.0,
              angle=(46.0, 55.0), spawns: int = 256) -> ProcMap:
    """Eight (by default) wedge surf ramps in two rows over a teleport kill
    volume at floor level; spawns are drops onto the ramps."""
    rng = np.random.default_rng(seed)
    b = MapBuilder()
    ramps = []
    cols = (n_ramps + 1) // 2
    for i in range(n_ramps):
        row, col = divmod(i, cols)
        ramps.append(Ramp(cx=(col - (cols - 1) / 2) * (width + 700), cy=(row - 0.5) * (length + 800),
                          z0=float(rng.uniform(200, 600)), yaw=90.0 + float(rng.uniform(-10, 10)),
                          length=length, width=width, angle=float(rng.uniform(*angle))))
    for r in ramps:
        b.world(r.planes())
    ext_x = cols * (width + 700) / 2 + 800
    ext_y = length + 1600
    b.world(box_planes((-ext_x, -ext_y, -16), (ext_x, ext_y, 0)))           # floor
    b.world(box_planes((ext_x - 16, ext_y - 16, 0), (ext_x, ext_y, 2400)))  # height marker
    spawn_top = (0.0, 0.0, 2300.0)
    _kill_net(b, (-ext_x, -ext_y, 0), (ext_x, ext_y, 64), spawn_top)
    for r in ramps:
        p = r.face_point(0.0, 1.0, 0.0) + np.array([0, 0, 600.0])
        b.point("info_player_start", p, angle=f"{r.yaw:g}")
    image = b.compile()
    core = _probe_core(image)
    pool = drop_spawns(core, ramps, rng, spawns, height=(200.0, 600.0), zmax=2400)
    core.close()
    meta = dict(kind="ramps", seed=seed, n_ramps=n_ramps, brushes=len(b.brushes))
    return ProcMap(f"proc_ramps_s{seed}", image, {"start": None, "end": None}, meta, ramps, pool)


def random_field_map(seed: int = 0, n_brushes: int = 512, cell: float = 16.0,
                     dims=(1024, 1024, 256), spawns: int = 4096) -> ProcMap:
    """``n_brushes`` seeded random boxes and wedge ramps (half each). The world
    bounds are chosen so the vision grid (bounds padded by 4 cells per side)
    is exactly ``dims`` voxels of ``cell`` units."""
    rng = np.random.default_rng(seed)
    ext = [(d - 8) * cell for d in dims]                  # world extent
    lo = np.array([-ext[0] / 2, -ext[1] / 2, 0.0])
    hi = lo + np.array(ext)
    b = MapBuilder()
    ramps = []
    n_ramp = n_brushes // 2
    for _ in range(n_ramp):
        L = float(rng.uniform(1000, 3000))
        W = float(rng.uniform(384, 1024))
        a = float(rng.uniform(46, 55))
        r = Ramp(cx=float(rng.uniform(lo[0] + L / 2, hi[0] - L / 2)), cy=float(rng.uniform(lo[1] + L / 2, hi[1] - L / 2)),
                 z0=0.0, yaw=float(rng.uniform(0, 180)), length=L, width=W, angle=a)
        r.z0 = float(rng.uniform(200, hi[2] - r.height - 200))
        ramps.append(r)
        b.world(r.planes())
    for _ in range(n_brushes - n_ramp):
        size = rng.uniform(64, 1024, 3)
        c = rng.uniform(lo + size / 2 + [0, 0, 200], hi - size / 2)
        b.world(box_planes(c - size / 2, c + size / 2))
    b.world(box_planes((lo[0], lo[1], -16), (hi[0], hi[1], 0)))            # floor slab
    b.world(box_planes((hi[0] - 16, hi[1] - 16, 0), (hi[0], hi[1], hi[2])))  # height marker
    _kill_net(b, (lo[0], lo[1], 0), (hi[0], hi[1], 64), (0.0, 0.0, hi[2] - 200))
    for r in ramps[:16]:
        b.point("info_player_start", r.face_point(0.0, 1.0, 0.0) + np.array([0, 0, 400.0]), angle=f"{r.yaw:g}")
    # a start platform whose -y edge drops onto a 50-degree face (the timed-map
    # convention; fixed geometry, so the seeded brushes above are unchanged)
    start = Ramp(cx=0.0, cy=0.0, z0=1600.0, yaw=0.0, length=2400.0, width=800.0, angle=50.0)
    b.world(start.planes())
    top = start.z0 + start.height + 64.0
    b.world(box_planes((-128.0, 250.0, top - 32.0), (128.0, 506.0, top)))
    b.point("info_player_start", (0.0, 378.0, top + 37.0), angle="270")
    image = b.compile()
    core = _probe_core(image)
    pool = drop_spawns(core, ramps, rng, spawns, zmax=hi[2])
    core.close()
    meta = dict(kind="random_field", seed=seed, n_brushes=n_brushes, cell=cell, dims=list(dims),
                grid_mins=[float(v) for v in (lo - 4 * cell)], brushes=len(b.brushes))
    return ProcMap(f"proc_field_s{seed}", image, {"start": None, "end": None}, meta, ramps, pool)


def race_track_map(seed: int = 0, n_ramps: int = 40, ramp_length: float = 4800.0, per_row: int = 5,
                   gap_jumps: int = 4, width: float = 640.0, angle: float = 50.0) -> ProcMap:
    """A descending serpentine surf track: rows of ``per_row`` chained ramps,
    connected row to row by drop transfers; ``gap_jumps`` of the in-row
    junctions are gaps over teleport fail-nets that must be jumped with carried
    speed. A 1u-thin finish curtain (trigger_multiple wired to a stop button,
    the timed-map convention) closes the track; the start platform carries the
    info_player_start entities. Track length ~ n_ramps * ramp_length."""
    rng = np.random.default_rng(seed)
    b = MapBuilder()
    ramps = []
    drop_per_ramp = 120.0
    row_pitch = 2600.0
    n_rows = (n_ramps + per_row - 1) // per_row
    top = 200.0 + n_ramps * drop_per_ramp + 800
    gap_at = set(rng.choice(np.arange(1, n_ramps - 1), size=min(gap_jumps, n_ramps - 2), replace=False).tolist())
    x_extent = per_row * ramp_length
    z = top - 800
    path = []
    for i in range(n_ramps):
        row, k = divmod(i, per_row)
        direction = 1.0 if row % 2 == 0 else -1.0
        col = k if direction > 0 else per_row - 1 - k
        cx = -x_extent / 2 + (col + 0.5) * ramp_length
        cy = -n_rows * row_pitch / 2 + (row + 0.5) * row_pitch
        length = ramp_length - (700.0 if i in gap_at else 40.0)
        r = Ramp(cx=cx, cy=cy, z0=0.0, yaw=0.0, length=length, width=width, angle=angle)
        r.z0 = z - r.height
        z -= drop_per_ramp
        ramps.append(r)
        b.world(r.planes())
        path.append((cx - direction * ramp_length / 2, cy, r.z0 + r.height + 64))
        path.append((cx + direction * ramp_length / 2, cy, r.z0 + r.height + 64))
        if k == per_row - 1 and i < n_ramps - 1:          # row transfer: a wide catch ramp turning 180 degrees
            ex = cx + direction * (ramp_length / 2 + 700)
            tr = Ramp(cx=ex, cy=cy + row_pitch / 2, z0=0.0, yaw=90.0, length=row_pitch + width, width=1000.0,
                      angle=angle)
            tr.z0 = r.z0 - 300 - tr.height
            ramps.append(tr)
            b.world(tr.planes())
    x_lo, x_hi = -x_extent / 2 - 2200, x_extent / 2 + 2200
    y_lo, y_hi = -n_rows * row_pitch / 2 - 1500, n_rows * row_pitch / 2 + 1500
    floor_z = min(r.z0 for r in ramps) - 1200
    b.world(box_planes((x_lo, y_lo, floor_z - 16), (x_hi, y_hi, floor_z)))
    b.world(box_planes((x_hi - 16, y_hi - 16, floor_z), (x_hi, y_hi, top + 600)))
    first = ramps[0]
    start = np.array([first.cx - first.length / 2 - 500, first.cy, first.z0 + first.height + 40])
    b.world(box_planes(start - [400, 400, 56], start + [300, 400, -40]))     # start platform
    _kill_net(b, (x_lo, y_lo, floor_z), (x_hi, y_hi, floor_z + 64), start + [0, 0, 40])
    for g in sorted(gap_at):                               # fail-nets under the gaps
        r = ramps[g] if g < len(ramps) else ramps[-1]
        direction = 1.0 if (g // per_row) % 2 == 0 else -1.0
        gx = r.cx + direction * (r.length / 2 + 330)
        b.brush_entity("trigger_teleport", [box_planes((gx - 380, r.cy - 700, r.z0 - 900), (gx + 380, r.cy + 700, r.z0 - 400))],
                       target="failnet_dest")
    last = ramps[-1]
    dirn = 1.0 if ((n_ramps - 1) // per_row) % 2 == 0 else -1.0
    fx = last.cx + dirn * (last.length / 2 + 200)
    fin_lo = (fx, last.cy - 900, last.z0 - 1000)
    fin_hi = (fx + 1, last.cy + 900, last.z0 + last.height + 1200)
    b.brush_entity("trigger_multiple", [box_planes(fin_lo, fin_hi)], target="counter_stop_button")
    b.brush_entity("func_button", [box_planes((x_hi - 200, y_hi - 200, floor_z + 100), (x_hi - 180, y_hi - 180, floor_z + 120))],
                   targetname="counter_stop_button", target="timer_stop")
    st_lo = (start[0] + 250, start[1] - 400, start[2] - 40)
    b.brush_entity("trigger_multiple", [box_planes(st_lo, (st_lo[0] + 1, start[1] + 400, start[2] + 300))],
                   target="counter_start_button")
    b.brush_entity("func_button", [box_planes((x_hi - 300, y_hi - 200, floor_z + 100), (x_hi - 280, y_hi - 180, floor_z + 120))],
                   targetname="counter_start_button", target="timer_start")
    for j in range(4):
        b.point("info_player_start", start + [-200 + 100 * j, 0, 40], angle="0")
    image = b.compile()
    core = _probe_core(image)
    pool = np.zeros(4, STATE_DTYPE)
    for j in range(4):
        pool[j]["origin"] = start + [-200 + 100 * j, 0, 40]
        pool[j]["yaw"] = 0.0
        pool[j]["onground"] = -1
    core.close()
    zones = {"start": {"mins": list(map(float, st_lo)), "maxs": [st_lo[0] + 1, float(start[1] + 400), float(start[2] + 300)]},
             "end": {"mins": list(map(float, fin_lo)), "maxs": list(map(float, fin_hi))}}
    meta = dict(kind="race_track", seed=seed, n_ramps=n_ramps, gap_jumps=sorted(int(g) for g in gap_at),
                approx_track_length=float(n_ramps * ramp_length + (n_rows - 1) * row_pitch), brushes=len(b.brushes),
                path=[list(map(float, p)) for p in path])
    return ProcMap(f"proc_race_s{seed}", image, zones, meta, ramps, pool)


MAP_KINDS = {"ramps": ramps_map, "field": random_field_map, "race": race_track_map}


def generate(kind: str, seed: int = 0, **kw) -> ProcMap:
    if kind not in MAP_KINDS:
        raise ValueError(f"unknown map kind {kind!r}; choose from {sorted(MAP_KINDS)}")
    return MAP_KINDS[kind](seed=seed, **kw)


def cached_map(kind: str, seed: int = 0, directory=None, **kw) -> Path:
    """Generate (or reuse) a procedural map on disk; returns the .bsp path."""
    d = Path(directory) if directory else Path(__file__).resolve().parents[2] / "maps"
    name = {"ramps": "proc_ramps", "field": "proc_field", "race": "proc_race"}[kind] + f"_s{seed}"
    p = d / f"{name}.bsp"
    if not p.exists() or not (d / f"{name}.meta.json").exists():
        generate(kind, seed, **kw).save(d)
    return p
