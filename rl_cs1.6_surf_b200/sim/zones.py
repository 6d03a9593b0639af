"""Race zones of timed surf maps: start / finish boxes and kill volumes.

Timed maps label themselves: a thin ``trigger_multiple`` at the start line
fires the timer's start ``func_button``, another at the finish fires its stop
button. The zone is that trigger brush's bounding box. Detection follows the
reference (python/surfgym/zones.py:150-191): a trigger_multiple whose target
is a func_button named (or targeting) something with start / stop|off|end|
finish, else a target named like mapend / finishzone / endzone. Zones are
stored in an editable ``<map>.zones.json`` next to the map; a file marked
``"source": "manual"`` always wins, an automatic one carries the map's
size + mtime signature and is re-extracted when the map changes.

Kill volumes (for kill-aware shaping): every trigger_teleport whose target
names a point entity (under the race rules any teleport is a failure) and
every trigger_hurt with dmg >= 90 (the simulator's lethal threshold).
Point-in-volume tests must use the simulator's hull containment
(``SimCore.trigger_contains``), not these boxes, which are broadphase only.

Pure Python on the BSP bytes (no native library needed).
"""
from __future__ import annotations

import json
import struct
from pathlib import Path
from typing import Union

LUMP_ENTITIES, LUMP_MODELS = 0, 14


def _image(src: Union[str, Path, bytes]) -> bytes:
    return bytes(src) if isinstance(src, (bytes, bytearray)) else Path(src).read_bytes()


def entities(src) -> list:
    """The entity lump as a list of key -> value dicts (quoted pairs inside braces)."""
    data = _image(src)
    if struct.unpack_from("<i", data, 0)[0] != 30:
        raise ValueError("not a BSP v30 file")
    off, n = struct.unpack_from("<ii", data, 4 + 8 * LUMP_ENTITIES)
    text = data[off:off + n].split(b"\0", 1)[0].decode("latin-1")
    out, cur, toks, i = [], None, [], 0
    while i < len(text):
        c = text[i]
        if c == "{":
            cur, toks = {}, []
        elif c == "}":
            if cur is not None:
                out.append(cur)
            cur = None
        elif c == '"':
            j = text.find('"', i + 1)
            if j < 0:
                break
            toks.append(text[i + 1:j])
            if len(toks) == 2 and cur is not None:
                cur[toks[0]] = toks[1]
                toks = []
            i = j
        i += 1
    return out


def model_bounds(src) -> list:
    """(mins, maxs) of every brush model; index N is the ``*N`` reference."""
    data = _image(src)
    off, n = struct.unpack_from("<ii", data, 4 + 8 * LUMP_MODELS)
    return [(list(struct.unpack_from("<3f", data, off + 64 * i)), list(struct.unpack_from("<3f", data, off + 64 * i + 12)))
            for i in range(n // 64)]


def _model(ent) -> int:
    m = ent.get("model", "")
    return int(m[1:]) if m.startswith("*") and m[1:].isdigit() else -1


def detect_zones(src) -> dict:
    ents, boxes = entities(src), model_bounds(src)
    buttons = {e["targetname"]: e for e in ents if e.get("classname") == "func_button" and e.get("targetname")}

    def role_of_button(name: str):
        low, tgt = name.lower(), buttons[name].get("target", "").lower()
        if any(w in low or w in tgt for w in ("stop", "off", "end", "finish")):
            return "end"
        if "start" in low or "start" in tgt:
            return "start"
        return None

    zones = {"start": None, "end": None}
    for e in ents:
        if e.get("classname") != "trigger_multiple":
            continue
        t = e.get("target", "")
        role = role_of_button(t) if t in buttons else None
        if role is None and any(w in t.lower() for w in ("mapend", "map_end", "finishzone", "endzone")):
            role = "end"
        mi = _model(e)
        if role and zones[role] is None and 0 <= mi < len(boxes):
            zones[role] = {"mins": boxes[mi][0], "maxs": boxes[mi][1]}
    return zones


def kill_zones(src) -> list:
    ents, boxes = entities(src), model_bounds(src)
    dests = {e.get("targetname") for e in ents if e.get("targetname") and _model(e) < 0}
    out = []
    for e in ents:
        mi = _model(e)
        if not 0 <= mi < len(boxes):
            continue
        cls = e.get("classname")
        try:
            dmg = float(e.get("dmg", 0.0))
        except ValueError:
            dmg = 0.0
        if (cls == "trigger_teleport" and e.get("target") in dests) or (cls == "trigger_hurt" and dmg >= 90.0):
            org = [float(v) for v in e.get("origin", "0 0 0").split()[:3]] if e.get("origin") else [0.0, 0.0, 0.0]
            out.append({"mins": boxes[mi][0], "maxs": boxes[mi][1], "class": cls, "model": f"*{mi}", "origin": org})
    return out


def zones_path(bsp_path) -> Path:
    p = Path(bsp_path)
    return p.with_name(p.stem + ".zones.json")


def _signature(bsp_path) -> str:
    st = Path(bsp_path).stat()
    return f"{st.st_size}_{st.st_mtime_ns}"


def load_zones(bsp_path, create: bool = True) -> dict:
    zp, sig = zones_path(bsp_path), _signature(bsp_path)
    if zp.exists():
        doc = json.loads(zp.read_text())
        if doc.get("source") in ("manual", "procedural") or doc.get("bsp_sig") == sig:
            return doc
    z = detect_zones(bsp_path)
    doc = {"map": Path(bsp_path).stem, "source": "auto", "bsp_sig": sig, **z}
    if create and (z["start"] or z["end"]):
        zp.write_text(json.dumps(doc, indent=2))
    return doc
