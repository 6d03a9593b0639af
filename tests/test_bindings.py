"""Every native entry point the package calls has a registered ctypes
signature and is exported by its library (an unregistered call would pass
64-bit device pointers as truncated C ints)."""
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "rl_cs1.6_surf_b200"


def _modules():
    import importlib
    for name in ("ops.vision", "ops.gemm", "ops.rl", "ops.geodesic", "ops.conv", "ops.conv_shift", "ops.framestack",
                 "ops.surfmask",
                 "rewards.spec", "parallel.p2p", "models.policy", "trainer.ppo"):
        importlib.import_module("surfb200." + name)


def test_called_entry_points_are_registered_and_exported():
    _modules()
    from surfb200.ops import _lib
    registered = {fn: lib for lib, sigs in _lib._SIGS.items() for fn in sigs}
    called = set()
    for p in PKG.rglob("*.py"):
        if p.parent.name == "sim":           # the simulator (surfsim_*) and the reference core have their own bindings
            continue
        for m in re.finditer(r"\.(surf_[a-z0-9_]+)\(", p.read_text()):
            called.add(m.group(1))
    called -= {n for n in called if n.startswith("surfsim_")}
    missing = sorted(n for n in called if n not in registered)
    assert not missing, f"called without a registered signature: {missing}"
    libdir = PKG / "_lib"
    for lib in sorted({registered[n] for n in called}):
        so = libdir / lib
        if not so.exists():
            pytest.skip(f"{lib} not built")
        syms = subprocess.run(["nm", "-D", "--defined-only", str(so)], capture_output=True, text=True).stdout
        exported = set(re.findall(r" T (surf_[a-z0-9_]+)", syms))
        absent = sorted(n for n in called if registered[n] == lib and n not in exported)
        assert not absent, f"{lib} does not export {absent}"


def test_unregistered_entry_point_raises():
    from surfb200.ops import _lib
    L = _lib.lib("libsurf_vision.so")
    with pytest.raises(AttributeError, match="no registered signature"):
        L.surf_edt_noalloc
