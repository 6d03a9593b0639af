"""Test configuration: the ``gpu`` marker and shared fixtures.

``pytest -m "not gpu"`` runs everything that needs no CUDA device (CPU
oracles, the simulator, multi-process gloo ranks); ``pytest -m gpu`` runs the
kernel tests on a B200.
"""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
import surfb200  # noqa: E402,F401  (binds the package alias)

# a real community map: the reference ships surf_ski_2.bsp, found in its
# installed copy under baseline/_ref unless SURF_REF_MAP names another file
REF_MAP = Path(os.environ.get("SURF_REF_MAP", ROOT / "baseline" / "_ref" / "maps" / "surf_ski_2.bsp"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        have_cuda = torch.cuda.is_available()
    except Exception:   # pragma: no cover
        have_cuda = False
    if have_cuda:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def maps_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("maps")


@pytest.fixture(scope="session")
def field_map(maps_dir):
    """The 512-brush random-field map (seed 0) on disk."""
    from surfb200.sim import mapgen
    m = mapgen.generate("field", 0)
    return m, m.save(maps_dir)


@pytest.fixture(scope="session")
def ramps_map(maps_dir):
    from surfb200.sim import mapgen
    m = mapgen.generate("ramps", 0)
    return m, m.save(maps_dir)


@pytest.fixture(scope="session")
def ski_map():
    """A real community map shipped with the reference, if present."""
    if not REF_MAP.is_file():
        pytest.skip(f"community map not present ({REF_MAP.name}; set SURF_REF_MAP)")
    return REF_MAP
