"""Loading of the in-tree native libraries (``_lib/*.so``).

CUDA libraries are required whenever a CUDA device is used: a missing or
stale library raises instead of silently falling back to PyTorch, so a GPU
run always executes the hand-written kernels.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "_lib"
_lock = threading.Lock()
_cache: dict[str, ctypes.CDLL] = {}


class NativeLibraryMissing(RuntimeError):
    pass


def load(name: str, build_if_missing: bool = True) -> ctypes.CDLL:
    """Load ``_lib/<name>`` (building it first if it is absent)."""
    with _lock:
        if name in _cache:
            return _cache[name]
        path = LIB_DIR / name
        if build_if_missing:
            # a library built from other sources than these would be called
            # with the wrong signatures: rebuild it first (nvcc / g++ exist
            # wherever the framework runs)
            from . import _build
            if _build.is_stale(name):
                # one process builds while the others (data-parallel ranks
                # starting together) wait on the lock, then find it fresh
                import fcntl
                LIB_DIR.mkdir(parents=True, exist_ok=True)
                with open(LIB_DIR / ".build.lock", "w") as lk:
                    fcntl.flock(lk, fcntl.LOCK_EX)
                    try:
                        if _build.is_stale(name):
                            _build.build(only=[name], verbose=False)
                    except Exception as e:                    # noqa: BLE001
                        raise NativeLibraryMissing(f"{path} is stale and could not be rebuilt: {e}") from e
                    finally:
                        fcntl.flock(lk, fcntl.LOCK_UN)
        if not path.exists():
            raise NativeLibraryMissing(
                f"{path} is not built; run `python -c 'import __graft_entry__ as g; g.build()'`")
        lib = ctypes.CDLL(str(path))
        _cache[name] = lib
        return lib


def loaded_paths() -> list[str]:
    return [str(LIB_DIR / n) for n in _cache]
