"""In-tree build of every native library of the framework.

Produces shared libraries under ``_lib/`` next to this file:

* ``libsurfsim.so``   — C++17 simulator (BSP reader/writer, hull traces,
  player movement, vectorized env with a persistent thread pool). Built with
  ``-ffp-contract=off`` so float results are bit-identical to the reference
  core built from source with the same flag (reference build.sh:10).
* ``libsurf_*.so``    — CUDA kernels for sm_100a (nvcc ``-gencode
  arch=compute_100a,code=sm_100a``), exported through a plain C ABI so they
  are launched on the caller's stream (CUDA-graph capturable) without
  compiling against torch headers.

A library is rebuilt only when a source, header or flag changed (content hash
stored beside the .so). ``python -m surfb200.build`` or ``__graft_entry__.build``
runs it; nvcc cross-compiles on a machine without a GPU.
"""
from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = ROOT / "csrc"
LIB = PKG / "_lib"

CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
             "-pthread", "-fvisibility=hidden", "-Wall", "-Wno-unused-function"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
                     "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
                     "-Xptxas", "-warn-spills"]


def _cutlass_include() -> list[str]:
    """CUTLASS/CuTe headers vendored with flashinfer (used for sm100 helpers)."""
    try:
        import site
        for sp in site.getsitepackages():
            p = Path(sp) / "flashinfer" / "data" / "cutlass" / "include"
            if p.is_dir():
                return ["-I", str(p)]
    except Exception:   # pragma: no cover
        pass
    return []


# name -> (compiler, sources, extra flags, extra link flags)
def _targets():
    sim = sorted(str(p) for p in (CSRC / "sim").glob("*.cpp"))
    kern = lambda *names: [str(CSRC / "kernels" / n) for n in names]
    comm = lambda *names: [str(CSRC / "comm" / n) for n in names]
    t = {"libsurfsim.so": ("g++", sim, [], []),
         # native acceptance gates of the simulator (an executable, run by tests/test_sim.py)
         "surfsim_gates": ("g++exe", [x for x in sim if not x.endswith("c_api.cpp")] +
                           [str(CSRC / "sim" / "tests" / "gates.cpp")], [], [])}
    groups = {
        "libsurf_vision.so": kern("march.cu", "sdf.cu", "geodesic.cu"),
        "libsurf_rl.so": kern("rl.cu", "reward.cu"),
        "libsurf_nn.so": kern("gemm_tc.cu", "conv_shift.cu", "nn_ops.cu", "adam.cu"),
        "libsurf_comm.so": comm("p2p.cu"),
    }
    for name, srcs in groups.items():
        srcs = [s for s in srcs if Path(s).exists()]
        if srcs:
            t[name] = ("nvcc", srcs, [], ["-lcuda"] if name in ("libsurf_nn.so", "libsurf_comm.so") else [])
    # the GPU env compiles the simulator's header-only per-env code for the
    # device; no FMA contraction, so float expressions round as on the host
    if (CSRC / "kernels" / "env_gpu.cu").exists():
        t["libsurf_env.so"] = ("nvcc", kern("env_gpu.cu"), ["-fmad=false", "-I", str(CSRC / "sim")], [])
    return t


# Sanitizer builds of the simulator (host code only), built on demand by
# tests/test_sanitizers.py rather than by build(): the native gates under
# AddressSanitizer + UndefinedBehaviorSanitizer, and the worker-pool stress
# program under ThreadSanitizer.
_SAN_COMMON = ["-O1", "-g", "-fno-omit-frame-pointer", "-fno-sanitize-recover=all"]


def _sanitizer_targets():
    sim = [str(p) for p in sorted((CSRC / "sim").glob("*.cpp")) if not p.name.endswith("c_api.cpp")]
    tests = CSRC / "sim" / "tests"
    return {"surfsim_gates_asan": ("g++exe", sim + [str(tests / "gates.cpp")],
                                   _SAN_COMMON + ["-fsanitize=address,undefined"], []),
            "surfsim_pool_tsan": ("g++exe", sim + [str(tests / "pool_stress.cpp")],
                                  _SAN_COMMON + ["-fsanitize=thread"], [])}


def build_sanitized(verbose: bool = False) -> dict:
    """Build the sanitizer executables (if stale); {name: path}."""
    out = {}
    for name, spec in _sanitizer_targets().items():
        msg = _compile(name, spec, False)
        if verbose:
            print(msg, flush=True)
        out[name] = LIB / name
    return out


def _digest(compiler: str, srcs: list[str], flags: list[str]) -> str:
    h = hashlib.sha256()
    h.update(" ".join([compiler] + flags).encode())
    dirs = {Path(s).parent for s in srcs}
    if any(Path(s).name == "env_gpu.cu" for s in srcs):
        dirs.add(CSRC / "sim")              # the simulator headers it compiles for the device
    files = set(srcs)
    for d in dirs:
        files |= {str(p) for p in d.glob("*.h*")} | {str(p) for p in d.glob("*.cuh")}
    files |= {str(p) for p in (CSRC / "common").glob("*")} if (CSRC / "common").is_dir() else set()
    for f in sorted(files):
        # repository-relative names: the digest must not depend on where the
        # checkout lives (the GPU box runs a copy under another path)
        try:
            name = str(Path(f).resolve().relative_to(ROOT))
        except ValueError:
            name = Path(f).name
        h.update(name.encode())
        h.update(Path(f).read_bytes())
    return h.hexdigest()


def _plan(name: str, spec):
    """(command, content digest) of one target."""
    compiler, srcs, extra, link = spec
    out = LIB / name
    if compiler == "g++exe":
        base = [f for f in CXX_FLAGS if f not in ("-shared", "-fPIC", "-fvisibility=hidden")]
        cmd = ["g++"] + base + extra + srcs + ["-o", str(out)] + link
        flags = base + extra + link
    elif compiler == "g++":
        cmd = ["g++"] + CXX_FLAGS + extra + srcs + ["-o", str(out)] + link
        flags = CXX_FLAGS + extra + link
    else:
        nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
        inc = ["-I", str(CSRC / "common")] + _cutlass_include()
        cmd = [nvcc] + NVCC_FLAGS + inc + extra + srcs + ["-o", str(out)] + link
        flags = NVCC_FLAGS + extra + link
    return cmd, _digest(compiler, srcs, flags)


def is_stale(name: str) -> bool:
    """True when ``_lib/<name>`` is missing or was built from other sources or flags."""
    spec = _targets().get(name)
    out, stamp = LIB / name, LIB / (name + ".sha")
    if spec is None:
        return not out.exists()
    if not out.exists() or not stamp.exists():
        return True
    return stamp.read_text() != _plan(name, spec)[1]


def _compile(name: str, spec, force: bool) -> str:
    out = LIB / name
    stamp = LIB / (name + ".sha")
    cmd, dig = _plan(name, spec)
    if not force and out.exists() and stamp.exists() and stamp.read_text() == dig:
        return f"{name}: up to date"
    LIB.mkdir(parents=True, exist_ok=True)
    tmp = out.with_name(f"{out.name}.{os.getpid()}.tmp")
    cmd[cmd.index(str(out))] = str(tmp)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build of {name} failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, out)
    stamp.write_text(dig)
    warn = (r.stderr or "").strip()
    return f"{name}: built" + (f"\n{warn}" if warn else "")


def build(force: bool = False, only: list[str] | None = None, verbose: bool = True) -> None:
    targets = _targets()
    if only:
        targets = {k: v for k, v in targets.items() if k in only}
    with cf.ThreadPoolExecutor(max_workers=min(8, len(targets) or 1)) as ex:
        futs = {ex.submit(_compile, n, s, force): n for n, s in targets.items()}
        for f in cf.as_completed(futs):
            msg = f.result()
            if verbose:
                print(msg, flush=True)


if __name__ == "__main__":
    import sys
    build(force="--force" in sys.argv)
