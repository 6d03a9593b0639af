"""The simulator's native code under sanitizers (CPU only, no GPU).

Reference strategy: the reference runs no sanitizers; its C safety net is
determinism flags, a NaN scan in its bench and ABI/argtype checks. Here the
native gates (load, traces, physics, throughput, start-node grids) run under
AddressSanitizer + UndefinedBehaviorSanitizer, and the env batch's worker
pool under ThreadSanitizer, stepping the same actions with 1 and 4 threads.
"""
import os
import subprocess

import pytest

from surfb200 import _build


@pytest.fixture(scope="module")
def exes():
    try:
        return _build.build_sanitized()
    except RuntimeError as e:      # no sanitizer runtime on this host
        if "sanitize" in str(e) and ("cannot find" in str(e) or "not supported" in str(e)):
            pytest.skip("sanitizer runtime not installed")
        raise


def _run(path, env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run([str(path)], capture_output=True, text=True, env=env, timeout=600)


def test_gates_under_address_and_undefined_sanitizers(exes):
    r = _run(exes["surfsim_gates_asan"], {"ASAN_OPTIONS": "detect_leaks=1:abort_on_error=0",
                                          "UBSAN_OPTIONS": "print_stacktrace=1"})
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "runtime error" not in r.stderr and "AddressSanitizer" not in r.stderr
    assert r.stdout.strip().splitlines()[-1].startswith("OK")


def test_worker_pool_under_thread_sanitizer(exes):
    r = _run(exes["surfsim_pool_tsan"], {"TSAN_OPTIONS": "halt_on_error=1"})
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "ThreadSanitizer" not in r.stderr
    assert r.stdout.strip().startswith("OK")
