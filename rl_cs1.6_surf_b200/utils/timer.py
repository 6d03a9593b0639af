"""Per-iteration phase timing and the ``TIMING`` line.

The line format is the reference's (``TIMING iter=N phase=ms ... total=ms``,
python/train_fast.py:311-401), so its perf tooling parses this trainer's
output; GPU phases carry an ``_ms`` suffix.

Design: host phases are ``with clock.phase(name):`` blocks timed with
``perf_counter``; device phases are ``with clock.gpu(name):`` blocks that
record a start and an end event on the current stream. The events come from
one ring that grows to the number of device spans of an iteration and is
reused afterwards, and the spans are only read at ``collect()`` (one
synchronize per iteration), so timing does not serialise the pipeline it
measures. Disabled, a block costs one branch.

With ``SURF_NVTX=1`` in the environment (or ``nvtx=True``) every block is
also an NVTX range (``torch.cuda.nvtx``), so a system profiler shows the
trainer's phases above its kernels; this works with timing off.
"""
from __future__ import annotations

import contextlib
import os
import time

import torch


class PhaseClock:
    """Host and device phase times of one training iteration."""

    def __init__(self, enabled: bool, cuda: bool, nvtx: bool = None) -> None:
        self.enabled = bool(enabled)
        self.device_spans = bool(cuda) and self.enabled
        want_nvtx = (os.environ.get("SURF_NVTX", "0") == "1") if nvtx is None else bool(nvtx)
        self.nvtx = want_nvtx and bool(cuda)
        self.host_ms: dict = {}
        self._ring: list = []          # torch.cuda.Event(enable_timing=True), reused every iteration
        self._spans: list = []         # (name, index of the start event in the ring)
        self._iter_start = 0.0

    # ---- blocks -------------------------------------------------------------------
    @contextlib.contextmanager
    def phase(self, name: str):
        """A host phase: wall time of the block, summed per name."""
        if self.nvtx:
            torch.cuda.nvtx.range_push(name)
        start = time.perf_counter() if self.enabled else 0.0
        try:
            yield
        finally:
            if self.enabled:
                self.host_ms[name] = self.host_ms.get(name, 0.0) + (time.perf_counter() - start) * 1e3
            if self.nvtx:
                torch.cuda.nvtx.range_pop()

    @contextlib.contextmanager
    def gpu(self, name: str):
        """A device phase: the stream time between two events around the block."""
        if self.nvtx:
            torch.cuda.nvtx.range_push(name)
        slot = None
        if self.device_spans:
            slot = 2 * len(self._spans)
            while len(self._ring) < slot + 2:
                self._ring.append(torch.cuda.Event(enable_timing=True))
            self._spans.append((name, slot))
            self._ring[slot].record()
        try:
            yield
        finally:
            if slot is not None:
                self._ring[slot + 1].record()
            if self.nvtx:
                torch.cuda.nvtx.range_pop()

    # ---- iteration bookkeeping ----------------------------------------------------------
    def new_iteration(self) -> None:
        if self.enabled:
            self.host_ms = {}
            self._spans = []
            self._iter_start = time.perf_counter()

    def collect(self) -> dict:
        """{phase: ms} of the iteration so far (empty when disabled); device
        phases are summed per name under ``<name>_ms``."""
        if not self.enabled:
            return {}
        out = dict(self.host_ms)
        if self._spans:
            torch.cuda.synchronize()
            for name, slot in self._spans:
                key = name + "_ms"
                out[key] = out.get(key, 0.0) + self._ring[slot].elapsed_time(self._ring[slot + 1])
            self._spans = []
        out["total"] = (time.perf_counter() - self._iter_start) * 1e3
        return out

    @staticmethod
    def timing_line(iteration: int, phases: dict) -> str:
        return f"TIMING iter={iteration} " + " ".join(f"{k}={v:.1f}" for k, v in phases.items())
