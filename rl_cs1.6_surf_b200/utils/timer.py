"""Per-iteration phase timing (reference: PhaseTimer, python/train_fast.py:311-401).

CPU phases are perf_counter brackets; GPU phases are pooled CUDA event pairs
read once per iteration (one synchronize), so timing does not serialise the
pipeline it measures. Disabled, every call is a single attribute test.

With ``SURF_NVTX=1`` in the environment (or ``nvtx=True``) every phase is
also an NVTX range (``torch.cuda.nvtx``), so a system profiler shows the
trainer's phases above its kernels; this works with timing off.
"""
from __future__ import annotations

import os
import time

import torch


class PhaseTimer:
    def __init__(self, enabled: bool, cuda: bool, nvtx: bool = None) -> None:
        self.on = bool(enabled)
        self.cuda = bool(cuda) and self.on
        self.nvtx = (os.environ.get("SURF_NVTX", "0") == "1") if nvtx is None else bool(nvtx)
        self.nvtx = self.nvtx and bool(cuda)
        self.acc: dict = {}
        self._pool: dict = {}
        self._used: dict = {}
        self._t0 = 0.0

    def now(self) -> float:
        return time.perf_counter() if self.on else 0.0

    def begin(self, name: str) -> float:
        """Start the CPU phase `name` (close it with add(name, t0))."""
        if self.nvtx:
            torch.cuda.nvtx.range_push(name)
        return time.perf_counter() if self.on else 0.0

    def add(self, name: str, t0: float) -> None:
        if self.on:
            self.acc[name] = self.acc.get(name, 0.0) + (time.perf_counter() - t0) * 1e3
        if self.nvtx:
            torch.cuda.nvtx.range_pop()

    def gpu_start(self, name: str):
        if self.nvtx:
            torch.cuda.nvtx.range_push(name)
        if not self.cuda:
            return None
        pool = self._pool.setdefault(name, [])
        k = self._used.get(name, 0)
        if k == len(pool):
            pool.append((torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)))
        self._used[name] = k + 1
        pool[k][0].record()
        return pool[k]

    def gpu_end(self, pair) -> None:
        if pair is not None:
            pair[1].record()
        if self.nvtx:
            torch.cuda.nvtx.range_pop()

    def start_iter(self) -> None:
        if self.on:
            self.acc = {}
            self._used.clear()
            self._t0 = time.perf_counter()

    def flush(self, iteration: int) -> dict:
        """Fold the event pairs in and return {phase: ms} (empty when off)."""
        if not self.on:
            return {}
        if self.cuda:
            torch.cuda.synchronize()
            for name, pool in self._pool.items():
                ms = sum(pool[k][0].elapsed_time(pool[k][1]) for k in range(self._used.get(name, 0)))
                self._used[name] = 0
                if ms:
                    self.acc[name + "_ms"] = self.acc.get(name + "_ms", 0.0) + ms
        self.acc["total"] = (time.perf_counter() - self._t0) * 1e3
        return dict(self.acc)

    @staticmethod
    def format(iteration: int, acc: dict) -> str:
        return f"TIMING iter={iteration} " + " ".join(f"{k}={v:.1f}" for k, v in acc.items())
