"""Respawn reservoir: exploring starts from the agent's own runs (Go-Explore style).

Behaviour of the reference (python/surfgym/respawn.py:29-229): full physics
states are snapshotted along live episodes every ``snap_every`` ticks; when
an episode ends (any way), only the snapshots taken at least ``margin``
ticks before that end are harvested into a FIFO reservoir (a state just
before a fatal mistake is usually already lost; the rule also keeps
next-to-the-finish states out). Each iteration a spawn pool is rebuilt: a
``fresh_frac`` share of map starts plus reservoir states with their speed
scaled by U(vel_scale) and their view pitch jittered (position and velocity
direction never change). With a distance function (race: the geodesic
distance to the finish) reservoir draws are spread uniformly over distance
bins, each bin capped at 4x its population, so the frontier is not starved
by the well-visited early track.

This implementation keeps the per-env pending snapshots in fixed numpy
arrays (no per-env Python lists), observes once per decision (``K`` ticks),
and under data parallelism merges every rank's harvest of the iteration in
(tick, global env id) order so that all ranks hold the same reservoir
(docs/ddp-plan.md:227-253).
"""
from __future__ import annotations

from typing import Callable, Optional

import numpy as np

from ..sim.core import STATE_DTYPE


def even_shares_under_caps(n: int, caps: np.ndarray) -> np.ndarray:
    """Split n draws over k groups as evenly as the per-group caps allow.

    Returns alloc with alloc <= caps and sum(alloc) = min(n, sum(caps)):
    every group gets min(cap, L) for the largest level L that does not
    overshoot n, and the remaining draws go one each to the lowest-index
    groups still below their cap (the nearest distance bins)."""
    caps = np.asarray(caps, np.int64)
    if n <= 0 or caps.size == 0:
        return np.zeros(caps.size, np.int64)
    if n >= int(caps.sum()):
        return caps.copy()
    lo, hi = 0, int(caps.max())
    while lo < hi:                                          # largest L with sum(min(caps, L)) <= n
        mid = (lo + hi + 1) // 2
        if int(np.minimum(caps, mid).sum()) <= n:
            lo = mid
        else:
            hi = mid - 1
    alloc = np.minimum(caps, lo)
    extra = n - int(alloc.sum())
    alloc[np.flatnonzero(alloc < caps)[:extra]] += 1
    return alloc

class RespawnReservoir:
    def __init__(self, n_envs: int, reservoir: int = 100_000, margin_ticks: int = 1000, snap_every: int = 100,
                 max_pending: int = 64, map_id: str = "", seed: int = 23, dist_fn: Optional[Callable] = None,
                 dist_max: Optional[float] = None, dist_valid_max: Optional[float] = None, bins: int = 16,
                 rank: int = 0):
        if dist_fn is not None and not dist_max:
            raise ValueError("dist_fn needs dist_max (the start distance)")
        self.n, self.cap, self.margin, self.snap_every = int(n_envs), int(reservoir), int(margin_ticks), int(snap_every)
        self.map_id = str(map_id)
        self.dist_fn, self.dist_max, self.dist_valid_max, self.bins = dist_fn, dist_max, dist_valid_max, int(bins)
        self.rank = int(rank)
        self.store = np.zeros(self.cap, STATE_DTYPE)
        self.d = np.zeros(self.cap, np.float32)
        self.size = 0
        self.head = 0
        self.tick = np.zeros(self.n, np.int64)
        self.last_snap = np.zeros(self.n, np.int64)
        self.P = int(max_pending)
        self.pend = np.zeros((self.n, self.P), STATE_DTYPE)
        self.pend_tick = np.zeros((self.n, self.P), np.int64)
        self.pend_n = np.zeros(self.n, np.int64)
        self.rng = np.random.default_rng(seed)
        self.harvested = 0
        self.new_rows: list = []          # this iteration's harvest: (tick, env, row) for the cross-rank merge

    # ---- collection ----------------------------------------------------------------------
    def observe(self, states: np.ndarray, ended: np.ndarray, stagnant: Optional[np.ndarray] = None,
                ticks: int = 1, step_index: int = 0) -> None:
        """``states``: post-step state rows (ended rows already hold the next
        episode's spawn); ``ended``: episodes that ended during these
        ``ticks``; ``stagnant``: envs making no progress (never snapshotted)."""
        self.tick += ticks
        ended = np.asarray(ended, bool)
        if ended.any():
            for i in np.flatnonzero(ended):
                k = int(self.pend_n[i])
                if k:
                    ok = self.pend_tick[i, :k] <= self.tick[i] - self.margin
                    for j in np.flatnonzero(ok):
                        self.new_rows.append((step_index, self.rank * self.n + int(i), self.pend[i, j].copy()))
            self.pend_n[ended] = 0
            self.tick[ended] = 0
            self.last_snap[ended] = 0
        snap = (~ended) & (self.tick - self.last_snap >= self.snap_every)
        if stagnant is not None:
            snap &= ~np.asarray(stagnant, bool)
        if snap.any():
            idx = np.flatnonzero(snap)
            slot = self.pend_n[idx]
            full = slot >= self.P                      # keep the newest: drop the oldest pending snapshot
            if full.any():
                f = idx[full]
                self.pend[f, :-1] = self.pend[f, 1:]
                self.pend_tick[f, :-1] = self.pend_tick[f, 1:]
                slot = np.minimum(slot, self.P - 1)
            self.pend[idx, slot] = states[idx]
            self.pend_tick[idx, slot] = self.tick[idx]
            self.pend_n[idx] = np.minimum(self.pend_n[idx] + 1, self.P)
            self.last_snap[idx] = self.tick[idx]

    def commit(self, comm=None) -> int:
        """Push this iteration's harvest (all ranks' under ``comm``) into the
        reservoir in (step, global env id) order; returns the rows added."""
        rows = self.new_rows
        self.new_rows = []
        if comm is not None:
            import torch.distributed as dist
            everyone = [None] * dist.get_world_size()
            payload = [(s, e, r.tobytes()) for s, e, r in rows]
            dist.all_gather_object(everyone, payload)
            rows = [(s, e, np.frombuffer(b, STATE_DTYPE)[0]) for part in everyone for (s, e, b) in part]
        rows.sort(key=lambda x: (x[0], x[1]))
        if not rows:
            return 0
        arr = np.array([r for _, _, r in rows], STATE_DTYPE)
        ds = self._dists(arr)
        for k in range(len(arr)):
            self._push(arr[k], 0.0 if ds is None else float(ds[k]))
        self.harvested += len(arr)
        return len(arr)

    def _dists(self, arr: np.ndarray) -> Optional[np.ndarray]:
        if self.dist_fn is None or len(arr) == 0:
            return None
        return np.asarray(self.dist_fn(arr["origin"].astype(np.float64)), np.float32)

    def _push(self, row, d: float) -> None:
        self.store[self.head] = row
        self.d[self.head] = d
        self.head = (self.head + 1) % self.cap
        self.size = min(self.size + 1, self.cap)

    # ---- sampling ------------------------------------------------------------------------
    def binned_pick(self, n: int) -> np.ndarray:
        """n reservoir indices spread evenly over the occupied goal-distance
        bins (uniform within a bin), no bin drawn more than 4x its population;
        demand the caps cannot absorb falls back to uniform draws over the
        whole reservoir (the reference's rule, python/surfgym/respawn.py:124-166).

        Vectorised: the candidates are grouped by bin with one stable sort,
        the per-bin counts come from ``even_shares_under_caps`` in closed form,
        and every draw is one offset into its bin's slice of the sorted
        candidates."""
        dist = self.d[:self.size]
        cand = np.flatnonzero(dist < self.dist_valid_max) if self.dist_valid_max else np.arange(self.size)
        if cand.size == 0:
            return self.rng.integers(0, self.size, n)
        nbins = int(self.bins)
        b = np.floor(dist[cand].astype(np.float64) * (nbins / float(self.dist_max)))
        b = np.clip(b, 0, nbins - 1).astype(np.int64)
        members = cand[np.argsort(b, kind="stable")]
        pop_all = np.bincount(b, minlength=nbins)
        first_all = np.concatenate(([0], np.cumsum(pop_all)[:-1]))
        occupied = np.flatnonzero(pop_all)
        pop, first = pop_all[occupied], first_all[occupied]
        take = even_shares_under_caps(int(n), 4 * pop)
        which = np.repeat(np.arange(occupied.size), take)
        offs = np.minimum((self.rng.random(which.size) * pop[which]).astype(np.int64), pop[which] - 1)
        out = members[first[which] + offs]
        if out.size < n:
            out = np.concatenate([out, self.rng.integers(0, self.size, n - out.size)])
        self.rng.shuffle(out)
        return out

    def build_pool(self, start_pool: np.ndarray, pool_size: int = 4096, fresh_frac: float = 0.10,
                   vel_scale=(0.9, 1.1), pitch_jitter: float = 5.0) -> np.ndarray:
        if self.size == 0:
            return start_pool
        n_fresh = max(1, int(round(pool_size * fresh_frac)))
        n_re = pool_size - n_fresh
        idx = self.binned_pick(n_re) if self.dist_fn is not None else self.rng.integers(0, self.size, n_re)
        re = self.store[idx].copy()
        re["velocity"] *= self.rng.uniform(vel_scale[0], vel_scale[1], n_re).astype(np.float32)[:, None]
        re["pitch"] = np.clip(re["pitch"] + self.rng.uniform(-pitch_jitter, pitch_jitter, n_re).astype(np.float32),
                              -70.0, 30.0)
        re["tick"] = 0
        fresh = start_pool[self.rng.integers(0, len(start_pool), n_fresh)]
        return np.concatenate([fresh, re])

    # ---- persistence ---------------------------------------------------------------------
    def state_dict(self, max_states: int = 20_000) -> dict:
        if self.size == 0:
            return {"states": None, "map_id": self.map_id}
        take = min(self.size, max_states)
        idx = (self.head - take + np.arange(take)) % self.cap
        return {"states": self.store[idx].copy(), "map_id": self.map_id}

    def load_state_dict(self, sd: dict) -> bool:
        arr = sd.get("states") if isinstance(sd, dict) else None
        if arr is None or len(arr) == 0:
            return False
        if sd.get("map_id") != self.map_id:
            return False                                    # raw map coordinates: never across maps
        arr = np.asarray(arr, STATE_DTYPE)[-self.cap:]
        ds = self._dists(arr)
        for k in range(len(arr)):
            self._push(arr[k], 0.0 if ds is None else float(ds[k]))
        return True
