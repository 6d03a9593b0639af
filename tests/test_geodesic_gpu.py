"""Geodesic distance bake (csrc/kernels/geodesic.cu) against the numpy
Bellman-Ford oracle on a synthetic maze, and against the host path (native
Dijkstra, the same fixed point) on the race map's goal field."""
import numpy as np
import pytest
import torch

from surfb200.ops.geodesic import bake_goal_field, geodesic, geodesic_reference

pytestmark = pytest.mark.gpu


def test_geodesic_matches_oracle_on_a_maze():
    rng = np.random.default_rng(0)
    occ = (rng.random((12, 40, 56)) < 0.25).astype(np.uint8)
    occ[:, 20, 5:50] = 1                                   # a wall with a gap forces detours
    lo, hi = (2, 2, 2), (4, 4, 4)
    occ[lo[2]:hi[2] + 1, lo[1]:hi[1] + 1, lo[0]:hi[0] + 1] = 0
    ref = geodesic_reference(occ, 16.0, lo, hi)
    got = geodesic(torch.as_tensor(occ, device="cuda"), 16.0, lo, hi).cpu().numpy()
    fin = ref < 1e30
    assert np.array_equal(fin, got < 1e30)
    np.testing.assert_allclose(got[fin], ref[fin], rtol=1e-5, atol=1e-2)


def test_goal_field_bake_gpu_matches_cpu():
    from surfb200.sim import mapgen
    from surfb200.sim.core import SimCore, default_config
    m = mapgen.generate("race", 0)
    core = SimCore.from_bytes(m.image, default_config(1), threads=4)
    end = m.zones["end"]
    g = bake_goal_field(core, end, cell=64.0, device="cuda")
    c = bake_goal_field(core, end, cell=64.0, device="cpu")
    assert g.grid.shape == c.grid.shape
    assert abs(g.reach_max - c.reach_max) < 1e-2 * max(1.0, c.reach_max)
    diff = np.abs(g.grid.astype(np.int64) - c.grid.astype(np.int64))
    assert diff.max() <= 1
    start = m.spawn_pool["origin"][:64].astype(np.float64)
    assert np.all(np.isfinite(g.sample(start)))


def test_kill_aware_goal_field_gpu_matches_cpu():
    """The race map's fail nets as walls of the goal graph: the GPU bake and
    the host bake agree, the starts stay connected, and no path through a
    kill volume shortens the distance."""
    from surfb200.sim import mapgen
    from surfb200.sim.core import SimCore, default_config
    m = mapgen.generate("race", 0)
    core = SimCore.from_bytes(m.image, default_config(1), threads=4)
    end = m.zones["end"]
    g = bake_goal_field(core, end, cell=64.0, device="cuda", kill_aware=True)
    c = bake_goal_field(core, end, cell=64.0, device="cpu", kill_aware=True)
    plain = bake_goal_field(core, end, cell=64.0, device="cuda")
    assert np.abs(g.grid.astype(np.int64) - c.grid.astype(np.int64)).max() <= 1
    start = m.spawn_pool["origin"][:64].astype(np.float64)
    d_k, d_p = g.sample(start), plain.sample(start)
    assert np.all(d_k < g.valid_max)                       # the starts still reach the finish
    assert np.all(d_k >= d_p - 1.0)                        # walls only lengthen the routes
    assert int((g.grid == np.uint16(round(g.sentinel / g.quant))).sum()) > \
        int((plain.grid == np.uint16(round(plain.sentinel / plain.quant))).sum())
