"""Data-parallel host logic on CPU ranks (gloo), no GPU involved.

Mirrors the reference's designed 2-rank gloo harness (docs/ddp-plan.md:506-562):
replicas stay identical after a training iteration; a rank that dies or stalls
between steps is detected by the survivor's next collective (process-group
timeout) instead of hanging it; a corrupted parameter replica is caught by the
periodic checksum comparison.
"""
import pytest

from dist_workers import gloo_corrupt_replica, gloo_dead_rank, gloo_stalled_rank, gloo_train, run_spawn


def test_gloo_two_ranks_train_identical_replicas():
    reports, codes = run_spawn(gloo_train, 2, timeout_s=300)
    assert len(reports) == 2, (reports, codes)
    for r, (ok, msg) in reports.items():
        assert ok, f"rank {r}: {msg}"


def test_gloo_dead_rank_is_detected():
    reports, codes = run_spawn(gloo_dead_rank, 2, timeout_s=120)
    assert codes[1] == 3
    ok, msg = reports[0]
    assert ok and msg.startswith("detected"), msg


def test_p2p_error_description():
    from surfb200.parallel.p2p import describe_error
    s = describe_error(0x201, 17)
    assert "norm exchange" in s and "rank 1" in s and "#17" in s


def test_gloo_stalled_rank_is_detected():
    reports, codes = run_spawn(gloo_stalled_rank, 2, timeout_s=120)
    ok, msg = reports[0]
    assert ok and msg.startswith("detected"), msg
    assert reports[1] == (True, "stalled")


def test_gloo_corrupt_replica_is_detected():
    reports, codes = run_spawn(gloo_corrupt_replica, 2, timeout_s=300)
    assert len(reports) == 2, (reports, codes)
    for r, (ok, msg) in reports.items():
        assert ok and msg.startswith("detected"), f"rank {r}: {msg}"


def test_rank_cpu_shares_are_disjoint_whole_cores(monkeypatch):
    """Each local rank gets whole physical cores (hyperthread siblings
    together), the shares are disjoint and cover every CPU."""
    from surfb200.parallel import dist as D
    # 16 logical CPUs = 8 cores x 2 siblings numbered i and i + 8
    topo = {c: (0, c % 8) for c in range(16)}
    monkeypatch.setattr(D, "physical_cores", lambda cpus: sorted(
        [[c for c in sorted(cpus) if topo[c] == k] for k in sorted({topo[c] for c in cpus})], key=lambda g: g[0]))
    for world in (1, 2, 3, 4, 8):
        shares = [D.rank_cpu_share(range(16), r, world) for r in range(world)]
        flat = sorted(c for s in shares for c in s)
        assert flat == list(range(16))
        for s in shares:
            assert all((c + 8) % 16 in s for c in s)          # siblings stay together
        if world == 8:
            assert shares[0] == [0, 8] and shares[7] == [7, 15]
