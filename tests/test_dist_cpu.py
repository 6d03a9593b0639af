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
