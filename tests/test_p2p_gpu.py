"""Peer-memory collectives (csrc/comm/p2p.cu).

Single GPU: a one-rank plan must reproduce the fused clip + Adam kernel (its
own gradient term is read in fp32), and
a wait on a flag that no peer ever sets must run out after its short limit
and report an error status while the context stays usable. Two or more GPUs:
two NCCL ranks compare the fused reduce-scatter / clip / Adam / push step
(peer terms in bf16, without and with the overlapped bucket launched on a
side stream), the moments all-reduce and the count merge with plain torch
(eager and inside CUDA graphs).
"""
import ctypes
from ctypes import c_int64, c_void_p

import pytest
import torch

from surfb200.ops import _lib
from surfb200.parallel import p2p as P

pytestmark = pytest.mark.gpu


def _arr(ptrs):
    return (c_void_p * len(ptrs))(*[c_void_p(int(p)) for p in ptrs])


def _buffers(n, dev, seed=0):
    g = torch.Generator().manual_seed(seed)
    flat = torch.randn(n, generator=g).to(dev)
    grad = (torch.randn(n, generator=g) * 0.05).to(dev)
    return flat, grad, flat.to(torch.bfloat16), torch.zeros(n, device=dev), torch.zeros(n, device=dev)


def test_single_rank_step_matches_fused_adam():
    from surfb200.ops.rl import Adam
    L = _lib.lib(P.CLIB)
    dev = torch.device("cuda")
    n = 300_008                                   # gradients cross NVLink in 16-byte bf16 groups
    flat, grad, flat16, m, v = _buffers(n, dev)
    g16 = torch.zeros(n, dtype=torch.bfloat16, device=dev)
    hyper = torch.tensor([1e-3, 0.9, 0.999, 1e-5, 0.5, 0.0], device=dev)
    sync = torch.zeros(int(L.surf_p2p_sync_words()), dtype=torch.int64, device=dev)
    plan = L.surf_p2p_create(0, 1, _arr([sync.data_ptr()]), 5.0)
    assert plan
    try:
        assert L.surf_p2p_set_grad(plan, n, _arr([grad.data_ptr()]), _arr([flat.data_ptr()]),
                                   _arr([flat16.data_ptr()]), m.data_ptr(), v.data_ptr(), hyper.data_ptr(), 0) == 0
        assert L.surf_p2p_set_grad16(plan, _arr([g16.data_ptr()])) == 0

        class Net:
            pass
        ref = Net()
        ref.flat, ref.grad, ref.flat16, ref.numel = flat.clone(), grad.clone(), flat16.clone(), n
        opt = Adam(ref, lr=1e-3, eps=1e-5, max_norm=0.5)
        for it in range(3):
            g = (torch.randn(n, generator=torch.Generator().manual_seed(it)) * 0.05).to(dev)
            grad.copy_(g)
            ref.grad.copy_(g)
            assert L.surf_p2p_grad_step(plan, c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
            opt.step()
            torch.cuda.synchronize()
            assert int(sync[P.W_ERR]) == 0
            torch.testing.assert_close(flat, ref.flat, rtol=1e-5, atol=1e-6)
            assert torch.equal(flat16, ref.flat16)
            assert not grad.any()
        assert int(sync[P.W_SEQ_GRAD]) == 3 and float(hyper[5]) == 3.0
    finally:
        L.surf_p2p_destroy(plan)


def test_wait_without_peer_times_out_with_status():
    """World of two where the second 'rank' never runs: its flags stay unset."""
    L = _lib.lib(P.CLIB)
    dev = torch.device("cuda")
    n = 4096
    flat, grad, flat16, m, v = _buffers(n, dev)
    peer = _buffers(n, dev, seed=1)
    hyper = torch.tensor([1e-3, 0.9, 0.999, 1e-5, 0.5, 0.0], device=dev)
    words = int(L.surf_p2p_sync_words())
    sync = torch.zeros(words, dtype=torch.int64, device=dev)
    ghost = torch.zeros(words, dtype=torch.int64, device=dev)
    plan = L.surf_p2p_create(0, 2, _arr([sync.data_ptr(), ghost.data_ptr()]), 0.5)
    try:
        assert L.surf_p2p_set_grad(plan, n, _arr([grad.data_ptr(), peer[1].data_ptr()]),
                                   _arr([flat.data_ptr(), peer[0].data_ptr()]),
                                   _arr([flat16.data_ptr(), peer[2].data_ptr()]), m.data_ptr(), v.data_ptr(),
                                   hyper.data_ptr(), 0) == 0
        g16 = torch.zeros(2, n, dtype=torch.bfloat16, device=dev)
        assert L.surf_p2p_set_grad16(plan, _arr([g16[0].data_ptr(), g16[1].data_ptr()])) == 0
        before = flat.clone()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        assert L.surf_p2p_grad_step(plan, c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
        e1.record()
        torch.cuda.synchronize()
        code, target = int(sync[P.W_ERR]), int(sync[P.W_ERR_TARGET])
        assert code == 0x101 and target == 1, hex(code)      # gradient barrier, waiting for rank 1
        assert 400 < e0.elapsed_time(e1) < 5000               # gave up after its 0.5 s limit
        assert torch.equal(flat, before)                       # no partial update was applied
        # later collectives return at once and keep the first error
        mom = torch.ones(4, dtype=torch.float64, device=dev)
        assert L.surf_p2p_moments(plan, mom.data_ptr(), 4, c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
        torch.cuda.synchronize()
        assert int(sync[P.W_ERR]) == 0x101
        # the context is still healthy
        x = torch.randn(256, 256, device=dev)
        assert torch.isfinite(x @ x).all()
        assert "gradient barrier" in P.describe_error(code, target)
    finally:
        L.surf_p2p_destroy(plan)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_peer_memory_collectives():
    from dist_workers import p2p_collectives, run_spawn
    reports, codes = run_spawn(p2p_collectives, 2, timeout_s=300)
    assert len(reports) == 2, (reports, codes)
    for r, (ok, msg) in reports.items():
        assert ok, f"rank {r}: {msg}"
