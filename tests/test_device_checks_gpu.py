"""Device-side index checks: the data-driven gathers (minibatch row gather,
frame-stack gather, PPO loss sample index) skip an out-of-range index, zero
the affected output and record an error code in the per-device flag, which
check_error_flag turns into a KernelError on the host. No fault, no trap:
the context stays usable. Oracles: plain torch indexing of the valid rows."""
import pytest
import torch

from surfb200.ops import _lib
from surfb200.ops import gemm as G
from surfb200.ops.framestack import FrameStacker

pytestmark = pytest.mark.gpu


def _expect_error(code):
    f = G.error_flag("cuda")
    assert int(f.item()) == code
    with pytest.raises(_lib.KernelError, match=hex(code)):
        G.check_error_flag("cuda")
    assert int(f.item()) == 0


def test_gather_rows_out_of_range_index():
    G.check_error_flag("cuda")
    src = torch.randn(10, 16, device="cuda")
    idx = torch.tensor([3, 9, 10, -1, 0], dtype=torch.int64, device="cuda")
    out = torch.full((5, 16), 7.0, device="cuda")
    G.gather_rows(src, idx, out)
    torch.cuda.synchronize()
    torch.testing.assert_close(out[[0, 1, 4]], src[[3, 9, 0]], rtol=0, atol=0)
    assert torch.all(out[[2, 3]] == 0)
    _expect_error(0x100)
    G.gather_rows(src, idx[[0, 1, 4]], out[:3])       # valid again: no error
    G.check_error_flag("cuda")


def test_frame_stack_gather_out_of_range_index():
    G.check_error_flag("cuda")
    st = FrameStacker(2, 64)
    T, N = 4, 8
    frames = torch.randn(st.pro + T + 1, N, st.fr, device="cuda").to(torch.bfloat16)
    ages = torch.zeros(T * N, dtype=torch.int32, device="cuda")
    idx = torch.tensor([0, 5, T * N, 31], dtype=torch.int64, device="cuda")
    out = torch.full((4, st.fr * 2), 3.0, device="cuda").to(torch.bfloat16)
    st.gather(frames, idx, ages, out)
    torch.cuda.synchronize()
    assert torch.all(out[2] == 0) and not torch.all(out[1] == 0)
    _expect_error(0x101)


def test_ppo_loss_out_of_range_sample_index():
    from surfb200.models.policy import HeadLayout
    from surfb200.ops import rl as R
    G.check_error_flag("cuda")
    layout = HeadLayout(("yaw", "pitch", "fwd", "side", "jump", "duck"), False)
    heads = R.HeadArgs(layout, torch.device("cuda"))
    B, n_src = 8, 6
    g = torch.Generator(device="cuda").manual_seed(0)
    out = torch.randn(B, 64, device="cuda", generator=g)
    act = torch.zeros(n_src, 8, dtype=torch.int32, device="cuda")
    old = torch.zeros(n_src, device="cuda")
    adv = torch.randn(n_src, device="cuda", generator=g)
    ret = torch.randn(n_src, device="cuda", generator=g)
    idx = torch.tensor([0, 1, 2, 3, 4, 5, 6, 2], dtype=torch.int64, device="cuda")    # 6 is out of range
    mom = torch.tensor([float(adv.sum()), float((adv * adv).sum())], dtype=torch.float64, device="cuda")
    coef = torch.tensor([0.2, 0.5, 0.005], device="cuda")
    dout = torch.full((B, 64), 5.0, device="cuda")
    dls = torch.zeros(1, device="cuda")
    stats = torch.zeros(6, device="cuda")
    log_std = torch.zeros(1, device="cuda")
    R.ppo_loss(out, layout.value_col, act, old, adv, ret, idx, mom, heads, log_std, coef, float(B), dout, dls, stats)
    torch.cuda.synchronize()
    assert torch.all(dout[6, :layout.value_col + 1] == 0)
    assert stats[5].item() == B - 1          # the skipped row adds no sample
    _expect_error(0x102)
