"""End-to-end GPU training iterations (small vision configuration)."""
import math

import numpy as np
import pytest
import torch

from surfb200.rewards.spec import RewardSpec
from surfb200.trainer.config import TrainConfig
from surfb200.trainer.ppo import Trainer

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("graphs,cont", [(True, False), (False, True)])
def test_vision_ppo_iterations(graphs, cont):
    cfg = TrainConfig(map="field", envs=256, n_steps=16, act_every=3, epochs=2, minibatches=4, ep_ticks=60,
                      graphs=graphs, continuous_yaw=cont,
                      reward=RewardSpec(mode="coverage", int_coef=0.25, int_view=8, int_speed=8))
    tr = Trainer(cfg, verbose=False)
    flat0 = tr.net.flat.clone()
    for _ in range(2):
        s = tr.train_iteration()
    torch.cuda.synchronize()
    from surfb200.ops.gemm import check_error_flag
    check_error_flag("cuda")
    assert s["global_step"] == 2 * 256 * 16 * 3
    for k in ("policy_loss", "value_loss", "entropy"):
        assert math.isfinite(s[k]), (k, s)
    assert s["episodes"] > 0                      # 60-tick episodes truncate inside the 96 ticks run
    assert torch.isfinite(tr.net.flat).all()
    assert not torch.equal(flat0, tr.net.flat)    # the optimizer moved the weights
    assert tr.b_img.float().std() > 0.01          # depth images were rendered
    # actions decode within range
    a = tr.b_act.view(-1, 8)
    assert int(a[:, 2].min()) >= 0 and int(a[:, 2].max()) <= 2


def test_async_host_rollout_matches_sync():
    """The overlapped host-env rollout (next group's env step started before
    this group's launches) fills the rollout buffers bit for bit like the
    one-group-at-a-time loop: same seed, same config, one rollout each."""
    def run(async_loop: bool):
        cfg = TrainConfig(map="field", envs=256, n_steps=12, act_every=3, epochs=1, minibatches=2, ep_ticks=20,
                          env_groups=2, reward=RewardSpec(mode="coverage", int_coef=0.25, int_view=8, int_speed=8))
        cfg.async_env = async_loop
        tr = Trainer(cfg, verbose=False)
        tr._host_bound = async_loop               # take the overlapped loop from the first rollout on
        tr.rollout_gpu()
        torch.cuda.synchronize()
        out = [t.clone() for t in (tr.b_act, tr.b_rew, tr.b_done, tr.b_img)] + [tr.hrec.clone()]
        assert tr.global_step == 256 * 12 * 3
        tr.release_graphs()
        return out

    for a, b in zip(run(True), run(False)):
        assert torch.equal(a, b)


@pytest.mark.parametrize("stack,mask", [(5, False), (3, True), (1, True)])
def test_frame_stack_and_surface_mask_training(stack, mask):
    """Rollout composition == update gather (same decision, same bytes), the
    next rollout's first decision reaches back into the carried prologue,
    and evaluation stacks through its own ring."""
    from surfb200.trainer.evaluate import evaluate
    cfg = TrainConfig(map="field", envs=256, n_steps=16, act_every=3, epochs=1, minibatches=4, ep_ticks=60,
                      frame_stack=stack, surf_mask=mask, reward=RewardSpec(mode="speed"))
    tr = Trainer(cfg, verbose=False)
    assert tr.net.cfg.img_c == (16 if tr.s2d else 1) * (2 if mask else 1) * max(stack, 1)
    N, T = tr.N, tr.T
    s = tr.train_iteration()
    assert math.isfinite(s["policy_loss"]) and torch.isfinite(tr.net.flat).all()
    if mask:
        slope = tr.b_img[tr.pro:tr.pro + T].float()[..., 1::2]
        assert 0.0 <= float(slope.min()) and float(slope.max()) <= 1.0
        assert (slope > 0).float().mean() > 0.2
    if stack > 1:
        st = tr.stacker
        idx = torch.arange(T * N, (T + 1) * N, device="cuda")
        tail = torch.zeros((N, tr.img_w), dtype=torch.bfloat16, device="cuda")
        st.gather(tr.b_img, idx, tr.b_age.view(-1), tail)
        assert torch.equal(tail, torch.cat(tr.stk_grp, 0))        # what the policy saw at the tail decision
        assert int(tr.b_age.max()) > 0 and int(tr.b_age.max()) <= st.pro
        tr.train_iteration()
        first = torch.zeros_like(tail)
        st.gather(tr.b_img, torch.arange(0, N, device="cuda"), tr.b_age.view(-1), first)
        assert torch.equal(first, tail)                              # t = 0 continues the previous tail
    summ = evaluate(tr, episodes=2, greedy=True, max_ticks=30)
    assert summ["episodes"] == 2
    tr.release_graphs()


def test_gpu_env_training_iterations():
    """The rollout with the env on the GPU: no host stepping, same buffers."""
    cfg = TrainConfig(map="field", envs=256, n_steps=16, act_every=3, epochs=1, minibatches=4, ep_ticks=60,
                      env_device="cuda", reward=RewardSpec(mode="coverage", int_coef=0.25, int_view=8, int_speed=8))
    tr = Trainer(cfg, verbose=False)
    assert tr.genv is not None and len(tr.groups) == 2
    flat0 = tr.net.flat.clone()
    for _ in range(2):
        s = tr.train_iteration()
    torch.cuda.synchronize()
    assert s["global_step"] == 2 * 256 * 16 * 3
    assert math.isfinite(s["policy_loss"]) and s["episodes"] > 0
    assert not torch.equal(flat0, tr.net.flat)
    assert int(tr.boot_overflow) >= 0
    st = tr.genv.get_states()
    assert (st["tick"] > 0).all() and np.isfinite(st["origin"]).all()
    tr.release_graphs()


@pytest.mark.parametrize("graphs", [True, False])
def test_pooled_update_stride_and_ez(graphs):
    """Train stride + ez-greedy on the GPU path: the pool kernel leaves burst
    rows and off-stride decisions out, the number of minibatches follows the
    pool, and the graphed and eager updates both train."""
    from surfb200.ops import rl as R
    cfg = TrainConfig(map="field", envs=256, n_steps=16, act_every=3, epochs=2, minibatches=4, ep_ticks=60,
                      graphs=graphs, train_stride=2, ez_eps=0.05, ez_max=8, fix_pitch=-10.0,
                      reward=RewardSpec(mode="coverage"))
    tr = Trainer(cfg, verbose=False)
    flat0 = tr.net.flat.clone()
    for it in range(3):
        s = tr.train_iteration()
        assert math.isfinite(s["policy_loss"])
        n = int(tr.pool_count)
        ref = R.train_pool_reference(tr.b_ez, tr.T, tr.N, 2, it % 2)
        assert n == len(ref) and torch.equal(tr.pool[:n].cpu(), ref)
        assert tr.last_minibatches == n // tr.mb
    assert int(tr.b_ez.sum()) > 0
    assert not torch.equal(flat0, tr.net.flat)
    # burst actions are written into the action rows the env received
    flags = tr.b_ez.bool()
    assert torch.all(tr.b_act[flags][:, 0] < 15)
    assert np.all(tr.core.states_view["pitch"] == np.float32(-10.0))        # fixed gaze held
    tr.release_graphs()


def test_host_truncation_bootstrap_values():
    """The host-env truncation bootstrap stages gamma * V(terminal state) for
    exactly the truncated envs of the group, the same values as a forward
    pass on the truncated rows gathered on the host."""
    from surfb200.models.policy import Workspace, forward_gpu
    from surfb200.trainer.ppo import C_OBS, C_REC, C_TOBS, C_TREC
    cfg = TrainConfig(map="field", envs=256, n_steps=4, act_every=3, epochs=1, minibatches=2, ep_ticks=60,
                      graphs=False, reward=RewardSpec(mode="coverage"))
    tr = Trainer(cfg, verbose=False)
    tr.reset()
    torch.cuda.synchronize()
    h = tr.hrec.numpy()
    lo, hi = tr.groups[1]
    trunc = np.array([lo + 3, lo + 40, hi - 1])
    h[trunc, C_TOBS:C_TOBS + 15] = h[trunc, C_OBS:C_OBS + 15]        # terminal obs / pose of a live state
    h[trunc, C_TREC:C_TREC + 6] = h[trunc, C_REC:C_REC + 6]
    h[trunc, C_TREC + 2] += 50.0
    h[trunc, C_REC + 12] = 1.0
    tr.reward.boot.zero_()
    tr._bootstrap_truncations(1, 0)
    got = tr.reward.boot.clone()
    rows = torch.from_numpy(h[trunc]).cuda()
    scal = torch.zeros((len(trunc), 16), dtype=torch.bfloat16, device="cuda")
    tr._features(rows[:, C_TOBS:C_TOBS + 15].contiguous(), scal)
    img = tr.camera.render(rows[:, C_TREC:C_TREC + 6].contiguous())
    out = forward_gpu(tr.net, Workspace(tr.net, len(trunc)), scal, img, B=len(trunc))
    want = cfg.gamma * out[:, tr.layout.value_col].float()
    torch.testing.assert_close(got[torch.from_numpy(trunc).cuda()].float(), want, rtol=1e-3, atol=1e-4)
    mask = torch.ones(len(got), dtype=torch.bool, device="cuda")
    mask[torch.from_numpy(trunc).cuda()] = False
    assert float(got[mask].abs().max()) == 0.0
    assert float(want.abs().max()) > 0.0
