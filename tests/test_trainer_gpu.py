"""End-to-end GPU training iterations (small vision configuration)."""
import math

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
