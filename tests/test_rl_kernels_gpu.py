"""RL kernels (csrc/kernels/rl.cu, reward.cu, adam.cu) against fp32 PyTorch oracles.

Reference checks these replace: the reference trainer's update is autograd
over log_softmax / ratio / clip (python/train_fast.py:1846-1864), its GAE a
Python reverse scan (:2119-2133), its optimizer clip_grad_norm_ + torch Adam
(:1505-1506, :2194-2195), and its numerics gate compares the compiled update
with eager (tools/bench_update.py:207-243). Here each hand-written kernel is
compared with the plain fp32 statement of the same rule in ops/rl.py or with
torch itself.
"""
import math

import numpy as np
import pytest
import torch

from surfb200.models.policy import HeadLayout
from surfb200.ops import _lib
from surfb200.ops import rl as R
from surfb200.ops._lib import check, ptr, stream_ptr

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")

LAYOUTS = [HeadLayout(), HeadLayout(("pitch", "fwd", "side", "jump", "duck"), continuous_yaw=True)]


def _logits(n, layout, seed, scale=2.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(n, layout.value_col + 1, generator=g) * scale).to(DEV)


# ---- sampling -------------------------------------------------------------------------
@pytest.mark.parametrize("layout", LAYOUTS, ids=["discrete", "cont_yaw"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_sample_logp_matches_reference(layout, dtype):
    n = 4096
    heads = R.HeadArgs(layout, DEV)
    logits = _logits(n, layout, 1).to(dtype)
    log_std = torch.tensor([-0.3], device=DEV)
    act = torch.zeros(n, 8, dtype=torch.int32, device=DEV)
    logp = torch.zeros(n, device=DEV)
    fail = (torch.arange(n, device=DEV) % 5 == 0).to(torch.uint8)
    R.sample_heads(logits, heads, log_std, act, logp, seed=1234, counter=7, fail_src=fail)
    torch.cuda.synchronize()
    ref_logp, _ = R.log_prob_reference(logits.float(), act, layout, log_std)
    torch.testing.assert_close(logp, ref_logp, rtol=1e-5, atol=2e-5)
    # every driven slot in range, undriven slots neutral, slot 7 carries the stall flag
    for size, slot in zip(layout.sizes, layout.slots):
        assert int(act[:, slot].min()) >= 0 and int(act[:, slot].max()) < size
    for s, v in enumerate(layout.neutral):
        if v >= 0:
            assert torch.all(act[:, s] == v)
    assert torch.equal(act[:, 7], fail.to(torch.int32))


@pytest.mark.parametrize("layout", LAYOUTS, ids=["discrete", "cont_yaw"])
def test_greedy_sample_is_argmax(layout):
    n = 1024
    heads = R.HeadArgs(layout, DEV)
    logits = _logits(n, layout, 2)
    log_std = torch.tensor([0.1], device=DEV)
    act = torch.zeros(n, 8, dtype=torch.int32, device=DEV)
    R.sample_heads(logits, heads, log_std, act, None, seed=5, counter=0, greedy=True)
    ref, _ = R.sample_reference(logits.cpu(), layout, log_std.cpu(), greedy=True)
    assert torch.equal(act.cpu()[:, :7], ref[:, :7])


@pytest.mark.parametrize("layout", LAYOUTS, ids=["discrete", "cont_yaw"])
def test_sample_distribution_chi_square(layout):
    """2^20 draws of one logits row: per-head category frequencies against the
    softmax (chi-square at p = 1e-6), the Gaussian yaw's standardised mean/std."""
    from scipy.stats import chi2
    n = 1 << 20
    heads = R.HeadArgs(layout, DEV)
    row = _logits(1, layout, 3, scale=1.0)
    logits = row.expand(n, -1).contiguous()
    log_std = torch.tensor([-0.5], device=DEV)
    act = torch.zeros(n, 8, dtype=torch.int32, device=DEV)
    R.sample_heads(logits, heads, log_std, act, None, seed=99, counter=3)
    off = 0
    for size, slot in zip(layout.sizes, layout.slots):
        p = torch.softmax(row[0, off:off + size].double(), -1).cpu().numpy()
        counts = torch.bincount(act[:, slot].long(), minlength=size).double().cpu().numpy()
        exp = p * n
        stat = float(((counts - exp) ** 2 / exp).sum())
        assert stat < chi2.ppf(1 - 1e-6, size - 1), (slot, stat)
        off += size
    if layout.continuous_yaw:
        mu = float(row[0, off])
        a = act[:, 6].view(torch.float32).double()
        z = (a - mu) / math.exp(-0.5)
        assert abs(float(z.mean())) < 6.0 / math.sqrt(n)
        assert abs(float(z.std()) - 1.0) < 6.0 * math.sqrt(0.5 / n)
    # a new counter draws new noise; the same counter repeats it
    act2 = torch.zeros_like(act)
    R.sample_heads(logits, heads, log_std, act2, None, seed=99, counter=3)
    assert torch.equal(act, act2)
    R.sample_heads(logits, heads, log_std, act2, None, seed=99, counter=4)
    assert not torch.equal(act, act2)


# ---- PPO loss ----------------------------------------------------------------------------
@pytest.mark.parametrize("layout", LAYOUTS, ids=["discrete", "cont_yaw"])
@pytest.mark.parametrize("norm_adv", [True, False])
def test_ppo_loss_gradient_matches_autograd(layout, norm_adv):
    torch.manual_seed(0)
    n_src, B = 8192, 2048
    heads = R.HeadArgs(layout, DEV)
    vc = layout.value_col
    src_logits = _logits(n_src, layout, 4)
    log_std = torch.tensor([-0.2], device=DEV)
    act = torch.zeros(n_src, 8, dtype=torch.int32, device=DEV)
    logp0 = torch.zeros(n_src, device=DEV)
    R.sample_heads(src_logits, heads, log_std, act, logp0, seed=11, counter=0)
    # the policy moved since the rollout: ratios spread well past the clip range
    old_logp = logp0 + 0.4 * torch.randn(n_src, device=DEV)
    adv = torch.randn(n_src, device=DEV) * 3.0 + 0.5
    ret = torch.randn(n_src, device=DEV)
    idx = torch.randperm(n_src, device=DEV)[:B]
    out = (src_logits[idx] + 0.05 * torch.randn(B, vc + 1, device=DEV)).contiguous()
    a_mb = adv[idx].double()
    moments = torch.stack([a_mb.sum(), (a_mb * a_mb).sum()])
    clip, vf, ent = 0.2, 0.5, 0.01
    coef = torch.tensor([clip, vf, ent], device=DEV)
    dout = torch.zeros(B, vc + 1, device=DEV)
    dls = torch.zeros(1, device=DEV)
    stats = torch.zeros(6, device=DEV)
    R.ppo_loss(out, vc, act, old_logp, adv, ret, idx, moments, heads, log_std, coef, float(B), dout, dls, stats,
               norm_adv=norm_adv)
    torch.cuda.synchronize()

    x = out.detach().clone().requires_grad_(True)
    ls = log_std.detach().clone().requires_grad_(True)
    loss, pg, vl, entropy = R.ppo_loss_reference(
        x, vc, act[idx], old_logp[idx], adv[idx], ret[idx], layout, ls, clip, vf, ent, norm_adv=norm_adv,
        moments=(float(moments[0]), float(moments[1]), float(B)) if norm_adv else None)
    loss.backward()
    if not norm_adv:
        pass
    ratio = torch.exp(R.log_prob_reference(out, act[idx], layout, log_std)[0] - old_logp[idx])
    assert float(((ratio - 1).abs() > clip).float().mean()) > 0.2            # clipping is active on many rows
    scale = float(x.grad.abs().max())
    torch.testing.assert_close(dout, x.grad, rtol=1e-3, atol=1e-4 * scale)
    if layout.continuous_yaw:
        torch.testing.assert_close(dls, ls.grad, rtol=1e-3, atol=1e-6)
    torch.testing.assert_close(stats[0] / B, pg.detach(), rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(stats[1] / B, vl.detach(), rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(stats[2] / B, entropy.detach(), rtol=1e-4, atol=1e-6)
    assert float(stats[5]) == B
    cos = torch.nn.functional.cosine_similarity(dout.flatten(), x.grad.flatten(), dim=0)
    assert float(cos) > 0.9999
    # the bf16 gradient (the backward GEMMs' operand) is the fp32 one rounded
    dout16 = torch.zeros(B, vc + 1, dtype=torch.bfloat16, device=DEV)
    R.ppo_loss(out, vc, act, old_logp, adv, ret, idx, moments, heads, log_std, coef, float(B), dout16,
               torch.zeros(1, device=DEV), torch.zeros(6, device=DEV), norm_adv=norm_adv)
    torch.cuda.synchronize()
    assert torch.equal(dout16, dout.to(torch.bfloat16))


# ---- GAE and moments -----------------------------------------------------------------------
def test_gae_matches_reference():
    T, n = 128, 4096
    g = torch.Generator(device="cpu").manual_seed(5)
    rew = torch.randn(T, n, generator=g).to(DEV)
    val = torch.randn(T, n, generator=g).to(DEV)
    done = (torch.rand(T, n, generator=g) < 0.03).float().to(DEV)
    last = torch.randn(n, generator=g).to(DEV)
    gamma, lam = 0.9995 ** 3, 0.95
    adv = torch.empty(T, n, device=DEV)
    ret = torch.empty(T, n, device=DEV)
    mom = torch.zeros(2, dtype=torch.float64, device=DEV)
    R.gae(rew, val, done, last, gamma, lam, adv, ret, mom)
    ra, rr = R.gae_reference(rew, val, done, last, gamma, lam)
    torch.testing.assert_close(adv, ra, rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(ret, rr, rtol=1e-5, atol=1e-4)
    a = adv.double()
    torch.testing.assert_close(mom, torch.stack([a.sum(), (a * a).sum()]), rtol=1e-9, atol=1e-6)


def test_gae_terminal_cuts_bootstrap():
    """A done flag at t stops both the value bootstrap and the trace at t."""
    T, n = 8, 32
    rew = torch.ones(T, n, device=DEV)
    val = torch.zeros(T, n, device=DEV)
    done = torch.zeros(T, n, device=DEV)
    done[3] = 1.0
    last = torch.full((n,), 100.0, device=DEV)
    adv = torch.empty(T, n, device=DEV)
    ret = torch.empty(T, n, device=DEV)
    R.gae(rew, val, done, last, 0.5, 1.0, adv, ret, None)
    torch.testing.assert_close(adv[3], torch.ones(n, device=DEV))                       # no bootstrap past t=3
    torch.testing.assert_close(adv[2], torch.full((n,), 1.5, device=DEV))
    torch.testing.assert_close(adv[T - 1], torch.full((n,), 51.0, device=DEV))          # 1 + 0.5 * 100


def test_adv_moments_over_permuted_minibatches():
    n, nmb = 3 * 4096 + 8, 6
    mb = n // nmb
    adv = torch.randn(n, device=DEV) * 2 + 1
    perm = torch.randperm(n, device=DEV)
    out = torch.zeros(nmb, 2, dtype=torch.float64, device=DEV)
    R.adv_moments(adv, perm, mb, nmb, out)
    for m in range(nmb):
        a = adv[perm[m * mb:(m + 1) * mb]].double()
        torch.testing.assert_close(out[m], torch.stack([a.sum(), (a * a).sum()]), rtol=1e-10, atol=1e-8)


@pytest.mark.parametrize("n", [1, 5, 1000, 262144, 2048 * 128 + 17])
def test_permutation_is_a_bijection(n):
    lib = _lib.lib("libsurf_rl.so")
    key = torch.tensor([12345], dtype=torch.int64, device=DEV)
    out = torch.empty(n, dtype=torch.int64, device=DEV)
    check(lib.surf_permutation(ptr(out), n, ptr(key), stream_ptr(DEV)), "surf_permutation")
    first = out.clone()
    assert torch.equal(torch.sort(first).values, torch.arange(n, device=DEV))
    check(lib.surf_permutation(ptr(out), n, ptr(key), stream_ptr(DEV)), "surf_permutation")
    assert torch.equal(torch.sort(out).values, torch.arange(n, device=DEV))
    if n > 4:
        assert not torch.equal(out, first)                   # the key advanced: a fresh permutation


# ---- optimizer ----------------------------------------------------------------------------
class _FlatNet:
    """The flat-buffer interface of PolicyNet that the optimizer uses."""

    def __init__(self, n, seed):
        g = torch.Generator(device="cpu").manual_seed(seed)
        self.flat = torch.randn(n, generator=g).to(DEV)
        self.grad = torch.zeros(n, device=DEV)
        self.flat16 = torch.zeros(n, dtype=torch.bfloat16, device=DEV)
        self.numel = n

    def sync_bf16(self):
        self.flat16.copy_(self.flat)


@pytest.mark.parametrize("grad_scale", [0.01, 10.0], ids=["unclipped", "clipped"])
def test_adam_matches_torch(grad_scale):
    n = 100_003
    net = _FlatNet(n, 0)
    opt = R.Adam(net, lr=3e-4, eps=1e-5, max_norm=0.5)
    ref_net = _FlatNet(n, 0)
    ref_opt = R.Adam(ref_net, lr=3e-4, eps=1e-5, max_norm=0.5)
    p = torch.nn.Parameter(net.flat.clone())
    topt = torch.optim.Adam([p], lr=3e-4, eps=1e-5)
    g = torch.Generator(device="cpu").manual_seed(1)
    for _ in range(5):
        grad = (torch.randn(n, generator=g) * grad_scale).to(DEV)
        net.grad.copy_(grad)
        ref_net.grad.copy_(grad)
        p.grad = grad.clone()
        opt.step()
        ref_opt.step_reference()
        torch.nn.utils.clip_grad_norm_([p], 0.5)
        topt.step()
        torch.cuda.synchronize()
        assert torch.all(net.grad == 0)                            # the kernel clears the gradient
    torch.testing.assert_close(net.flat, ref_net.flat, rtol=1e-5, atol=1e-7)
    torch.testing.assert_close(net.flat, p.detach(), rtol=1e-5, atol=1e-7)
    torch.testing.assert_close(opt.m, ref_opt.m, rtol=1e-5, atol=1e-9)
    torch.testing.assert_close(opt.v, ref_opt.v, rtol=1e-4, atol=1e-12)
    torch.testing.assert_close(net.flat16.float(), net.flat.to(torch.bfloat16).float())
    assert opt.steps == 5


# ---- training pool and ez-greedy bursts -------------------------------------------------------
def test_train_pool_matches_reference():
    T, n = 128, 2048
    ez = (torch.rand(T, n, device=DEV) < 0.07).to(torch.uint8)
    pool = torch.full((T * n,), -1, dtype=torch.int64, device=DEV)
    count = torch.zeros(1, dtype=torch.int64, device=DEV)
    for stride, offset, flags in ((1, 0, None), (3, 2, ez), (1, 0, ez), (4, 1, None)):
        R.train_pool(flags, T, n, stride, offset, pool, count)
        ref = R.train_pool_reference(flags, T, n, stride, offset)
        k = int(count)
        assert k == len(ref) and torch.equal(pool[:k].cpu(), ref)


def test_permutation_pool_is_a_bijection_of_the_pool():
    n_max = 262144
    pool = torch.randperm(n_max, device=DEV)[:100003].sort().values
    pool_full = torch.zeros(n_max, dtype=torch.int64, device=DEV)
    pool_full[:pool.numel()] = pool
    count = torch.tensor([pool.numel()], dtype=torch.int64, device=DEV)
    key = torch.tensor([99], dtype=torch.int64, device=DEV)
    out = torch.full((n_max,), -7, dtype=torch.int64, device=DEV)
    R.permutation_pool(out, pool_full, count, key)
    k = pool.numel()
    assert torch.equal(out[:k].sort().values, pool)
    assert torch.all(out[k:] == -7)                                 # nothing written past the count
    first = out[:k].clone()
    R.permutation_pool(out, pool_full, count, key)
    assert not torch.equal(out[:k], first)                          # the key advanced


def test_sampling_kernel_ez_bursts():
    """Burst rule in the sampling kernel: a running burst repeats its row, new
    bursts start only in envs without one, lengths follow floor(u^-1/(mu-1))
    clamped to [1, max]; rows without a burst are the plain samples."""
    layout = LAYOUTS[0]
    n = 65536
    heads = R.HeadArgs(layout, DEV)
    logits = _logits(n, layout, 21)
    log_std = torch.zeros(1, device=DEV)
    ez = R.EzGreedy(n, eps=0.05, mu=2.0, max_len=9, device=DEV)
    plain = torch.zeros(n, 8, dtype=torch.int32, device=DEV)
    act = torch.zeros(n, 8, dtype=torch.int32, device=DEV)
    flag = torch.zeros(n, dtype=torch.uint8, device=DEV)
    prev = None
    lens, starts = [], 0
    for c in range(40):
        before = ez.left.clone()
        R.sample_heads(logits, heads, log_std, plain, None, seed=3, counter=c)
        R.sample_heads(logits, heads, log_std, act, None, seed=3, counter=c, ez=ez.args(0, n, flag))
        f = flag.bool()
        cont = before > 0
        assert torch.all(f[cont])
        assert torch.equal(act[~f], plain[~f])
        if prev is not None:
            assert torch.equal(act[cont, :6], prev[cont, :6])
        for size, slot in zip(layout.sizes, layout.slots):
            col = act[f, slot]
            assert int(col.min()) >= 0 and int(col.max()) < size
        fresh = f & ~cont
        lens.append(ez.left[fresh] + 1)
        starts += int(fresh.sum())
        prev = act.clone()
    lens = torch.cat(lens).float()
    assert float(lens.min()) >= 1 and float(lens.max()) <= 9
    assert abs(float((lens == 1).float().mean()) - 0.5) < 0.03
    assert starts > 0.03 * 40 * n * 0.7
