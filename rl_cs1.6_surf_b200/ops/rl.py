"""RL math kernels (csrc/kernels/rl.cu, adam.cu) and their PyTorch oracles.

* ``sample_heads`` — multi-head action sampling + log-prob (one warp per env);
* ``gae`` — advantages/returns with the first two moments of the advantages;
* ``adv_moments`` — per-minibatch advantage moments for a whole epoch;
* ``ppo_loss`` — clipped PPO objective with its gradient w.r.t. the logits,
  value and log-std in closed form;
* ``Adam`` — global-norm clip fused with Adam on the flat parameter buffer.

Each ``*_reference`` function is the fp32 PyTorch statement of the same rule
(used on CPU and as the oracle of the kernel tests).
"""
from __future__ import annotations

import ctypes
import math
from ctypes import c_float, c_int, c_int64, c_uint64, c_void_p
from typing import Optional

import torch

from . import _lib
from ..rewards import spec as _spec  # noqa: F401  (registers surf_permutation_pool of libsurf_rl.so)
from . import gemm as _gemm  # noqa: F401  (registers the libsurf_nn.so signatures the optimizer uses)
from ._lib import check, ptr, stream_ptr

RLIB = "libsurf_rl.so"
NLIB = "libsurf_nn.so"
_lib.register(RLIB, {
    "surf_sample_heads": (c_int, [c_void_p, c_int, c_int64, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                  c_int, c_uint64, c_uint64, c_void_p, c_int, c_void_p, c_int64, c_void_p, c_void_p,
                                  c_int64, c_void_p, c_void_p, c_void_p, c_void_p]),
    "surf_train_pool": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "surf_counter_add": (c_int, [c_void_p, c_int64, c_void_p]),
    "surf_gae": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_float, c_void_p, c_void_p,
                         c_void_p, c_void_p]),
    "surf_adv_moments": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p]),
    "surf_ppo_loss": (c_int, [c_void_p, c_int, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p,
                              c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p,
                              c_float, c_int, c_int, c_void_p, c_int64, c_void_p, c_int64, c_int, c_void_p,
                              c_void_p, c_int64, c_void_p, c_void_p]),
})

LOG_SQRT_2PI = 0.9189385332046727


def _error_flag(device):
    from .gemm import error_flag
    return error_flag(device)


class EzArgs(ctypes.Structure):
    """ez-greedy burst state handed to the sampling kernel (see EzGreedy)."""
    _fields_ = [("eps", c_float), ("inv_mu1", c_float), ("max_len", c_int), ("left", c_void_p), ("act", c_void_p),
                ("flag", c_void_p)]


class EzGreedy:
    """Temporally-extended exploration state of N envs (reference --ez-eps,
    --ez-mu, --ez-max; python/train_fast.py:748-761, 1952-1971). With
    probability ``eps`` per decision an env without a running burst starts
    one: every discrete head gets a uniformly random category, held for
    floor(u^(-1/(mu-1))) decisions (u uniform) clamped to [1, max_len]. Burst
    decisions are flagged off-policy; the update leaves them out of its pool."""

    def __init__(self, n: int, eps: float, mu: float = 2.0, max_len: int = 60, device="cuda"):
        if eps > 0 and mu <= 1.0:
            raise ValueError("ez-greedy needs mu > 1")
        self.eps, self.mu, self.max_len = float(eps), float(mu), int(max_len)
        self.left = torch.zeros(n, dtype=torch.int32, device=device)
        self.act = torch.zeros(n, 8, dtype=torch.int32, device=device)

    def args(self, lo: int, hi: int, flag_out: torch.Tensor) -> EzArgs:
        a = EzArgs()
        a.eps, a.inv_mu1, a.max_len = self.eps, 1.0 / (self.mu - 1.0), self.max_len
        a.left, a.act, a.flag = ptr(self.left[lo:hi]), ptr(self.act[lo:hi]), ptr(flag_out)
        return a

    def apply_reference(self, act: torch.Tensor, layout, generator: Optional[torch.Generator] = None) -> torch.Tensor:
        """CPU statement of the burst rule on sampled action rows (in place);
        returns the off-policy flags (uint8 [N])."""
        n = act.shape[0]
        fresh = (self.left == 0) & (torch.rand(n, generator=generator) < self.eps)
        k = int(fresh.sum())
        if k:
            u = torch.rand(k, generator=generator).clamp_(1e-6, 1.0)
            self.left[fresh] = u.pow(-1.0 / (self.mu - 1.0)).to(torch.int32).clamp_(1, self.max_len)
            row = torch.zeros(k, 8, dtype=torch.int32)
            for s, v in enumerate(layout.neutral):
                if v >= 0:
                    row[:, s] = v
            for size, slot in zip(layout.sizes, layout.slots):
                row[:, slot] = (torch.rand(k, generator=generator) * size).to(torch.int32).clamp_(0, size - 1)
            self.act[fresh] = row
        live = self.left > 0
        act[live, :6] = self.act[live, :6]
        self.left[live] -= 1
        return live.to(torch.uint8)


def train_pool(ez_flag: Optional[torch.Tensor], T: int, n: int, stride: int, offset: int, pool: torch.Tensor,
               count: torch.Tensor) -> None:
    """pool[:count] = the rollout rows t * n + e the update samples from:
    decisions t = offset, offset + stride, ... whose action was on-policy."""
    check(_lib.lib(RLIB).surf_train_pool(ptr(ez_flag), int(T), int(n), int(stride), int(offset), ptr(pool),
                                         ptr(count), stream_ptr(pool.device)), "surf_train_pool")


def train_pool_reference(ez_flag: Optional[torch.Tensor], T: int, n: int, stride: int, offset: int) -> torch.Tensor:
    t = torch.arange(T).repeat_interleave(n)
    keep = (t >= offset) & ((t - offset) % stride == 0)
    if ez_flag is not None:
        keep &= ez_flag.reshape(-1).cpu() == 0
    return torch.nonzero(keep).squeeze(1)


def permutation_pool(out: torch.Tensor, pool: torch.Tensor, count: torch.Tensor, key: torch.Tensor) -> None:
    """out[:count] = pool[pi(i)], a keyed permutation of the pool's first
    ``count`` entries (count read on the device); the key advances."""
    check(_lib.lib(RLIB).surf_permutation_pool(ptr(out), ptr(pool), int(pool.numel()), ptr(count), ptr(key),
                                               stream_ptr(out.device)), "surf_permutation_pool")


class HeadArgs:
    """Device-resident head description shared by sampling and the loss."""

    def __init__(self, layout, device):
        self.layout = layout
        self.sizes = torch.tensor(layout.sizes, dtype=torch.int32)          # host arrays (ctypes pointers)
        self.slots = torch.tensor(layout.slots, dtype=torch.int32)
        self.neutral = torch.tensor(layout.neutral, dtype=torch.int32)
        self.n_heads = len(layout.sizes)
        self.cont = 1 if layout.continuous_yaw else 0

    def host_ptr(self, t):
        return ctypes.c_void_p(t.data_ptr())


# ---- sampling ---------------------------------------------------------------------
def sample_heads(logits: torch.Tensor, heads: HeadArgs, log_std: torch.Tensor, act_out: torch.Tensor,
                 logp_out: Optional[torch.Tensor], seed: int, counter: int, greedy: bool = False,
                 value_src: Optional[torch.Tensor] = None, value_out: Optional[torch.Tensor] = None,
                 fail_src: Optional[torch.Tensor] = None, counter_ptr: Optional[torch.Tensor] = None,
                 counter_offset: int = 0, ez: Optional[EzArgs] = None) -> None:
    """Sample every head for each row of ``logits`` ([N, >=n_logits] fp32);
    writes the int32 action rows (``act_out`` [N, 8]) and summed log-probs;
    optionally copies a strided value column to ``value_out`` and the stall
    flags ``fail_src`` into action slot 7. The Philox counter is
    ``counter + counter_offset`` (+ ``*counter_ptr`` when given, a device
    int64 the trainer advances, so graph replays draw fresh noise). ``ez``
    (``EzGreedy.args``) applies ez-greedy bursts to the sampled rows."""
    n = logits.shape[0]
    check(_lib.lib(RLIB).surf_sample_heads(
        ptr(logits), 1 if logits.dtype == torch.bfloat16 else 0, logits.stride(0), heads.host_ptr(heads.sizes),
        heads.n_heads, heads.host_ptr(heads.slots), heads.cont, heads.host_ptr(heads.neutral), ptr(log_std), n,
        int(seed) & (2 ** 64 - 1), (int(counter) + int(counter_offset)) & (2 ** 64 - 1), ptr(counter_ptr),
        1 if greedy else 0, ptr(act_out), act_out.stride(0),
        ptr(logp_out), ptr(value_src), value_src.stride(0) if value_src is not None else 0, ptr(value_out),
        ptr(fail_src), ctypes.byref(ez) if ez is not None else None, stream_ptr(logits.device)), "surf_sample_heads")


def log_prob_reference(logits: torch.Tensor, act: torch.Tensor, layout, log_std: torch.Tensor):
    """(logp [N], entropy [N]) of int32 action rows under the head layout."""
    logp = torch.zeros(logits.shape[0], dtype=torch.float32, device=logits.device)
    ent = torch.zeros_like(logp)
    off = 0
    for size, slot in zip(layout.sizes, layout.slots):
        lsm = torch.log_softmax(logits[:, off:off + size].float(), -1)
        logp = logp + lsm.gather(1, act[:, slot:slot + 1].long()).squeeze(1)
        ent = ent - (lsm.exp() * lsm).sum(-1)
        off += size
    if layout.continuous_yaw:
        mu = logits[:, off].float()
        a = act[:, 6].view(torch.float32) if act.dtype == torch.int32 else act[:, 6].float()
        z = (a - mu) * torch.exp(-log_std)
        logp = logp - 0.5 * z * z - log_std - LOG_SQRT_2PI
        ent = ent + 0.5 + LOG_SQRT_2PI + log_std
    return logp, ent


def sample_reference(logits: torch.Tensor, layout, log_std: torch.Tensor, generator: Optional[torch.Generator] = None,
                     greedy: bool = False):
    """CPU sampler with the same action-row format (Gumbel-max discrete heads,
    Gaussian yaw): returns (act int32 [N, 8], logp [N])."""
    from ..models.policy import NEUTRAL
    n = logits.shape[0]
    act = torch.zeros(n, 8, dtype=torch.int32)
    for s, v in enumerate(layout.neutral):
        if v >= 0:
            act[:, s] = v
    off = 0
    for size, slot in zip(layout.sizes, layout.slots):
        z = logits[:, off:off + size].float()
        if not greedy:
            u = torch.rand(z.shape, generator=generator).clamp_min(1e-20)
            z = z - torch.log(-torch.log(u))
        act[:, slot] = z.argmax(-1).to(torch.int32)
        off += size
    if layout.continuous_yaw:
        mu = logits[:, off].float()
        a = mu if greedy else mu + torch.exp(log_std) * torch.randn(n, generator=generator)
        act[:, 6] = a.to(torch.float32).view(torch.int32)
    logp, _ = log_prob_reference(logits, act, layout, log_std)
    del NEUTRAL
    return act, logp


def bump_counter(counter: torch.Tensor, inc: int) -> None:
    check(_lib.lib(RLIB).surf_counter_add(ptr(counter), int(inc), stream_ptr(counter.device)), "surf_counter_add")


# ---- GAE ----------------------------------------------------------------------------
def gae(rew, val, done, last_val, gamma: float, lam: float, adv, ret, moments=None) -> None:
    T, n = rew.shape
    check(_lib.lib(RLIB).surf_gae(ptr(rew), ptr(val), ptr(done), ptr(last_val), T, n, float(gamma), float(lam),
                                  ptr(adv), ptr(ret), ptr(moments), stream_ptr(rew.device)), "surf_gae")


def gae_reference(rew, val, done, last_val, gamma: float, lam: float):
    """Reverse scan (reference: python/train_fast.py:2119-2133)."""
    T = rew.shape[0]
    adv = torch.zeros_like(rew)
    last = torch.zeros_like(last_val)
    for t in range(T - 1, -1, -1):
        nv = last_val if t == T - 1 else val[t + 1]
        nonterm = 1.0 - done[t]
        delta = rew[t] + gamma * nv * nonterm - val[t]
        last = delta + gamma * lam * nonterm * last
        adv[t] = last
    return adv, adv + val


def adv_moments(adv_flat, perm, mb: int, n_mb: int, out) -> None:
    check(_lib.lib(RLIB).surf_adv_moments(ptr(adv_flat), ptr(perm), int(mb), int(n_mb), ptr(out),
                                          stream_ptr(adv_flat.device)), "surf_adv_moments")


# ---- PPO loss ---------------------------------------------------------------------------
def ppo_loss(out: torch.Tensor, value_col: int, act: torch.Tensor, old_logp, adv, ret, idx, moments, heads: HeadArgs,
             log_std, coef, count: float, dout: torch.Tensor, dlog_std: torch.Tensor, stats: torch.Tensor,
             norm_adv: bool = True, n: Optional[int] = None) -> None:
    """Fused PPO loss + gradient. ``out`` [B, >=value_col+1] head output (fp32);
    rollout tensors are indexed through ``idx`` (int64 [B]) when given.
    Writes dout [B, ...] (logit gradients + value gradient column; fp32, or
    bf16 -- the backward GEMMs' operand, rounded as a conversion would),
    adds the log-std gradient into ``dlog_std`` and loss sums into ``stats``
    (6 floats)."""
    B = out.shape[0] if n is None else n
    if dout.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("dout must be float32 or bfloat16")
    check(_lib.lib(RLIB).surf_ppo_loss(
        ptr(out), 0, out.stride(0), ptr(out[:, value_col:]), out.stride(0), ptr(act), act.stride(0), ptr(old_logp),
        ptr(adv), ptr(ret), ptr(idx), ptr(moments), heads.host_ptr(heads.sizes), heads.n_heads,
        heads.host_ptr(heads.slots), heads.cont, ptr(log_std), ptr(coef), float(count), 1 if norm_adv else 0, B,
        ptr(dout), dout.stride(0), ptr(dout[:, value_col:]), dout.stride(0), 1 if dout.dtype == torch.bfloat16 else 0,
        ptr(dlog_std), ptr(stats),
        min(act.shape[0], old_logp.numel(), adv.numel(), ret.numel()), ptr(_error_flag(out.device)),
        stream_ptr(out.device)), "surf_ppo_loss")


def ppo_loss_reference(logits_value, value_col: int, act, old_logp, adv, ret, layout, log_std, clip: float,
                       vf_coef: float, ent_coef: float, norm_adv: bool = True, moments=None):
    """Scalar loss in autograd form (reference mb_step, python/train_fast.py:1846-1864):
    returns (loss, pg, vl, entropy). ``moments`` = (sum, sum of squares, count)
    of the advantages over the whole (multi-rank) minibatch; by default the
    local minibatch's mean and std (ddof=1) normalise them."""
    logits = logits_value[:, :value_col]
    value = logits_value[:, value_col]
    logp, ent = log_prob_reference(logits, act, layout, log_std)
    ratio = torch.exp(logp - old_logp)
    a = adv
    if norm_adv and moments is not None:
        s, ss, n = (float(x) for x in moments)
        mean = s / n
        std = max((ss - s * mean) / max(n - 1.0, 1.0), 0.0) ** 0.5
        a = (a - mean) / (std + 1e-8)
    elif norm_adv:
        a = (a - a.mean()) / (a.std() + 1e-8)
    pg = torch.max(-a * ratio, -a * torch.clamp(ratio, 1 - clip, 1 + clip)).mean()
    vl = 0.5 * (value - ret).pow(2).mean()
    el = -ent.mean()
    return pg + vf_coef * vl + ent_coef * el, pg, vl, -el


# ---- optimizer ------------------------------------------------------------------------------
ADAM_ACC = 2 + 296                 # fp64 slots of surf_adam_norm's accumulator (surf_adam_acc_size)


class Adam:
    """Fused clip + Adam over a PolicyNet's flat buffers (GPU), or torch's Adam
    + clip_grad_norm_ over the same flat tensor (CPU)."""

    def __init__(self, net, lr: float = 3e-4, betas=(0.9, 0.999), eps: float = 1e-5, max_norm: float = 0.5):
        self.net = net
        dev = net.flat.device
        self.m = torch.zeros_like(net.flat)
        self.v = torch.zeros_like(net.flat)
        self.hyper = torch.tensor([lr, betas[0], betas[1], eps, max_norm, 0.0], dtype=torch.float32, device=dev)
        # squared norm, arrival counter and per-block partials of surf_adam_norm
        # (zero once; every launch leaves the counter at zero)
        self.acc = torch.zeros(ADAM_ACC, dtype=torch.float64, device=dev)
        if self.acc.is_cuda and _lib.lib(NLIB).surf_adam_acc_size() != ADAM_ACC:
            raise RuntimeError("libsurf_nn's Adam accumulator size differs from ADAM_ACC: rebuild the extensions")
        self.max_norm = max_norm

    @property
    def steps(self) -> int:
        return int(self.hyper[5].item())

    def set_lr(self, lr: float) -> None:
        self.hyper[0] = lr

    def step(self) -> None:
        net = self.net
        if net.flat.is_cuda:
            L = _lib.lib(NLIB)
            s = stream_ptr(net.flat.device)
            check(L.surf_adam_norm(ptr(net.grad), net.numel, ptr(self.acc), ptr(self.hyper), s), "surf_adam_norm")
            check(L.surf_adam_update(ptr(net.flat), ptr(net.grad), ptr(self.m), ptr(self.v), ptr(net.flat16),
                                     net.numel, ptr(self.acc), ptr(self.hyper), s), "surf_adam_update")
            return
        self.step_reference()

    def step_reference(self) -> None:
        """The same update in plain torch (CPU path and oracle)."""
        net = self.net
        lr, b1, b2, eps, max_norm, t = [float(x) for x in self.hyper.tolist()]
        t += 1
        self.hyper[5] = t
        g = net.grad
        norm = float(torch.sqrt((g.double() ** 2).sum()))
        coef = min(1.0, max_norm / (norm + 1e-6)) if max_norm > 0 else 1.0
        g = g * coef
        self.m.mul_(b1).add_(g, alpha=1 - b1)
        self.v.mul_(b2).addcmul_(g, g, value=1 - b2)
        bc1, bc2 = 1 - b1 ** t, 1 - b2 ** t
        denom = self.v.sqrt() / math.sqrt(bc2) + eps
        net.flat.addcdiv_(self.m, denom, value=-lr / bc1)
        net.grad.zero_()
        net.sync_bf16()

    def state_dict(self) -> dict:
        return {"m": self.m.cpu(), "v": self.v.cpu(), "hyper": self.hyper.cpu()}

    def load_state_dict(self, sd: dict) -> None:
        self.m.copy_(sd["m"].to(self.m.device))
        self.v.copy_(sd["v"].to(self.v.device))
        self.hyper.copy_(sd["hyper"].to(self.hyper.device))
