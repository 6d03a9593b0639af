"""Frame stacking: K depth frames of one env as K channels of one image.

Depth alone cannot show relative motion; with ``frame_stack = K`` the policy
sees the current render plus the renders of the decisions 1, 2, 4 (and 8)
before it, each reach-back clamped to the episode's age so that a freshly
spawned env sees its spawn frame in every slot (reference:
python/train_fast.py:177-293 and the ``--frame-stack`` option, :829-835).

The history is never copied per decision. The trainer's rollout buffer holds
one frame per decision slot (``slot = pro + t``; its first ``pro`` slots carry
the previous rollout's last frames) plus the per-decision age, and one kernel
(``surf_frame_stack``, csrc/kernels/nn_ops.cu) composes the policy input
straight from it in each of the three places it is needed:

* the rollout decision (mode 0), which also advances the per-env age from
  the previous decision's episode-end flags;
* the truncation bootstrap (mode 1), whose terminal frame sits one decision
  past the newest stored one;
* the minibatch gather of the update (mode 2), from the recorded ages.

Layout of a stacked row: pixel-major, frame index outer to the frame's own
channels (``[px][j][c]``) — channel fastest, the NHWC input of the first
convolution. ``stack_reference`` is the torch oracle of all three modes.
"""
from __future__ import annotations

from ctypes import c_int
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import check, ptr, stream_ptr

NLIB = "libsurf_nn.so"
STACK_STRIDES = (1, 2, 4, 8)
MAX_FRAMES = len(STACK_STRIDES) + 1

_V, _I, _L = _lib._V, _lib._I, _lib._L
_lib.register(NLIB, {
    "surf_frame_stack": (_I, [_V, _L, _I, _I, _I, _I, _V, _I, _I, _I, _I, _I, _I, _V, _V, _V, _V, _V, _L, _V, _L,
                              _I, _L, _V, _V]),
})

MODE_ROLLOUT, MODE_TERMINAL, MODE_GATHER = 0, 1, 2


def frame_offsets(k: int) -> tuple:
    """Decision offsets of a K-frame stack, newest first (k <= 1: no stacking)."""
    k = int(k)
    if k <= 1:
        return (0,)
    if k > MAX_FRAMES:
        raise ValueError(f"frame_stack {k}: at most {MAX_FRAMES} frames (strides {STACK_STRIDES})")
    return (0,) + STACK_STRIDES[:k - 1]


def _launch(frames: torch.Tensor, fr: int, C0: int, offs: Sequence[int], pro: int, ring: int, mode: int, N: int,
            lo: int, slot0: int, done, age_cur, age_rec, idx, cur, out: torch.Tensor, rows: int) -> torch.Tensor:
    K = len(offs)
    arr = (c_int * K)(*offs)
    if frames.dtype != torch.bfloat16 or out.dtype != torch.bfloat16:
        raise ValueError("frame stacking works on bf16 frames")
    from .gemm import error_flag
    # gather mode: flat sample indices must address the recorded ages
    bound = age_rec.numel() if (mode == MODE_GATHER and age_rec is not None) else 0
    check(_lib.lib(NLIB).surf_frame_stack(
        ptr(frames), frames.stride(0), frames.stride(1), int(fr), int(C0), K, arr, int(pro), int(ring), int(mode),
        int(N), int(lo), int(slot0), ptr(done), ptr(age_cur), ptr(age_rec), ptr(idx), ptr(cur),
        cur.stride(0) if cur is not None else 0, ptr(out), out.stride(0), int(rows), int(bound),
        ptr(error_flag(out.device)), stream_ptr(out.device)),
        "surf_frame_stack")
    return out


class FrameStacker:
    """Composes stacked policy inputs out of a slot-major frame buffer
    ``frames[S, N, >= fr]`` (bf16) for a K-frame stack of ``C0``-channel frames."""

    def __init__(self, k: int, fr: int, channels: int = 1, ring: int = 0):
        self.offs = frame_offsets(k)
        self.K = len(self.offs)
        self.pro = max(self.offs)
        self.fr = int(fr)
        self.C0 = int(channels)
        self.ring = int(ring)
        if self.fr % 8:
            raise ValueError("frame elements must be a multiple of 8")

    @property
    def width(self) -> int:
        return self.fr * self.K

    def rollout(self, frames, slot: int, lo: int, hi: int, done: Optional[torch.Tensor], age_cur: torch.Tensor,
                age_rec: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Decision at ``slot`` for envs [lo, hi): advance the ages (``done``:
        the previous decision's episode-end flags of these envs, None to keep
        them), record them in ``age_rec`` and compose ``out[hi - lo]``."""
        return _launch(frames, self.fr, self.C0, self.offs, self.pro, self.ring, MODE_ROLLOUT, frames.shape[1], lo,
                       slot, done, age_cur, age_rec, None, None, out, hi - lo)

    def terminal(self, frames, slot: int, env_idx: torch.Tensor, cur: torch.Tensor, age_cur: torch.Tensor,
                 out: torch.Tensor) -> torch.Tensor:
        """Stacks for terminal states one decision past ``slot`` (the newest
        stored decision): ``cur`` holds their renders, ``env_idx`` (int64) their envs."""
        return _launch(frames, self.fr, self.C0, self.offs, self.pro, self.ring, MODE_TERMINAL, frames.shape[1], 0,
                       slot + 1, None, age_cur, None, env_idx, cur, out, env_idx.numel())

    def gather(self, frames, idx: torch.Tensor, ages: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Minibatch rows: flat samples ``idx = t * N + n`` (int64) of a buffer
        whose decision t lives in slot pro + t, ``ages`` flat [T * N] int32."""
        return _launch(frames, self.fr, self.C0, self.offs, self.pro, self.ring, MODE_GATHER, frames.shape[1], 0, 0,
                       None, None, ages, idx, None, out, idx.numel())


def interleave(frames: Sequence[torch.Tensor], channels: int = 1) -> torch.Tensor:
    """K (B, P * C0) frames, newest first -> (B, P * K * C0), pixel-major with
    the frame index outer to the per-frame channels."""
    B = frames[0].shape[0]
    st = torch.stack([f.reshape(B, -1, channels) for f in frames], dim=2)      # B, P, K, C0
    return st.reshape(B, -1)


def stack_reference(frames: torch.Tensor, k: int, rows_env, rows_slot, rows_age, cur: Optional[torch.Tensor] = None,
                    fr: Optional[int] = None, channels: int = 1, ring: int = 0) -> torch.Tensor:
    """Torch oracle: row r stacks env rows_env[r] at slot rows_slot[r] with
    age rows_age[r]; a zero reach-back reads ``cur[r]`` when ``cur`` is given."""
    offs = frame_offsets(k)
    fr = frames.shape[-1] if fr is None else fr
    env = torch.as_tensor(rows_env, dtype=torch.long)
    slot = torch.as_tensor(rows_slot, dtype=torch.long)
    age = torch.as_tensor(rows_age, dtype=torch.long)
    outs = []
    for s in offs:
        back = torch.clamp(age, max=s)
        sl = slot - back
        if ring:
            sl = sl % ring
        f = frames[sl.clamp(min=0), env, :fr].clone()
        if cur is not None:
            zero = back == 0
            f[zero] = cur[zero.nonzero().flatten(), :fr]
        outs.append(f)
    return interleave(outs, channels)
