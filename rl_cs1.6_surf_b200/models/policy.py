"""Policy / value networks.

Two families (reference policy: python/train_fast.py:90-166, a conv trunk with
two tanh MLP towers; the B200 build trains the architectures its benchmark
configurations name):

* vision policy — Nature-CNN trunk over the 64x128 depth image
  (8x8/4 -> 32, 4x4/2 -> 64, 3x3/1 -> 64, ReLU) -> FC 512 (ReLU), concatenated
  with a proprioception MLP (scalars -> 256, tanh) -> shared tanh layer ->
  one linear head producing every action head's logits (plus the continuous
  yaw mean) and the value;
* eyeless policy — scalars -> MLP (2 x 256 tanh) -> the same head layout.

Parameters live in ONE flat fp32 buffer (master weights) with a flat fp32
gradient buffer and a bf16 shadow the tensor-core GEMMs read; every layer's
weight is a view into them. On a CUDA device the forward and backward run on
the hand-written kernels (explicit backward, activations kept in a
preallocated workspace, no autograd); on CPU the same views drive a float32
autograd implementation, which is also the numerics oracle of the GPU path.
Conv weights are stored (out, kh, kw, in) — the GEMM's patch order.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, replace
from typing import Optional

import numpy as np
import torch
import torch.nn.functional as F

# Action heads: (name, categories, action-row slot). The continuous yaw head
# (when enabled) replaces the discrete yaw bin.
DISCRETE_HEADS = {"yaw": (15, 0), "pitch": (7, 1), "fwd": (3, 2), "side": (3, 3), "jump": (2, 4), "duck": (2, 5)}
NEUTRAL = {0: 7, 1: 3, 2: 1, 3: 1, 4: 0, 5: 0}      # slot value when no head drives it


@dataclass
class HeadLayout:
    heads: tuple = ("yaw", "pitch", "fwd", "side", "jump", "duck")
    continuous_yaw: bool = False

    @property
    def sizes(self):
        return [DISCRETE_HEADS[h][0] for h in self.heads]

    @property
    def slots(self):
        return [DISCRETE_HEADS[h][1] for h in self.heads]

    @property
    def n_logits(self) -> int:
        return sum(self.sizes) + (1 if self.continuous_yaw else 0)

    @property
    def value_col(self) -> int:
        return self.n_logits

    @property
    def neutral(self):
        driven = set(self.slots) | ({0} if self.continuous_yaw else set())
        return [-1 if s in driven else NEUTRAL[s] for s in range(6)]

    def to_dict(self) -> dict:
        return {"heads": list(self.heads), "continuous_yaw": self.continuous_yaw}

    @classmethod
    def from_dict(cls, d) -> "HeadLayout":
        return cls(tuple(d["heads"]), bool(d["continuous_yaw"]))


@dataclass
class NetConfig:
    vision: bool = True
    img_h: int = 64
    img_w: int = 128
    img_c: int = 1                  # image channels, fastest (surface mask, stacked frames)
    n_scalar: int = 10              # proprioception features fed to the net
    scalar_pad: int = 16            # columns of the scalar operand (>= n_scalar, multiple of 8)
    conv: tuple = ((8, 4, 32), (4, 2, 64), (3, 1, 64))   # (kernel, stride, out channels)
    fc: int = 512
    proprio: int = 256
    hidden: int = 512               # shared tanh layer
    mlp: tuple = (256, 256)         # eyeless trunk
    heads: HeadLayout = field(default_factory=HeadLayout)
    out_pad: int = 64               # head output columns (logits + value, padded)

    def conv_shapes(self):
        h, w, c = self.img_h, self.img_w, self.img_c
        out = []
        for k, s, co in self.conv:
            oh, ow = (h - k) // s + 1, (w - k) // s + 1
            out.append(dict(H=h, W=w, C=c, k=k, s=s, CO=co, OH=oh, OW=ow))
            h, w, c = oh, ow, co
        return out

    @property
    def flat_conv(self) -> int:
        last = self.conv_shapes()[-1]
        return last["OH"] * last["OW"] * last["CO"]

    def to_dict(self) -> dict:
        d = dict(self.__dict__)
        d["heads"] = self.heads.to_dict()
        d["conv"] = [list(c) for c in self.conv]
        d["mlp"] = list(self.mlp)
        return d

    @classmethod
    def from_dict(cls, d) -> "NetConfig":
        d = dict(d)
        d["heads"] = HeadLayout.from_dict(d["heads"])
        d["conv"] = tuple(tuple(c) for c in d["conv"])
        d["mlp"] = tuple(d["mlp"])
        return cls(**d)


def space_to_depth_config(cfg: NetConfig) -> NetConfig:
    """The same network on the 4x4 space-to-depth image: an H x W x C depth
    image becomes H/4 x W/4 x 16C (pixel (r, c) -> super-pixel (r/4, c/4),
    channel ((r%4)*4 + c%4) * C + ch), and a first layer with kernel 4k' and
    stride 4 becomes kernel k', stride 1 over it — the identical convolution
    (the weight tensor is the same 64 numbers per output channel in
    (kh', kw', r, c) order). The depth camera renders this layout directly, and
    the tensor cores read its 16-channel taps as 32-byte slabs."""
    k, s_, co = cfg.conv[0]
    if cfg.img_h % 4 or cfg.img_w % 4 or k % 4 or s_ != 4:
        raise ValueError("space-to-depth needs H, W multiples of 4 and a first layer of stride 4, kernel 4k")
    return replace(cfg, img_h=cfg.img_h // 4, img_w=cfg.img_w // 4, img_c=cfg.img_c * 16,
                   conv=((k // 4, 1, co),) + tuple(cfg.conv[1:]))


def _param_specs(cfg: NetConfig):
    """(name, shape, fan_in, gain, is_bias) in storage order."""
    specs = []
    out_cols = cfg.heads.n_logits + 1
    if cfg.vision:
        for i, g in enumerate(cfg.conv_shapes()):
            specs.append((f"conv{i + 1}.w", (g["CO"], g["k"] * g["k"] * g["C"]), g["k"] * g["k"] * g["C"], math.sqrt(2), False))
            specs.append((f"conv{i + 1}.b", (g["CO"],), 0, 0.0, True))
        specs.append(("fc.w", (cfg.fc, cfg.flat_conv), cfg.flat_conv, math.sqrt(2), False))
        specs.append(("fc.b", (cfg.fc,), 0, 0.0, True))
        specs.append(("proprio.w", (cfg.proprio, cfg.scalar_pad), cfg.n_scalar, math.sqrt(2), False))
        specs.append(("proprio.b", (cfg.proprio,), 0, 0.0, True))
        specs.append(("hidden.w", (cfg.hidden, cfg.fc + cfg.proprio), cfg.fc + cfg.proprio, math.sqrt(2), False))
        specs.append(("hidden.b", (cfg.hidden,), 0, 0.0, True))
        last = cfg.hidden
    else:
        prev, prev_pad = cfg.n_scalar, cfg.scalar_pad
        for i, h in enumerate(cfg.mlp):
            specs.append((f"mlp{i + 1}.w", (h, prev_pad), prev, math.sqrt(2), False))
            specs.append((f"mlp{i + 1}.b", (h,), 0, 0.0, True))
            prev = prev_pad = h
        last = prev
    specs.append(("head.w", (cfg.out_pad, last), last, 0.01, False))
    specs.append(("head.b", (cfg.out_pad,), 0, 0.0, True))
    specs.append(("log_std", (1,), 0, 0.0, True))
    del out_cols
    return specs


class PolicyNet:
    """Flat-parameter policy; see the module docstring."""

    def __init__(self, cfg: NetConfig, device="cpu", seed: int = 0):
        self.cfg = cfg
        self.device = torch.device(device)
        self.specs = _param_specs(cfg)
        self.offsets = {}
        off = 0
        # storage: every weight matrix first, then the biases and log_std
        # (the parameters read in fp32 by the kernels) as one tail region
        # starting at fp32_from; data-parallel ranks keep full fp32 replicas
        # of the tail only and bf16 replicas of everything
        order = [s for s in self.specs if not s[4]] + [s for s in self.specs if s[4]]
        self.fp32_from = 0
        for name, shape, _, _, is_bias in order:
            if is_bias and not self.fp32_from:
                self.fp32_from = off
            self.offsets[name] = (off, shape)
            off += (int(np.prod(shape)) + 63) // 64 * 64       # 256-byte aligned views
        self.numel = off
        self.flat = torch.zeros(off, dtype=torch.float32, device=self.device)
        self.grad = torch.zeros(off, dtype=torch.float32, device=self.device)
        self.flat16 = torch.zeros(off, dtype=torch.bfloat16, device=self.device) if self.device.type == "cuda" else None
        self.implicit_conv = True           # implicit-GEMM convolutions where supported (else im2col + GEMM)
        # the flagship trunk's stacked shifted-grid kernels (ops/conv_shift.py)
        # where the geometry is theirs; else the 4-D implicit GEMMs above
        self.shift_conv = True
        self._trunk = None
        self.init_weights(seed)

    # ---- parameter views ------------------------------------------------------------
    def view(self, name: str, buf: Optional[torch.Tensor] = None) -> torch.Tensor:
        off, shape = self.offsets[name]
        b = self.flat if buf is None else buf
        return b[off:off + int(np.prod(shape))].view(*shape)

    def p(self, name):
        return self.view(name)

    def g(self, name):
        return self.view(name, self.grad)

    def w16(self, name):
        return self.view(name, self.flat16)

    @property
    def n_params(self) -> int:
        return sum(int(np.prod(s)) for _, s, *_ in self.specs)

    def init_weights(self, seed: int) -> None:
        """Orthogonal weights (gain sqrt 2 on hidden layers, 0.01 on the policy
        head, 1 on the value row), zero biases — the reference init scheme
        (python/train_fast.py:130-137)."""
        gen = torch.Generator().manual_seed(seed)
        cfg = self.cfg
        for name, shape, fan_in, gain, is_bias in self.specs:
            v = self.p(name)
            if is_bias:
                v.zero_()
                continue
            rows, cols = shape
            used = fan_in if name.startswith(("proprio", "mlp1")) else cols
            w = torch.empty(rows, used)
            torch.nn.init.orthogonal_(w, gain=gain, generator=gen)
            full = torch.zeros(rows, cols)
            full[:, :used] = w
            if name == "head.w":
                full[cfg.heads.n_logits + 1:] = 0.0             # padding rows stay zero
                vw = torch.empty(1, used)
                torch.nn.init.orthogonal_(vw, gain=1.0, generator=gen)
                full[cfg.heads.value_col] = vw[0]
            v.copy_(full.to(self.device))
        self.p("log_std").fill_(0.0)
        self.sync_bf16()

    def overlap_range(self):
        """[lo, hi) of the flat gradient that is final when ``backward_gpu``
        calls its ``on_towers`` hook (the tower, FC and head weight matrices,
        stored contiguously after the convolution weights), or None."""
        if not self.cfg.vision:
            return None
        lo = self.offsets["fc.w"][0]
        names = [n for n, _, _, _, b in self.specs if not b and not n.startswith("conv")]
        if any(self.offsets[n][0] < lo for n in names) or any(
                self.offsets[n][0] >= lo for n, *_ in self.specs if n.startswith("conv") and n.endswith(".w")):
            return None
        return lo, self.fp32_from

    def uses_shift_trunk(self) -> bool:
        from ..ops.conv_shift import Trunk
        return self.device.type == "cuda" and self.shift_conv and Trunk.supported(self.cfg)

    @property
    def trunk(self):
        """the stacked shifted-grid trunk over this network's bf16 weights (built on first use)"""
        if self._trunk is None:
            from ..ops.conv_shift import Trunk
            self._trunk = Trunk(self.device, [self.offsets[f"conv{i}.w"][0] for i in (1, 2, 3)])
        return self._trunk

    def sync_bf16(self) -> None:
        if self.flat16 is not None:
            self.flat16.copy_(self.flat)

    def state_dict(self) -> dict:
        return {"flat": self.flat.detach().cpu().clone(), "config": self.cfg.to_dict()}

    def load_state_dict(self, sd: dict) -> None:
        if sd["flat"].numel() != self.numel:
            raise ValueError("checkpoint parameter layout does not match this network")
        self.flat.copy_(sd["flat"].to(self.device))
        self.sync_bf16()

    # ---- float32 autograd path (CPU training and the GPU path's oracle) ---------------
    def forward_reference(self, scal: torch.Tensor, img: Optional[torch.Tensor], params: Optional[dict] = None):
        """scal [B, scalar_pad] (padding columns zero), img [B, H*W*C] NHWC ->
        head output [B, out_pad] fp32 (logits, value at value_col)."""
        cfg = self.cfg
        P = params if params is not None else {n: self.p(n) for n, *_ in self.specs}
        if cfg.vision:
            B = scal.shape[0]
            x = img[:, :cfg.img_h * cfg.img_w * cfg.img_c].float().reshape(B, cfg.img_h, cfg.img_w, cfg.img_c)
            x = x.permute(0, 3, 1, 2)
            for i, g in enumerate(cfg.conv_shapes()):
                w = P[f"conv{i + 1}.w"].reshape(g["CO"], g["k"], g["k"], g["C"]).permute(0, 3, 1, 2)
                x = F.relu(F.conv2d(x, w, P[f"conv{i + 1}.b"], stride=g["s"]))
            f = x.permute(0, 2, 3, 1).reshape(B, -1)             # (h, w, c) flattening
            f = F.relu(f @ P["fc.w"].t() + P["fc.b"])
            pr = torch.tanh(scal.float() @ P["proprio.w"].t() + P["proprio.b"])
            h = torch.tanh(torch.cat([f, pr], 1) @ P["hidden.w"].t() + P["hidden.b"])
        else:
            h = scal.float()
            for i in range(len(cfg.mlp)):
                h = torch.tanh(h @ P[f"mlp{i + 1}.w"].t() + P[f"mlp{i + 1}.b"])
        return h @ P["head.w"].t() + P["head.b"]

    def autograd_params(self) -> dict:
        """Leaf tensors sharing storage with the flat buffer; their .grad are
        copied into the flat gradient buffer by ``collect_grads``."""
        out = {}
        for name, *_ in self.specs:
            t = self.p(name).detach().requires_grad_(True)
            out[name] = t
        return out

    def collect_grads(self, params: dict) -> None:
        for name, t in params.items():
            if t.grad is not None:
                self.g(name).add_(t.grad)


# ---- tensor-core path -----------------------------------------------------------------
class Workspace:
    """Activations and gradients of one batch size, allocated once (so CUDA
    graphs capture stable addresses)."""

    def __init__(self, net: "PolicyNet", batch: int):
        cfg, dev, bf = net.cfg, net.device, torch.bfloat16
        self.B = batch
        self.col, self.y, self.dcol, self.dy, self.wt = [], [], [], [], []
        self.implicit = [False] * len(cfg.conv)
        self.img = None                         # conv1 input of the last forward (implicit weight gradient)
        self.shift = cfg.vision and net.uses_shift_trunk()
        if self.shift:
            # padded-grid layouts of the shifted trunk (ops/conv_shift.py): the
            # grids' padding rows are zeros that the kernels never write (dy3)
            # or write as zeros (y2, dy2)
            self.sy1 = torch.empty(batch * 512, 32, dtype=bf, device=dev)
            self.sy2 = torch.zeros(batch * 128, 64, dtype=bf, device=dev)
            self.y3 = torch.empty(batch * 48, 64, dtype=bf, device=dev)
            self.dy3 = torch.zeros(batch * 128, 64, dtype=bf, device=dev)
            self.dy2 = torch.zeros(batch * 128, 64, dtype=bf, device=dev)
            self.dy1 = torch.empty(batch * 512, 32, dtype=bf, device=dev)
            self.h0 = torch.empty(batch, cfg.fc + cfg.proprio, dtype=bf, device=dev)
            self.dh0 = torch.empty_like(self.h0)
            self.h = [torch.empty(batch, cfg.hidden, dtype=bf, device=dev)]
        elif cfg.vision:
            from ..ops.conv import SLACK_BYTES, ConvShape
            shapes = cfg.conv_shapes()
            for i, g in enumerate(shapes):
                rows = batch * g["OH"] * g["OW"]
                sh = ConvShape(batch, g["H"], g["W"], g["C"], g["k"], g["s"], g["CO"])
                # implicit GEMM (no patch matrix) wherever the kernel has an
                # operand mode for the input: >= 32 channels, or the 16-channel
                # space-to-depth depth image of the first layer (forward and
                # weight gradient only: the image needs no gradient)
                if i == 0:
                    imp = net.implicit_conv and sh.supported() and (sh.slabs or sh.C == 64) and sh.CO <= 64
                else:
                    imp = net.implicit_conv and sh.supported() and sh.CO == 64 and sh.k % sh.s == 0
                self.implicit[i] = imp
                patch = g["k"] * g["k"] * g["C"]
                self.col.append(None if imp else torch.empty(rows, patch, dtype=bf, device=dev))
                self.dcol.append(None if (imp or i == 0) else torch.empty(rows, patch, dtype=bf, device=dev))
                # activations carry slack after the last row: the implicit
                # convolution reading them may fetch a little past the end
                yb = torch.empty(rows * g["CO"] + SLACK_BYTES // 2, dtype=bf, device=dev)
                self.y.append(yb[:rows * g["CO"]].view(rows, g["CO"]))
                self.dy.append(torch.empty(rows, g["CO"], dtype=bf, device=dev))
                s_ = g["s"]
                self.wt.append(torch.empty(s_ * s_, g["C"], (g["k"] // s_) ** 2 * g["CO"], dtype=bf, device=dev)
                               if imp else None)
            self.h0 = torch.empty(batch, cfg.fc + cfg.proprio, dtype=bf, device=dev)
            self.dh0 = torch.empty_like(self.h0)
            self.h = [torch.empty(batch, cfg.hidden, dtype=bf, device=dev)]
        else:
            self.h = [torch.empty(batch, w, dtype=bf, device=dev) for w in cfg.mlp]
        self.dh = [torch.empty_like(t) for t in self.h]
        self.out = torch.empty(batch, cfg.out_pad, dtype=torch.float32, device=dev)
        self.dout16 = torch.zeros(batch, cfg.out_pad, dtype=bf, device=dev)


def _splits(M: int, N: int, K: int, bn: int, target: int = 296, min_kb: int = 16) -> int:
    """K splits of a weight gradient: enough units for two per SM, but at
    least min_kb 64-deep k-blocks per split -- a narrow gradient (a few
    tiles) split 148 ways spent its time in 148-way contended fp32 atomics
    (head at 32768 rows: 0.062 ms at 1 k-block per split, 0.037 at 8, 0.031
    at 16, 0.036 at 32)."""
    tiles = ((M + 127) // 128) * ((N + bn - 1) // bn)
    kb = (K + 63) // 64
    return max(1, min(kb // max(min_kb, 1), target // max(tiles, 1)))


def _wgrad(G, dy, x, gw, rows):
    """gw += dy^T x over `rows` batch rows (both operands MN-major)."""
    M, N = dy.shape[1], x.shape[1]
    bn = 64 if N <= 64 else (128 if N <= 128 else 256)
    G.gemm(dy, x, a_mn=True, b_mn=True, out=gw, accumulate=True, splits=_splits(M, N, rows, bn), bn=bn, K=rows)


def forward_gpu(net: "PolicyNet", ws: Workspace, scal16: torch.Tensor, img16: Optional[torch.Tensor],
                B: Optional[int] = None) -> torch.Tensor:
    """Head output [B, out_pad] fp32 into ws.out (bf16 operands, fp32 accumulate).
    scal16: [B, scalar_pad] bf16; img16: [B, H*W*C] bf16 NHWC (vision)."""
    from ..ops import gemm as G
    cfg = net.cfg
    B = ws.B if B is None else B
    w = net.w16
    if cfg.vision and ws.shift:
        T = net.trunk
        T.refresh(net.flat16)                   # stacked weight operands of the current parameters
        img = img16[:B].reshape(B * 512, 16)
        ws.img = img
        T.conv1_forward(img, net.p("conv1.b"), ws.sy1, B)
        T.conv2_forward(ws.sy1, net.p("conv2.b"), ws.sy2, B)
        T.conv3_forward(ws.sy2, net.p("conv3.b"), ws.y3, B)
        feat = ws.y3[:B * 48].view(B, cfg.flat_conv)
        G.gemm(feat, w("fc.w"), out=ws.h0[:B, :cfg.fc], bias=net.p("fc.b"), act="relu")
        G.gemm(scal16[:B], w("proprio.w"), out=ws.h0[:B, cfg.fc:], bias=net.p("proprio.b"), act="tanh")
        G.gemm(ws.h0[:B], w("hidden.w"), out=ws.h[0][:B], bias=net.p("hidden.b"), act="tanh")
    elif cfg.vision:
        from ..ops import conv as CV
        x = img16
        for i, g in enumerate(cfg.conv_shapes()):
            rows = B * g["OH"] * g["OW"]
            if ws.implicit[i]:
                sh = CV.ConvShape(B, g["H"], g["W"], g["C"], g["k"], g["s"], g["CO"])
                if i == 0:
                    ws.img = x                  # the weight gradient reads the image again
                CV.conv_forward(x, sh, w(f"conv{i + 1}.w"), net.p(f"conv{i + 1}.b"), ws.y[i][:rows])
            else:
                col = G.im2col(x, B, g["H"], g["W"], g["C"], g["k"], g["s"], out=ws.col[i][:rows])
                G.gemm(col, w(f"conv{i + 1}.w"), out=ws.y[i][:rows], bias=net.p(f"conv{i + 1}.b"), act="relu")
            x = ws.y[i][:rows]
        feat = ws.y[-1][:B * cfg.conv_shapes()[-1]["OH"] * cfg.conv_shapes()[-1]["OW"]].view(B, cfg.flat_conv)
        G.gemm(feat, w("fc.w"), out=ws.h0[:B, :cfg.fc], bias=net.p("fc.b"), act="relu")
        G.gemm(scal16[:B], w("proprio.w"), out=ws.h0[:B, cfg.fc:], bias=net.p("proprio.b"), act="tanh")
        G.gemm(ws.h0[:B], w("hidden.w"), out=ws.h[0][:B], bias=net.p("hidden.b"), act="tanh")
    else:
        x = scal16[:B]
        for i in range(len(cfg.mlp)):
            G.gemm(x, w(f"mlp{i + 1}.w"), out=ws.h[i][:B], bias=net.p(f"mlp{i + 1}.b"), act="tanh")
            x = ws.h[i][:B]
    G.gemm(ws.h[-1][:B], w("head.w"), out=ws.out[:B], bias=net.p("head.b"))
    return ws.out[:B]


def backward_gpu(net: "PolicyNet", ws: Workspace, scal16: torch.Tensor, B: Optional[int] = None,
                 on_towers=None) -> None:
    """Accumulate parameter gradients into net.grad from ws.dout16 (the
    gradient of the loss w.r.t. the head output, bf16). ``on_towers`` is
    called once the gradients of ``net.overlap_range()`` are final in stream
    order (before the convolutions' backward) -- the data-parallel step
    reduces that range on a side stream meanwhile."""
    from ..ops import gemm as G
    cfg = net.cfg
    B = ws.B if B is None else B
    w = net.w16
    dout = ws.dout16[:B]
    h_last = ws.h[-1][:B]
    _wgrad(G, dout, h_last, net.g("head.w"), B)
    G.colsum(dout, net.g("head.b"))
    G.gemm(dout, w("head.w"), b_mn=True, out=ws.dh[-1][:B], act="tanh_grad", aux=h_last)
    if cfg.vision:
        dh = ws.dh[0][:B]
        _wgrad(G, dh, ws.h0[:B], net.g("hidden.w"), B)
        G.colsum(dh, net.g("hidden.b"))
        G.gemm(dh, w("hidden.w"), b_mn=True, out=ws.dh0[:B], act="relu_grad", act2="tanh_grad", act_split=cfg.fc,
               aux=ws.h0[:B])
        dp = ws.dh0[:B, cfg.fc:]
        _wgrad(G, dp, scal16[:B], net.g("proprio.w"), B)
        G.colsum(dp, net.g("proprio.b"))
        df = ws.dh0[:B, :cfg.fc]
        if ws.shift:
            T = net.trunk
            feat = ws.y3[:B * 48].view(B, cfg.flat_conv)
            _wgrad(G, df, feat, net.g("fc.w"), B)
            G.colsum(df, net.g("fc.b"))
            if on_towers is not None:
                on_towers()
            # conv3's output gradient lands on its 8 x 16 input grid (row h*12 + w of the
            # dense feature -> h*16 + w), the padding staying zero
            dy3 = ws.dy3[:B * 128]
            G.gemm(df, w("fc.w"), b_mn=True, out=dy3.view(B, 8192), act="relu_grad", aux=feat, cmap=(768, 1024))
            # weight and bias gradients in one kernel per layer
            T.conv3_weight_grad(dy3, ws.sy2, net.g("conv3.w"), B, net.g("conv3.b"))
            T.conv3_input_grad(dy3, ws.sy2, ws.dy2, B)
            T.conv2_weight_grad(ws.dy2, ws.sy1, net.g("conv2.w"), B, net.g("conv2.b"))
            T.conv2_input_grad(ws.dy2, ws.sy1, ws.dy1, B)
            T.conv1_weight_grad(ws.dy1, ws.img, net.g("conv1.w"), B, net.g("conv1.b"))
            return
        shapes = cfg.conv_shapes()
        last_rows = B * shapes[-1]["OH"] * shapes[-1]["OW"]
        feat = ws.y[-1][:last_rows].view(B, cfg.flat_conv)
        _wgrad(G, df, feat, net.g("fc.w"), B)
        G.colsum(df, net.g("fc.b"))
        if on_towers is not None:
            on_towers()
        dfeat = ws.dy[-1][:last_rows].view(B, cfg.flat_conv)
        G.gemm(df, w("fc.w"), b_mn=True, out=dfeat, act="relu_grad", aux=feat)
        from ..ops import conv as CV
        for i in range(len(shapes) - 1, -1, -1):
            g = shapes[i]
            rows = B * g["OH"] * g["OW"]
            dy = ws.dy[i][:rows]
            prev_rows = B * g["H"] * g["W"]
            if ws.implicit[i]:
                sh = CV.ConvShape(B, g["H"], g["W"], g["C"], g["k"], g["s"], g["CO"])
                CV.conv_weight_grad(dy, ws.y[i - 1] if i > 0 else ws.img, sh, net.g(f"conv{i + 1}.w"))
            else:
                _wgrad(G, dy, ws.col[i][:rows], net.g(f"conv{i + 1}.w"), rows)
            G.colsum(dy, net.g(f"conv{i + 1}.b"))
            if i == 0:
                break
            if ws.implicit[i]:
                CV.weight_classes(w(f"conv{i + 1}.w"), sh, out=ws.wt[i])
                CV.conv_input_grad(dy, sh, ws.wt[i], ws.dy[i - 1][:prev_rows], ws.y[i - 1][:prev_rows])
            else:
                G.gemm(dy, w(f"conv{i + 1}.w"), b_mn=True, out=ws.dcol[i][:rows])
                G.col2im(ws.dcol[i][:rows], ws.y[i - 1][:prev_rows], B, g["H"], g["W"], g["C"], g["k"], g["s"],
                         out=ws.dy[i - 1][:prev_rows].view(B, g["H"], g["W"], g["C"]))
    else:
        for i in range(len(cfg.mlp) - 1, -1, -1):
            dh = ws.dh[i][:B]
            x = ws.h[i - 1][:B] if i > 0 else scal16[:B]
            _wgrad(G, dh, x, net.g(f"mlp{i + 1}.w"), B)
            G.colsum(dh, net.g(f"mlp{i + 1}.b"))
            if i > 0:
                G.gemm(dh, w(f"mlp{i + 1}.w"), b_mn=True, out=ws.dh[i - 1][:B], act="tanh_grad", aux=ws.h[i - 1][:B])
