"""Implicit-GEMM convolutions on the tcgen05 kernel (csrc/kernels/gemm_tc.cu).

No patch matrix is materialised: the GEMM's TMA producer reads the NHWC
activation through a 4-D tensor map (C, W, H, B) whose element strides are
the convolution stride, one box per (output tile, tap), and the epilogue
writes rows that are convolution-grid positions. Three products per layer:

* forward  Y = conv(X, W):   A = X (mode 1: rows = output positions,
  k-blocks = taps), B = W [CO, k*k*C] (K-major), out = Y with bias + ReLU;
* weight gradient dW += dY^T patches(X): A = dY, B = X (both mode 2:
  k-blocks = tiles of 64 output positions, n sub-blocks = taps), fp32 atomics;
* input gradient dX = conv^T(dY, W) * ReLU'(X): A = dY read at output
  coordinates (input position - tap); out-of-range coordinates load zeros,
  so the transposed convolution's halo costs nothing. Stride 2 splits into
  the four parity classes (py, px) of the input grid, each a stride-1
  convolution of dY with the sub-kernel W[:, py::2, px::2, :], stored to
  every other input position. B is that sub-kernel rearranged
  [C, taps x CO] by ``surf_conv_weight_t``.

A 64-byte-channel input (C = 32) with stride 2 along W is read as
"super-pixels" of two neighbouring positions (128 bytes), which turns the
stride along W into 1 and pairs the taps (kw, kw + 1); its buffer needs 64
bytes of slack after the last row (the unused 16th super-pixel of the last
row is fetched). A 16-channel input (the depth image in 4x4 space-to-depth
order) is read as windows of two neighbouring positions: the tensor map's W
stride is one position (32 bytes) and its inner extent two (64 bytes), so a
box row holds the taps (kw, kw + 1) -- half the box rows of one 32-byte tap
per row. Supported: C = 64 (any stride), C = 32 with stride 2 and even
kernel, C = 16 with even kernel; output-gradient channels (the dgrad A
operand) = 64.
Reference layer: the conv trunk of python/train_fast.py:115-121 (cuDNN there).
"""
from __future__ import annotations

import ctypes
from ctypes import c_int, c_int64, c_void_p
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from ._lib import check, ptr, stream_ptr
from .gemm import ACT, NLIB, Epilogue, error_flag


class MapDesc(ctypes.Structure):
    _fields_ = [("base", c_void_p), ("dims", c_int64 * 4), ("strides", c_int64 * 3), ("box", c_int * 4),
                ("estr", c_int * 4)]


class Geo(ctypes.Structure):
    _fields_ = [("mode", c_int), ("tw", c_int), ("th", c_int), ("tb", c_int), ("tiles_w", c_int),
                ("tiles_h", c_int), ("sw", c_int), ("sh", c_int), ("kw_n", c_int), ("sign", c_int),
                ("per_tap", c_int)]


class OutGeo(ctypes.Structure):
    _fields_ = [("on", c_int), ("gw", c_int), ("gh", c_int), ("gb", c_int), ("out_w", c_int), ("out_h", c_int),
                ("ys", c_int), ("xs", c_int), ("yo", c_int), ("xo", c_int), ("cls_cols", c_int)]


class ConvCfg(ctypes.Structure):
    _fields_ = [("a", Geo), ("b", Geo), ("o", OutGeo)]


_P = ctypes.POINTER
_lib.register(NLIB, {
    "surf_gemm_conv": (c_int, [c_void_p, c_int64, _P(MapDesc), c_int, c_void_p, c_int64, _P(MapDesc), c_int, c_int,
                               c_int, c_int, _P(Epilogue), _P(ConvCfg), c_int, c_int, c_void_p]),
    "surf_gemm_conv_sizes": (c_int, [_P(c_int)]),
    "surf_conv_weight_t": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
})

SLACK_BYTES = 128          # allocate activations with this much room after the last element
# Kernel diagnostics for timing studies only (Epilogue.dbg): bit 0 skips the
# epilogue's stores, bit 1 skips the MMAs (results are wrong with either);
# bit 2 streams a resident-able weight operand per k-block, bit 3 turns off the
# saved-activation prefetch of the derivative epilogues (results unchanged);
# shifted-grid kernels only: bit 4 reads every forward K step's A operand at
# the stage start, bit 5 skips the whole epilogue.
DEBUG = 0
TRACE = None               # a uint64 CUDA tensor of 5 * 256 stamps: CTA 0's pipeline timeline (diagnostics)
# 16-channel inputs: two-position windows (kernel mode 4) when True, one
# 32-byte tap per box row (mode 3) when False (A/B timing).
PAIR_WINDOWS = True


def _cdiv(a, b):
    return -(-a // b)


_SMS = {}


def _sm_count(dev) -> int:
    i = dev.index if dev.index is not None else torch.cuda.current_device()
    if i not in _SMS:
        _SMS[i] = torch.cuda.get_device_properties(i).multi_processor_count
    return _SMS[i]


def _pow2_at_least(n: int) -> int:
    p = 1
    while p < n:
        p *= 2
    return p


@dataclass(frozen=True)
class ConvShape:
    B: int
    H: int
    W: int
    C: int
    k: int
    s: int
    CO: int

    @property
    def OH(self):
        return (self.H - self.k) // self.s + 1

    @property
    def OW(self):
        return (self.W - self.k) // self.s + 1

    @property
    def superpixel(self) -> int:
        return 64 // self.C if self.C in (32, 64) else 1

    @property
    def slabs(self) -> bool:
        """16-channel input: taps load as 32-byte-swizzled slabs (kernel mode 3)
        or as two-position windows (mode 4)."""
        return self.C == 16

    @property
    def pairs(self) -> bool:
        """16-channel input read as 64-byte windows of taps (kw, kw + 1)."""
        return self.C == 16 and PAIR_WINDOWS

    def supported(self) -> bool:
        if self.C == 64:
            return True
        if self.C == 16:                  # 4 taps per 64-wide k-block
            return self.k % 2 == 0
        return self.C == 32 and self.s == 2 and self.k % 2 == 0


def _tile(gw: int, gh: int, rows: int):
    """(tw, th, tb) with tw * th * tb = rows covering a gw x gh grid with the least padding."""
    tw = min(_pow2_at_least(gw), rows)
    best = None
    th = 1
    while tw * th <= rows:
        waste = _cdiv(gh, th) * th / gh
        if best is None or waste < best[0] - 1e-9:
            best = (waste, th)
        th *= 2
    th = best[1]
    return tw, th, rows // (tw * th)


def _input_map(x: torch.Tensor, sh: ConvShape, tw: int, th: int, tb: int) -> MapDesc:
    """Map over the layer input (possibly as super-pixels) for a box of tw x th x tb output positions."""
    d = MapDesc()
    d.base = ptr(x)
    p = sh.superpixel
    if sh.pairs:
        # overlapping rows: W stride 32 bytes, inner extent 64 bytes; the last
        # position of a row has no right neighbour and is left out of the map
        d.dims[:] = [32, sh.W - 1, sh.H, sh.B]
        d.strides[:] = [sh.C * 2, sh.W * sh.C * 2, sh.H * sh.W * sh.C * 2]
        d.box[:] = [32, tw * sh.s, th * sh.s, tb]
        d.estr[:] = [1, sh.s, sh.s, 1]
    elif p == 2:
        d.dims[:] = [64, _cdiv(sh.W, 2), sh.H, sh.B]
        d.strides[:] = [128, sh.W * sh.C * 2, sh.H * sh.W * sh.C * 2]
        d.box[:] = [64, tw, th * sh.s, tb]
        d.estr[:] = [1, 1, sh.s, 1]
    else:
        d.dims[:] = [sh.C, sh.W, sh.H, sh.B]
        d.strides[:] = [sh.C * 2, sh.W * sh.C * 2, sh.H * sh.W * sh.C * 2]
        d.box[:] = [min(64, sh.C), tw * sh.s, th * sh.s, tb]     # 16 channels: one 32-byte slab row
        d.estr[:] = [1, sh.s, sh.s, 1]
    return d


def _grid_map(t: torch.Tensor, C: int, W: int, H: int, B: int, tw: int, th: int, tb: int) -> MapDesc:
    d = MapDesc()
    d.base = ptr(t)
    d.dims[:] = [C, W, H, B]
    d.strides[:] = [C * 2, W * C * 2, H * W * C * 2]
    d.box[:] = [64, tw, th, tb]
    d.estr[:] = [1, 1, 1, 1]
    return d


def _epilogue(out, accumulate=False, bias=None, act="none", aux=None, ld=None) -> Epilogue:
    ep = Epilogue()
    ep.c = ptr(out)
    ep.ldc = ld if ld is not None else out.shape[-1]
    ep.c_dtype = 1 if out.dtype == torch.bfloat16 else 0
    ep.c_mode = 1 if accumulate else 0
    ep.bias = ptr(bias)
    ep.act = ep.act2 = ACT[act]
    ep.act_split = 1 << 30
    if aux is not None:
        ep.aux = ptr(aux)
        ep.ld_aux = ld if ld is not None else aux.shape[-1]
    ep.err = ptr(error_flag(out.device))
    ep.dbg = int(DEBUG)
    ep.trace = ptr(TRACE)
    return ep


def _run(A, ad, a_mn, B, bd, b_mn, M, N, K, ep, cc, bn, splits=1, lda=0, ldb=0, dev=None):
    check(_lib.lib(NLIB).surf_gemm_conv(ptr(A), int(lda), ctypes.byref(ad) if ad is not None else None, int(a_mn),
                                        ptr(B), int(ldb), ctypes.byref(bd) if bd is not None else None, int(b_mn),
                                        int(M), int(N), int(K), ctypes.byref(ep), ctypes.byref(cc), int(bn),
                                        int(splits), stream_ptr(dev)), "surf_gemm_conv")


def conv_forward(x: torch.Tensor, sh: ConvShape, w16: torch.Tensor, bias: torch.Tensor, out: torch.Tensor,
                 act: str = "relu") -> torch.Tensor:
    """out [B*OH*OW, CO] (dense NHWC) = act(conv(x, W) + bias)."""
    if not sh.supported():
        raise ValueError(f"implicit convolution does not support {sh}")
    p = sh.superpixel
    tw, th, tb = _tile(sh.OW, sh.OH, 128)
    cc = ConvCfg()
    cc.a.mode, cc.a.tw, cc.a.th, cc.a.tb = (4 if sh.pairs else 3 if sh.slabs else 1), tw, th, tb
    cc.a.tiles_w, cc.a.tiles_h = _cdiv(sh.OW, tw), _cdiv(sh.OH, th)
    cc.a.sw, cc.a.sh = (1 if p == 2 else sh.s), sh.s
    cc.a.kw_n = sh.k // 2 if sh.pairs else sh.k // p
    cc.a.sign, cc.a.per_tap = 1, 1
    cc.o.on, cc.o.gw, cc.o.gh, cc.o.gb = 1, sh.OW, sh.OH, sh.B
    cc.o.out_w, cc.o.out_h, cc.o.ys, cc.o.xs = sh.OW, sh.OH, 1, 1
    ntiles = cc.a.tiles_w * cc.a.tiles_h * _cdiv(sh.B, tb)
    ad = _input_map(x, sh, tw, th, tb)
    ep = _epilogue(out, bias=bias, act=act, ld=sh.CO)
    K = sh.k * sh.k * sh.C
    bn = 32 if sh.CO <= 32 else (64 if sh.CO <= 64 else 128)
    _run(x, ad, 0, w16, None, 0, ntiles * 128, sh.CO, K, ep, cc, bn=bn, ldb=w16.stride(0), dev=x.device)
    return out


def conv_weight_grad(dy: torch.Tensor, x: torch.Tensor, sh: ConvShape, gw: torch.Tensor, splits: int = 0) -> None:
    """gw [CO, k*k*C] (fp32) += dY^T patches(X) over every output position."""
    if not sh.supported() or sh.CO > 128:
        raise ValueError(f"implicit weight gradient does not support {sh}")
    p = sh.superpixel
    tw, th, tb = _tile(sh.OW, sh.OH, 64)
    cc = ConvCfg()
    for g in (cc.a, cc.b):
        g.mode, g.tw, g.th, g.tb = 2, tw, th, tb
        g.tiles_w, g.tiles_h = _cdiv(sh.OW, tw), _cdiv(sh.OH, th)
    if sh.slabs:
        cc.b.mode = 4 if sh.pairs else 3
    cc.b.sw, cc.b.sh = (1 if p == 2 else sh.s), sh.s
    cc.b.kw_n = sh.k // 2 if sh.pairs else sh.k // p
    ktiles = cc.a.tiles_w * cc.a.tiles_h * _cdiv(sh.B, tb)
    ad = _grid_map(dy, sh.CO, sh.OW, sh.OH, sh.B, tw, th, tb)
    bd = _input_map(x, sh, tw, th, tb)
    N = sh.k * sh.k * sh.C
    bn = 64 if sh.slabs else (256 if N >= 256 else (128 if N >= 128 else 64))
    if not splits:
        # one (n tile, K split) per SM: a second tile per CTA would add a
        # second round of fp32 atomics into gw without adding parallelism
        tiles = _cdiv(N, bn)
        splits = max(1, min(ktiles, _sm_count(dy.device) // max(tiles, 1)))
    ep = _epilogue(gw, accumulate=True, ld=gw.stride(0))
    _run(dy, ad, 1, x, bd, 1, sh.CO, N, ktiles * 64, ep, cc, bn=bn, splits=splits, dev=dy.device)


def conv_input_grad(dy: torch.Tensor, sh: ConvShape, wt: torch.Tensor, dx: torch.Tensor,
                    x_act: Optional[torch.Tensor] = None) -> torch.Tensor:
    """dx [B*H*W, C] = conv^T(dY, W) (times ReLU'(x_act) when given).
    ``wt``: the rearranged weights of ``weight_classes`` ([s*s, C, taps*CO]).
    All s*s parity classes run as ONE GEMM: rows are positions (j, i) of the
    class grid, the A operand dY[j - a, i - b] is shared by every class, and
    the N = s*s*C columns are the classes' channels (class-major), each
    class block stored to its own input positions (2j + py, 2i + px)."""
    if sh.CO != 64 or (sh.s > 1 and sh.k % sh.s) or sh.C % 32:
        raise ValueError(f"implicit input gradient does not support {sh}")
    s = sh.s
    kt = sh.k // s                                   # taps per dimension of a parity class
    gh, gw_ = _cdiv(sh.H, s), _cdiv(sh.W, s)         # class grid (class (0, 0) is the largest)
    tw, th, tb = _tile(gw_, gh, 128)
    cc = ConvCfg()
    cc.a.mode, cc.a.tw, cc.a.th, cc.a.tb = 1, tw, th, tb
    cc.a.tiles_w, cc.a.tiles_h = _cdiv(gw_, tw), _cdiv(gh, th)
    cc.a.sw, cc.a.sh, cc.a.kw_n, cc.a.sign, cc.a.per_tap = 1, 1, kt, -1, 1
    cc.o.on, cc.o.gw, cc.o.gh, cc.o.gb = 1, gw_, gh, sh.B
    cc.o.out_w, cc.o.out_h, cc.o.ys, cc.o.xs, cc.o.yo, cc.o.xo = sh.W, sh.H, s, s, 0, 0
    cc.o.cls_cols = sh.C if s > 1 else 0
    ntiles = cc.a.tiles_w * cc.a.tiles_h * _cdiv(sh.B, tb)
    ad = _grid_map(dy, sh.CO, sh.OW, sh.OH, sh.B, tw, th, tb)
    w = wt.view(s * s * sh.C, kt * kt * sh.CO)
    N = s * s * sh.C
    ep = _epilogue(dx, act="relu_grad" if x_act is not None else "none", aux=x_act, ld=sh.C)
    _run(dy, ad, 0, w, None, 0, ntiles * 128, N, kt * kt * sh.CO, ep, cc, bn=min(256, max(32, N)),
         ldb=w.stride(0), dev=dy.device)
    return dx


def weight_classes(w16: torch.Tensor, sh: ConvShape, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[s*s, C, (k/s)^2 * CO] bf16: for parity class (py, px), row c holds
    W[co, py + s*a, px + s*b, c] in (a, b, co) order (s = 1: W transposed)."""
    s, kt = sh.s, sh.k // sh.s
    if out is None:
        out = torch.empty((s * s, sh.C, kt * kt * sh.CO), dtype=torch.bfloat16, device=w16.device)
    check(_lib.lib(NLIB).surf_conv_weight_t(ptr(w16), sh.CO, sh.C, sh.k, s, ptr(out), stream_ptr(w16.device)),
          "surf_conv_weight_t")
    return out


def weight_classes_reference(w: torch.Tensor, sh: ConvShape) -> torch.Tensor:
    s, kt = sh.s, sh.k // sh.s
    w4 = w.float().view(sh.CO, sh.k, sh.k, sh.C)
    out = []
    for py in range(s):
        for px in range(s):
            sub = w4[:, py::s, px::s, :][:, :kt, :kt, :]           # [CO, kt, kt, C]
            out.append(sub.permute(3, 1, 2, 0).reshape(sh.C, kt * kt * sh.CO))
    return torch.stack(out)
