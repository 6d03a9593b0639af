"""The vision trunk's convolutions on row-shifted views of flattened grids
(csrc/kernels/conv_shift.cu), for the flagship Nature-CNN geometry on the
4x4 space-to-depth depth image: conv1 2x2/1 (16 -> 32 channels) on the
16 x 32 image, conv2 4x4/2 (32 -> 64) and conv3 3x3/1 (64 -> 64).

An activation is a [rows, channels] matrix whose row p is grid position
(b, h, w), p = (b*GH + h)*GW + w. A stride-1 convolution computed at every
grid position reads, for tap (kh, kw), the same rows shifted by kh*GW + kw,
so a 128-row output tile needs one TMA box and each tap is an MMA at a row
offset into it. The layouts that make every layer a set of row shifts:

  img   [B][16][32][16]   read as rows of 4 positions (64 channels, conv1
                          forward: output class = position in the row) and
                          as rows of 2 positions (32 channels, conv1 weights)
  y1    [B][16][32][32]   conv1 output on the full 16 x 32 image grid (the
                          row h = 15 and column w = 31 are computed and never
                          read); read as rows of 2 positions (64 channels)
                          whose even / odd image rows form two "planes" of
                          8 x 16 rows (3-D boxes): conv2's stride 2 becomes
                          plane choice + row shifts
  y2    [B][8][16][64]    conv2 output on the 8 x 16 plane grid (valid 6 x 14,
                          zeros elsewhere)
  y3    [B][4][12][64]    conv3 output, dense (the FC layer's input)
  dy3   [B][8][16][64]    conv3's output gradient on its input grid, zeros
                          outside 4 x 12 (written there by the FC layer's
                          input-gradient GEMM through its column remap)
  dy2   [B][8][16][64]    zeros outside 6 x 14
  dy1   [B][16][32][32]   every position written (exact zeros where conv2
                          reads nothing)

Forward-kind products stack output-row offsets along N (one A operand
feeds up to three taps: the epilogue adds block j of row q + j into row q,
a warp shuffle; the grids put only invalid outputs in the lanes whose
partner row lies in the next warp). Weight gradients stack two position
ranges 16 rows apart along M. The stacked weight operands are gathered
from the bf16 parameters by one launch per optimizer step
(``Trunk.refresh``). The reference's trunk is cuDNN convolutions
(python/train_fast.py:115-121).
"""
from __future__ import annotations

import ctypes
from ctypes import c_int, c_int64, c_short, c_void_p
from typing import Optional

import numpy as np
import torch

from . import _lib
from ._lib import check, ptr, stream_ptr
from .gemm import ACT, NLIB, Epilogue, error_flag

SW128, SW64, SW32 = 2, 4, 6
_LAYOUT = {128: SW128, 64: SW64, 32: SW32}


class ShSeg(ctypes.Structure):
    _fields_ = [("rows", c_int), ("row_bytes", c_int), ("gw", c_int), ("udiv", c_int), ("mul_hi", c_int),
                ("mul_lo", c_int), ("add", c_int), ("soff", c_int)]


class ShOut(ctypes.Structure):
    _fields_ = [("gw", c_int), ("gh", c_int), ("vh", c_int), ("vw", c_int), ("ys", c_int), ("xs", c_int),
                ("cls_cols", c_int), ("hp", c_int), ("wp", c_int), ("owc", c_int), ("ob", c_int64), ("ohp", c_int64),
                ("oh", c_int64), ("ow", c_int64)]


class ShArgs(ctypes.Structure):
    _fields_ = [("kind", c_int), ("M", c_int), ("N", c_int), ("kt", c_int), ("mt", c_int), ("nt", c_int),
                ("splits", c_int), ("per", c_int), ("nseg_a", c_int), ("nseg_b", c_int), ("seg", ShSeg * 4),
                ("stage_bytes", c_int), ("unit_bytes", c_int), ("a_layout", c_int), ("a_lbo", c_int),
                ("a_sbo", c_int), ("b_layout", c_int), ("b_lbo", c_int), ("b_sbo", c_int), ("ksteps", c_int),
                ("a_koff", c_int * 64), ("nblk", c_int), ("bd", c_int * 4), ("zero_fill", c_int),
                ("stg_bytes", c_int), ("a_off", c_int), ("a_krow", c_int),
                ("subw", c_int), ("b_krow", c_int), ("b_noff", c_int * 16), ("kgrid", c_int), ("kmask", c_int),
                ("bias_rows", c_int), ("bias_mod", c_int),
                ("erow", c_int * 4),
                ("ecol", (c_short * 32) * 4), ("om", ShOut)]


class ShMap(ctypes.Structure):
    _fields_ = [("base", c_void_p), ("rows", c_int64), ("inner", c_int), ("gw", c_int), ("gstride", c_int64)]


class ShDesc(ctypes.Structure):
    _fields_ = [("a", ShArgs), ("maps", ShMap * 4), ("res", ShMap), ("res_ld", c_int64), ("bn", c_int)]


_lib.register(NLIB, {
    "surf_shconv": (c_int, [ctypes.POINTER(ShDesc), ctypes.POINTER(Epilogue), c_void_p]),
    "surf_shconv_weights": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "surf_shconv_sizes": (c_int, [ctypes.POINTER(c_int)]),
})

_checked = [False]
_SMS = {}


def _check_layout() -> None:
    if _checked[0]:
        return
    out = (c_int * 5)()
    _lib.lib(NLIB).surf_shconv_sizes(out)
    want = (ctypes.sizeof(ShDesc), ctypes.sizeof(ShArgs), ctypes.sizeof(ShSeg), ctypes.sizeof(ShOut),
            ctypes.sizeof(ShMap))
    if tuple(out) != want:
        raise RuntimeError(f"surf_shconv struct layout mismatch: native {tuple(out)} vs ctypes {want}")
    _checked[0] = True


def _sms(dev) -> int:
    if dev.type != "cuda":
        return 148
    i = dev.index if dev.index is not None else torch.cuda.current_device()
    if i not in _SMS:
        _SMS[i] = torch.cuda.get_device_properties(i).multi_processor_count
    return _SMS[i]


def _r1k(n: int) -> int:
    return (n + 1023) // 1024 * 1024


def _seg(rows, rb, soff, mul_hi, add=0, gw=0) -> ShSeg:
    """box of ``rows`` rows of ``rb`` bytes at stage offset ``soff``; unit u starts at row u*mul_hi + add"""
    s = ShSeg()
    s.rows, s.row_bytes, s.gw, s.udiv, s.mul_hi, s.mul_lo, s.add, s.soff = rows, rb, gw, 1, mul_hi, 0, add, soff
    return s


def _map(t: torch.Tensor, inner: int, rows: int, gw: int = 0, gstride: int = 0) -> ShMap:
    m = ShMap()
    m.base, m.rows, m.inner, m.gw, m.gstride = ptr(t), rows, inner, gw, gstride
    return m


def _out_map(gw, gh, vh, vw, ob, oh, ow=1, ys=1, xs=1, cls_cols=0) -> ShOut:
    o = ShOut()
    o.gw, o.gh, o.vh, o.vw, o.ys, o.xs, o.cls_cols = gw, gh, vh, vw, ys, xs, cls_cols
    o.hp, o.wp, o.owc, o.ob, o.ohp, o.oh, o.ow = 1, 1, 0, ob, 0, oh, ow
    return o


def _epi(out: torch.Tensor, ld: int, bias=None, act="none", aux=None, ld_aux=0, accumulate=False) -> Epilogue:
    from . import conv as CV
    ep = Epilogue()
    ep.c = ptr(out)
    ep.ldc = ld
    ep.c_dtype = 1 if out.dtype == torch.bfloat16 else 0
    ep.c_mode = 1 if accumulate else 0
    ep.bias = ptr(bias)
    ep.act = ep.act2 = ACT[act]
    ep.act_split = 1 << 30
    ep.aux = ptr(aux)
    ep.ld_aux = ld_aux
    ep.err = ptr(error_flag(out.device))
    ep.dbg = int(CV.DEBUG)
    ep.trace = ptr(CV.TRACE)
    return ep


def _launch(d: ShDesc, ep: Epilogue, dev) -> None:
    _check_layout()
    check(_lib.lib(NLIB).surf_shconv(ctypes.byref(d), ctypes.byref(ep), stream_ptr(dev)), "surf_shconv")


def shift_forward(segs, maps, koffs, w: torch.Tensor, tiles: int, M: int, om: ShOut, out: torch.Tensor, ld_out: int,
                  stg_bytes: int, nblk: int = 1, zero_fill: bool = False, bias=None, act="relu", aux=None,
                  ld_aux: int = 0) -> None:
    """Forward-kind product: ``segs`` / ``maps`` the tile's A boxes, ``koffs``
    the stage byte offset of each 16-wide K step's A operand (K-major, rows of
    segs[0].row_bytes), ``w`` [N, K] the resident B (nblk column blocks; block
    j of accumulator row p belongs to output row p - j), output rows through
    ``om`` -- rows outside the valid window stored as zeros with ``zero_fill``.
    The rows one epilogue warp writes (32 grid rows, every class) must form
    one contiguous, fully written range of ``out`` of at most ``stg_bytes``
    bytes: the warp stores it with a single bulk copy."""
    d = ShDesc()
    a = d.a
    N, K = w.shape
    for i, (sg, mp) in enumerate(zip(segs, maps)):
        a.seg[i] = sg
        d.maps[i] = mp
    last = segs[-1]
    a.stage_bytes = _r1k(last.soff + last.rows * last.row_bytes)
    a.unit_bytes = sum(s.rows * s.row_bytes for s in segs)
    a.kind, a.M, a.N, a.kt, a.mt = 0, M, N, (K + 63) // 64, tiles
    a.nseg_a, a.nseg_b = len(segs), 0
    rb = segs[0].row_bytes
    a.a_layout, a.a_lbo, a.a_sbo = _LAYOUT[rb], 16, 8 * rb
    a.ksteps = len(koffs)
    for k, off in enumerate(koffs):
        a.a_koff[k] = off
    a.nblk = nblk
    for j in range(nblk):
        a.bd[j] = j
    a.zero_fill = int(zero_fill)
    a.stg_bytes = stg_bytes
    a.om = om
    d.res = _map(w, K, N)
    d.res_ld = w.stride(0)
    d.bn = N
    _launch(d, _epi(out, ld_out, bias=bias, act=act, aux=aux, ld_aux=ld_aux), out.device)


def shift_wgrad(a_seg, a_map, b_segs, b_maps, groups, subw: int, b_lbo: int, R: int, L: int, kt: int, N: int,
                erow, ecol, gw: torch.Tensor, gb: Optional[torch.Tensor] = None, bias_mod: int = 64,
                kgrid: int = 0, kmask: int = 0) -> None:
    """Weight-gradient product, k = grid positions in load units of R rows:
    A (MN-major, 128-byte rows) holds the output gradient of rows
    [u*R - L, u*R + R); its upper MN block starts L rows in, so the upper
    accumulator half computes the taps L rows below the lower half's. ``groups``:
    per MMA group, (B box index, row inside the box) of its first N block; the
    group's blocks sit ``b_lbo`` bytes apart. ``erow`` / ``ecol``: destination
    of every (32-row, 16-column) accumulator block in ``gw`` (fp32, accumulated;
    column -1 = skipped). ``gb``: also accumulate the bias gradient, the sum
    of the first R rows of every A box (every position once), column c into
    channel c % bias_mod. ``kgrid`` / ``kmask``: K step ks of a unit covers
    grid row ((first A-box row) / 16 + ks) mod kgrid (both halves' rows: that
    row and the next); only rows whose bit is set in ``kmask`` are issued --
    the others' output gradient must be zero."""
    d = ShDesc()
    a = d.a
    a.seg[0] = a_seg
    d.maps[0] = a_map
    soff = _r1k(a_seg.rows * a_seg.row_bytes)
    xoff = []
    rbx = b_segs[0].row_bytes
    for j, (sg, mp) in enumerate(zip(b_segs, b_maps)):
        sg.soff = soff
        a.seg[1 + j] = sg
        d.maps[1 + j] = mp
        xoff.append(soff)
        soff = _r1k(soff + sg.rows * sg.row_bytes)
    a.kind, a.M, a.N, a.kt = 1, 128, N, kt
    a.nseg_a, a.nseg_b = 1, len(b_segs)
    a.stage_bytes = soff
    a.unit_bytes = a_seg.rows * a_seg.row_bytes + sum(s.rows * s.row_bytes for s in b_segs)
    ra = a_seg.row_bytes
    a.a_layout, a.a_lbo, a.a_sbo, a.a_off, a.a_krow = _LAYOUT[ra], L * ra, 8 * ra, 0, ra
    a.b_layout, a.b_lbo, a.b_sbo, a.b_krow = _LAYOUT[rbx], b_lbo, 8 * rbx, rbx
    a.subw = subw
    a.ksteps = R // 16
    for g, (box, row) in enumerate(groups):
        a.b_noff[g] = xoff[box] + row * rbx
    for q in range(4):
        a.erow[q] = erow[q]
        for nb in range(32):
            a.ecol[q][nb] = ecol[q][nb] if nb < len(ecol[q]) else -1
    a.nt = 1
    splits = max(1, min(kt, _sms(gw.device)))
    a.per = (kt + splits - 1) // splits
    a.splits = (kt + a.per - 1) // a.per
    if gb is not None:
        a.bias_rows, a.bias_mod = R, bias_mod
    a.kgrid, a.kmask = kgrid, kmask
    d.bn = subw * len(groups)
    ep = _epi(gw, gw.stride(0), accumulate=True)
    ep.ct = ptr(gb)
    _launch(d, ep, gw.device)


# ---- stacked weight operands ----------------------------------------------------------------
def _w1_index(co, kh, kw, ci):
    return ((co * 2 + kh) * 2 + kw) * 16 + ci


def _w2_index(co, kh, kw, ci):
    return ((co * 4 + kh) * 4 + kw) * 32 + ci


def _w3_index(co, kh, kw, ci):
    return ((co * 3 + kh) * 3 + kw) * 64 + ci


# conv1 forward K steps on the 4-position rows: (kh, position-row shift, quarter)
_C1_STEPS = [(kh, sp, q) for kh in range(2) for sp, q in ((0, 0), (0, 1), (0, 2), (0, 3), (1, 0))]


def stacked_weight_tables():
    """Index tables (into each layer's own [CO, kh, kw, C] weight, -1 = zero)
    of the five stacked B operands: conv1/2/3 forward, conv3/2 input gradient."""
    t = {}
    # conv1 forward [128 = (px, co)][192]: K step ks reads quarter q of the row sp rows on
    b = -np.ones((128, 192), np.int64)
    ci = np.arange(16)
    for ks, (kh, sp, q) in enumerate(_C1_STEPS):
        for px in range(4):
            kw = 4 * sp + q - px
            if 0 <= kw <= 1:
                for co in range(32):
                    b[px * 32 + co, ks * 16:(ks + 1) * 16] = _w1_index(co, kh, kw, ci)
    t["c1f"] = b
    # conv2 forward [128 = (j, co)][256]: K step (plane, a, kc); block j reads column shift c = j
    b = -np.ones((128, 256), np.int64)
    co = np.arange(64)
    for pl in range(2):
        for a_ in range(2):
            for e in range(64):
                px, c_i = e // 32, e % 32
                for j in range(2):
                    b[j * 64 + co, (pl * 2 + a_) * 64 + e] = _w2_index(co, 2 * a_ + pl, 2 * j + px, c_i)
    t["c2f"] = b
    # conv3 forward [192 = (j, co)][192 = (kh, ci)]: block j is tap column kw = j
    b = -np.ones((192, 192), np.int64)
    for kh in range(3):
        for c_i in range(64):
            for j in range(3):
                b[j * 64 + co, kh * 64 + c_i] = _w3_index(co, kh, j, c_i)
    t["c3f"] = b
    # conv3 input gradient [192 = (j, ci)][192 = (kh, co)]: block j is tap column kw = 2 - j
    b = -np.ones((192, 192), np.int64)
    cin = np.arange(64)
    for kh in range(3):
        for c_o in range(64):
            for j in range(3):
                b[j * 64 + cin, kh * 64 + c_o] = _w3_index(c_o, kh, 2 - j, cin)
    t["c3d"] = b
    # conv2 input gradient [256 = (j, py, px, ci)][128 = (a, co)]: block j is column shift c = 1 - j
    b = -np.ones((256, 128), np.int64)
    cin = np.arange(32)
    for a_ in range(2):
        for c_o in range(64):
            for j in range(2):
                for py in range(2):
                    for px in range(2):
                        b[j * 128 + py * 64 + px * 32 + cin, a_ * 64 + c_o] = _w2_index(c_o, py + 2 * a_,
                                                                                       px + 2 * (1 - j), cin)
    t["c2d"] = b
    return t


def wgrad_maps():
    """(erow, ecol) of the three weight gradients: where each (32-row, 16-column)
    accumulator block lands in the [CO, kh*kw*C] gradient (-1: not stored)."""
    m = {}
    # conv1: rows (h, px, co32), columns (c, half, ci16): kh = 1 - h, kw = 2c + half - px
    ecol = [[-1] * 4 for _ in range(4)]
    for q in range(4):
        h, px = q // 2, q % 2
        for nb in range(4):
            c, half = nb // 2, nb % 2
            kw = 2 * c + half - px
            if 0 <= kw <= 1:
                ecol[q][nb] = ((1 - h) * 2 + kw) * 16
    m["c1"] = ([0, 0, 0, 0], ecol)
    # conv2: rows (h, co64), columns (plane, c, px, ci32): kh = 2(1 - h) + plane, kw = 2c + px
    ecol = [[-1] * 16 for _ in range(4)]
    for q in range(4):
        h = q // 2
        for nb in range(16):
            n = nb * 16
            pl, c, px, ci0 = n // 128, (n // 64) % 2, (n // 32) % 2, n % 32
            ecol[q][nb] = ((2 * (1 - h) + pl) * 4 + 2 * c + px) * 32 + ci0
    m["c2"] = ([0, 32, 0, 32], ecol)
    # conv3: rows (h, co64), columns (g, kw, ci64): kh = g + 1 - h; (h = 1, g = 1) repeats (h = 0, g = 0)
    ecol = [[-1] * 24 for _ in range(4)]
    for q in range(4):
        h = q // 2
        for nb in range(24):
            n = nb * 16
            g, kw, ci0 = n // 192, (n % 192) // 64, n % 64
            if not (h == 1 and g == 1):
                ecol[q][nb] = ((g + 1 - h) * 3 + kw) * 64 + ci0
    m["c3"] = ([0, 32, 0, 32], ecol)
    return m


_TABLES = {}


class Trunk:
    """The flagship trunk's eight convolution products on the layouts of the
    module docstring. ``offsets``: flat bf16 parameter offsets of conv1.w,
    conv2.w and conv3.w (``refresh`` gathers the stacked operands from them)."""

    R1, L = 192, 16                  # weight-gradient load unit (positions) and stacking offset
    # weight-gradient K steps worth issuing on the 8 x 16 grids: a step covers
    # grid rows h (lower half) and h + 1 (upper half); dy3 is nonzero in rows
    # 0-3, dy2 in rows 0-5
    KMASK3 = sum(1 << h for h in range(8) if h < 4 or (h + 1) % 8 < 4)
    KMASK2 = sum(1 << h for h in range(8) if h < 6 or (h + 1) % 8 < 6)

    def __init__(self, device, offsets):
        dev = torch.device(device)
        key = (str(dev), tuple(int(o) for o in offsets))
        if key not in _TABLES:
            tabs = stacked_weight_tables()
            parts, where, pos = [], {}, 0
            for name, layer in (("c1f", 0), ("c2f", 1), ("c3f", 2), ("c3d", 2), ("c2d", 1)):
                t = tabs[name]
                size = (t.size + 63) // 64 * 64
                where[name] = (pos, t.shape)
                pos += size
                g = np.where(t >= 0, t + int(offsets[layer]), -1).reshape(-1)
                parts.append(np.pad(g, (0, size - t.size), constant_values=-1))
            idx = torch.from_numpy(np.concatenate(parts).astype(np.int32)).to(dev)
            _TABLES[key] = (idx, where)
        self.idx, self._where = _TABLES[key]
        self.w = torch.zeros(self.idx.numel(), dtype=torch.bfloat16, device=dev)
        self.maps = wgrad_maps()

    @staticmethod
    def supported(cfg) -> bool:
        """the geometry these layouts are written for (the Nature CNN on the
        64 x 128 depth image in 4x4 space-to-depth order)"""
        return bool(cfg.vision and (cfg.img_h, cfg.img_w, cfg.img_c) == (16, 32, 16)
                    and tuple(tuple(c) for c in cfg.conv) == ((2, 1, 32), (4, 2, 64), (3, 1, 64)))

    def weight(self, name: str) -> torch.Tensor:
        off, shape = self._where[name]
        return self.w[off:off + shape[0] * shape[1]].view(*shape)

    def refresh(self, flat16: torch.Tensor) -> None:
        """Rebuild the stacked weight operands from the bf16 parameters (one launch)."""
        check(_lib.lib(NLIB).surf_shconv_weights(ptr(flat16), ptr(self.idx), ptr(self.w), self.w.numel(),
                                                 stream_ptr(flat16.device)), "surf_shconv_weights")

    # ---- forward -------------------------------------------------------------------------
    def conv1_forward(self, img, b1, y1, B):
        """img [B*512, 16] -> y1 [B*512, 32] = relu(conv1 + b1) on the full 16 x 32 grid."""
        rows = B * 128                                   # rows of 4 positions
        sg = _seg(128 + 9, 128, 0, 128)
        koffs = [(8 * kh + sp) * 128 + q * 32 for kh, sp, q in _C1_STEPS]
        om = _out_map(8, 16, 16, 32, ob=512, oh=32, xs=4, cls_cols=32)
        shift_forward([sg], [_map(img, 64, rows)], koffs, self.weight("c1f"), B, rows, om, y1, 32, 4 * 32 * 64,
                      bias=b1)

    @staticmethod
    def _planes(y1, B):
        """the two row-parity planes of y1's 2-position rows (3-D maps of 16-row groups)"""
        return [_map(y1[pl * 32:], 64, B * 128, gw=16, gstride=2 * 16 * 128) for pl in range(2)]

    def conv2_forward(self, y1, b2, y2, B):
        """y1 [B*512, 32] -> y2 [B*128, 64] (8 x 16 plane grid) = relu(conv2 + b2) inside 6 x 14, zeros outside."""
        box = 160                                        # 10 plane rows: the tile's 8 + shifts up to 17 rows
        segs = [_seg(box, 128, pl * _r1k(box * 128), 128, gw=16) for pl in range(2)]
        koffs = [segs[pl].soff + 16 * a_ * 128 + kc * 32 for pl in range(2) for a_ in range(2) for kc in range(4)]
        om = _out_map(16, 8, 6, 14, ob=128, oh=16)
        shift_forward(segs, self._planes(y1, B), koffs, self.weight("c2f"), B, B * 128, om, y2, 64, 32 * 128, nblk=2,
                      zero_fill=True, bias=b2)

    def conv3_forward(self, y2, b3, y3, B):
        """y2 [B*128, 64] -> y3 [B*48, 64] (dense 4 x 12) = relu(conv3 + b3)."""
        sg = _seg(128 + 34, 128, 0, 128)
        koffs = [16 * kh * 128 + kc * 32 for kh in range(3) for kc in range(4)]
        om = _out_map(16, 8, 4, 12, ob=48, oh=12)
        shift_forward([sg], [_map(y2, 64, B * 128)], koffs, self.weight("c3f"), B, B * 128, om, y3, 64, 24 * 128,
                      nblk=3, bias=b3)

    # ---- input gradients -----------------------------------------------------------------
    def conv3_input_grad(self, dy3, y2, dy2, B):
        """dy3 [B*128, 64] (zeros outside 4 x 12) -> dy2 [B*128, 64] =
        conv3^T(dy3) * relu'(y2) inside 6 x 14, zeros outside."""
        sg = _seg(128 + 34, 128, 0, 128, add=-34)
        koffs = [(32 - 16 * kh) * 128 + kc * 32 for kh in range(3) for kc in range(4)]
        om = _out_map(16, 8, 6, 14, ob=128, oh=16)
        shift_forward([sg], [_map(dy3, 64, B * 128)], koffs, self.weight("c3d"), B, B * 128, om, dy2, 64, 32 * 128,
                      nblk=3, zero_fill=True, act="relu_grad", aux=y2, ld_aux=64)

    def conv2_input_grad(self, dy2, y1, dy1, B):
        """dy2 [B*128, 64] (zeros outside 6 x 14) -> dy1 [B*512, 32] (every
        position) = conv2^T(dy2) * relu'(y1)."""
        sg = _seg(128 + 17, 128, 0, 128, add=-17)
        koffs = [(16 - 16 * a_) * 128 + kc * 32 for a_ in range(2) for kc in range(4)]
        om = _out_map(16, 8, 16, 16, ob=256, oh=16, ys=2, cls_cols=64)
        shift_forward([sg], [_map(dy2, 64, B * 128)], koffs, self.weight("c2d"), B, B * 128, om, dy1, 64, 64 * 128,
                      nblk=2, act="relu_grad", aux=y1, ld_aux=64)

    # ---- weight gradients ----------------------------------------------------------------
    def conv1_weight_grad(self, dy1, img, gw1, B, gb1=None):
        """gw1 [32, 64] += dW of conv1 from dy1 [B*512, 32] and img [B*512, 16]
        (and gb1 [32] += the bias gradient)."""
        R, L = self.R1, self.L
        rows = B * 256                                   # rows of 2 positions
        kt = (rows + L + R - 1) // R
        a_seg = _seg(R + L, 128, 0, R, add=-L)
        b_seg = _seg(R + 1, 64, 0, R)
        erow, ecol = self.maps["c1"]
        shift_wgrad(a_seg, _map(dy1, 64, rows), [b_seg], [_map(img, 32, rows)], [(0, 0)], 64, 64, R, L, kt, 64,
                    erow, ecol, gw1, gb1, 32)

    def conv2_weight_grad(self, dy2, y1, gw2, B, gb2=None):
        """gw2 [64, 512] += dW of conv2 from dy2 [B*128, 64] (zeros outside 6 x 14) and y1
        (and gb2 [64] += the bias gradient)."""
        R, L = 128, self.L
        rows = B * 128
        kt = (rows + L + R - 1) // R
        a_seg = _seg(R + L, 128, 0, R, add=-L)
        b_segs = [_seg(R + 16, 128, 0, R, gw=16) for _ in range(2)]
        erow, ecol = self.maps["c2"]
        shift_wgrad(a_seg, _map(dy2, 64, rows), b_segs, self._planes(y1, B), [(0, 0), (1, 0)], 128, 128, R, L, kt,
                    256, erow, ecol, gw2, gb2, kgrid=8, kmask=self.KMASK2)

    def conv3_weight_grad(self, dy3, y2, gw3, B, gb3=None):
        """gw3 [64, 576] += dW of conv3 from dy3 [B*128, 64] (zeros outside 4 x 12) and y2
        (and gb3 [64] += the bias gradient)."""
        R, L = self.R1, self.L
        rows = B * 128
        kt = (rows + L + R - 1) // R
        a_seg = _seg(R + L, 128, 0, R, add=-L)
        b_seg = _seg(R + 18, 128, 0, R)
        erow, ecol = self.maps["c3"]
        shift_wgrad(a_seg, _map(dy3, 64, rows), [b_seg], [_map(y2, 64, rows)], [(0, 0), (0, 16)], 192, 128, R, L,
                    kt, 384, erow, ecol, gw3, gb3, kgrid=8, kmask=self.KMASK3)
