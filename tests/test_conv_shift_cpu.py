"""The shifted-grid trunk's launch descriptors (ops/conv_shift.py) run
through a CPU model of csrc/kernels/conv_shift.cu's semantics -- the TMA
boxes (2-D and 3-D, zero fill out of range), the K-major / MN-major operand
addressing by stage byte offsets, the row-stacked forward epilogue (block j
of row q + j, nothing from past the warp) and the position-stacked weight
gradient with its block map -- compared with torch fp32 convolutions. This
checks every table, offset and output map of the eight products without a
GPU; tests/test_conv_shift_gpu.py runs the same cases on the kernel."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from surfb200.ops import conv_shift as S

_REG = []       # tensors whose addresses the descriptors may hold


def _resolve(addr):
    """(tensor, element offset) of a descriptor address."""
    for t in _REG:
        base = t.data_ptr()
        if base <= addr < base + t.numel() * t.element_size():
            assert (addr - base) % t.element_size() == 0
            return t, (addr - base) // t.element_size()
    raise AssertionError("descriptor address outside the registered tensors")


def _rows(m, seg, u):
    """the box a segment lands for unit u: [rows, inner] fp32, zero outside the map"""
    t, off = _resolve(m.base)
    flat = t.reshape(-1).float()
    r0 = (u // seg.udiv) * seg.mul_hi + (u % seg.udiv) * seg.mul_lo + seg.add
    r = r0 + torch.arange(seg.rows)
    ok = (r >= 0) & (r < m.rows)
    rr = r.clamp(0, m.rows - 1)
    if m.gw:                                            # groups of gw rows, gstride bytes apart
        elem = off + (rr // m.gw) * (m.gstride // 2) + (rr % m.gw) * m.inner
    else:
        elem = off + rr * m.inner
    idx = elem[:, None] + torch.arange(m.inner)[None, :]
    return flat[idx] * ok[:, None]


def _stage(d, u, nseg):
    """the stage as a [stage_bytes / rb] x (rb / 2) matrix (all boxes of one row width)"""
    a = d.a
    rb = a.seg[0].row_bytes
    st = torch.zeros(a.stage_bytes // rb, rb // 2)
    for g in range(nseg):
        sg = a.seg[g]
        assert sg.row_bytes == rb and sg.soff % rb == 0
        st[sg.soff // rb: sg.soff // rb + sg.rows] = _rows(d.maps[g], sg, u)
    return st


def _run_fwd(d, ep):
    a = d.a
    w_t, w_off = _resolve(d.res.base)
    N, K = d.res.rows, d.res.inner
    W = w_t.reshape(-1)[w_off:w_off + N * d.res_ld].view(N, d.res_ld)[:, :K].float()
    out_t, out_off = _resolve(ep.c)
    out = out_t.reshape(-1)
    aux = _resolve(ep.aux) if ep.aux else None
    bias = _resolve(ep.bias) if ep.bias else None
    rb = a.seg[0].row_bytes
    nb = N // a.nblk
    o = a.om
    for t in range(a.mt):
        st = _stage(d, t, a.nseg_a)
        D = torch.zeros(128, N)
        for ks in range(a.ksteps):
            off = a.a_koff[ks]
            r0, c0 = off // rb, (off % rb) // 2
            D += st[r0:r0 + 128, c0:c0 + 16] @ W[:, ks * 16:(ks + 1) * 16].T
        acc = D[:, :nb].clone()
        for j in range(1, a.nblk):
            blk = D[:, j * nb:(j + 1) * nb]
            dj = a.bd[j]
            for r in range(128):
                if (r % 32) + dj < 32:
                    acc[r] += blk[r + dj]
        for quad in range(4):
            written = {}
            for r in range(quad * 32, quad * 32 + 32):
                p = t * 128 + r
                if p >= a.M:
                    continue
                b, rem = divmod(p, o.gw * o.gh)
                h, w = divmod(rem, o.gw)
                for c0 in range(0, nb, 32):
                    cls, col = (c0 // o.cls_cols, c0 % o.cls_cols) if o.cls_cols else (0, c0)
                    py, px = divmod(cls, o.xs)
                    hh, ww = h * o.ys + py, w * o.xs + px
                    valid = hh < o.vh and ww < o.vw
                    if not (valid or a.zero_fill):
                        continue
                    row = b * o.ob + (hh % o.hp) * o.ohp + (hh // o.hp) * o.oh + (ww // o.wp) * o.ow
                    dcol = col + (ww % o.wp) * o.owc
                    v = acc[r, c0:c0 + 32].clone()
                    if not valid:
                        v.zero_()
                    else:
                        if bias is not None:
                            bt, bo = bias
                            v += bt.reshape(-1)[bo + col:bo + col + 32].float()
                        if ep.act == 1:
                            v = v.clamp_min(0)
                        elif ep.act == 3:
                            at, ao = aux
                            sv = at.reshape(-1)[ao + row * ep.ld_aux + dcol:][:32].float()
                            v = v * (sv > 0)
                    for k in range(32):
                        assert (row, dcol + k) not in written
                        written[(row, dcol + k)] = v[k]
            if not written:
                continue
            # the kernel stores each warp's rows as one contiguous block
            rows = sorted({rc[0] for rc in written})
            lo, hi = rows[0], rows[-1]
            assert len(written) == (hi - lo + 1) * ep.ldc, "a warp's output rows must tile one contiguous block"
            assert (hi - lo + 1) * ep.ldc * 2 <= a.stg_bytes
            for (row, c), val in written.items():
                out[out_off + row * ep.ldc + c] = val.to(out.dtype)


def _run_wgrad(d, ep):
    a = d.a
    gw_t, gw_off = _resolve(ep.c)
    gw = gw_t.reshape(-1)
    ra, rbx = a.seg[0].row_bytes, a.seg[1].row_bytes
    na, nbx = ra // 2, rbx // 2
    blocks = a.subw // nbx
    ngrp = (a.N + a.subw - 1) // a.subw
    gb = _resolve(ep.ct) if a.bias_rows else None
    for sp in range(a.splits):
        D = torch.zeros(128, a.N)
        for u in range(sp * a.per, min(a.kt, (sp + 1) * a.per)):
            A = _rows(d.maps[0], a.seg[0], u)                         # A box [rows, 64]
            if gb is not None:
                bt, bo = gb
                col_sum = A[:a.bias_rows].sum(0)
                for c in range(col_sum.numel()):
                    bt.reshape(-1)[bo + c % a.bias_mod] += col_sum[c]
            Bs = {}
            for g in range(1, a.nseg_a + a.nseg_b):
                Bs[a.seg[g].soff] = _rows(d.maps[g], a.seg[g], u)
            row0 = u * a.seg[0].mul_hi + a.seg[0].add
            for ks in range(a.ksteps):
                if a.kgrid and (u, ks) != (sp * a.per, 0):
                    if not (a.kmask >> ((row0 // 16 + ks) % a.kgrid)) & 1:
                        continue
                k0 = a.a_off // ra + ks * 16
                Am = torch.cat([A[k0:k0 + 16], A[k0 + a.a_lbo // ra:k0 + a.a_lbo // ra + 16]], 1)  # [16, 128]
                for g in range(ngrp):
                    cols = []
                    for bb in range(blocks):
                        byte = a.b_noff[g] + bb * a.b_lbo
                        soff = max(s for s in Bs if s <= byte)
                        r = (byte - soff) // rbx + ks * 16
                        cols.append(Bs[soff][r:r + 16])
                    D[:, g * a.subw:(g + 1) * a.subw] += Am.T @ torch.cat(cols, 1)
        for q in range(4):
            for nb in range(a.N // 16):
                col = a.ecol[q][nb]
                if col < 0:
                    continue
                for lane in range(32):
                    s0 = gw_off + (lane + a.erow[q]) * ep.ldc + col
                    gw[s0:s0 + 16] += D[q * 32 + lane, nb * 16:(nb + 1) * 16]


def _emulate(d, ep, dev):
    if d.a.kind == 0:
        _run_fwd(d, ep)
    else:
        _run_wgrad(d, ep)


@pytest.fixture
def trunk(monkeypatch):
    monkeypatch.setattr(S, "_launch", _emulate)
    g = torch.Generator().manual_seed(0)
    w1, w2, w3 = (torch.randn(n, generator=g) * 0.05 for n in (32 * 64, 64 * 512, 64 * 576))
    flat = torch.cat([w1, torch.zeros(64), w2, w3]).to(torch.bfloat16)
    offs = [0, 32 * 64 + 64, 32 * 64 + 64 + 64 * 512]
    T = S.Trunk("cpu", offs)
    idx = T.idx.long()
    T.w.copy_(torch.where(idx >= 0, flat[idx.clamp_min(0)], torch.zeros((), dtype=torch.bfloat16)))
    ws = [flat[o:o + n].float() for o, n in zip(offs, (32 * 64, 64 * 512, 64 * 576))]
    _REG.clear()
    _REG.append(T.w)
    return T, ws, g


def _reg(*ts):
    _REG.extend(ts)
    return ts


def _conv(x_nhwc, w, co, k, c, s):
    wt = w.view(co, k, k, c).permute(0, 3, 1, 2)
    return F.conv2d(x_nhwc.permute(0, 3, 1, 2), wt, stride=s).permute(0, 2, 3, 1)


def _bf(t):
    return t.to(torch.bfloat16).float()


def test_forward_chain(trunk):
    T, (w1, w2, w3), g = trunk
    B = 2
    img = _bf(torch.randn(B, 16, 32, 16, generator=g)).to(torch.bfloat16)
    b1, b2, b3 = (torch.randn(n, generator=g) * 0.1 for n in (32, 64, 64))
    y1 = torch.zeros(B * 512, 32, dtype=torch.bfloat16)
    y2 = torch.zeros(B * 128, 64, dtype=torch.bfloat16)
    y3 = torch.zeros(B * 48, 64, dtype=torch.bfloat16)
    _reg(img, b1, b2, b3, y1, y2, y3)
    T.conv1_forward(img.view(-1, 16), b1, y1, B)
    r1 = torch.relu(_conv(img.float(), w1, 32, 2, 16, 1) + b1)                     # [B, 15, 31, 32]
    got1 = y1.float().view(B, 16, 32, 32)[:, :15, :31]
    torch.testing.assert_close(got1, r1, rtol=2e-2, atol=2e-2)
    T.conv2_forward(y1, b2, y2, B)
    r2 = torch.relu(_conv(got1, w2, 64, 4, 32, 2) + b2)                            # [B, 6, 14, 64]
    got2 = y2.float().view(B, 8, 16, 64)
    torch.testing.assert_close(got2[:, :6, :14], r2, rtol=2e-2, atol=2e-2)
    assert torch.all(got2[:, 6:] == 0) and torch.all(got2[:, :, 14:] == 0)        # padding untouched
    T.conv3_forward(y2, b3, y3, B)
    r3 = torch.relu(_conv(got2[:, :6, :14], w3, 64, 3, 64, 1) + b3)
    torch.testing.assert_close(y3.float().view(B, 4, 12, 64), r3, rtol=2e-2, atol=2e-2)


def test_input_grads(trunk):
    T, (w1, w2, w3), g = trunk
    B = 2
    a1 = _bf(torch.relu(torch.randn(B, 16, 32, 32, generator=g)))
    a2 = torch.zeros(B, 8, 16, 64)
    a2[:, :6, :14] = _bf(torch.relu(torch.randn(B, 6, 14, 64, generator=g)))
    d3 = torch.zeros(B, 8, 16, 64)
    d3[:, :4, :12] = _bf(torch.randn(B, 4, 12, 64, generator=g))
    y1, y2, dy3 = (t.to(torch.bfloat16).reshape(-1, t.shape[-1]).contiguous() for t in (a1, a2, d3))
    dy2 = torch.zeros(B * 128, 64, dtype=torch.bfloat16)
    dy1 = torch.full((B * 512, 32), 9.0, dtype=torch.bfloat16)
    _reg(y1, y2, dy3, dy2, dy1)
    T.conv3_input_grad(dy3, y2, dy2, B)
    x2 = torch.zeros(B, 64, 6, 14, requires_grad=True)
    F.conv2d(x2, w3.view(64, 3, 3, 64).permute(0, 3, 1, 2)).backward(d3[:, :4, :12].permute(0, 3, 1, 2))
    ref2 = x2.grad.permute(0, 2, 3, 1) * (a2[:, :6, :14] > 0)
    got2 = dy2.float().view(B, 8, 16, 64)
    torch.testing.assert_close(got2[:, :6, :14], ref2, rtol=2e-2, atol=2e-2)
    assert torch.all(got2[:, 6:] == 0) and torch.all(got2[:, :, 14:] == 0)
    T.conv2_input_grad(dy2, y1, dy1, B)
    x1 = torch.zeros(B, 32, 15, 31, requires_grad=True)
    F.conv2d(x1, w2.view(64, 4, 4, 32).permute(0, 3, 1, 2), stride=2).backward(_bf(ref2).permute(0, 3, 1, 2))
    ref1 = torch.zeros(B, 16, 32, 32)
    ref1[:, :15, :31] = x1.grad.permute(0, 2, 3, 1)
    ref1 = ref1 * (a1 > 0)
    torch.testing.assert_close(dy1.float().view(B, 16, 32, 32), ref1, rtol=2e-2, atol=2e-2)


def test_weight_grads(trunk):
    T, _, g = trunk
    B = 3
    img = _bf(torch.randn(B, 16, 32, 16, generator=g))
    a1 = _bf(torch.relu(torch.randn(B, 16, 32, 32, generator=g)))
    a2 = torch.zeros(B, 8, 16, 64)
    a2[:, :6, :14] = _bf(torch.relu(torch.randn(B, 6, 14, 64, generator=g)))
    d1 = torch.zeros(B, 16, 32, 32)
    d1[:, :15, :31] = _bf(torch.randn(B, 15, 31, 32, generator=g))
    d2 = torch.zeros(B, 8, 16, 64)
    d2[:, :6, :14] = _bf(torch.randn(B, 6, 14, 64, generator=g))
    d3 = torch.zeros(B, 8, 16, 64)
    d3[:, :4, :12] = _bf(torch.randn(B, 4, 12, 64, generator=g))
    ts = [t.to(torch.bfloat16).reshape(-1, t.shape[-1]).contiguous() for t in (img, a1, a2, d1, d2, d3)]
    x0, y1, y2, dy1, dy2, dy3 = ts
    gw1, gw2, gw3 = torch.full((32, 64), 0.5), torch.full((64, 512), 0.5), torch.full((64, 576), 0.5)
    _reg(*ts, gw1, gw2, gw3)

    def ref(x, d, co, k, c, s):
        w = torch.zeros(co, c, k, k, requires_grad=True)
        F.conv2d(x.permute(0, 3, 1, 2), w, stride=s).backward(d.permute(0, 3, 1, 2))
        return w.grad.permute(0, 2, 3, 1).reshape(co, -1)

    gb1, gb2, gb3 = torch.full((32,), 0.25), torch.full((64,), 0.25), torch.full((64,), 0.25)
    _reg(gb1, gb2, gb3)
    T.conv3_weight_grad(dy3, y2, gw3, B, gb3)
    torch.testing.assert_close(gw3, ref(a2[:, :6, :14], d3[:, :4, :12], 64, 3, 64, 1) + 0.5, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(gb3, d3.sum((0, 1, 2)) + 0.25, rtol=1e-3, atol=1e-3)
    T.conv2_weight_grad(dy2, y1, gw2, B, gb2)
    torch.testing.assert_close(gw2, ref(a1[:, :15, :31], d2[:, :6, :14], 64, 4, 32, 2) + 0.5, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(gb2, d2.sum((0, 1, 2)) + 0.25, rtol=1e-3, atol=1e-3)
    T.conv1_weight_grad(dy1, x0, gw1, B, gb1)
    torch.testing.assert_close(gw1, ref(img, d1[:, :15, :31], 32, 2, 16, 1) + 0.5, rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(gb1, d1.sum((0, 1, 2)) + 0.25, rtol=1e-3, atol=1e-3)


def test_stacked_tables_cover_every_weight_once():
    t = S.stacked_weight_tables()
    for name, n in (("c1f", 32 * 64), ("c2f", 64 * 512), ("c3f", 64 * 576), ("c3d", 64 * 576), ("c2d", 64 * 512)):
        v = t[name][t[name] >= 0]
        per = np.bincount(v, minlength=n)
        assert per.min() >= 1 and per.max() == (4 if name == "c1f" else 1), name
