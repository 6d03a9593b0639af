"""The shifted-grid trunk kernels (csrc/kernels/conv_shift.cu through
ops/conv_shift.py) on the B200 against torch fp32 convolutions: the three
forwards, the two input gradients (ReLU derivative from the saved
activation) and the three weight gradients on the trunk's padded-grid
layouts, plus the stacked-weight gather against its index tables. Batch
sizes that are not multiples of the persistent grid exercise every CTA's
tile loop; the padding of the output grids must stay untouched."""
import pytest
import torch
import torch.nn.functional as F

from surfb200.ops import conv_shift as S

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _trunk(g):
    w1, w2, w3 = (torch.randn(n, device=DEV, generator=g) * 0.05 for n in (32 * 64, 64 * 512, 64 * 576))
    flat = torch.cat([w1, torch.zeros(64, device=DEV), w2, w3]).to(torch.bfloat16)
    offs = [0, 32 * 64 + 64, 32 * 64 + 64 + 64 * 512]
    T = S.Trunk(DEV, offs)
    T.refresh(flat)
    ws = [flat[o:o + n].float() for o, n in zip(offs, (32 * 64, 64 * 512, 64 * 576))]
    return T, ws, flat


def _conv(x_nhwc, w, co, k, c, s):
    wt = w.view(co, k, k, c).permute(0, 3, 1, 2)
    return F.conv2d(x_nhwc.permute(0, 3, 1, 2), wt, stride=s).permute(0, 2, 3, 1)


def _bf(t):
    return t.to(torch.bfloat16).float()


def test_stacked_weight_gather():
    g = torch.Generator(device=DEV).manual_seed(5)
    T, _, flat = _trunk(g)
    idx = T.idx.long()
    want = torch.where(idx >= 0, flat[idx.clamp_min(0)], torch.zeros((), dtype=torch.bfloat16, device=DEV))
    assert torch.equal(T.w, want)


@pytest.mark.parametrize("B", [1, 3, 149, 300])
def test_forward_chain(B):
    g = torch.Generator(device=DEV).manual_seed(1)
    T, (w1, w2, w3), _ = _trunk(g)
    img = _bf(torch.randn(B, 16, 32, 16, device=DEV, generator=g))
    b1, b2, b3 = (torch.randn(n, device=DEV, generator=g) * 0.1 for n in (32, 64, 64))
    y1 = torch.full((B * 512, 32), 7.0, dtype=torch.bfloat16, device=DEV)
    y2 = torch.zeros(B * 128, 64, dtype=torch.bfloat16, device=DEV)
    y3 = torch.full((B * 48 + 32, 64), 7.0, dtype=torch.bfloat16, device=DEV)
    T.conv1_forward(img.to(torch.bfloat16).view(-1, 16), b1, y1, B)
    r1 = torch.relu(_conv(img, w1, 32, 2, 16, 1) + b1)                             # [B, 15, 31, 32]
    got1 = y1.float().view(B, 16, 32, 32)
    torch.testing.assert_close(got1[:, :15, :31], r1, rtol=2e-2, atol=2e-2)
    T.conv2_forward(y1, b2, y2, B)
    r2 = torch.relu(_conv(got1[:, :15, :31], w2, 64, 4, 32, 2) + b2)              # [B, 6, 14, 64]
    got2 = y2.float().view(B, 8, 16, 64)
    torch.testing.assert_close(got2[:, :6, :14], r2, rtol=2e-2, atol=2e-2)
    assert torch.all(got2[:, 6:] == 0) and torch.all(got2[:, :, 14:] == 0)
    T.conv3_forward(y2, b3, y3, B)
    r3 = torch.relu(_conv(got2[:, :6, :14], w3, 64, 3, 64, 1) + b3)
    torch.testing.assert_close(y3[:B * 48].float().view(B, 4, 12, 64), r3, rtol=2e-2, atol=2e-2)
    assert torch.all(y3[B * 48:] == 7.0)


@pytest.mark.parametrize("B", [2, 37, 300])
def test_input_grads(B):
    g = torch.Generator(device=DEV).manual_seed(2)
    T, (w1, w2, w3), _ = _trunk(g)
    a1 = _bf(torch.relu(torch.randn(B, 16, 32, 32, device=DEV, generator=g)))
    a2 = torch.zeros(B, 8, 16, 64, device=DEV)
    a2[:, :6, :14] = _bf(torch.relu(torch.randn(B, 6, 14, 64, device=DEV, generator=g)))
    d3 = torch.zeros(B, 8, 16, 64, device=DEV)
    d3[:, :4, :12] = _bf(torch.randn(B, 4, 12, 64, device=DEV, generator=g))
    y1, y2, dy3 = (t.to(torch.bfloat16).reshape(-1, t.shape[-1]).contiguous() for t in (a1, a2, d3))
    dy2 = torch.zeros(B * 128, 64, dtype=torch.bfloat16, device=DEV)
    dy1 = torch.full((B * 512, 32), 9.0, dtype=torch.bfloat16, device=DEV)
    T.conv3_input_grad(dy3, y2, dy2, B)
    x2 = torch.zeros(B, 64, 6, 14, device=DEV, requires_grad=True)
    F.conv2d(x2, w3.view(64, 3, 3, 64).permute(0, 3, 1, 2)).backward(d3[:, :4, :12].permute(0, 3, 1, 2))
    ref2 = x2.grad.permute(0, 2, 3, 1) * (a2[:, :6, :14] > 0)
    got2 = dy2.float().view(B, 8, 16, 64)
    torch.testing.assert_close(got2[:, :6, :14], ref2, rtol=2e-2, atol=2e-2)
    assert torch.all(got2[:, 6:] == 0) and torch.all(got2[:, :, 14:] == 0)
    T.conv2_input_grad(dy2, y1, dy1, B)
    x1 = torch.zeros(B, 32, 15, 31, device=DEV, requires_grad=True)
    F.conv2d(x1, w2.view(64, 4, 4, 32).permute(0, 3, 1, 2), stride=2).backward(_bf(ref2).permute(0, 3, 1, 2))
    ref1 = torch.zeros(B, 16, 32, 32, device=DEV)
    ref1[:, :15, :31] = x1.grad.permute(0, 2, 3, 1)
    ref1 = ref1 * (a1 > 0)
    torch.testing.assert_close(dy1.float().view(B, 16, 32, 32), ref1, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("B", [3, 41, 300])
def test_weight_grads(B):
    g = torch.Generator(device=DEV).manual_seed(3)
    T, _, _ = _trunk(g)
    img = _bf(torch.randn(B, 16, 32, 16, device=DEV, generator=g))
    a1 = _bf(torch.relu(torch.randn(B, 16, 32, 32, device=DEV, generator=g)))
    a2 = torch.zeros(B, 8, 16, 64, device=DEV)
    a2[:, :6, :14] = _bf(torch.relu(torch.randn(B, 6, 14, 64, device=DEV, generator=g)))
    d1 = torch.zeros(B, 16, 32, 32, device=DEV)
    d1[:, :15, :31] = _bf(torch.randn(B, 15, 31, 32, device=DEV, generator=g) * 0.1)
    d2 = torch.zeros(B, 8, 16, 64, device=DEV)
    d2[:, :6, :14] = _bf(torch.randn(B, 6, 14, 64, device=DEV, generator=g) * 0.1)
    d3 = torch.zeros(B, 8, 16, 64, device=DEV)
    d3[:, :4, :12] = _bf(torch.randn(B, 4, 12, 64, device=DEV, generator=g) * 0.1)
    x0, y1, y2, dy1, dy2, dy3 = (t.to(torch.bfloat16).reshape(-1, t.shape[-1]).contiguous()
                                 for t in (img, a1, a2, d1, d2, d3))
    gw1, gw2, gw3 = (torch.full(s, 0.5, device=DEV) for s in ((32, 64), (64, 512), (64, 576)))

    def ref(x, d, co, k, c, s):
        w = torch.zeros(co, c, k, k, device=DEV, requires_grad=True)
        F.conv2d(x.permute(0, 3, 1, 2), w, stride=s).backward(d.permute(0, 3, 1, 2))
        return w.grad.permute(0, 2, 3, 1).reshape(co, -1)

    gb1, gb2, gb3 = (torch.full((n,), 0.25, device=DEV) for n in (32, 64, 64))
    T.conv3_weight_grad(dy3, y2, gw3, B, gb3)
    torch.testing.assert_close(gw3, ref(a2[:, :6, :14], d3[:, :4, :12], 64, 3, 64, 1) + 0.5, rtol=1e-2, atol=3e-2)
    torch.testing.assert_close(gb3, d3.sum((0, 1, 2)) + 0.25, rtol=1e-3, atol=1e-2)
    T.conv2_weight_grad(dy2, y1, gw2, B, gb2)
    torch.testing.assert_close(gw2, ref(a1[:, :15, :31], d2[:, :6, :14], 64, 4, 32, 2) + 0.5, rtol=1e-2, atol=3e-2)
    torch.testing.assert_close(gb2, d2.sum((0, 1, 2)) + 0.25, rtol=1e-3, atol=1e-2)
    T.conv1_weight_grad(dy1, x0, gw1, B, gb1)
    torch.testing.assert_close(gw1, ref(img, d1[:, :15, :31], 32, 2, 16, 1) + 0.5, rtol=1e-2, atol=3e-2)
    torch.testing.assert_close(gb1, d1.sum((0, 1, 2)) + 0.25, rtol=1e-3, atol=1e-2)
