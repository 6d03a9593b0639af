"""Implicit-GEMM convolutions (ops/conv.py) against torch fp32 references:
forward with bias + ReLU, weight gradient, input gradient with the ReLU
derivative (stride 1 and the stride-2 parity classes), and the weight
rearrangement. Batch sizes that are not multiples of the tile's image count
exercise the out-of-range fills."""
import pytest
import torch
import torch.nn.functional as F

from surfb200.ops import conv as CV

pytestmark = pytest.mark.gpu

SHAPES = [CV.ConvShape(B=6, H=15, W=31, C=32, k=4, s=2, CO=64),      # the policy's conv2
          CV.ConvShape(B=5, H=6, W=14, C=64, k=3, s=1, CO=64),       # the policy's conv3
          CV.ConvShape(B=3, H=9, W=20, C=64, k=3, s=2, CO=64),
          CV.ConvShape(B=7, H=16, W=32, C=16, k=2, s=1, CO=32),      # conv1 on the space-to-depth image
          CV.ConvShape(B=3, H=16, W=32, C=64, k=2, s=1, CO=32)]      # conv1 with four stacked frames


def _nhwc(sh, gen, slack=True):
    n = sh.B * sh.H * sh.W * sh.C
    buf = torch.zeros(n + CV.SLACK_BYTES // 2, dtype=torch.bfloat16, device="cuda")
    buf[:n] = (torch.randn(n, device="cuda", generator=gen)).to(torch.bfloat16)
    return buf, buf[:n].view(sh.B, sh.H, sh.W, sh.C)


def _w(sh, gen):
    return (torch.randn(sh.CO, sh.k * sh.k * sh.C, device="cuda", generator=gen) * 0.05).to(torch.bfloat16)


def _ref_conv(x, w, sh):
    xt = x.float().permute(0, 3, 1, 2)
    wt = w.float().view(sh.CO, sh.k, sh.k, sh.C).permute(0, 3, 1, 2)
    return F.conv2d(xt, wt, stride=sh.s)                                 # [B, CO, OH, OW]


@pytest.mark.parametrize("sh", SHAPES, ids=lambda s: f"C{s.C}k{s.k}s{s.s}")
def test_forward(sh):
    g = torch.Generator(device="cuda").manual_seed(1)
    buf, x = _nhwc(sh, g)
    w = _w(sh, g)
    bias = torch.randn(sh.CO, device="cuda", generator=g) * 0.1
    out = torch.full((sh.B * sh.OH * sh.OW, sh.CO), 7.0, dtype=torch.bfloat16, device="cuda")
    if not sh.supported():
        pytest.skip("unsupported geometry")
    CV.conv_forward(buf, sh, w, bias, out)
    ref = torch.relu(_ref_conv(x, w, sh) + bias.view(1, -1, 1, 1)).permute(0, 2, 3, 1).reshape(-1, sh.CO)
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=3e-2)


@pytest.mark.parametrize("sh", SHAPES, ids=lambda s: f"C{s.C}k{s.k}s{s.s}")
def test_weight_grad(sh):
    g = torch.Generator(device="cuda").manual_seed(2)
    buf, x = _nhwc(sh, g)
    dy = (torch.randn(sh.B * sh.OH * sh.OW, sh.CO, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    gw = torch.full((sh.CO, sh.k * sh.k * sh.C), 0.25, device="cuda")
    CV.conv_weight_grad(dy, buf, sh, gw)
    xt = x.float().permute(0, 3, 1, 2)
    wt = torch.zeros(sh.CO, sh.C, sh.k, sh.k, device="cuda", requires_grad=True)
    y = F.conv2d(xt, wt, stride=sh.s)
    y.backward(dy.float().view(sh.B, sh.OH, sh.OW, sh.CO).permute(0, 3, 1, 2))
    ref = wt.grad.permute(0, 2, 3, 1).reshape(sh.CO, -1) + 0.25
    torch.testing.assert_close(gw, ref, rtol=1e-2, atol=5e-2)


@pytest.mark.parametrize("sh", SHAPES, ids=lambda s: f"C{s.C}k{s.k}s{s.s}")
def test_input_grad(sh):
    if sh.k % sh.s:
        pytest.skip("parity classes need k divisible by the stride")
    if sh.CO != 64 or sh.C % 32:
        pytest.skip("first-layer shapes: the image needs no input gradient")
    g = torch.Generator(device="cuda").manual_seed(3)
    buf, x = _nhwc(sh, g)
    x_act = torch.relu(x.float()).to(torch.bfloat16).reshape(-1, sh.C).contiguous()
    w = _w(sh, g)
    dy = (torch.randn(sh.B * sh.OH * sh.OW, sh.CO, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    wt = CV.weight_classes(w, sh)
    torch.testing.assert_close(wt.float(), CV.weight_classes_reference(w, sh), rtol=0, atol=0)
    dx = torch.full((sh.B * sh.H * sh.W, sh.C), 9.0, dtype=torch.bfloat16, device="cuda")
    CV.conv_input_grad(dy, sh, wt, dx, x_act)
    xt = torch.zeros(sh.B, sh.C, sh.H, sh.W, device="cuda", requires_grad=True)
    y = F.conv2d(xt, w.float().view(sh.CO, sh.k, sh.k, sh.C).permute(0, 3, 1, 2), stride=sh.s)
    y.backward(dy.float().view(sh.B, sh.OH, sh.OW, sh.CO).permute(0, 3, 1, 2))
    ref = xt.grad.permute(0, 2, 3, 1).reshape(-1, sh.C) * (x_act.float() > 0)
    torch.testing.assert_close(dx.float(), ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("sh", [CV.ConvShape(B=700, H=15, W=31, C=32, k=4, s=2, CO=64),
                                CV.ConvShape(B=300, H=6, W=14, C=64, k=3, s=1, CO=64),
                                CV.ConvShape(B=500, H=16, W=32, C=16, k=2, s=1, CO=32)],
                         ids=lambda s: f"C{s.C}k{s.k}s{s.s}")
def test_resident_weights_match_streamed(sh):
    """The forward and input-gradient GEMMs keep the weight operand resident
    in shared memory; streaming it per k-block instead (diagnostic bit 2)
    issues the same MMAs in the same order, so the outputs are bit-identical.
    The batches span several tiles per CTA."""
    g = torch.Generator(device="cuda").manual_seed(4)
    buf, x = _nhwc(sh, g)
    w = _w(sh, g)
    bias = torch.randn(sh.CO, device="cuda", generator=g) * 0.1
    outs = []
    try:
        for dbg in (0, 4):
            CV.DEBUG = dbg
            y = torch.empty(sh.B * sh.OH * sh.OW, sh.CO, dtype=torch.bfloat16, device="cuda")
            CV.conv_forward(buf, sh, w, bias, y)
            res = [y]
            if sh.CO == 64 and sh.C % 32 == 0:
                dy = (torch.randn(sh.B * sh.OH * sh.OW, sh.CO, device="cuda",
                                  generator=torch.Generator(device="cuda").manual_seed(5)) * 0.1).to(torch.bfloat16)
                x_act = torch.relu(x.float()).to(torch.bfloat16).reshape(-1, sh.C).contiguous()
                dx = torch.empty(sh.B * sh.H * sh.W, sh.C, dtype=torch.bfloat16, device="cuda")
                CV.conv_input_grad(dy, sh, CV.weight_classes(w, sh), dx, x_act)
                res.append(dx)
            outs.append(res)
    finally:
        CV.DEBUG = 0
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    ref = torch.relu(_ref_conv(x, w, sh) + bias.view(1, -1, 1, 1)).permute(0, 2, 3, 1).reshape(-1, sh.CO)
    torch.testing.assert_close(outs[0][0].float(), ref, rtol=2e-2, atol=3e-2)


def test_pair_windows_match_single_taps():
    """16-channel inputs read as two-position windows (64-byte rows of an
    overlapping tensor map) give the forward of one-tap slabs bit for bit
    (same MMAs, same order) and the same weight gradient up to the order of
    the split-K atomics."""
    sh = CV.ConvShape(B=300, H=16, W=32, C=16, k=2, s=1, CO=32)
    g = torch.Generator(device="cuda").manual_seed(6)
    buf, x = _nhwc(sh, g)
    w = _w(sh, g)
    bias = torch.randn(sh.CO, device="cuda", generator=g) * 0.1
    dy = (torch.randn(sh.B * sh.OH * sh.OW, sh.CO, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
    res = []
    try:
        for pairs in (True, False):
            CV.PAIR_WINDOWS = pairs
            y = torch.empty(sh.B * sh.OH * sh.OW, sh.CO, dtype=torch.bfloat16, device="cuda")
            CV.conv_forward(buf, sh, w, bias, y)
            gw = torch.zeros(sh.CO, sh.k * sh.k * sh.C, device="cuda")
            CV.conv_weight_grad(dy, buf, sh, gw)
            res.append((y, gw))
    finally:
        CV.PAIR_WINDOWS = True
    assert torch.equal(res[0][0], res[1][0])
    torch.testing.assert_close(res[0][1], res[1][1], rtol=1e-4, atol=1e-4)
