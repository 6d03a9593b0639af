"""im2col / col2im(+ReLU') / colsum kernels vs plain torch fp32 references,
on the policy's three convolution geometries and a ragged one."""
import pytest
import torch
import torch.nn.functional as F

from surfb200.ops import gemm as G

pytestmark = pytest.mark.gpu

GEOMS = [  # B, H, W, C, k, s
    (3, 64, 128, 1, 8, 4),
    (5, 15, 31, 32, 4, 2),
    (4, 6, 14, 64, 3, 1),
    (2, 9, 11, 8, 3, 2),
]


def _unfold(x, k, s):
    """NHWC -> [B*OH*OW, k*k*C] rows in (kh, kw, c) order."""
    B, H, W, C = x.shape
    u = F.unfold(x.permute(0, 3, 1, 2).float(), k, stride=s)          # [B, C*k*k, L]
    L = u.shape[-1]
    return u.view(B, C, k, k, L).permute(0, 4, 2, 3, 1).reshape(B * L, k * k * C)


@pytest.mark.parametrize("B,H,W,C,k,s", GEOMS)
def test_im2col_matches_unfold(B, H, W, C, k, s):
    x = torch.randn(B, H, W, C, device="cuda").to(torch.bfloat16)
    col = G.im2col(x, B, H, W, C, k, s)
    torch.testing.assert_close(col.float(), _unfold(x, k, s), rtol=0, atol=0)


@pytest.mark.parametrize("B,H,W,C,k,s", [g for g in GEOMS if g[3] % 8 == 0])
def test_col2im_relu_matches_fold(B, H, W, C, k, s):
    OH, OW = (H - k) // s + 1, (W - k) // s + 1
    dcol = torch.randn(B * OH * OW, k * k * C, device="cuda").to(torch.bfloat16)
    x_act = torch.relu(torch.randn(B, H, W, C, device="cuda")).to(torch.bfloat16)
    dx = G.col2im(dcol, x_act, B, H, W, C, k, s)
    d = dcol.float().view(B, OH * OW, k, k, C).permute(0, 4, 2, 3, 1).reshape(B, C * k * k, OH * OW)
    ref = F.fold(d, (H, W), k, stride=s).permute(0, 2, 3, 1) * (x_act.float() > 0)
    torch.testing.assert_close(dx.float(), ref, rtol=1e-2, atol=2e-2)


@pytest.mark.parametrize("M,N", [(15_237, 32), (100_003, 64), (4099, 512), (777, 72), (1000, 20)])
def test_colsum(M, N):
    x = torch.randn(M, N, device="cuda").to(torch.bfloat16)
    out = torch.full((N,), 0.5, device="cuda")
    G.colsum(x, out)
    torch.testing.assert_close(out, x.float().sum(0) + 0.5, rtol=1e-4, atol=1e-2)
