"""tcgen05 GEMM and conv helpers vs fp32 PyTorch references (GPU)."""
import pytest
import torch

from surfb200.ops import gemm as G

pytestmark = pytest.mark.gpu


def rand(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


def padded(rows, cols):
    """A [rows, cols] view whose row stride is padded to a multiple of 8 (TMA rule)."""
    ld = (cols + 7) // 8 * 8
    return rand(rows, ld)[:, :cols]


def operands(M, N, K, a_mn, b_mn):
    A = padded(K, M) if a_mn else padded(M, K)
    B = padded(K, N) if b_mn else padded(N, K)
    return A, B


def close(x, ref, tol=2e-2):
    err = (x.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= tol * scale, f"max err {err} vs scale {scale}"


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (True, False), (False, True), (True, True)])
@pytest.mark.parametrize("M,N,K", [(128, 64, 64), (300, 200, 150), (1024, 256, 512), (257, 96, 1000)])
def test_gemm_majorness_and_tails(a_mn, b_mn, M, N, K):
    torch.manual_seed(0)
    A, B = operands(M, N, K, a_mn, b_mn)
    out = G.gemm(A, B, a_mn=a_mn, b_mn=b_mn, out_dtype=torch.float32)
    torch.cuda.synchronize()
    G.check_error_flag("cuda")
    close(out, G.gemm_reference(A, B, a_mn=a_mn, b_mn=b_mn), 1e-2)


@pytest.mark.parametrize("bn", [32, 64, 128, 256])
def test_gemm_tile_widths(bn):
    A, B = operands(512, 250, 320, False, False)
    out = G.gemm(A, B, bn=bn, out_dtype=torch.float32)
    close(out, G.gemm_reference(A, B), 1e-2)


def test_epilogue_bias_act_bf16_and_transpose():
    A, B = operands(384, 192, 256, False, False)
    bias = torch.randn(192, device="cuda")
    out = torch.empty(384, 200, dtype=torch.bfloat16, device="cuda")        # row stride 200 > N
    out_t = torch.empty(192, 384, dtype=torch.bfloat16, device="cuda")
    G.gemm(A, B, out=out[:, :192], out_t=out_t, bias=bias, act="tanh")
    ref = G.gemm_reference(A, B, bias=bias, act="tanh")
    close(out[:, :192], ref)
    close(out_t.t(), ref)
    G.gemm(A, B, out=out[:, :192], bias=bias, act="relu")
    close(out[:, :192], G.gemm_reference(A, B, bias=bias, act="relu"))


def test_epilogue_derivatives_and_split():
    A, B = operands(256, 128, 64, False, True)
    aux = rand(256, 128)
    out = G.gemm(A, B, b_mn=True, act="relu_grad", act2="tanh_grad", act_split=64, aux=aux, out_dtype=torch.float32)
    ref = G.gemm_reference(A, B, b_mn=True, act="relu_grad", act2="tanh_grad", act_split=64, aux=aux)
    close(out, ref)


@pytest.mark.parametrize("splits", [1, 7, 40])
def test_split_k_atomic_weight_gradient(splits):
    # dW = dY^T X with the batch as reduction: both operands MN-major
    dY, X = rand(4096, 64), rand(4096, 576)
    dW = torch.zeros(64, 576, device="cuda")
    G.gemm(dY, X, a_mn=True, b_mn=True, out=dW, accumulate=True, splits=splits)
    close(dW, dY.float().t() @ X.float(), 1e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_column_remap_onto_padded_grid(dtype):
    """cmap = (n_in, n_out): dense column n lands at (n // n_in) * n_out +
    n % n_in of a wider row (the FC input gradient written onto the trunk's
    zero-padded grid); the padding columns stay untouched, the saved
    activation of the derivative epilogue stays dense."""
    torch.manual_seed(3)
    M, N, K = 1000, 3072, 512
    A, B = operands(M, N, K, False, True)
    aux = rand(M, N)
    out = torch.full((M, 8192), 7.0, dtype=dtype, device="cuda")
    G.gemm(A, B, b_mn=True, out=out, act="relu_grad", aux=aux, cmap=(768, 1024))
    torch.cuda.synchronize()
    G.check_error_flag("cuda")
    ref = G.gemm_reference(A, B, b_mn=True, act="relu_grad", aux=aux)
    cols = torch.arange(N, device="cuda")
    dst = (cols // 768) * 1024 + cols % 768
    close(out[:, dst], ref)
    pad = torch.ones(8192, dtype=torch.bool, device="cuda")
    pad[dst] = False
    assert bool((out[:, pad] == 7.0).all())


def test_narrow_mn_operand():
    """Weight gradient of a 32-channel layer: an MN-major operand narrower than the 64-wide box."""
    col, dy = rand(8192, 64), rand(8192, 32)
    dWt = torch.zeros(64, 32, device="cuda")
    G.gemm(col, dy, a_mn=True, b_mn=True, out=dWt, accumulate=True, splits=16)
    close(dWt, col.float().t() @ dy.float(), 1e-2)


def test_conv_via_im2col_matches_torch():
    torch.manual_seed(1)
    B, H, W, C, k, s, CO = 8, 15, 31, 32, 4, 2, 64
    x = torch.relu(torch.randn(B, H, W, C, device="cuda")).to(torch.bfloat16)
    w = (torch.randn(CO, C, k, k, device="cuda") * 0.1)
    wk = w.permute(0, 2, 3, 1).reshape(CO, k * k * C).to(torch.bfloat16)   # (kh, kw, c) order
    col = G.im2col(x, B, H, W, C, k, s)
    y = G.gemm(col, wk, out_dtype=torch.float32)
    ref = torch.nn.functional.conv2d(x.float().permute(0, 3, 1, 2), wk.float().reshape(CO, k, k, C).permute(0, 3, 1, 2),
                                     stride=s)
    close(y.reshape(B, *G.conv_out(H, W, k, s), CO), ref.permute(0, 2, 3, 1), 1e-2)
    # data gradient through col2im with the ReLU derivative of x
    dy = rand(B * y.shape[0] // B, CO)
    dcol = G.gemm(dy, wk, b_mn=True, out_dtype=torch.bfloat16)
    dx = G.col2im(dcol, x, B, H, W, C, k, s)
    xr = x.float().permute(0, 3, 1, 2).requires_grad_(True)
    yr = torch.nn.functional.conv2d(xr, wk.float().reshape(CO, k, k, C).permute(0, 3, 1, 2), stride=s)
    yr.backward(dy.float().reshape(B, *G.conv_out(H, W, k, s), CO).permute(0, 3, 1, 2))
    ref_dx = (xr.grad * (x.float().permute(0, 3, 1, 2) > 0)).permute(0, 2, 3, 1)
    close(dx, ref_dx, 3e-2)


def test_colsum_and_gather():
    x = rand(1000, 70)
    out = torch.zeros(70, device="cuda")
    G.colsum(x, out)
    close(out, x.float().sum(0), 1e-3)
    src = torch.randn(500, 16, device="cuda")
    idx = torch.randint(0, 400, (123,), device="cuda")
    dst = torch.empty(123, 16, device="cuda")
    G.gather_rows(src, idx, dst, offset=50)
    torch.testing.assert_close(dst, src[idx + 50])
    # image-sized rows (16 KB): the 16-byte vector path, bit-exact
    img = rand(3000, 8192)
    idx = torch.randint(0, 2900, (777,), device="cuda")
    got = torch.empty(777, 8192, dtype=torch.bfloat16, device="cuda")
    G.gather_rows(img, idx, got, offset=7)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), img[idx + 7].view(torch.int16))
