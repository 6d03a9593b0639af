"""Tensor-core GEMM and the convolution helpers built on it.

``gemm(A, B, ...)`` computes D = A @ B^T on the sm_100a tcgen05 kernel
(csrc/kernels/gemm_tc.cu) with a fused epilogue. Operand conventions:

* ``A`` is (M, K) row-major, or with ``a_mn=True`` (K, M) row-major;
* ``B`` is (N, K) row-major, or with ``b_mn=True`` (K, N) row-major.

So the three products of a linear layer Y = X W^T are, with no transposes:
forward ``gemm(X, W)``; data gradient ``gemm(dY, W, b_mn=True)``; weight
gradient ``gemm(dY, X, a_mn=True, b_mn=True)`` (reduction over the batch).

``gemm_reference`` is the fp32 PyTorch oracle of the same contract.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_void_p
from typing import Optional

import torch

from . import _lib
from ._lib import check, ptr, stream_ptr

NLIB = "libsurf_nn.so"
ACT = {"none": 0, "relu": 1, "tanh": 2, "relu_grad": 3, "tanh_grad": 4}


class Epilogue(ctypes.Structure):
    _fields_ = [("c", c_void_p), ("ldc", c_int64), ("c_dtype", c_int), ("c_mode", c_int), ("ct", c_void_p),
                ("ldct", c_int64), ("ct_dtype", c_int), ("bias", c_void_p), ("act", c_int), ("act2", c_int),
                ("act_split", c_int), ("aux", c_void_p), ("ld_aux", c_int64), ("err", c_void_p), ("dbg", c_int),
                ("trace", c_void_p), ("cmap_in", c_int), ("cmap_out", c_int)]
TRACE_N = 256              # stamps per kind in an Epilogue.trace buffer (kTraceN in gemm_tc.cu)


_SIG = {
    "surf_gemm_bf16": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_int64, c_int, c_int, c_int, c_int,
                               ctypes.POINTER(Epilogue), c_int, c_int, c_void_p]),
    "surf_gemm_epilogue_size": (c_int, []),
    "surf_im2col": (c_int, [c_void_p] + [c_int] * 7 + [c_void_p, c_int64, c_void_p]),
    "surf_col2im": (c_int, [c_void_p, c_int64, c_void_p, c_void_p] + [c_int] * 8 + [c_void_p]),
    "surf_colsum": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int, c_void_p, c_void_p]),
    "surf_gather_rows": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int, c_void_p, c_int64, c_int64,
                                 c_void_p, c_void_p]),
    "surf_f32_to_bf16": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int, c_void_p]),
    "surf_adam_norm": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p]),
    "surf_adam_acc_size": (c_int, []),
    "surf_adam_update": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p,
                                 c_void_p]),
}
_lib.register(NLIB, _SIG)

_err_flags: dict = {}


ERROR_CODES = {1: "GEMM producer wait timed out", 2: "GEMM MMA wait timed out", 3: "GEMM epilogue wait timed out",
               4: "GEMM accumulator wait timed out", 5: "GEMM resident-operand wait timed out",
               0x100: "row gather index out of range", 0x101: "frame-stack index out of range",
               0x102: "PPO loss sample index out of range"}


def error_flag(device) -> torch.Tensor:
    """Per-device int32 flag the kernels set on a bounded-wait timeout or an
    out-of-range index (first code wins; see ERROR_CODES)."""
    key = torch.device(device)
    if key.type == "cuda" and key.index is None:      # "cuda" and "cuda:<current>" share one flag
        key = torch.device("cuda", torch.cuda.current_device())
    if key not in _err_flags:
        _err_flags[key] = torch.zeros(1, dtype=torch.int32, device=key)
    return _err_flags[key]


def check_error_flag(device) -> None:
    """Raise KernelError (and clear the flag) if a kernel reported an error."""
    f = error_flag(device)
    v = int(f.item())
    if v:
        f.zero_()
        raise _lib.KernelError(f"device error {v:#x}: {ERROR_CODES.get(v, 'unknown code')}")


def _pick_bn(n: int, b_mn: bool, m: Optional[int] = None) -> int:
    """Tile width: the narrowest that covers N, else 256 -- unless the GEMM
    has few 128-row tiles (small M), where wider tiles leave most SMs idle
    and a handful of CTAs run every epilogue: then the widest width that
    still gives at least 148 tiles (64 at the least; measured at M = 1024:
    N = 512 x K = 768 takes 10.9 us at 64 against 19.3 us at 256)."""
    cover = next((bn for bn in (32, 64, 128, 256) if n <= bn and (bn >= 64 or not b_mn)), 256)
    if m is not None and cover > 64:
        mt = (m + 127) // 128
        for bn in (256, 128):
            if bn <= cover and mt * ((n + bn - 1) // bn) >= 148:
                return bn
        return 64
    return cover


def gemm(A: torch.Tensor, B: torch.Tensor, *, a_mn: bool = False, b_mn: bool = False,
         out: Optional[torch.Tensor] = None, out_dtype=torch.bfloat16, accumulate: bool = False,
         out_t: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None, act: str = "none",
         act2: Optional[str] = None, act_split: Optional[int] = None, aux: Optional[torch.Tensor] = None,
         splits: int = 1, bn: Optional[int] = None, M: Optional[int] = None, N: Optional[int] = None,
         K: Optional[int] = None, debug: int = 0, cmap: Optional[tuple] = None) -> Optional[torch.Tensor]:
    """D = A @ B^T (bf16 operands, fp32 accumulation) with a fused epilogue:
    ``+ bias``, activation (``relu``/``tanh``) or activation derivative
    (``relu_grad``/``tanh_grad`` against ``aux``, the saved activation), and
    stores to ``out`` (fp32/bf16, any row stride), ``out_t`` (transposed) or
    fp32 atomic accumulation (``accumulate=True``; required for ``splits>1``).
    ``act2``/``act_split`` switch the activation at a column boundary.
    ``cmap = (n_in, n_out)`` stores column n of ``out`` at (n // n_in) * n_out
    + n % n_in (a dense row onto a zero-padded grid; bias and aux stay dense)."""
    if A.dtype != torch.bfloat16 or B.dtype != torch.bfloat16:
        raise TypeError("gemm operands must be bfloat16")
    _lib.require_cuda(A, "gemm")
    if A.stride(-1) != 1 or B.stride(-1) != 1:
        raise ValueError("gemm operands need unit column stride")
    if (A.data_ptr() | B.data_ptr()) & 15 or (A.stride(0) | B.stride(0)) & 7:
        raise ValueError("gemm operands need 16-byte aligned bases and row strides (TMA)")
    if M is None:
        M = A.shape[1] if a_mn else A.shape[0]
    if K is None:
        K = A.shape[0] if a_mn else A.shape[1]
    if N is None:
        N = B.shape[1] if b_mn else B.shape[0]
    if out is None and out_t is None:
        out = torch.empty((M, N), dtype=torch.float32 if accumulate else out_dtype, device=A.device)
    ep = Epilogue()
    if out is not None:
        ep.c = ptr(out)
        ep.ldc = out.stride(0)
        ep.c_dtype = 1 if out.dtype == torch.bfloat16 else 0
        ep.c_mode = 1 if accumulate else 0
        if accumulate and out.dtype != torch.float32:
            raise TypeError("accumulate needs a float32 output")
    if out_t is not None:
        ep.ct = ptr(out_t)
        ep.ldct = out_t.stride(0)
        ep.ct_dtype = 1 if out_t.dtype == torch.bfloat16 else 0
    ep.bias = ptr(bias)
    ep.act = ACT[act]
    ep.act2 = ACT[act2 or act]
    ep.act_split = N if act_split is None else int(act_split)
    if aux is not None:
        ep.aux = ptr(aux)
        ep.ld_aux = aux.stride(0)
    elif ep.act in (3, 4) or ep.act2 in (3, 4):
        raise ValueError("activation-derivative epilogues need aux")
    ep.err = ptr(error_flag(A.device))
    ep.dbg = int(debug)
    if cmap is not None:
        ep.cmap_in, ep.cmap_out = int(cmap[0]), int(cmap[1])
    lda, ldb = A.stride(0), B.stride(0)
    check(_lib.lib(NLIB).surf_gemm_bf16(ptr(A), lda, int(a_mn), ptr(B), ldb, int(b_mn), int(M), int(N), int(K),
                                        ctypes.byref(ep), int(bn or _pick_bn(N, b_mn, None if splits > 1 else M)),
                                        int(splits),
                                        stream_ptr(A.device)), "surf_gemm_bf16")
    return out if out is not None else out_t


_ACT_FN = {
    "none": lambda x, a: x, "relu": lambda x, a: torch.relu(x), "tanh": lambda x, a: torch.tanh(x),
    "relu_grad": lambda x, a: x * (a > 0).to(x.dtype), "tanh_grad": lambda x, a: x * (1 - a * a),
}


def gemm_reference(A, B, *, a_mn=False, b_mn=False, bias=None, act="none", act2=None, act_split=None, aux=None):
    """fp32 oracle of ``gemm`` (returns the fp32 result)."""
    a = A.float().t() if a_mn else A.float()
    b = B.float() if b_mn else B.float().t()
    d = a @ b
    if bias is not None:
        d = d + bias.float()
    auxf = aux.float() if aux is not None else None
    split = d.shape[1] if act_split is None else act_split
    lo = _ACT_FN[act](d[:, :split], None if auxf is None else auxf[:, :split])
    hi = _ACT_FN[act2 or act](d[:, split:], None if auxf is None else auxf[:, split:])
    return torch.cat([lo, hi], 1)


# ---- convolution helpers ------------------------------------------------------
def conv_out(h: int, w: int, k: int, s: int):
    return (h - k) // s + 1, (w - k) // s + 1


def im2col(x: torch.Tensor, B: int, H: int, W: int, C: int, k: int, s: int, out: Optional[torch.Tensor] = None):
    """NHWC bf16 -> patch rows [B*OH*OW, k*k*C] in (kh, kw, c) order."""
    oh, ow = conv_out(H, W, k, s)
    if out is None:
        out = torch.empty((B * oh * ow, k * k * C), dtype=torch.bfloat16, device=x.device)
    check(_lib.lib(NLIB).surf_im2col(ptr(x), B, H, W, C, k, k, s, ptr(out), out.stride(0), stream_ptr(x.device)),
          "surf_im2col")
    return out


def col2im(dcol: torch.Tensor, x_act: Optional[torch.Tensor], B: int, H: int, W: int, C: int, k: int, s: int,
           out: Optional[torch.Tensor] = None):
    """Patch-row gradients -> NHWC input gradient, times ReLU'(x_act) if given."""
    if out is None:
        out = torch.empty((B, H, W, C), dtype=torch.bfloat16, device=dcol.device)
    check(_lib.lib(NLIB).surf_col2im(ptr(dcol), dcol.stride(0), ptr(x_act), ptr(out), B, H, W, C, k, k, s,
                                     1 if x_act is not None else 0, stream_ptr(dcol.device)), "surf_col2im")
    return out


def colsum(x: torch.Tensor, out: torch.Tensor, rows: Optional[int] = None, cols: Optional[int] = None):
    """out += x.sum(0) (fp32 accumulation; x bf16 or fp32, any row stride)."""
    M = x.shape[0] if rows is None else rows
    N = x.shape[1] if cols is None else cols
    check(_lib.lib(NLIB).surf_colsum(ptr(x), 1 if x.dtype == torch.bfloat16 else 0, x.stride(0), M, N, ptr(out),
                                     stream_ptr(x.device)), "surf_colsum")
    return out


def gather_rows(src: torch.Tensor, idx: torch.Tensor, out: torch.Tensor, offset: int = 0):
    """out[i] = src[idx[i] + offset] for 2-D tensors (row bytes multiple of 4)."""
    row_bytes = src.shape[1] * src.element_size()
    check(_lib.lib(NLIB).surf_gather_rows(ptr(src), src.stride(0) * src.element_size(), ptr(idx), int(offset),
                                          idx.numel(), row_bytes, ptr(out), out.stride(0) * out.element_size(),
                                          src.shape[0], ptr(error_flag(src.device)), stream_ptr(src.device)),
          "surf_gather_rows")
    return out


def to_bf16(x: torch.Tensor, out: torch.Tensor):
    check(_lib.lib(NLIB).surf_f32_to_bf16(ptr(x), x.stride(0), ptr(out), out.stride(0), x.shape[0], x.shape[1],
                                          stream_ptr(x.device)), "surf_f32_to_bf16")
    return out
