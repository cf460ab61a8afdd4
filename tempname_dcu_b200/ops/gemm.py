"""tcgen05 GEMM entry points (``csrc/gemm.cuh`` + ``csrc/gemm.cu``).

``gemm`` is the general form ``C = epilogue(A_logical @ B_logical^T)`` with
A_logical [M, K] and B_logical [N, K]; each operand may be supplied either in
its logical layout (K contiguous, "K-major") or transposed (its M/N dimension
contiguous, "MN-major").  The three shapes of a linear layer map to:

* forward        ``x[M,K] @ w[N,K]^T``           ``linear(x, w)``
* data gradient  ``dy[M,N] @ w[N,K]``            ``matmul_nt(dy, w)``  (B MN-major)
* weight grad    ``dw[N,K] (+)= dy^T @ x``        ``weight_grad(dy, x)`` (A, B MN-major)

Epilogues are fused into the kernel: bias, bias+GELU (saving the
pre-activation), GELU backward, bias+residual, fp32 accumulate.
"""
from __future__ import annotations

import ctypes

from . import native

STORE, BIAS, BIAS_GELU, GELU_BWD, ACC_F32, BIAS_RESIDUAL = range(6)

native.register("tdb_gemm", [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int,
                             ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                             ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                             ctypes.c_void_p, ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_void_p])


def _torch():
    import torch
    return torch


def _ptr(t):
    return 0 if t is None else t.data_ptr()


def gemm(a, b, *, a_mn=False, b_mn=False, out=None, mode=STORE, bias=None, aux=None, aux_out=None,
         alpha=1.0, beta=0.0, bn=0, stream=None):
    """General entry.  ``a`` is [M,K] (or [K,M] if a_mn); ``b`` is [N,K] (or
    [K,N] if b_mn).  Inner dimensions must be contiguous (row stride is taken
    from ``stride(0)``)."""
    torch = _torch()
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise TypeError("gemm operands must be bf16")
    if a.stride(-1) != 1 or b.stride(-1) != 1:
        raise ValueError("gemm operands need a contiguous inner dimension")
    M, K = (a.shape[1], a.shape[0]) if a_mn else (a.shape[0], a.shape[1])
    N, Kb = (b.shape[1], b.shape[0]) if b_mn else (b.shape[0], b.shape[1])
    if K != Kb:
        raise ValueError(f"gemm inner dimensions differ: {K} vs {Kb}")
    if out is None:
        dtype = torch.float32 if mode == ACC_F32 else torch.bfloat16
        out = torch.empty((M, N), dtype=dtype, device=a.device)
    if out.stride(-1) != 1 or tuple(out.shape) != (M, N):
        raise ValueError("gemm output must be [M, N] with a contiguous last dimension")
    if mode == ACC_F32 and out.dtype != torch.float32:
        raise TypeError("ACC_F32 writes an fp32 output")
    if mode != ACC_F32 and out.dtype != torch.bfloat16:
        raise TypeError("bf16 epilogues write a bf16 output")
    ld_aux = 0
    if aux is not None:
        ld_aux = aux.stride(0)
    if aux_out is not None:
        ld_aux = aux_out.stride(0)
    if bias is not None and (bias.dtype != torch.bfloat16 or not bias.is_contiguous() or bias.numel() != N):
        raise ValueError("bias must be a contiguous bf16 vector of length N")
    native.check(native.lib().tdb_gemm(a.data_ptr(), int(a_mn), a.stride(0), b.data_ptr(), int(b_mn), b.stride(0),
                                       out.data_ptr(), out.stride(0), M, N, K, mode, _ptr(bias), _ptr(aux), ld_aux,
                                       _ptr(aux_out), float(alpha), float(beta), int(bn),
                                       native.stream_ptr(stream)), "tcgen05 gemm")
    return out


def linear(x, w, bias=None, out=None):
    """``x @ w^T (+ bias)``; x [M,K], w [N,K]."""
    return gemm(x, w, out=out, mode=BIAS if bias is not None else STORE, bias=bias)


def linear_gelu(x, w, bias, pre_out=None, out=None):
    """Returns (gelu(x@w^T+b), pre-activation) from one kernel."""
    torch = _torch()
    M, N = x.shape[0], w.shape[0]
    if pre_out is None:
        pre_out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    y = gemm(x, w, out=out, mode=BIAS_GELU, bias=bias, aux_out=pre_out)
    return y, pre_out


def linear_residual(x, w, bias, residual, out=None):
    """``x @ w^T + bias + residual``."""
    return gemm(x, w, out=out, mode=BIAS_RESIDUAL, bias=bias, aux=residual)


def matmul_nt(dy, w, out=None, gelu_pre=None):
    """``dy[M,N] @ w[N,K] -> [M,K]`` (optionally times gelu'(gelu_pre))."""
    if gelu_pre is not None:
        return gemm(dy, w, b_mn=True, out=out, mode=GELU_BWD, aux=gelu_pre)
    return gemm(dy, w, b_mn=True, out=out)


def weight_grad(dy, x, out_f32=None, accumulate=True):
    """``out_f32[N,K] (+)= dy[M,N]^T @ x[M,K]`` in fp32."""
    torch = _torch()
    if out_f32 is None:
        out_f32 = torch.zeros((dy.shape[1], x.shape[1]), dtype=torch.float32, device=dy.device)
        accumulate = False
    return gemm(dy, x, a_mn=True, b_mn=True, out=out_f32, mode=ACC_F32, beta=1.0 if accumulate else 0.0)
