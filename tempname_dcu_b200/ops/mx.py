"""Block-scaled FP8 ("MXFP8") quantizer and tcgen05 ``kind::mxf8f6f4`` GEMM
(``csrc/gemm_mx.cu`` on the mainloop of ``csrc/gemm.cuh``).

Format: e4m3 values, one power-of-two scale (ue8m0 byte ``e + 127``) per 32
consecutive K values of a row.  The scale of a block with absolute maximum
``a`` is the smallest ``2^e`` with ``a / 2^e <= 448``, so nothing saturates.
Scales are stored in 512-byte atoms (one per 128 rows x 128 K values, in
K-chunk-major order) laid out as the tensor cores read them; ``scales_dense``
unpacks them to ``[rows, K/32]`` for inspection and for the references.

The selective arm can run its calibrated blocks through this path (the
reference quantizes those blocks on the wire only: python/flux_dcu/runtime.py:
196-197).
"""
from __future__ import annotations

import ctypes

from . import native

native.register("tdb_mx_scale_bytes", [ctypes.c_longlong, ctypes.c_longlong], restype=ctypes.c_longlong)
native.register("tdb_mx_quantize", [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                    ctypes.c_void_p, ctypes.c_void_p])
native.register("tdb_mx_quantize_versioned", [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_void_p])
native.register("tdb_gemm_mx", [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                 ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_void_p, ctypes.c_void_p])

E4M3_MAX = 448.0


def scale_bytes(rows: int, k: int) -> int:
    return rows // 128 * (k // 128) * 512


def quantize(x, q=None, sf=None, stream=None, version=None, seen=None):
    """bf16 ``x`` [rows, K] (rows, K multiples of 128) -> (q uint8 [rows, K]
    holding e4m3 bits, sf uint8 scale atoms).  With ``version`` / ``seen``
    (device int32 scalars) the work is skipped on the device while
    ``version == seen`` and ``seen`` takes ``version`` afterwards."""
    import torch
    rows, k = x.shape
    if x.dtype != torch.bfloat16 or x.stride(-1) != 1:
        raise TypeError("quantize expects bf16 rows with a contiguous last dimension")
    if rows % 128 or k % 128:
        raise ValueError("rows and K must be multiples of 128")
    if q is None:
        q = torch.empty((rows, k), dtype=torch.uint8, device=x.device)
    if sf is None:
        sf = torch.empty(scale_bytes(rows, k), dtype=torch.uint8, device=x.device)
    if (version is None) != (seen is None):
        raise ValueError("version and seen go together")
    for t in (version, seen):
        if t is not None and (t.dtype != torch.int32 or t.numel() != 1 or not t.is_cuda):
            raise ValueError("version / seen must be device int32 scalars")
    native.check(native.lib().tdb_mx_quantize_versioned(
        x.data_ptr(), x.stride(0), rows, k, q.data_ptr(), sf.data_ptr(), 0 if version is None else version.data_ptr(),
        0 if seen is None else seen.data_ptr(), native.stream_ptr(stream)), "mx quantize")
    return q, sf


def gemm(qa, sfa, qb, sfb, *, bias=None, out=None, stream=None):
    """``out[M, N] = dequant(qa) @ dequant(qb)^T (+ bias)`` in bf16 with fp32
    accumulation; qa [M, K], qb [N, K] from ``quantize``."""
    import torch
    m, k = qa.shape
    n, kb = qb.shape
    if k != kb or m % 128 or n % 128 or k % 128:
        raise ValueError("M, N, K must be multiples of 128 and the K extents equal")
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=qa.device)
    if bias is not None and (bias.dtype != torch.bfloat16 or bias.numel() != n or not bias.is_contiguous()):
        raise ValueError("bias must be a contiguous bf16 vector of length N")
    native.check(native.lib().tdb_gemm_mx(qa.data_ptr(), sfa.data_ptr(), qb.data_ptr(), sfb.data_ptr(),
                                          out.data_ptr(), out.stride(0), m, n, k, 1 if bias is not None else 0,
                                          0 if bias is None else bias.data_ptr(), native.stream_ptr(stream)),
                 "mx gemm")
    return out


def scales_dense(sf, rows: int, k: int):
    """Scale atoms -> ue8m0 bytes [rows, K/32] (row r, K block j)."""
    import torch
    atoms = sf.view(k // 128, rows // 128, 32, 4, 4)  # kc, blk, row % 32, row group, j
    # [blk, group, lane, kc, j] -> rows in order blk*128 + group*32 + lane
    return atoms.permute(1, 3, 2, 0, 4).reshape(rows, k // 32)


def dequantize(q, sf):
    """fp32 values of an operand produced by ``quantize``."""
    import torch
    rows, k = q.shape
    scale = torch.exp2(scales_dense(sf, rows, k).float() - 127.0)
    values = q.view(torch.float8_e4m3fn).float()
    return (values.view(rows, k // 32, 32) * scale.unsqueeze(-1)).view(rows, k)


def quantize_reference(x):
    """CPU/torch restatement of the quantizer: (e4m3 values as fp32, scale
    exponents [rows, K/32]) -- used to check the kernel bit for bit."""
    import torch
    rows, k = x.shape
    blocks = x.float().view(rows, k // 32, 32)
    amax = blocks.abs().amax(-1)
    mant, exp = torch.frexp(amax)  # amax = mant * 2^exp, mant in [0.5, 1)
    # amax = (2 mant) 2^(exp-1); need the smallest e with amax / 2^e <= 448 = 1.75 * 2^8
    e = (exp - 1 - 8) + (2 * mant > 1.75).to(exp.dtype)
    e = torch.where(amax > 0, e, torch.full_like(e, -127)).clamp(-127, 127)
    scaled = blocks / torch.exp2(e.float()).unsqueeze(-1)
    values = scaled.to(torch.float8_e4m3fn).float()
    return values.view(rows, k), e


def pack_scales(e, rows: int, k: int):
    """Inverse of ``scales_dense``: exponents [rows, K/32] -> scale atoms."""
    import torch
    dense = (e + 127).to(torch.uint8).view(rows // 128, 4, 32, k // 128, 4)  # blk, group, lane, kc, j
    return dense.permute(3, 0, 2, 1, 4).contiguous().view(-1)  # kc, blk, lane, group, j
