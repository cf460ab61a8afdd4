"""Python entry points of the non-GEMM sm_100a kernels.

Each function validates shapes/dtypes, allocates outputs when not given and
launches one native entry point on the current stream.  Kernels:
``csrc/layernorm.cu``, ``csrc/attention.cu``, ``csrc/xent.cu``,
``csrc/optim.cu``, ``csrc/embedding.cu``.
"""
from __future__ import annotations

import ctypes
import math

from . import native

V, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float

native.register("tdb_layernorm_fwd", [V, V, V, V, V, V, I, I, F, V])
native.register("tdb_layernorm_bwd", [V, V, V, V, V, V, V, V, V, V, I, I, I, V])
native.register("tdb_layernorm_bwd_scratch_floats", [I, I])
native.register("tdb_attn_fwd", [V, I64, V, I64, V, I, I, I, F, V])
native.register("tdb_attn_fwd_tc", [V, I64, V, I64, V, I, I, I, F, V])
native.register("tdb_attn_bwd", [V, I64, V, I64, V, I64, V, V, V, I64, I, I, I, F, V])
native.register("tdb_attn_bwd_tc", [V, I64, V, I64, V, I64, V, V, V, I64, I, I, I, F, V])
native.register("tdb_xent_stats", [V, I64, V, I64, I, I, I, V, V])
native.register("tdb_xent_combine", [V, I, I, V, V, V, F, I, V])
native.register("tdb_xent_grad", [V, I64, V, I64, I, I, I, V, F, V])
native.register("tdb_sumsq_partials_count", [])
native.register("tdb_sumsq", [V, I64, V, V, I, V])
native.register("tdb_clip_coef", [V, F, V, V, V, V, V, V])
native.register("tdb_adamw", [V, V, V, V, V, I64, I64, I64, I64, I64, F, F, F, F, F, I, V, V, I, V, V])
native.register("tdb_to_bf16", [V, V, I64, V])
native.register("tdb_embedding_fwd", [V, V, I64, I64, V, I64, I, I, I, V, V])
native.register("tdb_add_positions", [V, V, I64, I, I, I, V])
native.register("tdb_embedding_bwd", [V, V, I, V, I64, I64, I, V, V])
native.register("tdb_position_bwd", [V, I, I64, I, I, V, V])


def _t():
    import torch
    return torch


def _p(x):
    return 0 if x is None else x.data_ptr()


def _s(stream=None):
    return native.stream_ptr(stream)


def _need(cond, msg):
    if not cond:
        raise ValueError(msg)


# ---------------------------------------------------------------- LayerNorm
def layernorm_fwd(x, weight, bias, eps=1e-5, out=None, mean=None, rstd=None):
    torch = _t()
    rows, H = x.shape
    _need(x.is_contiguous() and x.dtype == torch.bfloat16, "layernorm input must be contiguous bf16")
    out = torch.empty_like(x) if out is None else out
    mean = torch.empty(rows, dtype=torch.float32, device=x.device) if mean is None else mean
    rstd = torch.empty(rows, dtype=torch.float32, device=x.device) if rstd is None else rstd
    native.check(native.lib().tdb_layernorm_fwd(x.data_ptr(), weight.data_ptr(), bias.data_ptr(), out.data_ptr(),
                                                mean.data_ptr(), rstd.data_ptr(), rows, H, float(eps), _s()),
                 "layernorm fwd")
    return out, mean, rstd


def layernorm_scratch_floats(rows, H):
    return int(native.lib().tdb_layernorm_bwd_scratch_floats(rows, H))


def layernorm_bwd(x, weight, mean, rstd, dy, dgamma, dbeta, scratch, dres=None, dx=None, accumulate=True):
    """dx = LN backward (+ dres); dgamma/dbeta (fp32) (+)= parameter grads."""
    torch = _t()
    rows, H = x.shape
    dx = torch.empty_like(x) if dx is None else dx
    _need(scratch.numel() >= layernorm_scratch_floats(rows, H), "layernorm scratch too small")
    native.check(native.lib().tdb_layernorm_bwd(x.data_ptr(), weight.data_ptr(), mean.data_ptr(), rstd.data_ptr(),
                                                dy.data_ptr(), _p(dres), dx.data_ptr(), dgamma.data_ptr(),
                                                dbeta.data_ptr(), scratch.data_ptr(), rows, H, int(accumulate), _s()),
                 "layernorm bwd")
    return dx


# ---------------------------------------------------------------- attention
def attention_fwd(qkv, mb, seq, heads_local, out=None, lse=None, scale=None, impl=None):
    """qkv [mb*seq, 3*Hl*128] -> (out [mb*seq, Hl*128], lse [mb, Hl, seq]).

    impl "tc" = tcgen05/TMEM kernel (attn_tc.cu, needs seq % 128 == 0 and
    16-byte aligned rows), "mma" = the mma.sync kernel (attention.cu, any
    seq); default: "tc" whenever it applies."""
    torch = _t()
    D = 128
    _need(qkv.shape[1] >= 3 * heads_local * D and qkv.stride(1) == 1, "qkv must be [tokens, 3*Hl*128]")
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    out = torch.empty((mb * seq, heads_local * D), dtype=torch.bfloat16, device=qkv.device) if out is None else out
    lse = torch.empty((mb, heads_local, seq), dtype=torch.float32, device=qkv.device) if lse is None else lse
    if impl is None:
        impl = "tc" if seq % 128 == 0 and qkv.stride(0) % 8 == 0 and out.stride(0) % 8 == 0 \
            and qkv.data_ptr() % 16 == 0 and out.data_ptr() % 16 == 0 else "mma"
    fn = native.lib().tdb_attn_fwd_tc if impl == "tc" else native.lib().tdb_attn_fwd
    native.check(fn(qkv.data_ptr(), qkv.stride(0), out.data_ptr(), out.stride(0), lse.data_ptr(), mb, seq,
                    heads_local, float(scale), _s()), f"attention fwd ({impl})")
    return out, lse


def attention_bwd(qkv, out, dout, lse, mb, seq, heads_local, dqkv=None, dsum=None, scale=None, impl=None):
    """dqkv [mb*seq, 3*Hl*128] from (qkv, out, dout, lse); deterministic.

    impl "tc" = tcgen05 kernels (attn_tc.cu, seq % 128 == 0, 16-byte aligned
    rows), "mma" = mma.sync kernels (attention.cu); default "tc" when it applies."""
    torch = _t()
    D = 128
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    dqkv = torch.empty_like(qkv) if dqkv is None else dqkv
    dsum = torch.empty((mb, heads_local, seq), dtype=torch.float32, device=qkv.device) if dsum is None else dsum
    if impl is None:
        aligned = all(t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0 for t in (qkv, dout, dqkv)) \
            and lse.data_ptr() % 16 == 0 and dsum.data_ptr() % 16 == 0
        impl = "tc" if seq % 128 == 0 and aligned else "mma"
    fn = native.lib().tdb_attn_bwd_tc if impl == "tc" else native.lib().tdb_attn_bwd
    native.check(fn(qkv.data_ptr(), qkv.stride(0), out.data_ptr(), out.stride(0), dout.data_ptr(), dout.stride(0),
                    lse.data_ptr(), dsum.data_ptr(), dqkv.data_ptr(), dqkv.stride(0), mb, seq, heads_local,
                    float(scale), _s()), f"attention bwd ({impl})")
    return dqkv


# ---------------------------------------------------------------- cross-entropy
def xent_stats(logits, targets, vocab_start, valid_cols, stats=None):
    torch = _t()
    rows, cols = logits.shape
    stats = torch.empty((rows, 3), dtype=torch.float32, device=logits.device) if stats is None else stats
    native.check(native.lib().tdb_xent_stats(logits.data_ptr(), logits.stride(0), targets.data_ptr(),
                                             int(vocab_start), int(valid_cols), cols, rows, stats.data_ptr(), _s()),
                 "xent stats")
    return stats


def xent_combine(all_stats, world, rows, gstats, row_loss, loss_out=None, loss_scale=1.0, accumulate=False):
    native.check(native.lib().tdb_xent_combine(all_stats.data_ptr(), world, rows, gstats.data_ptr(),
                                               row_loss.data_ptr(), _p(loss_out), float(loss_scale),
                                               int(accumulate), _s()), "xent combine")


def xent_grad(logits, targets, vocab_start, valid_cols, gstats, scale):
    rows, cols = logits.shape
    native.check(native.lib().tdb_xent_grad(logits.data_ptr(), logits.stride(0), targets.data_ptr(),
                                            int(vocab_start), int(valid_cols), cols, rows, gstats.data_ptr(),
                                            float(scale), _s()), "xent grad")


# ---------------------------------------------------------------- optimizer
def sumsq_partials_count():
    return int(native.lib().tdb_sumsq_partials_count())


def sumsq(g, partial, out, accumulate=False):
    native.check(native.lib().tdb_sumsq(g.data_ptr(), g.numel(), partial.data_ptr(), out.data_ptr(),
                                        int(accumulate), _s()), "sumsq")


def clip_coef(total, max_norm, norm_out, coef, loss=None, finite=None, step_counter=None):
    """norm = sqrt(total); coef = min(1, max_norm / (norm + 1e-6)); clears
    ``finite`` on a non-finite norm or loss; increments ``step_counter``
    (device int32) when given."""
    native.check(native.lib().tdb_clip_coef(total.data_ptr(), float(max_norm), norm_out.data_ptr(),
                                            coef.data_ptr(), _p(loss), _p(finite), _p(step_counter), _s()),
                 "clip coef")


def adamw(master, grad, m, v, param_bf16, *, wd_ranges, lr, beta1, beta2, eps, weight_decay, step=0, coef=None,
          finite=None, zero_grad=True, step_dev=None):
    """Fused AdamW over flat buffers.  The step number comes from ``step`` or,
    when given, from the device int32 ``step_dev`` (CUDA-graph replayable)."""
    (a0, a1), (b0, b1) = (list(wd_ranges) + [(0, 0), (0, 0)])[:2]
    native.check(native.lib().tdb_adamw(master.data_ptr(), grad.data_ptr(), m.data_ptr(), v.data_ptr(),
                                        param_bf16.data_ptr(), master.numel(), a0, a1, b0, b1, float(lr),
                                        float(beta1), float(beta2), float(eps), float(weight_decay), int(step),
                                        _p(coef), _p(finite), int(zero_grad), _p(step_dev), _s()), "adamw")


def to_bf16(src, dst):
    native.check(native.lib().tdb_to_bf16(src.data_ptr(), dst.data_ptr(), src.numel(), _s()), "to_bf16")


# ---------------------------------------------------------------- embedding
def embedding_fwd(tokens, table, vocab_start, out, pos=None, pos_offset=0, seq=1):
    rows, H = out.shape
    native.check(native.lib().tdb_embedding_fwd(tokens.data_ptr(), table.data_ptr(), int(vocab_start),
                                                table.shape[0], _p(pos), int(pos_offset), int(seq), rows, H,
                                                out.data_ptr(), _s()), "embedding fwd")
    return out


def add_positions(x, pos, offset, seq):
    rows, H = x.shape
    native.check(native.lib().tdb_add_positions(x.data_ptr(), pos.data_ptr(), int(offset), int(seq), rows, H, _s()),
                 "add positions")


native.register("tdb_sort_tokens", [V, I, V, V, V])


def sort_tokens(tokens, sorted_tokens=None, order=None):
    """Stable ascending sort of int64 token ids (at most 16384, one CTA):
    returns (sorted ids, original positions)."""
    torch = _t()
    n = tokens.numel()
    if tokens.dtype != torch.int64 or not tokens.is_contiguous():
        raise ValueError("tokens must be a contiguous int64 vector")
    sorted_tokens = torch.empty_like(tokens) if sorted_tokens is None else sorted_tokens
    order = torch.empty_like(tokens) if order is None else order
    native.check(native.lib().tdb_sort_tokens(tokens.data_ptr(), n, sorted_tokens.data_ptr(), order.data_ptr(), _s()),
                 "sort tokens")
    return sorted_tokens, order


def embedding_bwd(sorted_tokens, sorted_rows, dy, vocab_start, local_vocab, grad):
    rows, H = dy.shape
    native.check(native.lib().tdb_embedding_bwd(sorted_tokens.data_ptr(), sorted_rows.data_ptr(), rows,
                                                dy.data_ptr(), int(vocab_start), int(local_vocab), H,
                                                grad.data_ptr(), _s()), "embedding bwd")


def position_bwd(dy, offset, seq, grad_pos):
    rows, H = dy.shape
    native.check(native.lib().tdb_position_bwd(dy.data_ptr(), rows, int(offset), int(seq), H, grad_pos.data_ptr(),
                                               _s()), "position bwd")


# ---------------------------------------------------------------- elementwise
native.register("tdb_bias_residual", [V, V, V, V, I64, I, V])
native.register("tdb_colsum_scratch_floats", [I, I])
native.register("tdb_colsum", [V, I64, I, I, V, V, I, V])


def bias_residual(x, bias, residual, out=None):
    """out = x + bias[col] + residual (bf16, any of bias/residual may be None)."""
    torch = _t()
    rows, cols = x.shape
    out = torch.empty_like(x) if out is None else out
    native.check(native.lib().tdb_bias_residual(x.data_ptr(), _p(bias), _p(residual), out.data_ptr(), rows, cols,
                                                _s()), "bias_residual")
    return out


def colsum_scratch_floats(rows, cols):
    return int(native.lib().tdb_colsum_scratch_floats(rows, cols))


def colsum(x, out, scratch, accumulate=True):
    """out (fp32, [cols]) (+)= x.sum(0), deterministic."""
    rows, cols = x.shape
    native.check(native.lib().tdb_colsum(x.data_ptr(), x.stride(0), rows, cols, scratch.data_ptr(), out.data_ptr(),
                                         int(accumulate), _s()), "colsum")
    return out
