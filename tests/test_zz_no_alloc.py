"""The allocation-free LayerNorm backward, called through its exported C symbol.

``tdb_layernorm_bwd_noalloc`` (declared in ``csrc/tdb.h``) serves callers that
cannot allocate device memory when they run the LayerNorm backward (their
memory is already fully planned, or they must not risk the device
synchronisation an allocation can cause): it keeps its partial sums in a
fixed array inside the library.  This test calls that symbol directly with
ctypes, on two calls in a row with different gradients, and checks dx /
dgamma / dbeta against

* the regular entry point that takes caller-provided scratch, and
* an fp32 PyTorch restatement of the LayerNorm backward,

for the GPT-6.7B row count that exactly fills the built-in array, for hidden
sizes that select other kernel widths, with and without the residual
gradient, and with ``accumulate`` 0 (overwrite) and 1 (add to dgamma / dbeta).
It also checks that a problem larger than the built-in array is refused with a
clear message.

The file name makes pytest collect it last.
"""
import ctypes

import pytest

pytestmark = pytest.mark.gpu


def _rel(a, b):
    import torch
    return (torch.linalg.vector_norm(a.float() - b.float()) /
            torch.linalg.vector_norm(b.float()).clamp_min(1e-30)).item()


def _symbol():
    from tempname_dcu_b200.ops import native
    lib = native.lib()
    fn = lib.tdb_layernorm_bwd_noalloc
    v, i = ctypes.c_void_p, ctypes.c_int
    fn.argtypes = [v, v, v, v, v, v, v, v, v, i, i, i, v]
    fn.restype = i
    limit = lib.tdb_layernorm_bwd_noalloc_max_floats
    limit.argtypes, limit.restype = [], ctypes.c_longlong
    return fn, int(limit()), lib


def _torch_ln_bwd(x, w, mean, rstd, dy, dres):
    """fp32 restatement: xhat = (x - mean) * rstd; dgamma = sum dy * xhat;
    dbeta = sum dy; dx = rstd * (g - mean(g) - xhat * mean(g * xhat)) + dres
    with g = dy * gamma."""
    xf, dyf = x.float(), dy.float()
    xhat = (xf - mean[:, None]) * rstd[:, None]
    g = dyf * w.float()[None, :]
    dx = rstd[:, None] * (g - g.mean(1, keepdim=True) - xhat * (g * xhat).mean(1, keepdim=True))
    if dres is not None:
        dx = dx + dres.float()
    return dx, (dyf * xhat).sum(0), dyf.sum(0)


@pytest.mark.parametrize("rows,H,with_dres,accumulate", [
    (2048, 4096, True, 0),   # GPT-6.7B rows at TP=1: exactly fills the built-in array
    (2048, 4096, True, 1),
    (1000, 1536, False, 0),  # another kernel width, no residual gradient, a partial last row block
    (512, 768, True, 1),
])
def test_noalloc_layernorm_bwd_matches_allocating_entry_point(cuda, rows, H, with_dres, accumulate):
    import torch
    from tempname_dcu_b200.ops import kernels as K
    from tempname_dcu_b200.ops import native
    fn, limit, lib = _symbol()
    assert ((rows + 15) // 16) * 2 * H <= limit
    gen = torch.Generator(device=cuda).manual_seed(11 + rows + H)
    x = (torch.randn(rows, H, device=cuda, generator=gen) * 2 + 0.5).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H, device=cuda, generator=gen)).to(torch.bfloat16)
    b = (0.1 * torch.randn(H, device=cuda, generator=gen)).to(torch.bfloat16)
    _, mean, rstd = K.layernorm_fwd(x, w, b)
    scratch = torch.empty(K.layernorm_scratch_floats(rows, H), device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    # dgamma / dbeta carry over between the two calls when accumulating
    dg = torch.randn(H, device=cuda, generator=gen) if accumulate else torch.full((H,), float("nan"), device=cuda)
    db = torch.randn(H, device=cuda, generator=gen) if accumulate else torch.full((H,), float("nan"), device=cuda)
    ref_dg, ref_db = dg.clone(), db.clone()
    torch_dg, torch_db = dg.clone(), db.clone()
    for call in range(2):
        dy = torch.randn(rows, H, device=cuda, generator=gen).to(torch.bfloat16)
        dres = torch.randn(rows, H, device=cuda, generator=gen).to(torch.bfloat16) if with_dres else None
        ref_dx = K.layernorm_bwd(x, w, mean, rstd, dy, ref_dg, ref_db, scratch, dres=dres,
                                 accumulate=bool(accumulate))
        dx = torch.empty_like(x)
        rc = fn(x.data_ptr(), w.data_ptr(), mean.data_ptr(), rstd.data_ptr(), dy.data_ptr(),
                dres.data_ptr() if dres is not None else None, dx.data_ptr(), dg.data_ptr(), db.data_ptr(), rows, H,
                accumulate, stream)
        assert rc == 0, lib.tdb_last_error()
        t_dx, t_dg, t_db = _torch_ln_bwd(x, w, mean, rstd, dy, dres)
        if accumulate:
            torch_dg += t_dg
            torch_db += t_db
        else:
            torch_dg, torch_db = t_dg, t_db
        torch.cuda.synchronize()
        assert _rel(dx, ref_dx) < 1e-3, call
        assert _rel(dg, ref_dg) < 1e-3, call
        assert _rel(db, ref_db) < 1e-3, call
        # against fp32 torch: dx is stored in bf16 (relative rounding 2^-9)
        assert _rel(dx, t_dx) < 1e-2, call
        assert _rel(dg, torch_dg) < 1e-3, call
        assert _rel(db, torch_db) < 1e-3, call
    native.raise_on_status()


def test_noalloc_layernorm_bwd_rejects_oversized_problem(cuda):
    import torch
    fn, limit, lib = _symbol()
    rows, H = 4096, 4096  # needs twice the built-in array
    assert ((rows + 15) // 16) * 2 * H > limit
    t = torch.empty(1, device=cuda)
    p = t.data_ptr()
    rc = fn(p, p, p, p, p, p, p, p, p, rows, H, 0, torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    message = lib.tdb_last_error().decode()
    assert "at most" in message and "tdb_layernorm_bwd" in message
