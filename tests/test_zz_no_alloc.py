"""The allocation-free LayerNorm backward, called through its exported C symbol.

``tdb_layernorm_bwd_noalloc`` serves callers that cannot allocate device
memory when they run the LayerNorm backward (their memory is already fully
planned, or they must not risk the device synchronisation an allocation can
cause): it keeps its partial sums in a fixed array inside the library.  This
test calls that symbol directly with ctypes and checks, on two calls in a row
with different gradients, that it gives the same dx / dgamma / dbeta as the
regular entry point that takes caller-provided scratch.  It also checks that
a problem larger than the built-in array is refused with a clear message.

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


def test_noalloc_layernorm_bwd_matches_allocating_entry_point(cuda):
    import torch
    from tempname_dcu_b200.ops import kernels as K
    from tempname_dcu_b200.ops import native
    fn, limit, lib = _symbol()
    # GPT-6.7B rows of one rank at TP=1: exactly fills the built-in array.
    rows, H = 2048, 4096
    assert ((rows + 15) // 16) * 2 * H <= limit
    torch.manual_seed(11)
    x = (torch.randn(rows, H, device=cuda) * 2 + 0.5).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H, device=cuda)).to(torch.bfloat16)
    b = (0.1 * torch.randn(H, device=cuda)).to(torch.bfloat16)
    _, mean, rstd = K.layernorm_fwd(x, w, b)
    scratch = torch.empty(K.layernorm_scratch_floats(rows, H), device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        dy = torch.randn(rows, H, device=cuda).to(torch.bfloat16)
        dres = torch.randn(rows, H, device=cuda).to(torch.bfloat16)
        ref_dg = torch.zeros(H, device=cuda)
        ref_db = torch.zeros(H, device=cuda)
        ref_dx = K.layernorm_bwd(x, w, mean, rstd, dy, ref_dg, ref_db, scratch, dres=dres, accumulate=False)
        dx = torch.empty_like(x)
        dg = torch.full((H,), float("nan"), device=cuda)
        db = torch.full((H,), float("nan"), device=cuda)
        rc = fn(x.data_ptr(), w.data_ptr(), mean.data_ptr(), rstd.data_ptr(), dy.data_ptr(), dres.data_ptr(),
                dx.data_ptr(), dg.data_ptr(), db.data_ptr(), rows, H, 0, stream)
        assert rc == 0, lib.tdb_last_error()
        torch.cuda.synchronize()
        assert _rel(dx, ref_dx) < 1e-3, call
        assert _rel(dg, ref_dg) < 1e-3, call
        assert _rel(db, ref_db) < 1e-3, call
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
