"""Bounded device waits run out, report, and poison -- on one GPU, no fault.

A ``LoopbackGroup`` stands in for a two-rank tensor-parallel group whose
peer heap is this GPU's own memory: the missing rank never delivers its
blocks or publishes its rows, so the fused kernels' waits for it must expire.
The tests check that

* the fused GEMM -> reduce-scatter consumer gives up after its wait limit,
  records a peer-flag timeout in the status word, and returns (the call ends
  in milliseconds, not at the 20 s production limit);
* ``FluxB200.check_status`` raises, and the operator AND its context are
  poisoned: a later call and a new operator on the same group are refused
  (reference: python/flux_dcu/runtime.py:264-266, tested there at
  tests/test_runtime_contract.py:206-217 with an injected transport failure);
* the fused all-gather GEMM's wait for a peer's rows expires the same way,
  naming the source rank that never published;
* the CUDA context stays usable afterwards.

Nothing here traps or hangs: every wait is bounded by %globaltimer and the
kernels unwind normally.
"""
import time

import pytest

pytestmark = pytest.mark.gpu


def test_fused_reduce_scatter_wait_expires_and_poisons(cuda):
    import torch
    from tempname_dcu_b200.ops import native
    from tempname_dcu_b200.parallel.tp import LoopbackGroup
    from tempname_dcu_b200.runtime import FluxB200, initialize_context, shutdown_context
    native.clear_status()
    group = LoopbackGroup(2)
    m, n, k = 512, 1024, 256
    op = FluxB200(m, n, k, group, "flux", wait_seconds=0.005)
    x = torch.randn(m, k, device=cuda).to(torch.bfloat16)
    w = torch.randn(n, k, device=cuda).to(torch.bfloat16)
    start = time.monotonic()
    op.forward(x, w)
    with pytest.raises(native.NativeError, match="peer flag timeout"):
        op.check_status()
    assert time.monotonic() - start < 30.0
    assert op.failed and op.context.failed
    with pytest.raises(RuntimeError, match="previously failed"):
        op.forward(x, w)
    with pytest.raises(RuntimeError, match="previously failed"):
        initialize_context(group)
    assert native.read_status()[0] == 0  # the report was consumed
    y = x.float() @ w.float().t()  # the CUDA context still works
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
    shutdown_context(group)


def test_fused_allgather_wait_expires_and_names_the_source(cuda):
    import torch
    from tempname_dcu_b200.ops import native
    from tempname_dcu_b200.parallel.allgather import SymmAgGemm
    from tempname_dcu_b200.parallel.tp import LoopbackGroup
    native.clear_status()
    agg = SymmAgGemm(LoopbackGroup(2), 256, 256, wait_seconds=0.005)
    x = torch.randn(256, 256, device=cuda).to(torch.bfloat16)
    w = torch.randn(512, 256, device=cuda).to(torch.bfloat16)
    agg(x, w)
    torch.cuda.synchronize()
    code, where, source, _ = native.read_status()
    assert (code, where, source) == (2, 310, 1)  # peer-flag timeout at the pull, rank 1 never published
    native.clear_status()
    assert (x.float().sum() + 1).isfinite()
    agg.close()
