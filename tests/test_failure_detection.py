"""Failure detection on the host (no GPU fault is ever provoked): the
rank-coordinated MIN gate, a rank that never joins a collective (the process
group timeout ends the survivor's call with an error), and a rank that raises
between steps.  Reference: python/flux_dcu/worker.py:31-37 (require_all) and
the worker failure rows (:438-441)."""
import datetime


def _vote_worker(rank, world, init_file, queue):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        from tempname_dcu_b200.worker import require_all
        require_all(True, "all good", dist.group.WORLD)
        try:
            require_all(rank != 1, "rank 1 objects", dist.group.WORLD)
            queue.put((rank, "passed"))
        except RuntimeError as exc:
            queue.put((rank, str(exc)))
    finally:
        dist.destroy_process_group()


def test_min_vote_fails_every_rank(tmp_path):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_vote_worker, args=(r, 2, str(tmp_path / "rdv"), queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert results[0] == results[1] == "rank 1 objects (failed on at least one rank)"


def _dead_rank_worker(rank, world, init_file, queue):
    import time
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        queue.put((rank, "left"))  # leaves between steps, with nothing in flight
        return
    t0 = time.time()
    try:
        t = torch.ones(4)
        dist.all_reduce(t)
        queue.put((rank, "completed"))
    except Exception as exc:  # noqa: BLE001 - the timeout / connection error is the point
        queue.put((rank, f"error after {time.time() - t0:.1f}s: {type(exc).__name__}"))


def test_rank_that_never_joins_ends_the_survivor_with_an_error(tmp_path):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_dead_rank_worker, args=(r, 2, str(tmp_path / "rdv"), queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert results[1] == "left"
    assert results[0].startswith("error after"), results[0]
    import re
    assert float(re.match(r"error after ([0-9.]+)s", results[0]).group(1)) < 60.0


def test_operator_poisoning_refuses_reuse():
    """A failure inside a fused call marks the operator and its context failed;
    both then refuse further calls (host logic of runtime.FluxB200)."""
    import threading
    import types
    import pytest
    from tempname_dcu_b200 import runtime
    ctx = types.SimpleNamespace(failed=False, closed=False, submission_lock=threading.Lock(),
                                next_call=lambda signals: (_ for _ in ()).throw(RuntimeError("peer flag timeout")))
    op = runtime.FluxB200.__new__(runtime.FluxB200)
    op.context, op.failed = ctx, False
    op._check = lambda *a: None
    op.world, op.m, op.n, op.device, op.signals = 2, 256, 128, "cpu", 4
    op.epilogue_reduction = False
    import torch
    with pytest.raises(RuntimeError, match="peer flag timeout"):
        op.forward(torch.zeros(1), torch.zeros(1), out=torch.zeros(1))
    assert op.failed and ctx.failed
    ctx.next_call = lambda signals: (0, 4)
    op2 = runtime.FluxB200.__new__(runtime.FluxB200)   # a fresh operator on the poisoned context
    op2.context, op2.failed = ctx, False
    with pytest.raises(RuntimeError, match="previously failed"):
        op2.forward(torch.zeros(1), torch.zeros(1))
    assert not ctx.submission_lock.locked()
