"""Host model of the fused all-gather's push protocol (variant 3, CPU).

Per call every rank advances its epoch e (``advance_ag_state``: e += 1,
parity = e & 1), then ONE kernel of that rank runs, in any interleaving of
its CTAs:

* push(s -> d): write this rank's rows into rank d's receive buffer
  [parity][s], then stamp flag[d][s] = e (release);
* collect(s): wait until flag[r][s] >= e (acquire), then read the receive
  buffer [parity][s] of this rank.

Pushes never wait.  A rank's next kernel starts only after its current one has
ended (stream order).  The simulation interleaves ranks and CTAs at random and
checks that every collect reads exactly the rows of its own call (never the
call two earlier nor two later), that no push overwrites rows a collect has
not read yet -- the two-buffer reuse argument of ``csrc/ag_gemm.cu`` -- and
that the run never deadlocks.
"""
import random

import pytest


def _simulate(world, calls, rng):
    # receive[d][parity][s] = (call written, read yet?)
    receive = [[[None] * world for _ in range(2)] for _ in range(world)]
    flag = [[0] * world for _ in range(world)]
    epoch = [0] * world
    pending = [None] * world  # events left in the rank's current kernel
    done_calls = [0] * world
    violations = []

    def start(r):
        epoch[r] += 1
        e = epoch[r]
        pending[r] = [("push", d) for d in range(world) if d != r] + [("collect", s) for s in range(world) if s != r]
        return e

    for r in range(world):
        start(r)
    steps = 0
    while any(done_calls[r] < calls for r in range(world)):
        steps += 1
        if steps > 100000:
            raise AssertionError("no progress: deadlock")
        enabled = []
        for r in range(world):
            if done_calls[r] >= calls:
                continue
            e = epoch[r]
            for i, (kind, other) in enumerate(pending[r]):
                if kind == "push" or flag[r][other] >= e:
                    enabled.append((r, i))
        if not enabled:
            raise AssertionError("deadlock: no event enabled")
        r, i = rng.choice(enabled)
        kind, other = pending[r].pop(i)
        e, parity = epoch[r], epoch[r] & 1
        if kind == "push":
            d = other
            slot = receive[d][parity][r]
            if slot is not None and not slot[1]:
                violations.append(f"rank {r} call {e} overwrote unread rows of call {slot[0]} at rank {d}")
            receive[d][parity][r] = [e, False]
            flag[d][r] = max(flag[d][r], e)
        else:
            s = other
            slot = receive[r][parity][s]
            if slot is None or slot[0] != e:
                violations.append(f"rank {r} call {e} read rows of call {slot and slot[0]} from {s}")
            else:
                slot[1] = True
        if not pending[r]:
            done_calls[r] += 1
            if done_calls[r] < calls:
                start(r)
    return violations


@pytest.mark.parametrize("seed", range(16))
def test_push_receive_buffers_are_reused_safely(seed):
    rng = random.Random(seed)
    world = rng.choice([2, 3, 4, 8])
    assert _simulate(world, 12, rng) == []


def test_model_catches_a_single_receive_buffer():
    """The same protocol with one receive buffer instead of two (parity
    ignored) must show an overwrite of unread rows in some interleaving: the
    check is not vacuous."""
    rng = random.Random(0)
    found = False
    for _ in range(200):
        world, calls = 2, 6
        receive = [[None] * world for _ in range(world)]
        flag = [[0] * world for _ in range(world)]
        epoch, pending, done = [1] * world, [None] * world, [0] * world
        for r in range(world):
            pending[r] = [("push", 1 - r), ("collect", 1 - r)]
        while any(d < calls for d in done):
            enabled = [(r, i) for r in range(world) if done[r] < calls
                       for i, (k, o) in enumerate(pending[r]) if k == "push" or flag[r][o] >= epoch[r]]
            r, i = rng.choice(enabled)
            kind, o = pending[r].pop(i)
            if kind == "push":
                slot = receive[o][r]
                if slot is not None and not slot[1]:
                    found = True
                receive[o][r] = [epoch[r], False]
                flag[o][r] = max(flag[o][r], epoch[r])
            else:
                receive[r][o][1] = True
            if not pending[r]:
                done[r] += 1
                epoch[r] += 1
                pending[r] = [("push", 1 - r), ("collect", 1 - r)]
        if found:
            break
    assert found
