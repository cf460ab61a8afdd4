"""Host model of the fused GEMM -> reduce-scatter signalling protocol (CPU).

Every rank makes the same sequence of calls.  Call c uses receive set
``epoch & 1`` and counter target ``targets[set] += signals(c)``
(``runtime.Context.next_call``, mirrored on the device by rs_advance_kernel).
A producer writes its blocks into the destination's slots of that set and adds
``signals`` to the (block, source) counters; a consumer waits until every
counter of its blocks reaches the target, then reads.  On a rank the producer
of call c+1 starts only after that rank's consumer of call c finished (stream
order).  The simulation interleaves ranks at random and checks that a
consumer never accepts a stale counter, never reads a slot still holding an
older call, and that no producer overwrites a slot a consumer has not read
yet -- the reuse argument for two receive sets.
"""
import random
from types import SimpleNamespace

import pytest

from tempname_dcu_b200.runtime import Context


@pytest.fixture(scope="module")
def native_state():
    """csrc/call_state.cuh (the arithmetic of rs_advance_kernel and
    ag_advance_kernel) compiled for the host."""
    import ctypes
    import shutil
    import subprocess
    import tempfile
    from pathlib import Path
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).is_file():
        pytest.skip("nvcc unavailable")
    csrc = Path(__file__).resolve().parents[1] / "tempname_dcu_b200" / "csrc"
    folder = Path(tempfile.mkdtemp(prefix="tdb-state-"))
    (folder / "s.cu").write_text('#include "call_state.cuh"\n'
                                 'extern "C" void rs(unsigned* st, unsigned n) { tdb::advance_rs_state(st, n); }\n'
                                 'extern "C" void ag(unsigned* st) { tdb::advance_ag_state(st); }\n')
    subprocess.run([nvcc, "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "-I", str(csrc), str(folder / "s.cu"),
                    "-o", str(folder / "s.so")], check=True, capture_output=True, text=True)
    lib = ctypes.CDLL(str(folder / "s.so"))
    lib.rs.argtypes, lib.ag.argtypes = [ctypes.c_void_p, ctypes.c_uint], [ctypes.c_void_p]
    return lib


def _device_advance(lib, state, signals):
    """One rs_advance_kernel step on a host copy of the device call state
    {set, expected, epoch, target0, target1}."""
    lib.rs(state, signals)
    return state[0], state[1]


@pytest.mark.parametrize("seed", range(12))
def test_two_receive_sets_are_reused_safely(seed, native_state):
    import ctypes
    rng = random.Random(seed)
    world, per, calls = rng.choice([2, 4, 8]), 2, 40
    signals = [rng.choice([4, 8, 64]) for _ in range(calls)]  # operators of different shapes interleave
    host = SimpleNamespace(epoch=0, targets=[0, 0])
    device = (ctypes.c_uint * 5)()
    plan = []
    for c in range(calls):
        expect = Context.next_call(host, signals[c])
        assert _device_advance(native_state, device, signals[c]) == expect
        plan.append(expect)
    # shared memory of every rank: counters[set][within][source], slots[set][source][within] = call id
    counters = [[[[0] * world for _ in range(per)] for _ in range(2)] for _ in range(world)]
    slots = [[[[None] * per for _ in range(world)] for _ in range(2)] for _ in range(world)]
    unread = [[[[False] * per for _ in range(world)] for _ in range(2)] for _ in range(world)]
    # per rank: next call to produce / consume
    produced, consumed = [0] * world, [0] * world
    steps = 0
    while min(consumed) < calls:
        steps += 1
        assert steps < 100000, "the protocol deadlocked"
        r = rng.randrange(world)
        if produced[r] == consumed[r] and produced[r] < calls:
            c = produced[r]
            s, _ = plan[c]
            for dest in range(world):
                for w in range(per):
                    assert not unread[dest][s][r][w], "a producer overwrote a slot before it was read"
                    slots[dest][s][r][w] = c
                    unread[dest][s][r][w] = True
                    counters[dest][s][w][r] += signals[c]
            produced[r] += 1
        elif consumed[r] < produced[r]:
            c = consumed[r]
            s, target = plan[c]
            if all(counters[r][s][w][src] >= target for w in range(per) for src in range(world)):
                for w in range(per):
                    for src in range(world):
                        assert counters[r][s][w][src] == target, "a counter ran ahead into the next use of the set"
                        assert slots[r][s][src][w] == c, "consumer accepted a stale or newer slot"
                        unread[r][s][src][w] = False
                consumed[r] += 1


def test_a_stale_counter_never_satisfies_the_next_use_of_its_set():
    host = SimpleNamespace(epoch=0, targets=[0, 0])
    seq = [Context.next_call(host, n) for n in (4, 8, 4, 8, 64)]
    assert [s for s, _ in seq] == [0, 1, 0, 1, 0]
    for (s0, t0), (s1, t1) in zip(seq, seq[2:]):
        assert s0 == s1 and t1 > t0  # the counters left by call c are below call c+2's target


def test_all_gather_state_counts_epochs_and_alternates_slots(native_state):
    import ctypes
    st = (ctypes.c_uint * 2)()
    seen = []
    for _ in range(5):
        native_state.ag(st)
        seen.append((st[0], st[1]))
    assert seen == [(1, 1), (2, 0), (3, 1), (4, 0), (5, 1)]  # call c: epoch c + 1, slot (c + 1) & 1


@pytest.mark.parametrize("seed", range(12))
def test_all_gather_slots_are_reused_safely(seed):
    """The NVLink all-gather (csrc/allgather.cu, csrc/ag_gemm.cu): a call
    advances the epoch, stages this rank's rows into its send slot
    [epoch & 1], publishes the epoch to every peer, then pulls each source's
    slot once that source's published epoch reaches the call's.  A rank
    starts call c+1 only after its pulls of call c finished.  No pull may read
    a slot restaged for a later call, none may return an older call's rows."""
    rng = random.Random(1000 + seed)
    world, calls = rng.choice([2, 4, 8]), 30
    slot = [[None, None] for _ in range(world)]          # slot[rank][parity] = call staged there
    published = [[0] * world for _ in range(world)]      # published[reader][source] = epoch
    pending = [set() for _ in range(world)]              # sources still to pull in the current call
    call = [-1] * world
    wanted = {}                                           # (source, parity) -> {reader: call it will pull}
    steps = 0
    while min(call) < calls - 1 or any(pending):
        steps += 1
        assert steps < 100000, "the all-gather deadlocked"
        r = rng.randrange(world)
        if not pending[r] and call[r] < calls - 1:
            call[r] += 1
            c, parity = call[r], (call[r] + 1) & 1          # epoch = c + 1
            waiting = wanted.get((r, parity), {})
            assert all(w >= c for w in waiting.values()), "a rank restaged a slot that a peer had not pulled"
            slot[r][parity] = c
            for peer in range(world):
                published[peer][r] = c + 1
            pending[r] = set(range(world))
            for s in range(world):
                wanted.setdefault((s, parity), {})[r] = c
        elif pending[r]:
            s = rng.choice(sorted(pending[r]))
            c, parity = call[r], (call[r] + 1) & 1
            if s == r or published[r][s] >= c + 1:
                assert slot[s][parity] == c, "pulled rows of another call"
                pending[r].discard(s)
                del wanted[(s, parity)][r]
