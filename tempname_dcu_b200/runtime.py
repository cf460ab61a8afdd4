"""The five-arm tensor-parallel overlap operator on B200.

``FluxB200(m, n, k, group, arm, codec=None, chunk_rows=128, plan=None)``
computes the row-parallel projection ``out = RS(input @ weight^T) (+ residual
+ bias)`` with a fused producer / consumer kernel pair (``csrc/gemm_rs.cu``):
tcgen05 GEMM tiles are produced in the arm's schedule (``mapping.schedule``)
and pushed by the epilogue into the destination rank's receive slot over
NVLink (BF16, or TACO-encoded for the selected blocks; with
``selective_mode="fp8-mma"`` the selected blocks are computed as block-scaled
FP8 MMAs instead), and the consumer performs the ordered BF16 reduction of
this rank's blocks, polling per-block counters -- in schedule order
("ordered") or per lane, ready block first ("per-lane ready", arrival arms).

``initialize_context`` / ``shutdown_context`` manage the per-(device, group)
state shared by all operators: the symmetric heap (receive slots for two
alternating buffer sets and the per-block counters), the call epoch and the
failure flag.  Any exception during a call poisons the operator and the
context; a poisoned context refuses further calls.

Reference parity: python/flux_dcu/runtime.py:18-321 (initialize_context,
shutdown_context, FluxDCU.forward / profile_call / state) and
mapping.py (schedules, selection, wire bytes).
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import threading

from .mapping import (ARRIVAL_ARMS, BACKEND, block_selection, mma_row_blocks, remote_first_order, schedule,
                      selection_statistics, tile_table, tiles_for_order)
from .ops import native

native.register("tdb_gemm_rs", [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_int64,
                                ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_uint64,
                                ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int, ctypes.c_uint, ctypes.c_void_p,
                                ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_double,
                                ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p])
native.register("tdb_gemm_rs_mx", list(native.SIGNATURES["tdb_gemm_rs"][:-2])
                + [ctypes.c_void_p] * 5 + [ctypes.c_void_p])
native.register("tdb_rs_advance", [ctypes.c_void_p, ctypes.c_uint, ctypes.c_void_p])
native.register("tdb_rs_set_variant", [ctypes.c_int])
native.register("tdb_gemm_rs_signals_per_block", [ctypes.c_int, ctypes.c_int, ctypes.c_int])


def set_rs_variant(variant):
    """Signalling / consumer variant of the following fused GEMM-RS calls on
    this process (bit 0: per-tile signals; bit 1: consumer inside the
    producer kernel; bit 2: BF16 tiles pushed with TMA bulk stores and
    signalled per tile once written).  Results are bitwise the same for
    every variant; all ranks must use the same one.  Returns the previous
    variant."""
    if variant not in range(8):
        raise ValueError("variant must be 0..7")
    return int(native.lib().tdb_rs_set_variant(int(variant)))


# Default of FluxB200(epilogue_reduction=None) for eligible operators (see
# FluxB200); a process-wide switch for A/B measurements.  Off: on 8 B200 the
# epilogue form took 116 / 128 us per attention-out / FC2 call against 66 / 80
# for the consumer kernel (its producer CTAs stall on peers' tiles), and the
# training step 311 against 271 ms.
_EPILOGUE_REDUCTION = False
FINE_FLAG_BYTES = 32768


def set_epilogue_reduction(on):
    """Whether eligible operators created from now on reduce their own blocks
    in the producer's epilogue (True) or in a separate consumer kernel (False,
    the default).  Results are bitwise the same.  Returns the previous
    setting."""
    global _EPILOGUE_REDUCTION
    old, _EPILOGUE_REDUCTION = _EPILOGUE_REDUCTION, bool(on)
    return old


def epilogue_reduction_default():
    """The current process-wide setting of ``set_epilogue_reduction``."""
    return _EPILOGUE_REDUCTION


_CONTEXTS = {}
_LOCK = threading.Lock()
FLAGS_BYTES = 1 << 16
PEER_WAIT_SECONDS = 20.0


class Context:
    """Per-(device, group) shared state of the fused operators."""

    def __init__(self, tp, capacity_bytes):
        import torch
        from .parallel.symmetric import SymmetricHeap
        self.tp = tp
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.recv_bytes = int(capacity_bytes)
        self.heap = SymmetricHeap(tp, FLAGS_BYTES + self.recv_bytes)
        self.flags_off = 0
        self.recv_off = FLAGS_BYTES
        self.epoch = 0
        self.targets = [0, 0]
        # device copy of (set, expected, epoch, targets), advanced by a kernel
        # before every call so that CUDA-graph replays see fresh values
        self.call_state = torch.zeros(8, dtype=torch.int32, device=self.device)
        self.failed = False
        self.closed = False
        self.submission_lock = threading.Lock()
        self.calls = 0

    def next_call(self, signals_per_block):
        """(set, expected counter) for the next fused call; identical on all
        ranks because every rank makes the same sequence of calls."""
        s = self.epoch & 1
        self.targets[s] += signals_per_block
        self.epoch += 1
        return s, self.targets[s]


def initialize_context(group, capacity_bytes=None):
    """Collectively create (or return) the context of ``group`` on the current
    device.  All ranks must call it in the same order."""
    import torch
    from .parallel.tp import TPGroup
    key = (torch.cuda.current_device(), id(group))
    with _LOCK:
        ctx = _CONTEXTS.get(key)
        if ctx is not None:
            if ctx.closed or ctx.failed:
                raise RuntimeError("this FluxB200 context is closed or previously failed")
            if capacity_bytes is not None and capacity_bytes > ctx.recv_bytes:
                raise ValueError("context receive capacity too small for this operator; create the context "
                                 "with the model's largest projection first")
            return ctx
        tp = group if getattr(group, "loopback", False) else TPGroup(group)
        if tp.world < 2:
            raise ValueError("the fused operator needs a group of at least two ranks")
        ctx = Context(tp, capacity_bytes or (64 << 20))
        _CONTEXTS[key] = ctx
        return ctx


def shutdown_context(group):
    """Collective, ordered teardown (call on every rank before destroying the group)."""
    import torch
    key = (torch.cuda.current_device(), id(group))
    with _LOCK:
        ctx = _CONTEXTS.pop(key, None)
    if ctx is None:
        return
    if not ctx.submission_lock.acquire(blocking=False):
        raise RuntimeError("cannot shut down a context during operator submission")
    try:
        ctx.heap.close()
        ctx.closed = True
    finally:
        ctx.submission_lock.release()


def receive_bytes(m, n, chunk_rows):
    """Receive capacity of one operator shape: 2 sets x (m / chunk_rows) slots
    of chunk_rows x n BF16 (a TACO packet fits in a BF16 slot)."""
    return 2 * (m // chunk_rows) * chunk_rows * n * 2


def operator_layout(m, n, k, world, rank, arm, plan=None, chunk_rows=128, bn=256):
    """Pure (CPU) description of one fused call: production schedule, wire
    format per physical block, the device tile table, this rank's
    consumption order and the number of counter signals per (block, source).
    Every rank derives the same tables from the same arguments."""
    order = schedule(m, n, k, world, chunk_rows, arm, plan)
    mask = block_selection(m, n, k, world, chunk_rows, arm, plan)
    tiles = tile_table(m, n, world, chunk_rows, arm, plan, block_m=128, block_n=bn, k=k)
    consume = [item["within"] for item in order if item["destination"] == rank]
    signals = (chunk_rows // 128) * (n // bn) * 4
    first0 = next((item for item in order if item["lane"] == 0), None)
    delay_tile = (first0["row"] // 128, 0) if first0 else (-1, -1)
    return dict(order=order, selection_mask=mask, tiles=tiles, consume=consume, signals=signals,
                per=m // world // chunk_rows, delay_tile=delay_tile,
                consumer_policy="per_lane_ready" if arm in ARRIVAL_ARMS else "ordered")


class FluxB200:
    """Fused GEMM + reduce-scatter for one projection shape and arm."""

    def __init__(self, m, n, k, group, arm, codec=None, chunk_rows=128, plan=None, diagnostic_delay_cycles=0,
                 b_mn=False, tile_n=None, remote_first=False, selective_mode="wire", wait_seconds=PEER_WAIT_SECONDS,
                 epilogue_reduction=None):
        """``remote_first`` (first three arms only): produce the blocks bound for
        other ranks first and this rank's own blocks last, so the NVLink
        transfers overlap the local tiles; results are bitwise unchanged (the
        receiving side reduces sources in fixed order).  Off for the
        reference experiment arms, whose production order is part of their
        definition.

        ``selective_mode`` (selective arm only): ``"wire"`` quantizes the
        calibrated blocks on the link (TACO packets, the reference's mode);
        ``"fp8-mma"`` instead computes their GEMM tiles as block-scaled FP8
        tcgen05 MMAs (e4m3 with one power-of-two scale per 32 K values) and
        sends every block as BF16.

        ``wait_seconds`` bounds every wait of the consumer for other ranks'
        blocks; on expiry the kernel records a peer-flag timeout in the status
        word and returns (``check_status`` raises and poisons).

        ``epilogue_reduction`` (remote-first BF16 operators, up to 8 ranks):
        no consumer kernel -- the producer's epilogue reduces this rank's own
        tiles (produced last) once every peer's copy of the tile has arrived,
        in the same rank order and rounding as the consumer kernel, so the
        result is bitwise the same.  None follows ``set_epilogue_reduction``
        (off by default: slower on 2 and 8 B200s)."""
        import torch
        if not 0 < wait_seconds <= 600:
            raise ValueError("wait_seconds must be in (0, 600]")
        self.wait_seconds = float(wait_seconds)
        if selective_mode not in ("wire", "fp8-mma"):
            raise ValueError("selective_mode must be 'wire' or 'fp8-mma'")
        if selective_mode == "fp8-mma" and (not arm.endswith("_selective") or b_mn or tile_n not in (None, 128, 256)
                                            or k % 128 or m % 128 or n % 128 or (tile_n == 256 and n % 256)):
            raise ValueError("fp8-mma runs the selective arm with a K-major weight and m, n, k multiples of 128")
        self.selective_mode = selective_mode
        if type(diagnostic_delay_cycles) is not int or not 0 <= diagnostic_delay_cycles <= 100_000_000:
            raise ValueError("diagnostic_delay_cycles must be an integer in [0, 100000000]")
        self.context = initialize_context(group, receive_bytes(m, n, chunk_rows))
        tp = self.context.tp
        self.group, self.arm, self.codec = group, arm, codec
        self.rank, self.world = tp.rank, tp.world
        self.device = self.context.device
        self.m, self.n, self.k, self.chunk_rows = m, n, k, chunk_rows
        self.b_mn = bool(b_mn)
        self.diagnostic_delay_cycles = diagnostic_delay_cycles
        self.last_profile_delay = None
        self.plan = json.loads(json.dumps(plan, allow_nan=False)) if plan is not None else None
        self.order = schedule(m, n, k, self.world, chunk_rows, arm, self.plan)
        self.selection_mask = block_selection(m, n, k, self.world, chunk_rows, arm, self.plan)
        self.consumer_policy = "per_lane_ready" if arm in ARRIVAL_ARMS else "ordered"
        self.quantized = any(self.selection_mask)
        self.mapping_sha256 = hashlib.sha256(json.dumps(self.order, sort_keys=True).encode()).hexdigest()
        if self.plan is not None:
            from .planning import role_digest
            self.plan_sha256 = role_digest(self.plan)
        else:
            self.plan_sha256 = None
        base = schedule(m, n, k, self.world, chunk_rows, "flux_taco_interleaved")
        self.arrival_order_changed = ([x["physical"] for x in self.order] != [x["physical"] for x in base]
                                      if self.plan else False)
        self.selection = selection_statistics(m, n, self.world, chunk_rows, self.selection_mask)
        # Tile width: every rank derives it from the shape alone.
        sms = native.lib().tdb_sm_count(torch.cuda.current_device())
        if selective_mode == "fp8-mma":  # FP8 outruns BF16 only with 256-wide tiles
            self.bn = tile_n or (256 if n % 256 == 0 else 128)
        else:
            self.bn = tile_n or (256 if (m // 128) * (n // 256) >= sms else 128)
        self.remote_first = bool(remote_first) and arm not in ARRIVAL_ARMS
        if self.remote_first:
            self.tiles = tiles_for_order(remote_first_order(self.order, self.world, self.rank), n, chunk_rows,
                                         block_m=128, block_n=self.bn)
        else:
            self.tiles = tile_table(m, n, self.world, chunk_rows, arm, self.plan, block_m=128, block_n=self.bn, k=k)
        self.tile_table = torch.tensor(self.tiles, dtype=torch.int32, device=self.device)
        # wire_mask: blocks that cross the link as TACO packets; mma_mask: blocks computed in block-scaled FP8
        fp8 = selective_mode == "fp8-mma"
        self.wire_mask = [False] * len(self.selection_mask) if fp8 else list(self.selection_mask)
        self.mma_mask = list(self.selection_mask) if fp8 else [False] * len(self.selection_mask)
        self.qmask = torch.tensor([int(x) for x in self.wire_mask], dtype=torch.uint8, device=self.device)
        self.mx = None
        self.weight_version = None  # optional device int32 scalar that changes when the weight does
        if fp8:
            from .ops import mx as _mx
            rows_mask = mma_row_blocks(self.order, self.mma_mask, m, chunk_rows)
            self.mx = dict(
                mask=torch.tensor(rows_mask, dtype=torch.uint8, device=self.device),
                a8=torch.empty((m, k), dtype=torch.uint8, device=self.device),
                sfa=torch.empty(_mx.scale_bytes(m, k), dtype=torch.uint8, device=self.device),
                b8=torch.empty((n, k), dtype=torch.uint8, device=self.device),
                sfb=torch.empty(_mx.scale_bytes(n, k), dtype=torch.uint8, device=self.device),
                seen=torch.full((), -1, dtype=torch.int32, device=self.device))
        self.per = m // self.world // chunk_rows
        fine_bytes = 2 * self.per * (chunk_rows // 128) * (n // self.bn) * 4 * self.world * 4
        eligible = (self.remote_first and not any(self.wire_mask) and self.mx is None and self.world <= 8
                    and fine_bytes <= FINE_FLAG_BYTES)
        if epilogue_reduction is None:
            epilogue_reduction = eligible and _EPILOGUE_REDUCTION
        elif epilogue_reduction and not eligible:
            raise ValueError("epilogue reduction needs a remote-first BF16 operator of at most 8 ranks")
        self.epilogue_reduction = bool(epilogue_reduction)
        if self.epilogue_reduction:
            self.consumer_policy = "epilogue"
        local_in_order = [item["within"] for item in self.order if item["destination"] == self.rank]
        self.consume = torch.tensor(local_in_order, dtype=torch.int32, device=self.device)
        self.signals = int(native.lib().tdb_gemm_rs_signals_per_block(chunk_rows, n, self.bn))
        self.slot_bytes = chunk_rows * n * 2
        self.packet_bytes = chunk_rows * n // 128 * 136
        self.calls = self.validation_calls = 0
        self.failed = False
        self.profile_enabled = False
        self.validate_next_call = False
        self.events = []
        self._last = None
        # optional per-CTA phase stamps (globaltimer): [grid, 4]
        self.phase_buffer = None
        # delay target: first tile (in production order) of the first lane-0 block
        first0 = next((it for it in self.order if it["lane"] == 0), None)
        n_tiles = n // self.bn
        self._delay_tile = ((first0["row"] // 128), 0) if first0 else (-1, -1)
        self._n_tiles = n_tiles

    # ------------------------------------------------------------------ call
    def _check(self, input_, weight):
        import torch
        if self.failed or self.context.failed or self.context.closed:
            raise RuntimeError("this operator/context previously failed or was closed and cannot be reused")
        wshape = (self.k, self.n) if self.b_mn else (self.n, self.k)
        for label, value, shape in (("input", input_, (self.m, self.k)), ("weight", weight, wshape)):
            if (tuple(value.shape) != shape or value.dtype != torch.bfloat16 or not value.is_cuda
                    or not value.is_contiguous()):
                raise ValueError(f"{label} must be contiguous BF16 {shape} on the current device")

    def forward(self, input_, weight, bias=None, residual=None, out=None):
        if getattr(self, "profile_enabled", False):  # a named range per call in profiler traces
            import torch
            with torch.profiler.record_function(f"tdb/gemm_rs/{self.arm}/{self.m}x{self.n}x{self.k}"):
                return self._forward(input_, weight, bias, residual, out)
        return self._forward(input_, weight, bias, residual, out)

    def _forward(self, input_, weight, bias=None, residual=None, out=None):
        import torch
        self._check(input_, weight)
        ctx = self.context
        if not ctx.submission_lock.acquire(blocking=False):
            raise RuntimeError("concurrent submissions to one FluxB200 context are unsupported")
        try:
            rows = self.m // self.world
            if out is None:
                out = torch.empty((rows, self.n), dtype=torch.bfloat16, device=self.device)
            # epilogue-reduction calls signal per-tile epoch flags, not the
            # per-block counters: their targets must not move
            counted = 0 if self.epilogue_reduction else self.signals
            set_, expected = ctx.next_call(counted)
            timeline = None
            delay = 0
            if self.profile_enabled:
                timeline = torch.full((2 * self.per,), 2 ** 63 - 1, dtype=torch.int64, device=self.device)
                if self.diagnostic_delay_cycles and self.rank == 0:
                    delay = self.diagnostic_delay_cycles
                    first0 = next(it for it in self.order if it["lane"] == 0)
                    self.last_profile_delay = dict(physical=first0["physical"], lane=0, rank=0,
                                                   cycles=self.diagnostic_delay_cycles)
            heap = ctx.heap
            lib = native.lib()
            stream = native.stream_ptr()
            native.check(lib.tdb_rs_advance(ctx.call_state.data_ptr(), counted, stream), "rs advance")
            args = (input_.data_ptr(), input_.stride(0), weight.data_ptr(), int(self.b_mn), weight.stride(0), self.m,
                    self.n, self.k, self.bn, self.tile_table.data_ptr(), heap.peers.data_ptr(), self.world, self.rank,
                    self.chunk_rows, ctx.recv_off, self.slot_bytes, ctx.flags_off, set_, expected,
                    self.qmask.data_ptr(), out.data_ptr(), 0 if bias is None else bias.data_ptr(),
                    0 if residual is None else residual.data_ptr(), self.consume.data_ptr(),
                    {"ordered": 0, "per_lane_ready": 1, "epilogue": 2}[self.consumer_policy],
                    0 if timeline is None else timeline.data_ptr(), delay, self._delay_tile[0], self._delay_tile[1],
                    self.wait_seconds, 0 if self.phase_buffer is None else self.phase_buffer.data_ptr(),
                    ctx.call_state.data_ptr())
            if self.mx is None:
                native.check(lib.tdb_gemm_rs(*args, int(any(self.wire_mask)), stream), "fused gemm_rs")
            else:
                from .ops import mx as _mx
                q = self.mx
                # activations change every call; the weight only when the device counter in
                # ``weight_version`` (the optimizer's step) moved -- decided on the device, so
                # captured graphs replay it correctly; without a counter it is quantized every call
                _mx.quantize(input_, q["a8"], q["sfa"])
                if self.weight_version is None:
                    _mx.quantize(weight, q["b8"], q["sfb"])
                else:
                    _mx.quantize(weight, q["b8"], q["sfb"], version=self.weight_version, seen=q["seen"])
                native.check(lib.tdb_gemm_rs_mx(*args, q["a8"].data_ptr(), q["sfa"].data_ptr(), q["b8"].data_ptr(),
                                                q["sfb"].data_ptr(), q["mask"].data_ptr(), stream),
                             "fused gemm_rs (block-scaled fp8)")
            self._last = (set_, expected, timeline)
            self.calls += 1
            ctx.calls += 1
            if self.validate_next_call:
                from .validation import validate_operator_buffers
                validate_operator_buffers(self, input_, weight, out)
                native.raise_on_status()
                self.validate_next_call = False
                self.validation_calls += 1
            return out
        except BaseException:
            self.failed = ctx.failed = True
            raise
        finally:
            ctx.submission_lock.release()

    __call__ = forward

    def freeze_selection(self, mask):
        """Adopt a frozen per-physical-block wire format (TACO arms): True
        blocks cross NVLink as TACO packets, False blocks as BF16 -- e.g. the
        mask chosen on the first training steps (warmup_calibration).  Call
        between steps, before a CUDA graph of the step is captured."""
        import torch
        if self.arm == "flux" or self.mx is not None:
            raise ValueError("only the TACO wire-format arms take a selection mask")
        mask = list(mask)
        if len(mask) != len(self.selection_mask) or any(type(v) is not bool for v in mask):
            raise ValueError("the mask needs one bool per physical output block")
        self.selection_mask = list(mask)
        self.wire_mask = list(mask)
        self.qmask.copy_(torch.tensor([int(v) for v in mask], dtype=torch.uint8))
        self.quantized = any(mask)
        self.selection = selection_statistics(self.m, self.n, self.world, self.chunk_rows, self.selection_mask)
        if self.plan is not None:
            from .planning import role_digest
            self.plan["selective_mask"] = list(mask)
            self.plan_sha256 = role_digest(self.plan)
        self.frozen_selection = True

    def check_status(self):
        """Wait for this device's queued work, then read the library status
        word; if a kernel recorded a bounded-wait expiry (a peer that never
        delivered) or another device-side error, poison this operator and its
        context -- both refuse every later call -- and raise NativeError.
        Reference parity: python/flux_dcu/runtime.py:264-266 (an exception
        during a call marks the operator and the shared context failed)."""
        import torch
        torch.cuda.synchronize(self.device)
        try:
            native.raise_on_status()
        except native.NativeError:
            self.failed = self.context.failed = True
            raise

    def enable_phase_profile(self, on=True):
        """Record per-CTA {start, produce done, first block ready, end} device
        timestamps of every following call (diagnostics only)."""
        import torch
        self.phase_buffer = torch.zeros((1024, 4), dtype=torch.int64, device=self.device) if on else None

    def phase_summary(self):
        """Mean/max over CTAs of produce, wait and consume durations (us) of the last call."""
        import torch
        t = self.phase_buffer.cpu().double()
        prod = t[t[:, 0] > 0]
        cons = t[t[:, 2] > 0]
        if cons.shape[0] == 0:  # epilogue reduction: no consumer kernel
            produce = (prod[:, 1] - prod[:, 0]) / 1e3
            return dict(ctas=int(prod.shape[0]), kernel_span_us=round((prod[:, 1].max() - prod[:, 0].min()).item() / 1e3, 2),
                        produce_mean_us=round(produce.mean().item(), 2), produce_max_us=round(produce.max().item(), 2),
                        consumer="epilogue")
        produce = (prod[:, 1] - prod[:, 0]) / 1e3
        end_of_produce = prod[:, 1].max()
        wait = (cons[:, 2] - end_of_produce).clamp_min(0) / 1e3
        consume = (cons[:, 3] - cons[:, 2]) / 1e3
        total = (t[:, 3].max() - prod[:, 0].min()).item() / 1e3
        return dict(ctas=int(prod.shape[0]), kernel_span_us=round(total, 2),
                    produce_mean_us=round(produce.mean().item(), 2), produce_max_us=round(produce.max().item(), 2),
                    wait_mean_us=round(wait.mean().item(), 2), wait_max_us=round(wait.max().item(), 2),
                    consume_mean_us=round(consume.mean().item(), 2), consume_max_us=round(consume.max().item(), 2))

    # ---------------------------------------------------- validation hooks
    def _slot_view(self, set_, source, within, nbytes, dtype, shape):
        ctx = self.context
        off = ctx.recv_off + ((set_ * self.world + source) * self.per + within) * self.slot_bytes
        return ctx.heap.view(off, shape, dtype)

    def validation_tensors(self):
        import torch
        set_ = self._last[0] if self._last else 0
        out = []
        for within in range(self.per):
            physical = self.rank * self.per + within
            for s in range(self.world):
                if self.wire_mask[physical] and s != self.rank:
                    continue
                out.append((f"receive.{within}.{s}", self._slot_view(set_, s, within, self.slot_bytes,
                                                                     torch.bfloat16, (self.chunk_rows, self.n))))
        return out

    def validation_packets(self):
        import torch
        set_ = self._last[0] if self._last else 0
        out = []
        elements = self.chunk_rows * self.n
        for within in range(self.per):
            physical = self.rank * self.per + within
            if not self.wire_mask[physical]:
                continue
            for s in range(self.world):
                if s == self.rank:
                    continue
                out.append((f"packet.{within}.{s}", self._slot_view(set_, s, within, self.packet_bytes,
                                                                    torch.uint8, (self.packet_bytes,)), elements))
        return out

    # ------------------------------------------------------------ profiling
    def profile_call(self, input_, weight, bias=None, residual=None):
        """Separate diagnostic call recording per-block ready / consumed device
        timestamps (globaltimer, ns) of this rank's blocks; with a diagnostic
        delay, rank 0 holds back the signal of the first lane-0 tile."""
        import torch
        torch.cuda.synchronize()
        self.profile_enabled = True
        try:
            result = self.forward(input_, weight, bias, residual)
            torch.cuda.synchronize()
            native.raise_on_status()
            timeline = self._last[2].cpu().tolist()
        finally:
            self.profile_enabled = False
        origin = min(t for t in timeline[0::2]) if timeline else 0
        rows = []
        for within in range(self.per):
            physical = self.rank * self.per + within
            rows.append(dict(stage="consumer", physical=physical, lane=within % 2,
                             start_ms=(timeline[2 * within] - origin) / 1e6,
                             end_ms=(timeline[2 * within + 1] - origin) / 1e6))
        self.events = rows
        return result, dict(events=rows, transport_lanes=2, consumer_policy=self.consumer_policy,
                            diagnostic_delay=self.last_profile_delay,
                            clock="device globaltimer (ns), receiver-local",
                            diagnostic_limitation="Artificial skew tests mechanism availability, not normal-workload "
                                                  "performance")

    # ----------------------------------------------------------------- state
    def state(self):
        quantization = ("selective_remote_h128_e4m3" if self.arm.endswith("_selective") else
                        "all_remote_h128_e4m3" if self.arm != "flux" else "none")
        if getattr(self, "frozen_selection", False):
            quantization = "warmup_calibrated_remote_h128_e4m3"
        extra = {}
        if self.mx is not None:
            quantization = "selective_mma_e4m3_ue8m0_k32"
            bf16 = self.chunk_rows * self.n * 2 * self.per
            extra = dict(selective_mode="fp8-mma", mma_block_mask=list(self.mma_mask),
                         remote_wire_bytes_by_source=[bf16 * (self.world - 1)] * self.world,
                         remote_wire_bytes_per_source=bf16 * (self.world - 1),
                         actual_remote_wire_bytes_per_rank=bf16 * (self.world - 1),
                         fused_kernel="tdb::rs::gemm_rs_mx_kernel")
        return dict(backend=BACKEND, arm=self.arm, rank=self.rank, calls=self.calls,
                    shape=[self.m, self.n, self.k], chunk_rows=self.chunk_rows,
                    production_schedule=self.order, mapping_sha256=self.mapping_sha256,
                    production_order="remote_first" if self.remote_first else "schedule",
                    gemms_per_call=1, collectives_per_call=1, fused_kernel="tdb::rs::gemm_rs_kernel",
                    tile_n=self.bn, tiles_per_call=len(self.tiles), quantization=quantization,
                    selection_mask=list(self.selection_mask),
                    selection_granularity="physical_receiver_block_all_remote_sources",
                    selected_remote_blocks_by_source=self.selection["selected_remote_blocks_by_source"],
                    remote_wire_bytes_by_source=self.selection["remote_wire_bytes_by_source"],
                    remote_wire_bytes_per_source=self.selection["remote_wire_bytes_by_source"][self.rank],
                    actual_remote_wire_bytes_per_rank=self.selection["remote_wire_bytes_by_source"][self.rank],
                    plan_sha256=self.plan_sha256, arrival_order_changed=self.arrival_order_changed,
                    reduction_order=list(range(self.world)), rounding="bf16_after_each_source",
                    scratch_bytes=receive_bytes(self.m, self.n, self.chunk_rows), original_cuda_flux=False,
                    cta_level_swizzle=True, transport_lanes=2, lane_assignment="physical_within_destination_mod_2",
                    consumer_policy=self.consumer_policy, validation_calls=self.validation_calls,
                    diagnostic_delay_cycles=self.diagnostic_delay_cycles, diagnostic_delay_in_normal_forward=False,
                    scheduling_granularity="tcgen05_tile_128x%d" % self.bn,
                    overlap_claim="epilogue peer stores overlap the MMA of later tiles in one kernel") | extra


def operator_factory_for(arm, remote_first=True, selective_mode="wire"):
    """Factory for ``GPT(operator_factory=...)``: a FluxB200 per row-parallel
    projection (training uses the remote-first production order;
    ``selective_mode`` applies to the selective arm's forward projections)."""
    def factory(m, n, k, group, arm=arm, chunk_rows=128, plan=None, **kw):
        if arm.endswith("_selective") and not kw.get("b_mn"):
            kw.setdefault("selective_mode", selective_mode)
        return FluxB200(m, n, k, group, arm, chunk_rows=chunk_rows, plan=plan, remote_first=remote_first, **kw)
    return factory
