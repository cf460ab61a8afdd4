"""Rank-independent tile-to-rank production schedules for the five arms.

Pure functions, no device imports.  For an output of M rows split over
``world`` destinations, each destination owns ``per = M / world / chunk_rows``
row blocks ("physical" block ``p = destination * per + within``).  A schedule
lists the order in which every rank produces the blocks:

* ``flux`` / ``flux_taco``: contiguous by destination (``slot -> divmod(slot, per)``);
* ``flux_taco_interleaved``: the common interleave shared by all ranks,
  ``destination = slot % world, within = slot // world`` (Entwine v1 eq. (1));
* arrival arms: a calibrated permutation of physical blocks that keeps every
  slot's destination (``plan['arrival_order']``).

Every block carries a transport lane ``within % 2``; the selective arm carries
a per-physical-block quantization mask.  On B200 the schedule is what the
fused kernels read as their device tile-order table.

Reference parity: ``python/flux_dcu/mapping.py:7-124`` (arm ids, shape
validation, schedule, plan check, block selection, selection statistics,
wire bytes, sparse all-to-all split sizes).
"""
from __future__ import annotations

ARMS = ("flux", "flux_taco", "flux_taco_interleaved",
        "flux_taco_interleaved_arrival", "flux_taco_interleaved_arrival_selective")
ARRIVAL_ARMS = ARMS[3:]
# Backend identity recorded in operator state and rank rows.
BACKEND = "b200-tcgen05-nvlink-fused-lanes-v1"

GROUP = 128
GROUP_BYTES = 136


def validate_shape(m, n, k, world, chunk_rows):
    for value in (m, n, k, world, chunk_rows):
        if type(value) is not int or value <= 0:
            raise ValueError("M, N, K, world and chunk_rows must be positive integers")
    if world < 2:
        raise ValueError("the overlapped operator needs world >= 2")
    if m % (world * chunk_rows):
        raise ValueError("M must be divisible by world_size * chunk_rows")
    if n % GROUP:
        raise ValueError("N must be a multiple of the H128 codec group")


def blocks_per_destination(m, world, chunk_rows):
    return m // world // chunk_rows


def _entry(slot, destination, within, per, chunk_rows):
    physical = destination * per + within
    return dict(slot=slot, destination=destination, within=within, physical=physical,
                row=physical * chunk_rows, rows=chunk_rows, lane=within % 2)


def schedule(m, n, k, world, chunk_rows, arm, plan=None):
    """Production order as a list of block dicts (slot, destination, within,
    physical, row, rows, lane)."""
    validate_shape(m, n, k, world, chunk_rows)
    if arm not in ARMS:
        raise ValueError(f"unknown arm: {arm}")
    per = blocks_per_destination(m, world, chunk_rows)
    count = per * world
    if arm in ARRIVAL_ARMS:
        validate_runtime_plan(plan, m, n, k, world, chunk_rows)
        return [_entry(slot, *divmod(plan["arrival_order"][slot], per), per, chunk_rows)
                for slot in range(count)]
    if plan is not None:
        raise ValueError("the first three arms take no arrival/selection plan")
    if arm == "flux_taco_interleaved":
        return [_entry(slot, slot % world, slot // world, per, chunk_rows) for slot in range(count)]
    return [_entry(slot, *divmod(slot, per), per, chunk_rows) for slot in range(count)]


def validate_runtime_plan(plan, m, n, k, world, chunk_rows):
    """Scheduling/wire contract of a role plan, then the planner's full check."""
    validate_shape(m, n, k, world, chunk_rows)
    if not isinstance(plan, dict):
        raise ValueError("arrival/selective arms need an explicit role plan")
    if plan.get("shape") != [m, n, k] or plan.get("chunk_rows") != chunk_rows:
        raise ValueError("role plan shape or chunk_rows differs from the operator")
    count = m // chunk_rows
    per = count // world
    order, mask = plan.get("arrival_order"), plan.get("selective_mask")
    if (not isinstance(order, list) or len(order) != count or any(type(v) is not int for v in order)
            or sorted(order) != list(range(count))):
        raise ValueError("arrival_order must be a complete permutation of physical blocks")
    if any(physical // per != slot % world for slot, physical in enumerate(order)):
        raise ValueError("arrival order must keep the destination of every interleaved slot")
    if not isinstance(mask, list) or len(mask) != count or any(type(v) is not bool for v in mask):
        raise ValueError("selective_mask needs one bool per physical block")
    if not isinstance(plan.get("diagnostics"), dict):
        raise ValueError("role plan diagnostics must be a dictionary")
    from .planning import validate_role_plan
    validate_role_plan(plan, shape=[m, n, k], world_size=world, chunk_rows=chunk_rows)
    return plan


def block_selection(m, n, k, world, chunk_rows, arm, plan=None):
    """Per-physical-block wire format (True = TACO) after closure: all remote
    sources of one receiver block use the same format."""
    schedule(m, n, k, world, chunk_rows, arm, plan)
    if arm == ARMS[-1]:
        return list(plan["selective_mask"])
    return [arm != "flux"] * (m // chunk_rows)


def selection_statistics(m, n, world, chunk_rows, mask):
    validate_shape(m, n, 1, world, chunk_rows)
    count = m // chunk_rows
    if not isinstance(mask, list) or len(mask) != count or any(type(v) is not bool for v in mask):
        raise ValueError("invalid closed-block selection mask")
    per = count // world
    plain = chunk_rows * n * 2
    packed = chunk_rows * n // GROUP * GROUP_BYTES
    chosen, wire = [], []
    for source in range(world):
        remote = [p for p in range(count) if p // per != source]
        q = sum(1 for p in remote if mask[p])
        chosen.append(q)
        wire.append(q * packed + (len(remote) - q) * plain)
    return dict(selected_remote_blocks_by_source=chosen, remote_blocks_per_source=count - per,
                remote_wire_bytes_by_source=wire, selected_physical_blocks=sum(mask), physical_blocks=count,
                bf16_bytes_per_block=plain, quantized_bytes_per_block=packed)


def wire_bytes(m, n, world, quantized):
    """Bytes each rank sends to remote destinations for one projection."""
    elements = (world - 1) * (m // world) * n
    return elements // GROUP * GROUP_BYTES if quantized else elements * 2


def split_sizes(world, rank, destination, elements):
    """Send/receive split sizes of the sparse exchange of one destination
    block: every remote source sends one block; the destination receives
    world-1 blocks in ascending source order; self data is not exchanged."""
    if not 0 <= rank < world or not 0 <= destination < world or elements <= 0:
        raise ValueError("invalid rank/destination/count")
    send = [0] * world
    receive = [0] * world
    if rank != destination:
        send[destination] = elements
    else:
        receive = [0 if source == rank else elements for source in range(world)]
    return send, receive


def remote_first_order(order, world, rank):
    """The same blocks with this rank's destinations rotated so that blocks
    for rank+1, rank+2, ... are produced first and this rank's own blocks
    last (their data then crosses NVLink while the local tiles compute).
    Block order within a destination is kept."""
    return sorted(order, key=lambda item: ((item["destination"] - rank - 1) % world, item["slot"]))


def tiles_for_order(order, n, chunk_rows, *, block_m=128, block_n=256):
    """Expand a block order to the device tile table (see tile_table)."""
    if chunk_rows % block_m:
        raise ValueError("chunk_rows must be a multiple of the tile height")
    n_tiles = -(-n // block_n)
    table = []
    for item in order:
        first = item["row"] // block_m
        for sub in range(chunk_rows // block_m):
            for nt in range(n_tiles):
                table.append((first + sub) * n_tiles + nt)
    return table


def tile_table(m, n, world, chunk_rows, arm, plan=None, *, block_m=128, block_n=256, k=1):
    """Device tile-order table for the fused GEMM-RS: the production schedule
    expanded to (block_m x block_n) output tiles, row blocks in schedule order
    and the N tiles of each row block consecutively.  Values are
    ``m_tile * n_tiles + n_tile``."""
    order = schedule(m, n, k, world, chunk_rows, arm, plan)
    return tiles_for_order(order, n, chunk_rows, block_m=block_m, block_n=block_n)


def mma_row_blocks(order, mask, m, chunk_rows, block_m=128):
    """Per ``block_m``-row block of a rank's [m, n] partial output: 1 if the
    block belongs to a physical block selected by ``mask`` (the selective
    arm's block-scaled FP8 MMA tiles), else 0."""
    rows = [0] * (m // block_m)
    for item in order:
        if mask[item["physical"]]:
            for mb in range(item["row"] // block_m, (item["row"] + chunk_rows) // block_m):
                rows[mb] = 1
    return rows
