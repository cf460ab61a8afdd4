"""Calibrate-then-freeze planning of the arrival order and the selective mask.

Pure orchestration with injected timing (``evaluate(plan, seed, arm, label)``
returns the max-over-ranks elapsed time of a complete operator run, or a dict
holding it): no device code, so the whole planner is exercised on CPU and can
be replayed from recorded samples.

Protocol (identical in steps to the reference, so frozen plans and replayed
calibrations are interchangeable):

1. Arrival order.  Candidates are per-destination transforms of the base
   interleave (identity, reverse_all, reverse_odd, reverse_even, rotate,
   deduplicated).  Each non-identity candidate is measured against identity in
   ``training_pairs`` AB/BA pairs; the best gain above ``min_gain`` is
   re-measured on disjoint seeds (``confirmation_pairs``) and accepted only if
   the geometric-mean gain and every confirmation pair beat ``min_gain``.
   Otherwise identity is kept.
2. Selective mask (under the frozen order).  With ``cap = floor(blocks *
   quant_budget)`` > 0, every single block is measured against the all-BF16
   plan Q0; blocks with positive gain are ranked; prefixes of sizes
   {1, 2, 4, 8, cap} are measured; the best above ``min_gain`` is confirmed
   like step 1.  The all-quantized control Qall is always measured and wins
   only when the budget allows every block.
3. The frozen plan records every measurement in ``diagnostics``.

Optional error-budget mode (``selection_mode="error_budget"``, not in the
reference): step 2 instead ranks blocks by the TACO round-trip error measured
on a calibration batch and keeps the largest prefix whose predicted relative
error of the projection output stays within ``error_budget``
(``_fit_mask_error``); the statistics are frozen into the plan, so replay
reproduces the mask from the plan alone.

Reference parity: ``python/flux_dcu/planning.py:11-280`` (schema, digest,
base order, validation, candidates, quantization statistics, settings,
paired measurement, confirmation, fit_role).
"""
from __future__ import annotations

import hashlib
import json
import math
import statistics

SCHEMA = "dcu-arrival-selective-plan-v2"
ARRIVAL_ARM = "flux_taco_interleaved_arrival"
SELECTIVE_ARM = "flux_taco_interleaved_arrival_selective"
DEFAULTS = dict(warmup=2, iterations=5, training_pairs=3, confirmation_pairs=3, min_gain=0.002,
                quant_budget=0.25)
# Optional settings (absent = the reference's timing-based selection, so plans
# frozen in that mode stay byte-compatible): selection_mode "error_budget"
# picks the selective mask from measured codec error instead of timing.
SELECTION_MODES = ("timing", "error_budget")
OPTIONAL = dict(selection_mode="timing", error_budget=0.01)
PLAN_KEYS = frozenset({"shape", "chunk_rows", "arrival_order", "selective_mask", "diagnostics"})


def canonical_json(value) -> bytes:
    return json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False).encode()


def role_digest(plan) -> str:
    """sha256 of canonical JSON (sorted keys, compact separators, no NaN)."""
    return hashlib.sha256(canonical_json(plan)).hexdigest()


def _per_destination(m, n, k, world, chunk_rows) -> int:
    if any(type(x) is not int or x <= 0 for x in (m, n, k, world, chunk_rows)):
        raise ValueError("positive integer shape/world/chunk_rows required")
    if world < 2 or m % (world * chunk_rows) or n % 128:
        raise ValueError("need M divisible by world*chunk_rows, N by 128 and world >= 2")
    return m // world // chunk_rows


def base_order(m, n, k, world, chunk_rows):
    """Physical blocks in the common interleaved order."""
    per = _per_destination(m, n, k, world, chunk_rows)
    return [(slot % world) * per + slot // world for slot in range(per * world)]


def validate_role_plan(plan, m=None, n=None, k=None, world=None, chunk_rows=None, *, shape=None,
                       world_size=None):
    if shape is not None:
        if not isinstance(shape, (list, tuple)) or len(shape) != 3:
            raise ValueError("shape must be [M, N, K]")
        if any(v is not None for v in (m, n, k)):
            raise ValueError("give shape or M/N/K, not both")
        m, n, k = shape
    if world_size is not None:
        if world is not None and world != world_size:
            raise ValueError("conflicting world/world_size")
        world = world_size
    per = _per_destination(m, n, k, world, chunk_rows)
    if not isinstance(plan, dict) or set(plan) != PLAN_KEYS:
        raise ValueError("unexpected or missing role-plan fields")
    if plan["shape"] != [m, n, k] or plan["chunk_rows"] != chunk_rows:
        raise ValueError("plan shape/chunk_rows differs from the actual operator")
    count = per * world
    order, mask = plan["arrival_order"], plan["selective_mask"]
    if (not isinstance(order, list) or len(order) != count or any(type(v) is not int for v in order)
            or sorted(order) != list(range(count))):
        raise ValueError("arrival order must be a bijection of physical blocks")
    if any(physical // per != slot % world for slot, physical in enumerate(order)):
        raise ValueError("arrival order must keep every interleaved destination slot")
    if not isinstance(mask, list) or len(mask) != count or any(type(v) is not bool for v in mask):
        raise ValueError("selective mask needs one bool per physical output block")
    if not isinstance(plan["diagnostics"], dict):
        raise ValueError("plan diagnostics must be a dictionary")
    role_digest(plan)  # rejects NaN / non-JSON content before freezing
    return plan


def make_role(m, n, k, world, chunk_rows, order=None, mask=None):
    base = base_order(m, n, k, world, chunk_rows)
    plan = dict(shape=[m, n, k], chunk_rows=chunk_rows,
                arrival_order=list(base if order is None else order),
                selective_mask=list([True] * len(base) if mask is None else mask),
                diagnostics={})
    return validate_role_plan(plan, m, n, k, world, chunk_rows)


_TRANSFORMS = (
    ("identity", lambda d, idx: idx),
    ("reverse_all", lambda d, idx: idx[::-1]),
    ("reverse_odd", lambda d, idx: idx[::-1] if d % 2 else idx),
    ("reverse_even", lambda d, idx: idx if d % 2 else idx[::-1]),
    ("rotate", lambda d, idx: idx[1:] + idx[:1]),
)


def candidates(m, n, k, world, chunk_rows):
    """Legal candidate orders (the first is always the base interleave)."""
    per = _per_destination(m, n, k, world, chunk_rows)
    result, seen = [], set()
    for name, transform in _TRANSFORMS:
        within = [transform(d, list(range(per))) for d in range(world)]
        order = [d * per + within[d][w] for w in range(per) for d in range(world)]
        if tuple(order) not in seen:
            seen.add(tuple(order))
            result.append(dict(name=name, arrival_order=order))
    return result


def quantized_blocks(plan):
    return [index for index, flag in enumerate(plan["selective_mask"]) if flag]


def quantization_statistics(plan, world):
    m, n, k = plan["shape"]
    per = _per_destination(m, n, k, world, plan["chunk_rows"])
    validate_role_plan(plan, m, n, k, world, plan["chunk_rows"])
    chosen = quantized_blocks(plan)
    per_source = [sum(1 for p in chosen if p // per != source) for source in range(world)]
    elements = plan["chunk_rows"] * n
    plain, packed = elements * 2, elements // 128 * 136
    remote = (world - 1) * per
    wire = [remote * plain - q * (plain - packed) for q in per_source]
    return dict(selection_unit="physical-output-macroblock-all-remote-sources",
                total_output_blocks=per * world, quantized_output_blocks=len(chosen),
                selected_physical_blocks=chosen,
                total_remote_contributions=(world - 1) * per * world,
                quantized_remote_contributions=(world - 1) * len(chosen),
                actual_remote_fraction=len(chosen) / (per * world),
                selected_per_source=per_source, remote_wire_bytes_per_source=wire,
                bf16_remote_wire_bytes_per_source=[remote * plain] * world,
                full_quantized_remote_wire_bytes_per_source=[remote * packed] * world,
                mixed_source_blocks=0)


def settings(values=None):
    cfg = dict(DEFAULTS)
    if values is not None:
        if not isinstance(values, dict) or set(values) - set(DEFAULTS) - set(OPTIONAL):
            raise ValueError("unknown calibration settings")
        cfg.update(values)
    mode = cfg.get("selection_mode", "timing")
    if mode not in SELECTION_MODES:
        raise ValueError(f"selection_mode must be one of {SELECTION_MODES}")
    if mode == "timing":
        if "error_budget" in cfg:
            raise ValueError("error_budget applies to selection_mode 'error_budget' only")
        cfg.pop("selection_mode", None)
    else:
        budget = cfg.setdefault("error_budget", OPTIONAL["error_budget"])
        if type(budget) not in (int, float) or not math.isfinite(budget) or not 0 < budget <= 1:
            raise ValueError("error_budget must be in (0, 1]")
        cfg["error_budget"] = float(budget)
    for key in ("warmup", "iterations", "training_pairs", "confirmation_pairs"):
        floor = 0 if key == "warmup" else 1
        if type(cfg[key]) is not int or cfg[key] < floor:
            raise ValueError(f"invalid calibration {key}")
    for key in ("min_gain", "quant_budget"):
        value = cfg[key]
        if type(value) not in (int, float) or not math.isfinite(value) or not 0 <= value <= 1:
            raise ValueError(f"invalid calibration {key}")
        cfg[key] = float(value)
    if cfg["min_gain"] >= 1:
        raise ValueError("min_gain must be below one")
    return cfg


def _elapsed(result) -> float:
    if isinstance(result, dict):
        if result.get("correctness_passed", True) is not True:
            raise ValueError("a calibration candidate failed its numerical gate; it cannot be selected or hidden")
        result = result.get("elapsed_seconds")
    if type(result) not in (int, float) or not math.isfinite(result) or result <= 0:
        raise ValueError("the evaluator must return a positive complete-operator elapsed time")
    return float(result)


def paired_measure(reference, candidate, evaluate, *, arm, pairs, seed, phase, name):
    """AB/BA pairs on identical inputs (input seed = seed + pair); the order
    inside a pair alternates so drift cancels."""
    records = []
    for pair in range(pairs):
        sides = [("reference", reference), ("candidate", candidate)]
        if pair % 2:
            sides.reverse()
        times = {}
        for side, plan in sides:
            times[side] = _elapsed(evaluate(plan, seed + pair, arm, f"{phase}/{name}/pair{pair}/{side}"))
        records.append(dict(pair=pair, seed=seed + pair, execution_order=[s for s, _ in sides],
                            reference_seconds=times["reference"], candidate_seconds=times["candidate"],
                            fractional_gain=1 - times["candidate"] / times["reference"]))
    gain = 1 - math.exp(statistics.mean(math.log(r["candidate_seconds"] / r["reference_seconds"])
                                        for r in records))
    return dict(name=name, phase=phase, paired_samples=records, fractional_gain=gain,
                worst_pair_gain=min(r["fractional_gain"] for r in records),
                candidate_digest=role_digest(candidate), reference_digest=role_digest(reference))


def confirmed(record, minimum_gain) -> bool:
    """Every confirmation pair, and their geometric mean, must beat the
    pre-declared threshold; nothing is trimmed or re-selected."""
    return record["fractional_gain"] > minimum_gain and all(
        r["fractional_gain"] > minimum_gain for r in record["paired_samples"])


def _fit_order(shape, evaluate, cfg, seed):
    m, n, k, world, chunk_rows = shape
    identity = make_role(*shape)
    trials, best, best_name, best_gain = [], identity, "identity", 0.0
    for cand in candidates(*shape)[1:]:
        plan = make_role(*shape, order=cand["arrival_order"])
        record = paired_measure(identity, plan, evaluate, arm=ARRIVAL_ARM, pairs=cfg["training_pairs"],
                                seed=seed, phase="arrival_training", name=cand["name"])
        trials.append(record)
        if record["fractional_gain"] > max(cfg["min_gain"], best_gain):
            best, best_name, best_gain = plan, cand["name"], record["fractional_gain"]
    confirmation, accepted = None, False
    if best_name != "identity":
        confirmation = paired_measure(identity, best, evaluate, arm=ARRIVAL_ARM,
                                      pairs=cfg["confirmation_pairs"], seed=seed + 1_000_000,
                                      phase="arrival_confirmation", name=best_name)
        accepted = confirmed(confirmation, cfg["min_gain"])
    order = (best if accepted else identity)["arrival_order"]
    diag = dict(selected_candidate=best_name if accepted else "identity", proposed_candidate=best_name,
                accepted=accepted, identity_fallback=not accepted, training_candidates=trials,
                confirmation=confirmation,
                changed_slots=sum(a != b for a, b in zip(identity["arrival_order"], order)))
    return order, diag


def _fit_mask(shape, order, evaluate, cfg, seed):
    blocks = len(order)
    q0 = make_role(*shape, order=order, mask=[False] * blocks)
    qall = make_role(*shape, order=order, mask=[True] * blocks)
    cap = math.floor(blocks * cfg["quant_budget"])
    singles, positive = [], []
    if cap:
        for physical in range(blocks):
            mask = [i == physical for i in range(blocks)]
            record = paired_measure(q0, make_role(*shape, order=order, mask=mask), evaluate, arm=SELECTIVE_ARM,
                                    pairs=cfg["training_pairs"], seed=seed + 2_000_000,
                                    phase="selective_singleton_training", name=f"block{physical}")
            record["physical_block"] = physical
            singles.append(record)
            if record["fractional_gain"] > 0:
                positive.append((record["fractional_gain"], physical))
    ranked = [physical for _, physical in sorted(positive, key=lambda item: (-item[0], item[1]))]
    limit = min(cap, len(ranked))
    sizes = sorted({c for c in (1, 2, 4, 8, limit) if 0 < c <= limit})
    prefixes, best, best_name, best_gain = [], q0, "Q0", 0.0
    for size in sizes:
        chosen = set(ranked[:size])
        plan = make_role(*shape, order=order, mask=[i in chosen for i in range(blocks)])
        record = paired_measure(q0, plan, evaluate, arm=SELECTIVE_ARM, pairs=cfg["training_pairs"],
                                seed=seed + 3_000_000, phase="selective_prefix_training", name=f"prefix{size}")
        record["selected_physical_blocks"] = sorted(chosen)
        prefixes.append(record)
        if record["fractional_gain"] > max(cfg["min_gain"], best_gain):
            best, best_name, best_gain = plan, f"prefix{size}", record["fractional_gain"]
    full = paired_measure(q0, qall, evaluate, arm=SELECTIVE_ARM, pairs=cfg["training_pairs"],
                          seed=seed + 4_000_000, phase="selective_full_control", name="Qall")
    if cap == blocks and full["fractional_gain"] > max(cfg["min_gain"], best_gain):
        best, best_name, best_gain = qall, "Qall", full["fractional_gain"]
    confirmation, accepted = None, False
    if best_name != "Q0":
        confirmation = paired_measure(q0, best, evaluate, arm=SELECTIVE_ARM, pairs=cfg["confirmation_pairs"],
                                      seed=seed + 5_000_000, phase="selective_confirmation", name=best_name)
        accepted = confirmed(confirmation, cfg["min_gain"])
    mask = (best if accepted else q0)["selective_mask"]
    diag = dict(selected_candidate=best_name if accepted else "Q0", proposed_candidate=best_name,
                accepted=accepted, zero_fallback=not accepted, budget_fraction=cfg["quant_budget"],
                budget_cap_blocks=cap, positive_singleton_blocks=ranked, singletons=singles,
                prefix_candidates=prefixes, full_control=full, confirmation=confirmation)
    return mask, diag


def validate_block_statistics(stats, blocks):
    """Codec statistics of one role on a calibration batch, per physical
    output block: ``error_sq`` = sum over the block's remote sources of the
    squared TACO round-trip error of their partial products, ``output_sq`` =
    squared norm of the reduced output block."""
    if not isinstance(stats, dict) or set(stats) != {"error_sq", "output_sq"}:
        raise ValueError("block statistics need exactly error_sq and output_sq")
    for key in ("error_sq", "output_sq"):
        values = stats[key]
        if (not isinstance(values, list) or len(values) != blocks
                or any(type(v) not in (int, float) or not math.isfinite(v) or v < 0 for v in values)):
            raise ValueError(f"block statistics {key}: one finite non-negative number per physical block")
    if sum(stats["output_sq"]) <= 0:
        raise ValueError("block statistics: the reduced output is all zero")
    return stats


def _fit_mask_error(shape, order, stats, cfg):
    """Selective mask by error budget: blocks in ascending order of their
    codec error (ties by block index) are added while the predicted relative
    L2 error of the whole projection output, sqrt(sum chosen error_sq / sum
    output_sq), stays within ``error_budget`` and the count within the block
    budget.  Every block saves the same wire bytes, so the cheapest-error
    blocks are the ones worth compressing.  No timing is involved."""
    blocks = len(order)
    validate_block_statistics(stats, blocks)
    cap = math.floor(blocks * cfg["quant_budget"])
    err, out_total = stats["error_sq"], sum(stats["output_sq"])
    ranked = sorted(range(blocks), key=lambda p: (err[p], p))
    chosen, spent = [], 0.0
    for physical in ranked:
        if len(chosen) == cap or math.sqrt((spent + err[physical]) / out_total) > cfg["error_budget"]:
            break
        chosen.append(physical)
        spent += err[physical]
    mask = [p in set(chosen) for p in range(blocks)]
    diag = dict(method="error_budget", selected_candidate=f"error_budget{len(chosen)}", accepted=bool(chosen),
                zero_fallback=not chosen, budget_fraction=cfg["quant_budget"], budget_cap_blocks=cap,
                error_budget=cfg["error_budget"], ranked_blocks=ranked, selected_physical_blocks=sorted(chosen),
                predicted_relative_l2=math.sqrt(spent / out_total),
                block_statistics=dict(error_sq=list(err), output_sq=list(stats["output_sq"])))
    return mask, diag


def fit_role(m, n, k, world, chunk_rows, evaluate, *, config=None, seed=8_000_000, block_stats=None):
    """Measure, confirm and freeze one role plan.  With ``selection_mode``
    "error_budget" the selective mask comes from ``block_stats`` (see
    ``validate_block_statistics``) instead of paired timing; the arrival
    order is always chosen by timing."""
    cfg = settings(config)
    shape = (m, n, k, world, chunk_rows)
    order, arrival = _fit_order(shape, evaluate, cfg, seed)
    if cfg.get("selection_mode") == "error_budget":
        if block_stats is None:
            raise ValueError("selection_mode 'error_budget' needs the calibration batch's block statistics")
        mask, selective = _fit_mask_error(shape, order, block_stats, cfg)
    else:
        mask, selective = _fit_mask(shape, order, evaluate, cfg, seed)
    final = make_role(*shape, order=order, mask=mask)
    final["diagnostics"] = dict(
        method="same-codec-paired-complete-operator-selection-v2", settings=cfg,
        arrival=arrival, selective=selective, actual_selection=quantization_statistics(final, world),
        limitation="Role-shape operator calibration, not a guarantee of layer-specific or full-step "
                   "benefit; confirmation does not reselect.")
    return validate_role_plan(final, m, n, k, world, chunk_rows)
