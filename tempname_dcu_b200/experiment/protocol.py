"""CPU-only contract of the calibrated five-arm experiment (no torch import).

Defines the protocol identity, the model presets, the counterbalanced arm
orders, the job list (preflight -> calibrate -> operator windows -> training
windows), the per-job configuration (with the frozen plan injected after
calibration), and the validators that every rank row, operator state and
arrival diagnostic must pass before a result is accepted.

Reference parity: tools/dcu/phase6/protocol.py:1-390.  The B200 operator is
one fused kernel per call, so its state reports ``gemms_per_call ==
collectives_per_call == 1`` and ``fused_kernel``; every other field and rule
(schedules, mapping hash, wire bytes, plan hash, reduction order, rounding,
diagnostic-delay isolation) is checked as in the reference.
"""
from __future__ import annotations

import hashlib
import json
import math
import os
from pathlib import Path
import re
import tempfile

from ..mapping import ARMS, BACKEND
from ..planning import OPTIONAL as OPTIONAL_CALIBRATION
from ..planning import SCHEMA as PLAN_SCHEMA
from ..planning import SELECTION_MODES

PROTOCOL = "b200-flux-five-arm-arrival-selective-v1"
ARRIVAL = "flux_taco_interleaved_arrival"
SELECTIVE = "flux_taco_interleaved_arrival_selective"
FULL_TACO_ARMS = ("flux_taco", "flux_taco_interleaved", ARRIVAL)
CALIBRATION = dict(warmup=2, iterations=5, training_pairs=3, confirmation_pairs=3, min_gain=0.002,
                   quant_budget=0.25)
RECOMMENDED_IMAGE = "CUDA 12.9 / PyTorch 2.11 (cu128) / NCCL 2.28, sm_100a"
MODEL = dict(layers=32, hidden=4096, ffn=16384, heads=32, sequence=2048, micro_batch=1, accumulation_steps=4,
             vocab=33792, chunk_rows=128)
# The benchmark's GPT-6.7B: vocab 50257 padded, 8 micro-batches per step.
BENCH_MODEL = dict(MODEL, vocab=50257, accumulation_steps=8, pad_vocab=True)
# Diagnostic model: head_dim 128 (the attention kernel's size) and 128-row
# chunks (the fused kernel's tile) at up to 8 ranks.
SMALL_MODEL = dict(layers=2, hidden=1024, ffn=4096, heads=8, sequence=2048, micro_batch=1, accumulation_steps=1,
                   vocab=8192, chunk_rows=128)
_OPTIONAL_MODEL_KEYS = {"pad_vocab"}


# --------------------------------------------------------------- basic checks and files

class _Missing:
    def __repr__(self):
        return "<missing>"


MISSING = _Missing()
_HASH = re.compile(r"[0-9a-f]{64}")


def require(condition, message):
    """The protocol's single failure path: a violated rule raises ValueError."""
    if not condition:
        raise ValueError(message)


def positive_int(value):
    return isinstance(value, int) and not isinstance(value, bool) and value > 0


def finite_number(value, nonnegative=False):
    if isinstance(value, bool) or not isinstance(value, (int, float)) or not math.isfinite(value):
        return False
    return value >= 0 or not nonnegative


def valid_hash(value):
    return isinstance(value, str) and _HASH.fullmatch(value) is not None


def canonical(value):
    """Canonical JSON bytes of a plan or manifest: sorted keys, no spaces, no NaN."""
    return json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False).encode()


def digest(value):
    return hashlib.sha256(canonical(value)).hexdigest()


def sha(path):
    with open(path, "rb") as fh:
        return hashlib.file_digest(fh, "sha256").hexdigest()


def read(path):
    with open(path, encoding="utf-8") as fh:
        return json.load(fh)


def write(path, value):
    """Write JSON atomically: a temporary file in the same directory, then a rename."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    text = json.dumps(value, indent=2, ensure_ascii=False, allow_nan=False) + "\n"
    fd, tmp = tempfile.mkstemp(dir=path.parent, prefix=path.name + ".", suffix=".tmp")
    try:
        with os.fdopen(fd, "w", encoding="utf-8") as fh:
            fh.write(text)
        os.replace(tmp, path)
    except BaseException:
        Path(tmp).unlink(missing_ok=True)
        raise


# --------------------------------------------------------------- declarative field checks
#
# A rule is (dotted path, predicate, reason).  check_fields looks every path
# up in a rank row / record / state and raises with the reason and the value
# found when the predicate does not hold.

def lookup(obj, path):
    for key in path.split("."):
        if not isinstance(obj, dict) or key not in obj:
            return MISSING
        obj = obj[key]
    return obj


def check_fields(obj, rules, what):
    for path, ok, reason in rules:
        value = lookup(obj, path)
        require(value is not MISSING and ok(value), f"{what}: {reason} ({path} = {value!r:.80})")


def equals(expected):
    return lambda v: v == expected


def is_true(v):
    return v is True


def is_false(v):
    return v is False


def positive_finite(v):
    return finite_number(v) and v > 0


def at_most(limit):
    return lambda v: finite_number(v, True) and v <= limit


def nonnegative_int(v):
    return isinstance(v, int) and not isinstance(v, bool) and v >= 0


def series(length):
    """A list of ``length`` finite non-negative numbers (losses, norms)."""
    return lambda v: isinstance(v, list) and len(v) == length and all(finite_number(x, True) for x in v)


def validate_calibration_options(options):
    require(isinstance(options, dict) and set(CALIBRATION) <= set(options) <= set(CALIBRATION) | set(OPTIONAL_CALIBRATION),
            "wrong calibration option keys")
    mode = options.get("selection_mode", "timing")
    require(mode in SELECTION_MODES, f"selection_mode must be one of {SELECTION_MODES}")
    require(("error_budget" in options) == (mode == "error_budget"),
            "error_budget is given exactly when selection_mode is 'error_budget'")
    if mode == "error_budget":
        require(finite_number(options["error_budget"]) and 0 < options["error_budget"] <= 1,
                "error_budget must lie in (0, 1]")
    check_fields(options, [
        ("iterations", positive_int, "positive integer required"),
        ("training_pairs", positive_int, "positive integer required"),
        ("confirmation_pairs", positive_int, "positive integer required"),
        ("warmup", nonnegative_int, "non-negative integer required"),
        ("quant_budget", lambda v: finite_number(v) and 0 <= v <= 1, "must lie in [0, 1]"),
        ("min_gain", lambda v: finite_number(v) and 0 <= v < 1, "must lie in [0, 1)"),
    ], "calibration options")


def validate_model(model, world):
    require(world in (1, 2, 4, 8), "world_size must be 1, 2, 4 or 8")
    require(set(MODEL) <= set(model) <= set(MODEL) | _OPTIONAL_MODEL_KEYS, "unexpected or missing model dimensions")
    require(all(positive_int(model[k]) for k in MODEL), "positive integer dimensions required")
    require(type(model.get("pad_vocab", False)) is bool, "pad_vocab must be a bool")
    require(model["hidden"] % model["heads"] == 0 and model["hidden"] // model["heads"] == 128,
            "head_dim must be 128")
    require(all(model[k] % world == 0 for k in ("hidden", "ffn", "heads")), "TP dimensions must divide world_size")
    require(model.get("pad_vocab") or model["vocab"] % world == 0, "vocab must divide world_size (or pad_vocab)")
    rows = model["sequence"] * model["micro_batch"]
    require(rows % world == 0 and (rows // world) % model["chunk_rows"] == 0,
            "chunk_rows must divide the per-rank output rows")
    require(model["chunk_rows"] % 128 == 0, "chunk_rows must be a multiple of the 128-row tile")
    require(model["hidden"] % 128 == 0, "the H128 codec needs hidden divisible by 128")
    return model


def select_arms(arms=None):
    """The arms one experiment compares, in the canonical order (all five by
    default).  A subset keeps the rotation/reverse counterbalancing among the
    chosen arms; the calibrate job runs only when an arrival arm is chosen."""
    if arms is None:
        return ARMS
    arms = list(arms)
    require(arms and len(set(arms)) == len(arms) and set(arms) <= set(ARMS), f"arms must be distinct names of {ARMS}")
    return tuple(a for a in ARMS if a in arms)


def needs_calibration(arms):
    return any(a in (ARRIVAL, SELECTIVE) for a in arms)


def orders(trials, blocks, arms=ARMS):
    """Counterbalanced arm orders: the rotations of the arm list and their
    reverses, the cycle reversed on odd trials."""
    require(positive_int(trials) and positive_int(blocks), "trials and blocks must be positive")
    arms = select_arms(arms)
    rotations = [list(arms[i:] + arms[:i]) for i in range(len(arms))]
    cycle = rotations + [r[::-1] for r in rotations]
    out = []
    for trial in range(trials):
        seq = cycle if trial % 2 == 0 else cycle[::-1]
        for block in range(blocks):
            out.append(dict(trial=trial + 1, block=block, arms=list(seq[block % len(seq)])))
    return out


def jobs(trials, blocks, scope, arms=ARMS, world=None):
    """preflight, then calibrate (arrival arms only), then the operator windows
    (skipped on one rank: no reduce-scatter), then the training windows."""
    require(scope in ("preflight", "operator", "train"), "invalid experiment scope")
    require(world != 1 or scope != "operator", "the operator windows need at least two ranks")
    arms = select_arms(arms)
    out = [dict(stage="preflight", arm=arms[0], trial=0, block=0, index=0, directory="preflight")]
    if scope == "preflight":
        return out
    if needs_calibration(arms):
        out.append(dict(stage="calibrate", arm=ARRIVAL, trial=0, block=0, index=1, directory="calibrate"))
    for stage in ("operator", "train"):
        if stage == "train" and scope != "train":
            break
        if stage == "operator" and world == 1:
            continue
        for block in orders(trials, blocks, arms):
            for arm in block["arms"]:
                out.append(dict(stage=stage, arm=arm, trial=block["trial"], block=block["block"], index=len(out),
                                directory=f"{stage}/trial{block['trial']}/block{block['block']:03d}-{arm}"))
    return out


def balanced(blocks, arms=ARMS):
    """Every rotation and its reverse appear equally often."""
    cycle = 2 * len(select_arms(arms))
    return blocks >= cycle and blocks % cycle == 0


# --------------------------------------------------------------- frozen plans and job configs

def role_shape(model, world, role):
    """[M, N, K] of a role's projection: M = rows of a micro-batch, N = hidden,
    K = the input width on one rank (attention-out h/W, FC2 f/W)."""
    k = model["hidden"] if role == "attn" else model["ffn"]
    return [model["sequence"] * model["micro_batch"], model["hidden"], k // world]


def physical_blocks(model):
    return model["sequence"] * model["micro_batch"] // model["chunk_rows"]


def validate_execution_plan(bundle, config):
    model, world = config["model"], config["world_size"]
    require(isinstance(bundle, dict), "calibrated execution plan missing")
    check_fields(bundle, [("schema", equals(PLAN_SCHEMA), "unknown plan schema"),
                          ("world_size", equals(world), "plan for another world size"),
                          ("transport_lanes", equals(2), "two transport lanes required")], "execution plan")
    require(isinstance(bundle.get("roles"), dict) and set(bundle["roles"]) == {"attn", "mlp"},
            "the plan needs exactly the attn and mlp roles")
    count = physical_blocks(model)
    per = count // world
    budget = math.floor(count * config["calibration"]["quant_budget"] + 1e-12)

    def bijection(order):
        return isinstance(order, list) and all(type(i) is int for i in order) and sorted(order) == list(range(count))

    def keeps_slots(order):  # slot s still feeds destination s % W (the interleaved slot structure)
        return all(physical // per == slot % world for slot, physical in enumerate(order))

    def block_mask(mask):
        return isinstance(mask, list) and len(mask) == count and all(type(x) is bool for x in mask)

    for role, plan in bundle["roles"].items():
        check_fields(plan, [
            ("shape", equals(role_shape(model, world, role)), "calibrated for another shape"),
            ("chunk_rows", equals(model["chunk_rows"]), "calibrated for another chunk size"),
            ("arrival_order", bijection, "arrival order must permute the physical blocks"),
            ("arrival_order", keeps_slots, "arrival order must keep the interleaved destination slots"),
            ("selective_mask", block_mask, "selection mask needs one bool per physical block"),
            ("selective_mask", lambda m: sum(m) <= budget, "selection exceeds the frozen block budget"),
            ("diagnostics", lambda d: isinstance(d, dict), "calibration diagnostics missing"),
        ], f"{role} plan")
    digest(bundle)  # must be canonical JSON (finite numbers only)
    return bundle


def config_for_job(base, job, execution_plan=None):
    """The job's config: the immutable base config plus the job, and -- for
    operator / training windows of an experiment that calibrates -- the
    frozen plan with its digest."""
    require(base.get("execution_plan") is None and base.get("execution_plan_sha256") is None,
            "the base plan must stay uncalibrated and immutable")
    config = {**base, "job": job}
    windowed = job["stage"] in ("operator", "train")
    if windowed and (execution_plan is not None or needs_calibration(base.get("arms", ARMS))):
        config["execution_plan"] = validate_execution_plan(execution_plan, base)
        config["execution_plan_sha256"] = digest(execution_plan)
    return config


def calibration_from_rows(rows, config):
    """The plan every rank froze; ranks must agree byte for byte."""
    require(rows, "no calibration rows")
    found = {canonical(row.get("calibration_plan")) for row in rows}
    require(len(found) == 1, "ranks disagree on the calibrated execution plan")
    return validate_execution_plan(rows[0].get("calibration_plan"), config)


# --------------------------------------------------------------- the operator contract

def _production_pairs(arm, world, per, role_plan):
    """(destination, block within destination) in production order."""
    if arm in (ARRIVAL, SELECTIVE):
        return [divmod(physical, per) for physical in role_plan["arrival_order"]]
    if arm == "flux_taco_interleaved":
        return [(d, w) for w in range(per) for d in range(world)]
    return [(d, w) for d in range(world) for w in range(per)]


def expected_schedule(model, world, arm, role_plan=None):
    """The arm's production schedule as the operator must report it."""
    per = physical_blocks(model) // world
    rows = model["chunk_rows"]
    return [dict(slot=slot, destination=d, within=w, physical=d * per + w, row=(d * per + w) * rows, rows=rows,
                 lane=w % 2)
            for slot, (d, w) in enumerate(_production_pairs(arm, world, per, role_plan))]


def expected_consumer_policy(arm, stage):
    """Arrival arms consume per lane, ready block first; the other arms in
    order, in every stage (the optional epilogue reduction of remote-first
    BF16 operators is off by default and not part of an experiment)."""
    del stage
    if arm in (ARRIVAL, SELECTIVE):
        return "per_lane_ready"
    return "ordered"


def expected_operator_state(model, world, arm, rank, role, calls, stage, execution_plan=None,
                            selective_mode="wire"):
    """Every exactly-known field of a correct operator's ``state()`` for this
    job: identity, shape, schedule and its hash, the one fused kernel, codec
    and reduction contract, per-source wire bytes from the frozen selection,
    plan hash, lanes / consumer policy, validation calls, no diagnostic delay."""
    arrival = arm in (ARRIVAL, SELECTIVE)
    role_plan = execution_plan["roles"][role] if arrival else None
    schedule = expected_schedule(model, world, arm, role_plan)
    count = len(schedule)
    per = count // world
    mask = list(role_plan["selective_mask"]) if arm == SELECTIVE else [arm != "flux"] * count
    # remote blocks each source quantizes: masked blocks owned by another rank
    selected = [sum(1 for phys, q in enumerate(mask) if q and phys // per != src) for src in range(world)]
    elements = model["chunk_rows"] * model["hidden"]
    packet, plain = elements // 128 * 136, elements * 2
    remote = (world - 1) * per
    fp8 = selective_mode == "fp8-mma" and arm == SELECTIVE
    wires = [remote * plain] * world if fp8 else [q * packet + (remote - q) * plain for q in selected]
    if fp8:
        quantization = "selective_mma_e4m3_ue8m0_k32"
    elif arm == SELECTIVE:
        quantization = "selective_remote_h128_e4m3"
    else:
        quantization = "none" if arm == "flux" else "all_remote_h128_e4m3"
    state = dict(
        backend=BACKEND, arm=arm, rank=rank, shape=role_shape(model, world, role), chunk_rows=model["chunk_rows"],
        calls=calls, production_schedule=schedule,
        mapping_sha256=hashlib.sha256(json.dumps(schedule, sort_keys=True).encode()).hexdigest(),
        gemms_per_call=1, collectives_per_call=1,
        fused_kernel="tdb::rs::gemm_rs_mx_kernel" if fp8 else "tdb::rs::gemm_rs_kernel",
        quantization=quantization, reduction_order=list(range(world)), rounding="bf16_after_each_source",
        selection_mask=mask, selected_remote_blocks_by_source=selected, remote_wire_bytes_by_source=wires,
        remote_wire_bytes_per_source=wires[rank], actual_remote_wire_bytes_per_rank=wires[rank],
        plan_sha256=digest(role_plan) if role_plan is not None else None, original_cuda_flux=False,
        transport_lanes=2, consumer_policy=expected_consumer_policy(arm, stage),
        validation_calls=2 if stage == "operator" else 1, diagnostic_delay_cycles=0,
        diagnostic_delay_in_normal_forward=False)
    if fp8:
        state.update(selective_mode="fp8-mma", mma_block_mask=mask)
    return state


def validate_operator_state(state, row, model, world, role, calls, execution_plan=None, selective_mode="wire"):
    """Compare the operator's own account field by field with the contract
    (expected_operator_state) of this job."""
    require(isinstance(state, dict), "operator state missing")
    expected = expected_operator_state(model, world, row["arm"], row["rank"], role, calls, row["stage"],
                                       execution_plan, selective_mode)
    for key, want in expected.items():
        got = state.get(key, MISSING)
        require(got == want, f"{role} operator state: {key} is {got!r:.80}, the frozen contract says {want!r:.80}")
    require(nonnegative_int(state.get("scratch_bytes")), "invalid scratch accounting")


# --------------------------------------------------------------- the artificial lane-skew diagnostic

LANE_SKEW = dict(delayed_rank=0, delayed_lane=0, delay_cycles=50_000_000)


def _first_lane0_block(config):
    """Physical block of the first lane-0 slot of the common interleave (the
    block whose signal the diagnostic holds back)."""
    schedule = expected_schedule(config["model"], config["world_size"], "flux_taco_interleaved")
    return next(item["physical"] for item in schedule if item["lane"] == 0)


def _consumer_event(e):
    return (isinstance(e, dict) and e.get("stage") == "consumer" and type(e.get("physical")) is int
            and e.get("lane") in (0, 1) and finite_number(e.get("start_ms")) and finite_number(e.get("end_ms"))
            and e["end_ms"] >= e["start_ms"] - 1e-9)


def validate_arrival_diagnostic(record, row, config):
    """Arrival arms carry a passed artificial lane-skew check whose bypass
    claim is recomputed here from its own consumer events; control arms
    carry none."""
    diag = record.get("arrival_diagnostic")
    if row["arm"] not in (ARRIVAL, SELECTIVE):
        require(diag is None, "unexpected arrival diagnostic on a control arm")
        return
    require(isinstance(diag, dict), "missing artificial lane-skew check")
    pending = _first_lane0_block(config)
    rules = [("passed", is_true, "the check did not pass"),
             ("numerical_bitwise_equal", is_true, "delayed and normal outputs differ"),
             ("artificial", is_true, "must be labelled artificial"),
             ("ordinary_speedup_claim", is_false, "claims an ordinary speed-up"),
             ("delayed_physical", equals(pending), "wrong delayed physical block"),
             ("evidence.events", lambda v: isinstance(v, list) and all(_consumer_event(e) for e in v),
              "invalid consumer event intervals")]
    rules += [(key, equals(value), "artificial lane-skew protocol changed") for key, value in LANE_SKEW.items()]
    check_fields(diag, rules, "arrival diagnostic")
    events = diag["evidence"]["events"]
    held = [e for e in events if e["physical"] == pending]
    bypass = [e["physical"] for e in events if held and e["lane"] != 0 and e["end_ms"] < held[0]["end_ms"]]
    require(diag.get("later_blocks_completed_before_pending") == bypass
            and diag.get("ready_bypass_observed") is bool(bypass),
            "artificial bypass claim disagrees with receiver-local evidence")


# --------------------------------------------------------------- rank rows

def expected_parameter_counts(model, world):
    from ..models.config import parameter_counts
    return parameter_counts(model, world)


def _identity_rules(job, config):
    world = config["world_size"]
    return [
        ("world_size", equals(world), "worker world size does not match the job"),
        ("stage", equals(job["stage"]), "worker stage does not match the job"),
        ("arm", equals(job["arm"]), "worker arm does not match the job"),
        ("completed", is_true, "the rank did not complete"),
        ("passed", is_true, "the rank's correctness checks failed"),
        ("run_id", equals(config["run_id"]), "worker run_id mismatch"),
        ("environment_identity", lambda v: isinstance(v, dict) and bool(v), "missing hardware/software identity"),
        ("backend", equals(BACKEND), "wrong worker backend"),
        ("original_cuda_flux", is_false, "the B200 operator is not upstream CUDA Flux"),
        ("codec_build.library_sha256", valid_hash, "missing native library hash"),
        ("codec_build.identity.source_sha256", valid_hash, "missing native source hash"),
        ("execution_plan_sha256", equals(config.get("execution_plan_sha256")), "worker plan hash changed"),
    ]


def _train_rules(config, world):
    model, timing = config["model"], config["timing"]
    steps = timing["timed_steps"]
    counts = expected_parameter_counts(model, world)
    layers2 = 2 * model["layers"]
    rules = [
        ("timed_steps", equals(steps), "wrong timed step count"),
        ("warmup_steps", equals(timing["warmup_steps"]), "wrong warm-up step count"),
        ("elapsed_seconds", positive_finite, "invalid training elapsed time"),
        ("losses", series(steps), "incomplete or non-finite losses"),
        ("grad_norms", series(steps), "incomplete or non-finite gradient norms"),
        ("initialization_sha256", valid_hash, "missing initial-weight hash"),
        ("input_sha256", valid_hash, "missing input hash"),
        ("final_parameters_sha256", valid_hash, "missing final-parameter hash"),
        ("actual_model_config", lambda v: isinstance(v, dict) and all(v.get(k) == x for k, x in model.items()),
         "the trained model differs from the frozen config"),
        ("parameter_counts", equals(counts), "wrong trainable parameter count"),
        ("actual_parameters_per_rank", equals(counts["parameters_per_rank"]), "wrong parameters per rank"),
        ("tokens_per_step", equals(model["sequence"] * model["micro_batch"] * model["accumulation_steps"]),
         "token budget changed"),
        ("dtype", equals("bfloat16"), "compute dtype changed"),
        ("optimizer", equals("AdamW-fp32-master"), "optimizer changed"),
        ("operator_counters.model_forwards", equals(steps * model["accumulation_steps"]), "wrong forward count"),
        ("operator_counters.target_modules", equals(layers2), "wrong projection module count"),
        ("memory.peak_allocated_bytes", nonnegative_int, "missing allocator peak"),
        ("memory.peak_reserved_bytes", nonnegative_int, "missing allocator peak"),
    ]
    if world > 1:
        total = (steps + timing["warmup_steps"]) * model["accumulation_steps"]
        rules += [("operator_counters.actual_calls_per_instance", equals([total] * layers2),
                   "a projection bypassed the fused operator"),
                  ("operator_states", lambda v: isinstance(v, list) and len(v) == layers2, "missing operator state")]
    return rules


def _check_train_row(row, config, world):
    check_fields(row, _train_rules(config, world), f"rank {row['rank']} training window")
    if world > 1:
        model, timing = config["model"], config["timing"]
        total = (timing["timed_steps"] + timing["warmup_steps"]) * model["accumulation_steps"]
        for index, state in enumerate(row["operator_states"]):
            validate_operator_state(state, row, model, world, ("attn", "mlp")[index % 2], total,
                                    config["execution_plan"], config.get("selective_mode", "wire"))


def _check_operator_row(row, config, world):
    records = row.get("operator_results")
    require(isinstance(records, list) and len(records) == 2 and {r.get("role") for r in records} == {"attn", "mlp"},
            "need both output-projection roles")
    timing = config["timing"]
    calls = 2 + int(bool(config["profile"])) + timing["operator_warmup"] + timing["operator_iterations"]
    plain_limit = 0.01 if row["arm"] == "flux" else 0.05
    rules = [
        ("correctness_passed", is_true, "independent operator correctness check failed"),
        ("timed_iterations", equals(timing["operator_iterations"]), "wrong operator timing denominator"),
        ("elapsed_seconds", positive_finite, "invalid operator elapsed time"),
        ("bf16_relative_l2", at_most(plain_limit), "gate vs plain BF16 failed"),
        ("codec_reference_relative_l2", at_most(0.01), "gate vs the codec reference failed"),
        ("changed_input_relative_l2", at_most(0.01), "changed-input reuse gate failed"),
        ("full_gemm_only_seconds", positive_finite, "missing full-GEMM control timing"),
    ]
    if row["arm"] != "flux":
        rules.append(("order_bitwise_equal", is_true, "order-only numerical equivalence not verified"))
    for record in records:
        check_fields(record, rules, f"rank {row['rank']} {record['role']} operator window")
        validate_arrival_diagnostic(record, row, config)
        validate_operator_state(record.get("execution"), row, config["model"], world, record["role"], calls,
                                config["execution_plan"], config.get("selective_mode", "wire"))
        require(bool(record.get("profile")) == bool(config["profile"]), "requested profile missing/unexpected")
    check_fields(row, [("initialization_sha256", valid_hash, "missing operator weight hash"),
                       ("input_sha256", valid_hash, "missing operator input hash")], f"rank {row['rank']}")


def _check_calibrate_row(row, config, world):
    validate_execution_plan(row.get("calibration_plan"), config)
    require(isinstance(row.get("calibration_results"), dict) and row["calibration_results"],
            "missing rank-local calibration evidence")


_STAGE_CHECKS = {"train": _check_train_row, "operator": _check_operator_row, "calibrate": _check_calibrate_row}


def validate_rows(rows, job, config):
    """All rank rows of one job against the job's frozen config; returns
    them sorted by rank."""
    world = config["world_size"]
    ranks = [r.get("rank") for r in rows]
    require(len(ranks) == world and set(ranks) == set(range(world)), "missing, duplicate or unexpected rank")
    identity = _identity_rules(job, config)
    stage_check = _STAGE_CHECKS.get(job["stage"])
    for row in rows:
        check_fields(row, identity, f"rank {row['rank']}")
        if stage_check is not None:
            stage_check(row, config, world)
    if job["stage"] == "calibrate":
        calibration_from_rows(rows, config)
    return sorted(rows, key=lambda r: r["rank"])


# --------------------------------------------------------------- training trajectories

IDENTITY_KEYS = ("initialization_sha256", "input_sha256")


def training_identity(rows):
    """Per rank, the hashes of the initial weights and the input batch."""
    return [[row[key] for key in IDENTITY_KEYS] for row in rows]


def compare_taco_trajectories(left, right):
    """Arms that only reorder production must train bitwise identically:
    same start, same loss and gradient-norm series, same final parameters."""
    require(training_identity(left) == training_identity(right), "TACO arms have different initialisation/input")
    for a, b in zip(left, right):
        differs = [key for key in ("losses", "grad_norms") if a[key] != b[key]]
        require(not differs, f"TACO ordering changed {', '.join(differs)}; investigate before timing claims")
        final = a.get("final_parameters_sha256")
        require(final and final == b.get("final_parameters_sha256"), "TACO final parameters differ")
