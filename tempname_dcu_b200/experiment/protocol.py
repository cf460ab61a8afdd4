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
from pathlib import Path

from ..mapping import ARMS, BACKEND
from ..planning import SCHEMA as PLAN_SCHEMA

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


def require(value, message):
    if not value:
        raise ValueError(message)


def positive_int(value):
    return type(value) is int and value > 0


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


def sha(path):
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def digest(value):
    return hashlib.sha256(json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False).encode()).hexdigest()


def read(path):
    return json.loads(Path(path).read_text())


def write(path, value):
    """Atomic JSON write (temp file + replace)."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + ".tmp")
    tmp.write_text(json.dumps(value, indent=2, ensure_ascii=False, allow_nan=False) + "\n")
    tmp.replace(path)


def finite_number(value, nonnegative=False):
    return type(value) in (int, float) and math.isfinite(value) and (not nonnegative or value >= 0)


def valid_hash(value):
    return isinstance(value, str) and len(value) == 64 and all(c in "0123456789abcdef" for c in value)


def validate_calibration_options(options):
    require(set(options) == set(CALIBRATION), "wrong calibration option keys")
    for key in ("iterations", "training_pairs", "confirmation_pairs"):
        require(positive_int(options[key]), f"positive calibration {key} required")
    require(type(options["warmup"]) is int and options["warmup"] >= 0, "invalid calibration warmup")
    require(finite_number(options["quant_budget"]) and 0 <= options["quant_budget"] <= 1, "quant_budget in [0,1]")
    require(finite_number(options["min_gain"]) and 0 <= options["min_gain"] < 1, "min_gain in [0,1)")


def role_shape(model, world, role):
    return [model["sequence"] * model["micro_batch"], model["hidden"],
            model["hidden" if role == "attn" else "ffn"] // world]


def validate_execution_plan(bundle, config):
    model, world = config["model"], config["world_size"]
    require(isinstance(bundle, dict) and bundle.get("schema") == PLAN_SCHEMA and bundle.get("world_size") == world
            and bundle.get("transport_lanes") == 2, "wrong calibrated execution-plan identity")
    require(set(bundle.get("roles", {})) == {"attn", "mlp"}, "missing calibrated role")
    count = model["sequence"] * model["micro_batch"] // model["chunk_rows"]
    for role, plan in bundle["roles"].items():
        require(plan.get("shape") == role_shape(model, world, role) and plan.get("chunk_rows") == model["chunk_rows"],
                "calibrated plan shape/chunk mismatch")
        order, mask = plan.get("arrival_order"), plan.get("selective_mask")
        require(isinstance(order, list) and len(order) == count and all(type(i) is int for i in order)
                and sorted(order) == list(range(count)), "arrival order must be a physical-block bijection")
        require(all(p // (count // world) == slot % world for slot, p in enumerate(order)),
                "arrival plan must keep interleaved destination slots")
        require(isinstance(mask, list) and len(mask) == count and all(type(x) is bool for x in mask),
                "selection mask needs one bool per physical block")
        require(sum(mask) <= math.floor(count * config["calibration"]["quant_budget"] + 1e-12),
                "selection exceeds the frozen block budget")
        require(isinstance(plan.get("diagnostics"), dict), "missing calibration diagnostics")
    digest(bundle)
    return bundle


def config_for_job(base, job, execution_plan=None):
    require(base.get("execution_plan") is None and base.get("execution_plan_sha256") is None,
            "the base plan must stay uncalibrated and immutable")
    out = dict(base, job=job)
    if job["stage"] in ("operator", "train") and (execution_plan is not None
                                                   or needs_calibration(base.get("arms", ARMS))):
        validate_execution_plan(execution_plan, base)
        out.update(execution_plan=execution_plan, execution_plan_sha256=digest(execution_plan))
    return out


def calibration_from_rows(rows, config):
    plans = [row.get("calibration_plan") for row in rows]
    require(plans and all(p == plans[0] for p in plans), "ranks disagree on the calibrated execution plan")
    return validate_execution_plan(plans[0], config)


def expected_schedule(model, world, arm, role_plan=None):
    per = model["sequence"] * model["micro_batch"] // world // model["chunk_rows"]
    out = []
    for slot in range(world * per):
        if arm in (ARRIVAL, SELECTIVE):
            physical = role_plan["arrival_order"][slot]
            destination, within = divmod(physical, per)
        else:
            destination, within = ((slot % world, slot // world) if arm == "flux_taco_interleaved"
                                   else divmod(slot, per))
            physical = destination * per + within
        out.append(dict(slot=slot, destination=destination, within=within, physical=physical,
                        row=physical * model["chunk_rows"], rows=model["chunk_rows"], lane=within % 2))
    return out


def validate_operator_state(state, row, model, world, role, calls, execution_plan=None, selective_mode="wire"):
    """The operator's own account of a call sequence against the frozen arm
    contract.  With selective_mode "fp8-mma" the selective arm computes its
    calibrated blocks as block-scaled FP8 MMAs and sends every block as BF16."""
    shape = role_shape(model, world, role)
    fp8 = selective_mode == "fp8-mma" and row["arm"] == SELECTIVE
    role_plan = execution_plan["roles"][role] if row["arm"] in (ARRIVAL, SELECTIVE) else None
    sched = expected_schedule(model, world, row["arm"], role_plan)
    mapping_sha = hashlib.sha256(json.dumps(sched, sort_keys=True).encode()).hexdigest()
    mask = role_plan["selective_mask"] if row["arm"] == SELECTIVE else [row["arm"] != "flux"] * len(sched)
    per = len(sched) // world
    selected = [sum(flag and p // per != s for p, flag in enumerate(mask)) for s in range(world)]
    remote = (world - 1) * per
    elements = model["chunk_rows"] * model["hidden"]
    wires = [q * (elements // 128 * 136) + (remote - q) * elements * 2 for q in selected]
    if fp8:
        wires = [remote * elements * 2] * world
    require(state.get("backend") == BACKEND and state.get("arm") == row["arm"] and state.get("rank") == row["rank"],
            "wrong operator backend/arm/rank")
    require(state.get("shape") == shape and state.get("chunk_rows") == model["chunk_rows"],
            "wrong projection shape/chunk size")
    require(state.get("calls") == calls, f"wrong actual {role} projection call count")
    require(state.get("production_schedule") == sched and state.get("mapping_sha256") == mapping_sha,
            "actual production mapping is not the frozen arm schedule")
    kernel = "tdb::rs::gemm_rs_mx_kernel" if fp8 else "tdb::rs::gemm_rs_kernel"
    require(state.get("gemms_per_call") == 1 and state.get("collectives_per_call") == 1
            and state.get("fused_kernel") == kernel, "the operator must be one fused kernel")
    quant = ("selective_mma_e4m3_ue8m0_k32" if fp8 else "selective_remote_h128_e4m3" if row["arm"] == SELECTIVE else
             "none" if row["arm"] == "flux" else "all_remote_h128_e4m3")
    require(not fp8 or (state.get("selective_mode") == "fp8-mma" and state.get("mma_block_mask") == mask),
            "the FP8 MMA block mask is not the calibrated selective mask")
    require(state.get("quantization") == quant and state.get("reduction_order") == list(range(world))
            and state.get("rounding") == "bf16_after_each_source", "codec/reduction contract changed")
    require(state.get("remote_wire_bytes_per_source") == wires[row["rank"]]
            and state.get("actual_remote_wire_bytes_per_rank") == wires[row["rank"]]
            and state.get("remote_wire_bytes_by_source") == wires
            and state.get("selected_remote_blocks_by_source") == selected and state.get("selection_mask") == mask,
            "remote wire-byte accounting mismatch")
    require(state.get("plan_sha256") == (digest(role_plan) if role_plan is not None else None),
            "actual role-plan hash changed")
    require(state.get("original_cuda_flux") is False, "the B200 operator is not upstream CUDA Flux")
    require(type(state.get("scratch_bytes")) is int and state["scratch_bytes"] >= 0, "invalid scratch accounting")
    require(state.get("transport_lanes") == 2 and state.get("consumer_policy") ==
            ("per_lane_ready" if row["arm"] in (ARRIVAL, SELECTIVE) else "ordered")
            and state.get("validation_calls") == (2 if row["stage"] == "operator" else 1),
            "missing untimed per-instance validation or unexpected consumer policy")
    require(state.get("diagnostic_delay_cycles") == 0 and state.get("diagnostic_delay_in_normal_forward") is False,
            "the artificial lane delay must not enter measured operators")


def validate_arrival_diagnostic(record, row, config):
    diag = record.get("arrival_diagnostic")
    if row["arm"] not in (ARRIVAL, SELECTIVE):
        require(diag is None, "unexpected arrival diagnostic on a control arm")
        return
    require(isinstance(diag, dict) and diag.get("passed") is True and diag.get("numerical_bitwise_equal") is True
            and diag.get("artificial") is True and diag.get("ordinary_speedup_claim") is False,
            "missing successful artificial lane-skew check")
    require(diag.get("delayed_rank") == 0 and diag.get("delayed_lane") == 0 and diag.get("delay_cycles") == 50_000_000,
            "artificial lane-skew protocol changed")
    base = expected_schedule(config["model"], config["world_size"], "flux_taco_interleaved")
    pending = next(item["physical"] for item in base if item["lane"] == 0)
    require(diag.get("delayed_physical") == pending, "wrong delayed physical block")
    events = diag.get("evidence", {}).get("events")
    require(isinstance(events, list), "missing lane-skew event evidence")
    for event in events:
        require(event.get("stage") == "consumer" and type(event.get("physical")) is int
                and event.get("lane") in (0, 1) and finite_number(event.get("start_ms"))
                and finite_number(event.get("end_ms")) and event["end_ms"] >= event["start_ms"] - 1e-9,
                "invalid lane-skew event interval")
    rows = [e for e in events if e["physical"] == pending]
    overtakes = []
    if rows:
        overtakes = [e["physical"] for e in events if e["lane"] != 0 and e["end_ms"] < rows[0]["end_ms"]]
    require(diag.get("later_blocks_completed_before_pending") == overtakes
            and diag.get("ready_bypass_observed") is bool(overtakes),
            "artificial bypass claim disagrees with receiver-local evidence")


def expected_parameter_counts(model, world):
    from ..models.config import parameter_counts
    return parameter_counts(model, world)


def validate_rows(rows, job, config):
    world = config["world_size"]
    require(len(rows) == world and {r.get("rank") for r in rows} == set(range(world)),
            "missing, duplicate or unexpected rank")
    for row in rows:
        require(row.get("world_size") == world and row.get("stage") == job["stage"] and row.get("arm") == job["arm"],
                "worker identity does not match the job")
        require(row.get("completed") is True and row.get("passed") is True,
                f"rank {row.get('rank')} did not complete its correctness checks")
        require(row.get("run_id") == config["run_id"], "worker run_id mismatch")
        require(isinstance(row.get("environment_identity"), dict) and row["environment_identity"],
                "missing hardware/software identity")
        require(row.get("backend") == BACKEND and row.get("original_cuda_flux") is False,
                "wrong worker implementation identity")
        build = row.get("codec_build", {})
        require(valid_hash(build.get("library_sha256")) and valid_hash(build.get("identity", {}).get("source_sha256")),
                "missing native library provenance")
        require(row.get("execution_plan_sha256") == config.get("execution_plan_sha256"), "worker plan hash changed")
        if job["stage"] == "train":
            model, steps = config["model"], config["timing"]["timed_steps"]
            require(row.get("timed_steps") == steps and row.get("warmup_steps") == config["timing"]["warmup_steps"],
                    "wrong training step counts")
            require(finite_number(row.get("elapsed_seconds")) and row["elapsed_seconds"] > 0,
                    "invalid training elapsed time")
            for key in ("losses", "grad_norms"):
                values = row.get(key)
                require(isinstance(values, list) and len(values) == steps and all(finite_number(v, True) for v in values),
                        f"incomplete or non-finite {key}")
            for key in ("initialization_sha256", "input_sha256", "final_parameters_sha256"):
                require(valid_hash(row.get(key)), f"missing/invalid {key}")
            actual = row.get("actual_model_config", {})
            require(all(actual.get(k) == v for k, v in model.items()), "actual training model changed")
            counts = expected_parameter_counts(model, world)
            require(row.get("parameter_counts") == counts and
                    row.get("actual_parameters_per_rank") == counts["parameters_per_rank"],
                    "wrong trainable parameter count")
            tokens = model["sequence"] * model["micro_batch"] * model["accumulation_steps"]
            require(row.get("tokens_per_step") == tokens and row.get("dtype") == "bfloat16"
                    and row.get("optimizer") == "AdamW-fp32-master", "training dtype/optimizer/token budget changed")
            forwards = steps * model["accumulation_steps"]
            counters = row.get("operator_counters", {})
            require(counters.get("model_forwards") == forwards and counters.get("target_modules") == 2 * model["layers"],
                    "wrong formal model/module coverage")
            if world > 1:
                total = (steps + config["timing"]["warmup_steps"]) * model["accumulation_steps"]
                require(counters.get("actual_calls_per_instance") == [total] * (2 * model["layers"]),
                        "a projection bypassed the fused operator")
                states = row.get("operator_states", [])
                require(len(states) == 2 * model["layers"], "missing operator state")
                for index, state in enumerate(states):
                    validate_operator_state(state, row, model, world, "attn" if index % 2 == 0 else "mlp", total,
                                            config["execution_plan"], config.get("selective_mode", "wire"))
            memory = row.get("memory", {})
            require(all(type(memory.get(k)) is int and memory[k] >= 0 for k in
                        ("peak_allocated_bytes", "peak_reserved_bytes")), "missing allocator peak memory")
        elif job["stage"] == "operator":
            records = row.get("operator_results", [])
            require(len(records) == 2 and {r.get("role") for r in records} == {"attn", "mlp"},
                    "need both output-projection roles")
            for record in records:
                require(record.get("correctness_passed") is True, "independent operator correctness check failed")
                require(record.get("timed_iterations") == config["timing"]["operator_iterations"],
                        "wrong operator timing denominator")
                require(finite_number(record.get("elapsed_seconds")) and record["elapsed_seconds"] > 0,
                        "invalid operator elapsed time")
                for key, limit in (("bf16_relative_l2", 0.01 if row["arm"] == "flux" else 0.05),
                                   ("codec_reference_relative_l2", 0.01), ("changed_input_relative_l2", 0.01)):
                    require(finite_number(record.get(key), True) and record[key] <= limit,
                            f"operator numerical gate failed: {key}")
                require(row["arm"] == "flux" or record.get("order_bitwise_equal") is True,
                        "order-only numerical equivalence not verified")
                validate_arrival_diagnostic(record, row, config)
                require(finite_number(record.get("full_gemm_only_seconds")) and record["full_gemm_only_seconds"] > 0,
                        "missing full-GEMM control timing")
                validate_operator_state(record.get("execution", {}), row, config["model"], world, record["role"],
                                        2 + int(bool(config["profile"])) + config["timing"]["operator_warmup"]
                                        + config["timing"]["operator_iterations"], config["execution_plan"],
                                        config.get("selective_mode", "wire"))
                profile = record.get("profile")
                require(bool(profile) == bool(config["profile"]), "requested profile missing/unexpected")
            for key in ("initialization_sha256", "input_sha256"):
                require(valid_hash(row.get(key)), f"missing operator {key}")
        elif job["stage"] == "calibrate":
            validate_execution_plan(row.get("calibration_plan"), config)
            require(isinstance(row.get("calibration_results"), dict) and row["calibration_results"],
                    "missing rank-local calibration evidence")
    if job["stage"] == "calibrate":
        calibration_from_rows(rows, config)
    return sorted(rows, key=lambda r: r["rank"])


def training_identity(rows):
    return [[r["initialization_sha256"], r["input_sha256"]] for r in rows]


def compare_taco_trajectories(left, right):
    """Arms that only reorder production must train bitwise identically."""
    require(training_identity(left) == training_identity(right), "TACO arms have different initialisation/input")
    for a, b in zip(left, right):
        for key in ("losses", "grad_norms"):
            require(a[key] == b[key], f"TACO ordering changed {key}; investigate before timing claims")
        require(a.get("final_parameters_sha256") == b.get("final_parameters_sha256")
                and a.get("final_parameters_sha256"), "TACO final parameters differ")
