"""Synthetic rank rows of a five-arm batch for the protocol / controller
tests: what a correct worker would write for each job (calibration samples
from the real planner with injected timings, operator records, training
windows in which the order-only TACO arms trained identically)."""
import hashlib
import json

from tempname_dcu_b200.experiment import protocol as p
from tempname_dcu_b200.runtime import operator_layout

ENV = dict(device_name="B200", host="h")


def _sha(data: bytes):
    return hashlib.sha256(data).hexdigest()


def _state(model, world, rank, arm, role, calls, plan_bundle, selective_mode="wire"):
    m = model["sequence"] * model["micro_batch"]
    k = (model["hidden"] if role == "attn" else model["ffn"]) // world
    role_plan = plan_bundle["roles"][role] if arm in (p.ARRIVAL, p.SELECTIVE) else None
    lay = operator_layout(m, model["hidden"], k, world, rank, arm, role_plan, model["chunk_rows"])
    from tempname_dcu_b200.mapping import selection_statistics
    sel = selection_statistics(m, model["hidden"], world, model["chunk_rows"], lay["selection_mask"])
    return dict(backend=p.BACKEND, arm=arm, rank=rank, calls=calls, shape=p.role_shape(model, world, role),
                chunk_rows=model["chunk_rows"], production_schedule=lay["order"],
                mapping_sha256=hashlib.sha256(json.dumps(lay["order"], sort_keys=True).encode()).hexdigest(),
                gemms_per_call=1, collectives_per_call=1, fused_kernel="tdb::rs::gemm_rs_kernel",
                quantization=("selective_remote_h128_e4m3" if arm == p.SELECTIVE else
                              "none" if arm == "flux" else "all_remote_h128_e4m3"),
                selection_mask=lay["selection_mask"],
                selected_remote_blocks_by_source=sel["selected_remote_blocks_by_source"],
                remote_wire_bytes_by_source=sel["remote_wire_bytes_by_source"],
                remote_wire_bytes_per_source=sel["remote_wire_bytes_by_source"][rank],
                actual_remote_wire_bytes_per_rank=sel["remote_wire_bytes_by_source"][rank],
                plan_sha256=p.digest(role_plan) if role_plan is not None else None, reduction_order=list(range(world)),
                rounding="bf16_after_each_source", scratch_bytes=1, original_cuda_flux=False, transport_lanes=2,
                consumer_policy=lay["consumer_policy"], validation_calls=2, diagnostic_delay_cycles=0,
                diagnostic_delay_in_normal_forward=False) | _fp8_fields(model, world, arm, lay, selective_mode)


def _fp8_fields(model, world, arm, lay, selective_mode):
    if selective_mode != "fp8-mma" or arm != p.SELECTIVE:
        return {}
    per = model["sequence"] * model["micro_batch"] // world // model["chunk_rows"]
    bf16 = (world - 1) * per * model["chunk_rows"] * model["hidden"] * 2
    return dict(selective_mode="fp8-mma", mma_block_mask=lay["selection_mask"], fused_kernel="tdb::rs::gemm_rs_mx_kernel",
                quantization="selective_mma_e4m3_ue8m0_k32", remote_wire_bytes_by_source=[bf16] * world,
                remote_wire_bytes_per_source=bf16, actual_remote_wire_bytes_per_rank=bf16)


def _diag(config, arm):
    if arm not in (p.ARRIVAL, p.SELECTIVE):
        return None
    base = p.expected_schedule(config["model"], config["world_size"], "flux_taco_interleaved")
    pending = next(it["physical"] for it in base if it["lane"] == 0)
    events = [dict(stage="consumer", physical=pending, lane=0, start_ms=0.0, end_ms=5.0),
              dict(stage="consumer", physical=pending + 1, lane=1, start_ms=0.0, end_ms=1.0)]
    return dict(passed=True, numerical_bitwise_equal=True, artificial=True, delayed_rank=0, delayed_lane=0,
                delayed_physical=pending, delay_cycles=50_000_000, later_blocks_completed_before_pending=[pending + 1],
                ready_bypass_observed=True, evidence=dict(events=events), ordinary_speedup_claim=False)



def fake_rows(job, job_config, directory, library_sha256, world=2):
    """Rank rows of one job (and, for calibrate, the raw sample files in
    ``directory``).  Returns (rows, calibrated bundle or None)."""
    from tempname_dcu_b200 import planning as P
    config, model = job_config, job_config["model"]
    execution_plan = job_config.get("execution_plan")
    build = dict(library_sha256=library_sha256, identity=dict(source_sha256="e" * 64))
    env = ENV
    bundle = None
    rows = []
    for rank in range(world):
        row = dict(rank=rank, world_size=world, stage=job["stage"], arm=job["arm"], run_id=config["run_id"],
                   completed=True, passed=True, execution_plan_sha256=job_config.get("execution_plan_sha256"),
                   backend=p.BACKEND, original_cuda_flux=False, environment_identity=env, codec_build=build)
        rows.append(row)
    if job["stage"] == "calibrate":
        samples = []
        roles = {}
        for index, role in enumerate(("attn", "mlp")):
            m, n, k = p.role_shape(model, world, role)

            def evaluate(cand, seed, arm, label, role=role):
                t = 1.0 - 0.001 * sum(cand["selective_mask"])
                samples.append(dict(role=role, label=label, seed=seed, arm=arm,
                                    plan_digest=P.role_digest(cand), arrival_order=cand["arrival_order"],
                                    selective_mask=cand["selective_mask"], iterations=config["calibration"]["iterations"],
                                    warmup=config["calibration"]["warmup"], max_rank_elapsed_seconds=t,
                                    bf16_relative_l2=0.01, codec_reference_relative_l2=0.001,
                                    correctness_passed=True))
                return t
            stats = None
            if config["calibration"].get("selection_mode") == "error_budget":
                blocks = m // model["chunk_rows"]
                stats = dict(error_sq=[1e-5 * (1 + (7 * b) % 5) for b in range(blocks)], output_sq=[1.0] * blocks)
            roles[role] = P.fit_role(m, n, k, world, model["chunk_rows"], evaluate, config=config["calibration"],
                                     seed=8_000_000 + 10_000_000 * index + config["seed"], block_stats=stats)
        bundle = dict(schema=P.SCHEMA, world_size=world, transport_lanes=2, roles=roles)
        for row in rows:
            mine = [dict(s, local_elapsed_seconds=s["max_rank_elapsed_seconds"] * (1 if row["rank"] else 0.9))
                    for s in samples]
            name = f"calibration-rank{row['rank']}-samples.json"
            p.write(directory / name, dict(schema="b200-calibration-samples-v1", rank=row["rank"], samples=mine))
            row.update(calibration_plan=bundle, calibration_results=dict(
                plan_sha256=p.digest(bundle), raw_samples=mine, raw_samples_file=name))
    elif job["stage"] == "operator":
        calls = 2 + config["timing"]["operator_warmup"] + config["timing"]["operator_iterations"]
        for row in rows:
            results = []
            for role in ("attn", "mlp"):
                results.append(dict(role=role, elapsed_seconds=0.001 * (1 + row["rank"]),
                                    timed_iterations=config["timing"]["operator_iterations"],
                                    correctness_passed=True, bf16_relative_l2=0.004,
                                    codec_reference_relative_l2=0.001, changed_input_relative_l2=0.001,
                                    order_bitwise_equal=True if job["arm"] != "flux" else None,
                                    full_gemm_only_seconds=0.0005, profile=None,
                                    arrival_diagnostic=_diag(config, job["arm"]),
                                    execution=_state(model, world, row["rank"], job["arm"], role, calls,
                                                     execution_plan, config.get("selective_mode", "wire"))))
            row.update(operator_results=results, initialization_sha256="a" * 64, input_sha256="b" * 64)
    elif job["stage"] == "train":
        steps, warm = config["timing"]["timed_steps"], config["timing"]["warmup_steps"]
        total = (steps + warm) * model["accumulation_steps"]
        counts = p.expected_parameter_counts(model, world)
        # order-only TACO arms train bitwise identically; flux and the selective arm differ
        same = job["arm"] in p.FULL_TACO_ARMS
        tag = "taco" if same else job["arm"]
        for row in rows:
            states = [_state(model, world, row["rank"], job["arm"], "attn" if i % 2 == 0 else "mlp", total,
                             execution_plan, config.get("selective_mode", "wire")) for i in range(2 * model["layers"])]
            for st in states:
                st["validation_calls"] = 1
                st["consumer_policy"] = p.expected_consumer_policy(job["arm"], "train")
            row.update(timed_steps=steps, warmup_steps=warm, elapsed_seconds=0.5 + 0.01 * row["rank"],
                       losses=[9.0 - 0.1 * i - (0 if same else 0.001) for i in range(steps)],
                       grad_norms=[1.0 + 0.01 * i for i in range(steps)],
                       initialization_sha256="c" * 64, input_sha256="d" * 64,
                       final_parameters_sha256=_sha(tag.encode()), actual_model_config=dict(model),
                       parameter_counts=counts, actual_parameters_per_rank=counts["parameters_per_rank"],
                       tokens_per_step=model["sequence"] * model["micro_batch"] * model["accumulation_steps"],
                       dtype="bfloat16", optimizer="AdamW-fp32-master",
                       operator_counters=dict(model_forwards=steps * model["accumulation_steps"],
                                              target_modules=2 * model["layers"],
                                              actual_calls_per_instance=[total] * (2 * model["layers"])),
                       operator_states=states,
                       memory=dict(peak_allocated_bytes=1 << 30, peak_reserved_bytes=1 << 31))
    return rows, bundle
