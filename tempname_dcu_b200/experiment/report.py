"""Read-only audit, replay and paired statistics of a completed experiment.

``replay(out_dir)`` re-validates everything the controller wrote -- the
frozen source snapshot and its manifest, each job's configuration and
command, every rank row (through ``protocol.validate_rows``), the native
library bytes recorded in the rows, the calibration evidence (re-running the
frozen planner from the raw per-rank samples must reproduce the frozen plan),
and the trajectory identity of the TACO arms -- and then summarises operator
and training windows with paired log-ratio gains and a block bootstrap CI.
``markdown(report)`` renders the summary.

Reference parity: tools/dcu/phase6/report.py:10-405 (same statistics: gain
``100 * (1 - exp(mean log(Tc / Tr)))``, 10,000 bootstrap draws with seed
20261108 for balanced runs of >= 10 blocks, window time = max over ranks).
"""
from __future__ import annotations

import importlib.util
import math
from pathlib import Path
import random
import statistics

from ..mapping import selection_statistics
from . import protocol as p

BOOTSTRAP_SEED = 20261108


def pair_statistics(candidate, reference, balanced, bootstrap=10_000):
    p.require(len(candidate) == len(reference) and candidate, "unpaired samples")
    logs = [math.log(c / r) for c, r in zip(candidate, reference)]
    estimate = 100 * (1 - math.exp(statistics.mean(logs)))
    interval = None
    if balanced and len(logs) >= 10:
        rng = random.Random(BOOTSTRAP_SEED)
        draws = sorted(100 * (1 - math.exp(statistics.mean(rng.choices(logs, k=len(logs)))))
                       for _ in range(bootstrap))
        interval = [draws[int((bootstrap - 1) * 0.025)], draws[int((bootstrap - 1) * 0.975)]]
    return dict(percent=estimate, ci95=interval, paired_blocks=len(logs),
                faster_blocks=sum(c < r for c, r in zip(candidate, reference)))


def summary(values):
    return dict(mean=statistics.mean(values), median=statistics.median(values), min=min(values), max=max(values),
                windows=len(values))


PAIRS = (("flux_taco", "flux"), ("flux_taco_interleaved", "flux_taco"), (p.ARRIVAL, "flux_taco_interleaved"),
         (p.SELECTIVE, p.ARRIVAL), ("flux_taco_interleaved", "flux"), (p.ARRIVAL, "flux"), (p.SELECTIVE, "flux"))


def summarize_stage(samples, stage, trials, blocks, arms=p.ARMS):
    out = {}
    roles = ("attn", "mlp") if stage == "operator" else ("full_step",)
    for trial in range(1, trials + 1):
        by_role = {}
        for role in roles:
            values = {arm: [next(s["value"] for s in samples if s["trial"] == trial and s["block"] == b
                                 and s["arm"] == arm and s["role"] == role) for b in range(blocks)] for arm in arms}
            pairs = {f"{x}/{y}": pair_statistics(values[x], values[y], p.balanced(blocks, arms))
                     for x, y in PAIRS if x in values and y in values}
            result = {a: summary(v) for a, v in values.items()}
            for arm in arms:
                chosen = [s for s in samples if s["trial"] == trial and s["arm"] == arm and s["role"] == role]
                if stage == "train":
                    result[arm].update(
                        tokens_per_second=chosen[0]["tokens_per_step"] * 1000 / result[arm]["mean"],
                        mean_training_loss=statistics.mean(s["mean_loss"] for s in chosen),
                        mean_final_loss=statistics.mean(s["final_loss"] for s in chosen),
                        mean_grad_norm=statistics.mean(s["mean_grad_norm"] for s in chosen),
                        mean_final_grad_norm=statistics.mean(s["final_grad_norm"] for s in chosen),
                        max_peak_allocated_gib=max(s["peak_allocated_bytes"] for s in chosen) / 2 ** 30,
                        max_peak_reserved_gib=max(s["peak_reserved_bytes"] for s in chosen) / 2 ** 30)
                else:
                    result[arm].update(
                        full_gemm_only_mean_us=statistics.mean(s["full_gemm_only_us"] for s in chosen),
                        max_bf16_relative_l2=max(s["bf16_relative_l2"] for s in chosen),
                        max_codec_reference_relative_l2=max(s["codec_reference_relative_l2"] for s in chosen),
                        artificial_bypass_rank_windows=sum(len(s["artificial_bypass_ranks"]) for s in chosen),
                        artificial_diagnostic_rank_windows=sum(s["artificial_diagnostic_ranks"] for s in chosen))
            by_role[role] = dict(unit="us/call" if stage == "operator" else "ms/step", arms=result, pairs=pairs)
        out[f"trial{trial}"] = by_role
    return out


def validate_artifacts(root, directory, rows, config):
    """Re-hash the native library recorded by every rank (the snapshot keeps
    it under build/); fails if it is missing or changed."""
    root = Path(root)
    evidence = {}
    for row in rows:
        build = row["codec_build"]
        library = root / "build" / "libtdb.so"
        p.require(library.is_file(), "native library missing from the experiment directory")
        p.require(p.sha(library) == build["library_sha256"], "on-disk native library bytes changed")
        evidence[str(library.relative_to(root))] = build["library_sha256"]
        if row["stage"] == "operator" and config["profile"]:
            for record in row["operator_results"]:
                p.require(isinstance(record.get("profile"), dict), "missing requested profile")
    return evidence


def _frozen_planner(root):
    source = Path(root) / "sources" / "tempname_dcu_b200" / "planning.py"
    spec = importlib.util.spec_from_file_location("tdb_frozen_planner_audit", source)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def validate_calibration_evidence(root, directory, rows, config):
    """Replay the frozen planner from the raw per-rank samples without a GPU."""
    planner = _frozen_planner(root)
    plan = p.calibration_from_rows(rows, config)
    evidence, per_rank = {}, []
    for row in rows:
        record = row["calibration_results"]
        p.require(record.get("plan_sha256") == p.digest(plan), "calibration digest mismatch")
        samples = record.get("raw_samples")
        p.require(isinstance(samples, list) and samples, "missing raw calibration measurements")
        name = record.get("raw_samples_file")
        p.require(isinstance(name, str) and Path(name).name == name, "invalid calibration sample path")
        file = Path(directory) / name
        p.require(p.read(file) == dict(schema="b200-calibration-samples-v1", rank=row["rank"], samples=samples),
                  "calibration sample file differs from the rank row")
        evidence[str(file.relative_to(root))] = p.sha(file)
        per_rank.append(samples)
    p.require(all(len(s) == len(per_rank[0]) for s in per_rank), "calibration sample counts differ across ranks")
    for items in zip(*per_rank):
        strip = [{k: v for k, v in it.items() if k != "local_elapsed_seconds"} for it in items]
        p.require(all(x == strip[0] for x in strip), "calibration labels/inputs/aggregate times differ across ranks")
        p.require(all(p.finite_number(it.get("local_elapsed_seconds")) and it["local_elapsed_seconds"] > 0
                      for it in items), "invalid rank-local calibration time")
        p.require(items[0].get("max_rank_elapsed_seconds") == max(it["local_elapsed_seconds"] for it in items),
                  "calibration timing must be the maximum over ranks")
        for it in items:
            p.require(it.get("correctness_passed") is True and it.get("bf16_relative_l2", 1) <= 0.05
                      and it.get("codec_reference_relative_l2", 1) <= 0.01, "calibration candidate failed its gates")
    model, cfg, world = config["model"], config["calibration"], config["world_size"]
    stream = iter(per_rank[0])
    for index, role in enumerate(("attn", "mlp")):
        def evaluate(candidate, seed, arm, label):
            sample = next(stream, None)
            p.require(sample is not None, "missing calibration measurement during replay")
            expected = dict(role=role, label=label, seed=seed, arm=arm, plan_digest=planner.role_digest(candidate),
                            arrival_order=candidate["arrival_order"], selective_mask=candidate["selective_mask"],
                            iterations=cfg["iterations"], warmup=cfg["warmup"])
            p.require(all(sample.get(k) == v for k, v in expected.items()),
                      "calibration candidate/seed/order differs from the frozen planner replay")
            return sample["max_rank_elapsed_seconds"]
        shape = p.role_shape(model, world, role)
        # error-budget mode: the mask is recomputed from the statistics frozen in the plan
        stats = (plan["roles"][role]["diagnostics"].get("selective", {}).get("block_statistics")
                 if cfg.get("selection_mode") == "error_budget" else None)
        rebuilt = planner.fit_role(shape[0], shape[1], shape[2], world, model["chunk_rows"], evaluate, config=cfg,
                                   seed=8_000_000 + 10_000_000 * index + config["seed"], block_stats=stats)
        p.require(rebuilt == plan["roles"][role], "calibration replay does not reproduce the frozen role plan")
    p.require(next(stream, None) is None, "unexpected extra calibration samples")
    return evidence


def _role_bytes(model, world, mask):
    """Remote bytes one projection call puts on the links, summed over all
    sources, for a selection mask (from the mapping's per-source accounting)."""
    m = model["sequence"] * model["micro_batch"]
    stats = selection_statistics(m, model["hidden"], world, model["chunk_rows"], list(mask))
    return sum(stats["remote_wire_bytes_by_source"])


def execution_plan_summary(bundle, config):
    """Per role of the frozen plan: how far the arrival order moved from the
    common interleave, how many blocks the selective arm quantizes, and the
    remote bytes that selection puts on the links against all-BF16 and
    all-TACO traffic."""
    if bundle is None:
        return None
    model, world = config["model"], config["world_size"]
    interleave = [item["physical"] for item in p.expected_schedule(model, world, "flux_taco_interleaved")]
    count = len(interleave)
    bf16 = _role_bytes(model, world, [False] * count)
    full = _role_bytes(model, world, [True] * count)
    roles = {}
    for role, plan in bundle["roles"].items():
        order, mask = plan["arrival_order"], plan["selective_mask"]
        moved = sum(1 for slot, physical in enumerate(order) if physical != interleave[slot])
        wire = _role_bytes(model, world, mask)
        chosen = sum(mask)
        roles[role] = dict(
            arrival_identity=moved == 0, arrival_changed_slots=moved, selective_blocks=chosen,
            physical_blocks=count, actual_quantized_remote_fraction=chosen / count,
            remote_bytes_all_sources=wire, bf16_remote_bytes_all_sources=bf16,
            full_quantized_remote_bytes_all_sources=full, remote_bytes_ratio_to_bf16=wire / bf16,
            remote_bytes_ratio_to_full_quantized=wire / full,
            remote_bytes_reduction_vs_bf16_percent=100.0 * (bf16 - wire) / bf16,
            role_plan_sha256=p.digest(plan), diagnostics=plan["diagnostics"])
    return dict(execution_plan_sha256=p.digest(bundle), budget=config["calibration"]["quant_budget"],
                transport_lanes=2, roles=roles,
                limitation="The arrival order changes which blocks are produced first; the arrival arms "
                           "still consume with per-lane ready consumers whatever the order.")


def replay(root):
    root = Path(root)
    plan = p.read(root / "plan.json")
    config = plan["config"]
    p.require(config["protocol"] == p.PROTOCOL, "wrong protocol")
    p.validate_model(config["model"], config["world_size"])
    p.validate_calibration_options(config["calibration"])
    p.require(config.get("execution_plan") is None and config.get("execution_plan_sha256") is None,
              "the immutable base plan must not be rewritten after calibration")
    arms = p.select_arms(plan.get("arms"))
    p.require(config.get("arms", list(p.ARMS)) == list(arms), "plan and config disagree on the arms")
    p.require(plan["jobs"] == p.jobs(plan["trials"], plan["blocks"], plan["scope"], arms, config["world_size"]),
              "frozen schedule changed")
    manifest = p.read(root / "source-manifest.json")
    p.require(p.digest(manifest) == config["source_manifest_sha256"], "source manifest changed")
    for name, expected in manifest.items():
        p.require(p.sha(root / "sources" / name) == expected, f"frozen source changed: {name}")
    completed = p.read(root / "completed-jobs.json")
    p.require(len(completed) == len(plan["jobs"]), "incomplete worker sequence")
    samples = {"operator": [], "train": []}
    trajectories, rank_files, artifacts = {}, {}, {}
    identities = operator_identities = environment = native_identity = execution_plan = None
    calibration_files = {}
    for job, done in zip(plan["jobs"], completed):
        p.require(job == done["job"], "completed job order/identity mismatch")
        directory = root / "results" / job["directory"]
        job_config = p.read(directory / "config.json")
        p.require(job_config == p.config_for_job(config, job, execution_plan), "job configuration drift")
        command = p.read(directory / "command.json")
        p.require(command.get("job") == job and p.sha(directory / "command.json") == done["command_sha256"],
                  "worker command identity drift")
        rows = []
        for rank in range(config["world_size"]):
            name = f"rank{rank}.json"
            file = directory / name
            p.require(p.sha(file) == done["rank_sha256"][name], "rank result bytes changed")
            rank_files[str(file.relative_to(root))] = done["rank_sha256"][name]
            rows.append(p.read(file))
        rows = p.validate_rows(rows, job, job_config)
        env = [r["environment_identity"] for r in rows]
        p.require(environment is None or env == environment, "hardware/software identity changed between workers")
        environment = env
        native = [r["codec_build"] for r in rows]
        p.require(native_identity is None or native == native_identity, "native library changed between workers")
        native_identity = native
        artifacts.update(validate_artifacts(root, directory, rows, job_config))
        if job["stage"] == "calibrate":
            p.require(execution_plan is None, "repeated calibration in a frozen experiment")
            execution_plan = p.calibration_from_rows(rows, job_config)
            file = root / "selection-plan.json"
            p.require(p.read(file) == execution_plan, "selection plan differs from the calibration rows")
            p.require(done.get("execution_plan_sha256") == p.digest(execution_plan)
                      and done.get("selection_plan_file_sha256") == p.sha(file), "frozen selection-plan hash changed")
            artifacts["selection-plan.json"] = p.sha(file)
            calibration_files = {str((directory / n).relative_to(root)): v for n, v in done["rank_sha256"].items()}
            artifacts.update(validate_calibration_evidence(root, directory, rows, job_config))
        elif job["stage"] == "train":
            identity = p.training_identity(rows)
            p.require(identities is None or identity == identities, "training initialisation/input changed")
            identities = identity
            trajectories.setdefault((job["trial"], job["block"]), {})[job["arm"]] = rows
            samples["train"].append(dict(
                trial=job["trial"], block=job["block"], arm=job["arm"], role="full_step",
                value=max(r["elapsed_seconds"] for r in rows) * 1000 / config["timing"]["timed_steps"],
                tokens_per_step=rows[0]["tokens_per_step"], mean_loss=statistics.mean(rows[0]["losses"]),
                final_loss=rows[0]["losses"][-1], mean_grad_norm=statistics.mean(rows[0]["grad_norms"]),
                final_grad_norm=rows[0]["grad_norms"][-1],
                peak_allocated_bytes=max(r["memory"]["peak_allocated_bytes"] for r in rows),
                peak_reserved_bytes=max(r["memory"]["peak_reserved_bytes"] for r in rows)))
        elif job["stage"] == "operator":
            current = p.training_identity(rows)
            p.require(operator_identities is None or current == operator_identities, "operator inputs changed")
            operator_identities = current
            for role in ("attn", "mlp"):
                records = [next(v for v in r["operator_results"] if v["role"] == role) for r in rows]
                samples["operator"].append(dict(
                    trial=job["trial"], block=job["block"], arm=job["arm"], role=role,
                    value=max(r["elapsed_seconds"] for r in records) * 1e6 / config["timing"]["operator_iterations"],
                    full_gemm_only_us=max(r["full_gemm_only_seconds"] for r in records) * 1e6
                    / config["timing"]["operator_iterations"],
                    bf16_relative_l2=max(r["bf16_relative_l2"] for r in records),
                    codec_reference_relative_l2=max(r["codec_reference_relative_l2"] for r in records),
                    artificial_bypass_ranks=[row["rank"] for row, rec in zip(rows, records)
                                             if rec.get("arrival_diagnostic")
                                             and rec["arrival_diagnostic"]["ready_bypass_observed"]],
                    artificial_diagnostic_ranks=config["world_size"] if job["arm"] in (p.ARRIVAL, p.SELECTIVE) else 0))
    for group in trajectories.values():
        p.require(set(group) == set(arms), "incomplete training block")
        taco = [a for a in p.FULL_TACO_ARMS if a in arms]
        for other in taco[1:]:
            p.compare_taco_trajectories(group[taco[0]], group[other])
    report = dict(protocol=p.PROTOCOL, run_id=config["run_id"], completed=True, completed_scope=plan["scope"],
                  hardware_target="B200, single node", world_size=config["world_size"], model=config["model"],
                  standard_tp8_workload=config["world_size"] == 8 and config["model"] in (p.MODEL, p.BENCH_MODEL),
                  implementation="fused tcgen05 GEMM + NVLink reduce-scatter kernel (tempname_dcu_b200)",
                  backend=p.BACKEND, original_cuda_flux=False, environment_identity=environment,
                  timing=config["timing"], recommended_image=p.RECOMMENDED_IMAGE, trials=plan["trials"],
                  blocks=plan["blocks"], arms=list(arms), selective_mode=config.get("selective_mode", "wire"),
                  counterbalanced=p.balanced(plan["blocks"], arms),
                  ci_available=p.balanced(plan["blocks"], arms) and bool(samples["operator"]),
                  short_run=not p.balanced(plan["blocks"], arms), all_windows_retained=True, correctness_passed=True,
                  full_quantized_trajectories_identical=bool(trajectories)
                  and sum(a in arms for a in p.FULL_TACO_ARMS) > 1,
                  trajectory_equivalence_arms=[a for a in p.FULL_TACO_ARMS if a in arms],
                  formal_optimizer_steps=len(samples["train"]) * config["timing"]["timed_steps"],
                  training_windows=len(samples["train"]), rank_sha256=rank_files, artifact_sha256=artifacts,
                  native_build_by_rank=native_identity, profile_requested=config["profile"],
                  calibration_config=config["calibration"], calibration_rank_sha256=calibration_files,
                  selection=execution_plan_summary(execution_plan, config),
                  execution_plan_sha256=p.digest(execution_plan) if execution_plan is not None else None,
                  samples=samples, results={})
    for stage in ("operator", "train"):
        if samples[stage]:
            report["results"][stage] = summarize_stage(samples[stage], stage, plan["trials"], plan["blocks"], arms)
    return report


def markdown(report):
    lines = ["# B200 five-arm experiment", "",
             f"Protocol `{report['protocol']}`; completed scope `{report['completed_scope']}`; "
             f"world size {report['world_size']}.", "",
             "Implementation: one fused tcgen05 GEMM + NVLink reduce-scatter kernel per projection call.", "",
             f"Arms: {', '.join(report.get('arms', p.ARMS))}; selective arm mode: "
             f"{report.get('selective_mode', 'wire')} ("
             + ("calibrated blocks computed as block-scaled FP8 MMAs, BF16 on the wire"
                if report.get("selective_mode") == "fp8-mma" else "calibrated blocks sent as TACO packets") + ").",
             ""]
    if report["short_run"]:
        lines += ["Short run (not a balanced 10-block cycle): no confidence intervals.", ""]
    lines += [f"Training windows: {report['training_windows']}; formal optimizer steps: "
              f"{report['formal_optimizer_steps']} (each window freshly initialised).", ""]
    if report["selection"]:
        lines += [f"Frozen calibration plan `{report['execution_plan_sha256']}`; quantization budget "
                  f"{report['selection']['budget']:.4%}.", "",
                  "| role | arrival order = identity | changed slots | quantized block fraction | remote bytes / BF16 |"
                  " remote bytes / full TACO |", "| --- | --- | ---: | ---: | ---: | ---: |"]
        for role, v in report["selection"]["roles"].items():
            lines.append(f"| {role} | {v['arrival_identity']} | {v['arrival_changed_slots']} | "
                         f"{v['actual_quantized_remote_fraction']:.4%} | {v['remote_bytes_ratio_to_bf16']:.6f} | "
                         f"{v['remote_bytes_ratio_to_full_quantized']:.6f} |")
        lines += [""]
    for stage, trials in report["results"].items():
        for trial, roles in trials.items():
            for role, result in roles.items():
                lines += [f"## {stage} / {trial} / {role}", "",
                          f"Unit: {result['unit']}; every window is the maximum over ranks.", "",
                          "| arm | mean | median | slowest window |", "| --- | ---: | ---: | ---: |"]
                for arm, v in result["arms"].items():
                    lines.append(f"| {arm} | {v['mean']:.6f} | {v['median']:.6f} | {v['max']:.6f} |")
                if stage == "train":
                    lines += ["", "| arm | tokens/s | mean loss | final loss | mean grad norm | peak allocated GiB |",
                              "| --- | ---: | ---: | ---: | ---: | ---: |"]
                    for arm, v in result["arms"].items():
                        lines.append(f"| {arm} | {v['tokens_per_second']:.3f} | {v['mean_training_loss']:.8g} | "
                                     f"{v['mean_final_loss']:.8g} | {v['mean_grad_norm']:.8g} | "
                                     f"{v['max_peak_allocated_gib']:.4f} |")
                else:
                    lines += ["", "| arm | GEMM-only mean us | max rel-L2 vs BF16 | max rel-L2 vs codec ref |",
                              "| --- | ---: | ---: | ---: |"]
                    for arm, v in result["arms"].items():
                        lines.append(f"| {arm} | {v['full_gemm_only_mean_us']:.3f} | "
                                     f"{v['max_bf16_relative_l2']:.6g} | {v['max_codec_reference_relative_l2']:.6g} |")
                    lines += ["", "| artificial skew diagnostic | bypass rank-windows / diagnosed rank-windows |",
                              "| --- | ---: |"]
                    for arm in (a for a in (p.ARRIVAL, p.SELECTIVE) if a in result["arms"]):
                        v = result["arms"][arm]
                        lines.append(f"| {arm} | {v['artificial_bypass_rank_windows']}/"
                                     f"{v['artificial_diagnostic_rank_windows']} |")
                lines += ["", "| candidate / reference | paired reduction % | 95% CI | faster blocks |",
                          "| --- | ---: | --- | ---: |"]
                for pair, v in result["pairs"].items():
                    ci = "n/a" if v["ci95"] is None else f"[{v['ci95'][0]:+.4f}, {v['ci95'][1]:+.4f}]"
                    lines.append(f"| {pair} | {v['percent']:+.4f} | {ci} | {v['faster_blocks']}/{v['paired_blocks']} |")
                lines.append("")
    lines += ["A positive reduction means the candidate is faster.  CIs bootstrap whole blocks; ranks and steps are "
              "not independent samples.  Loss and grad norm come from rank 0.", ""]
    return "\n".join(lines)
