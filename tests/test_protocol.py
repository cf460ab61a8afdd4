"""Experiment protocol, controller and report replay on CPU (reference:
tests/test_protocol.py).  A synthetic batch directory (frozen sources, plan,
rank rows, a stand-in native library) must be accepted by ``replay`` and
every tamper must be rejected."""
import copy
import hashlib
import json
import os
from pathlib import Path
import signal
import subprocess
import sys
import time

import pytest

from tempname_dcu_b200.experiment import controller as C
from tempname_dcu_b200.experiment import protocol as p
from tempname_dcu_b200.experiment import report as R
from tempname_dcu_b200.runtime import operator_layout

ROOT = Path(__file__).resolve().parents[1]


def test_counterbalanced_orders():
    cycle = p.orders(2, 10)
    assert len(cycle) == 20
    first = [tuple(b["arms"]) for b in cycle[:10]]
    assert len(set(first)) == 10
    for arm in p.ARMS:
        assert sum(b["arms"].index(arm) == 0 for b in cycle[:10]) == 2
    assert [b["arms"] for b in cycle[10:]] == [b["arms"] for b in cycle[:10]][::-1]


def test_short_runs_have_no_ci():
    assert p.balanced(10) and p.balanced(20) and not p.balanced(1) and not p.balanced(15)
    assert R.pair_statistics([1.0] * 3, [2.0] * 3, False)["ci95"] is None
    stats = R.pair_statistics([1.0 + 0.01 * i for i in range(10)], [2.0] * 10, True)
    assert stats["ci95"] is not None and stats["percent"] > 0 and stats["faster_blocks"] == 10


def test_job_counts():
    assert len(p.jobs(1, 1, "preflight")) == 1
    assert len(p.jobs(1, 1, "operator")) == 2 + 5
    assert len(p.jobs(2, 10, "train")) == 2 + 2 * 2 * 10 * 5
    assert [j["stage"] for j in p.jobs(1, 1, "train")][:2] == ["preflight", "calibrate"]


def test_arm_subsets_keep_counterbalancing_and_skip_unused_stages():
    pair = ("flux", "flux_taco")
    cycle = p.orders(1, 4, pair)
    assert [b["arms"] for b in cycle] == [["flux", "flux_taco"], ["flux_taco", "flux"],
                                          ["flux_taco", "flux"], ["flux", "flux_taco"]]
    assert p.balanced(4, pair) and not p.balanced(2, ("flux", "flux_taco", p.ARRIVAL))
    stages = [j["stage"] for j in p.jobs(1, 2, "train", pair)]
    assert "calibrate" not in stages and stages.count("operator") == stages.count("train") == 4
    assert [j["stage"] for j in p.jobs(1, 1, "train", (p.SELECTIVE,))][:2] == ["preflight", "calibrate"]
    assert p.select_arms(["flux_taco", "flux"]) == pair  # canonical order
    single = p.jobs(1, 2, "train", ("flux",), world=1)
    assert [j["stage"] for j in single] == ["preflight", "train", "train"]
    with pytest.raises(ValueError):
        p.select_arms(["flux", "flux"])
    with pytest.raises(ValueError):
        p.jobs(1, 1, "operator", ("flux",), world=1)


def test_cli_model_and_arm_flags(tmp_path):
    args = C.arguments(["--out", str(tmp_path / "x"), "--arm", "flux_taco", "--arm", "flux", "--vocab", "50257",
                        "--vocab-pad", "--accum", "8", "--world-size", "8"])
    assert args.arms == ("flux", "flux_taco")
    assert args.model["vocab"] == 50257 and args.model["pad_vocab"] and args.model["accumulation_steps"] == 8
    plan = C.plan_for(args)
    assert plan["arms"] == plan["config"]["arms"] == ["flux", "flux_taco"]
    assert plan["config"]["selective_mode"] == "wire"
    assert {j["arm"] for j in plan["jobs"] if j["stage"] == "train"} == {"flux", "flux_taco"}
    one = C.arguments(["--out", str(tmp_path / "y"), "--world-size", "1", "--arm", "flux", "--small-model"])
    assert [j["stage"] for j in C.plan_for(one)["jobs"]][:2] == ["preflight", "train"]


@pytest.mark.parametrize("argv", [["--world-size", "1"], ["--world-size", "1", "--arm", "flux", "--operator-only"],
                                  ["--selective-mode", "fp8"], ["--arm", "nope"], ["--accum", "0"],
                                  ["--vocab", "50257"]])
def test_new_cli_flags_rejected(argv):
    with pytest.raises((ValueError, SystemExit)):
        C.arguments(argv)


@pytest.mark.parametrize("argv", [["--blocks", "0"], ["--world-size", "3"], ["--steps", "0"],
                                  ["--report"], ["--quant-budget", "2"], ["--chunk-rows", "96"],
                                  ["--small-model", "--bench-model"]])
def test_cli_validation(argv):
    with pytest.raises((ValueError, SystemExit)):
        C.arguments(argv)


def test_preview_imports_no_torch_and_writes_nothing(tmp_path):
    out = tmp_path / "never"
    script = ("import sys; sys.path.insert(0, %r); from tempname_dcu_b200.experiment import controller as c; "
              "c.main(['--out', %r, '--small-model', '--world-size', '2', '--blocks', '1']); "
              "assert 'torch' not in sys.modules" % (str(ROOT), str(out)))
    result = subprocess.run([sys.executable, "-c", script], capture_output=True, text=True, check=True)
    plan = json.loads(result.stdout)
    assert plan["preview"] is True and plan["uses_gpu"] is False and not out.exists()


def test_shell_entry_is_preview_by_default(tmp_path):
    out = tmp_path / "never"
    result = subprocess.run(["bash", str(ROOT / "tempname_dcu_b200/experiment/run_init.sh"), "--out", str(out),
                             "--small-model", "--world-size", "2", "--blocks", "1"],
                            capture_output=True, text=True, check=True, env=dict(os.environ, TDB_PYTHON=sys.executable))
    assert json.loads(result.stdout)["preview"] is True and not out.exists()


def test_snapshot_covers_package_sources():
    names = {str(f.relative_to(ROOT)) for f in C.source_files()}
    assert "tempname_dcu_b200/planning.py" in names
    assert "tempname_dcu_b200/csrc/gemm_rs.cu" in names
    assert not any(name.endswith(".so") for name in names)


def test_stop_process_kills_only_its_group():
    proc = subprocess.Popen([sys.executable, "-c", "import time; time.sleep(60)"], start_new_session=True)
    time.sleep(0.2)
    C.stop_process(proc)
    assert proc.poll() is not None
    assert os.getpgid(os.getpid()) != proc.pid


def test_trajectory_mismatch_rejected():
    row = dict(initialization_sha256="a" * 64, input_sha256="b" * 64, losses=[1.0], grad_norms=[2.0],
               final_parameters_sha256="c" * 64)
    p.compare_taco_trajectories([row], [dict(row)])
    with pytest.raises(ValueError):
        p.compare_taco_trajectories([row], [dict(row, losses=[1.0000001])])
    with pytest.raises(ValueError):
        p.compare_taco_trajectories([row], [dict(row, final_parameters_sha256="d" * 64)])


# --------------------------------------------------------------- fixture
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


def _fixture(tmp_path, extra=(), train=False):
    """A complete batch directory built by the real planner (calibration
    replays from synthetic timings): operator scope, or (``train``) the full
    scope with training windows whose order-only TACO arms trained
    identically."""
    from tempname_dcu_b200 import planning as P
    scope = ["--steps", "2", "--warmup-steps", "1"] if train else ["--operator-only"]
    args = C.arguments(["--out", str(tmp_path / "run"), "--small-model", "--world-size", "2", "--blocks", "1",
                        *scope, "--operator-warmup", "1", "--operator-iters", "2",
                        "--calibration-pairs", "1", "--quant-budget", "0.25", *extra])
    out = args.out
    files = C.source_files()
    manifest = {str(f.relative_to(ROOT)): p.sha(f) for f in files}
    plan = C.plan_for(args, manifest=manifest, run_id="r" * 32)
    for f in files:
        dest = out / "sources" / f.relative_to(ROOT)
        dest.parent.mkdir(parents=True, exist_ok=True)
        dest.write_bytes(f.read_bytes())
    library = b"stand-in native library"
    (out / "build").mkdir(parents=True)
    (out / "build" / "libtdb.so").write_bytes(library)
    build = dict(library_sha256=_sha(library), identity=dict(source_sha256="e" * 64))
    p.write(out / "source-manifest.json", manifest)
    p.write(out / "plan.json", plan)
    config, world, model = plan["config"], 2, plan["config"]["model"]
    env = dict(device_name="B200", host="h")
    completed, execution_plan = [], None
    for job in plan["jobs"]:
        directory = out / "results" / job["directory"]
        directory.mkdir(parents=True)
        job_config = p.config_for_job(config, job, execution_plan)
        p.write(directory / "config.json", job_config)
        p.write(directory / "command.json", dict(job=job, command=["x"], environment={}))
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
                roles[role] = P.fit_role(m, n, k, world, model["chunk_rows"], evaluate, config=config["calibration"],
                                         seed=8_000_000 + 10_000_000 * index + config["seed"])
            bundle = dict(schema=P.SCHEMA, world_size=world, transport_lanes=2, roles=roles)
            for row in rows:
                mine = [dict(s, local_elapsed_seconds=s["max_rank_elapsed_seconds"] * (1 if row["rank"] else 0.9))
                        for s in samples]
                name = f"calibration-rank{row['rank']}-samples.json"
                p.write(directory / name, dict(schema="b200-calibration-samples-v1", rank=row["rank"], samples=mine))
                row.update(calibration_plan=bundle, calibration_results=dict(
                    plan_sha256=p.digest(bundle), raw_samples=mine, raw_samples_file=name))
            execution_plan = bundle
            p.write(out / "selection-plan.json", bundle)
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
        for row in rows:
            p.write(directory / f"rank{row['rank']}.json", row)
        done = dict(job=job, command_sha256=p.sha(directory / "command.json"),
                    rank_sha256={f"rank{r}.json": p.sha(directory / f"rank{r}.json") for r in range(world)})
        if job["stage"] == "calibrate":
            done.update(execution_plan_sha256=p.digest(execution_plan),
                        selection_plan_file_sha256=p.sha(out / "selection-plan.json"))
        completed.append(done)
    p.write(out / "completed-jobs.json", completed)
    return out


def test_replay_accepts_fixture_and_renders_markdown(tmp_path):
    out = _fixture(tmp_path)
    report = R.replay(out)
    assert report["completed"] and report["results"]["operator"]
    text = R.markdown(report)
    assert "B200 five-arm experiment" in text and "flux_taco" in text


def test_replay_accepts_an_arm_subset(tmp_path):
    out = _fixture(tmp_path, ["--arm", "flux", "--arm", "flux_taco_interleaved"])
    report = R.replay(out)
    assert report["arms"] == ["flux", "flux_taco_interleaved"] and report["selection"] is None
    result = report["results"]["operator"]["trial1"]["attn"]
    assert set(result["arms"]) == {"flux", "flux_taco_interleaved"}
    assert set(result["pairs"]) == {"flux_taco_interleaved/flux"}
    assert "flux_taco_interleaved" in R.markdown(report)
    plan = json.loads((out / "plan.json").read_text())
    plan["arms"] = list(p.ARMS)  # a widened arm list no longer matches the frozen job list
    p.write(out / "plan.json", plan)
    with pytest.raises(ValueError):
        R.replay(out)


def test_replay_checks_the_fp8_mma_selective_contract(tmp_path):
    out = _fixture(tmp_path, ["--selective-mode", "fp8-mma"])
    report = R.replay(out)
    assert report["completed"] and report["selective_mode"] == "fp8-mma"
    assert "selective arm mode: fp8-mma" in R.markdown(report)
    sel = next(j["directory"] for j in json.loads((out / "plan.json").read_text())["jobs"]
               if j["stage"] == "operator" and j["arm"] == p.SELECTIVE)

    def wire_mode(row):  # a selective operator that still sent TACO packets breaks the fp8-mma contract
        row["operator_results"][0]["execution"]["fused_kernel"] = "tdb::rs::gemm_rs_kernel"
    _retamper(out, sel, 0, wire_mode)
    with pytest.raises(ValueError):
        R.replay(out)


def test_replay_accepts_training_windows(tmp_path):
    out = _fixture(tmp_path, train=True)
    report = R.replay(out)
    assert report["completed"] and report["training_windows"] == len(p.ARMS)
    assert report["full_quantized_trajectories_identical"]
    arms = report["results"]["train"]["trial1"]["full_step"]["arms"]
    assert set(arms) == set(p.ARMS) and all(v["tokens_per_second"] > 0 for v in arms.values())
    assert "tokens/s" in R.markdown(report)


@pytest.mark.parametrize("tamper", ["loss", "missing_window", "final_parameters", "bypassed_operator"])
def test_replay_rejects_training_tampering(tmp_path, tamper):
    out = _fixture(tmp_path, train=True)
    jobs = json.loads((out / "plan.json").read_text())["jobs"]
    taco = next(j["directory"] for j in jobs if j["stage"] == "train" and j["arm"] == "flux_taco_interleaved")
    if tamper == "loss":  # an order-only arm whose loss differs from the other TACO arms
        _retamper(out, taco, 0, lambda r: r["losses"].__setitem__(0, r["losses"][0] + 1e-6))
    elif tamper == "missing_window":
        completed = json.loads((out / "completed-jobs.json").read_text())
        p.write(out / "completed-jobs.json", completed[:-1])
    elif tamper == "final_parameters":
        _retamper(out, taco, 1, lambda r: r.update(final_parameters_sha256="0" * 64))
    elif tamper == "bypassed_operator":  # a projection that did not go through the fused operator
        _retamper(out, taco, 0, lambda r: r["operator_counters"]["actual_calls_per_instance"].__setitem__(0, 1))
    with pytest.raises((ValueError, FileNotFoundError, KeyError)):
        R.replay(out)


def _retamper(out, directory, rank, mutate):
    file = out / "results" / directory / f"rank{rank}.json"
    row = json.loads(file.read_text())
    mutate(row)
    p.write(file, row)
    completed = json.loads((out / "completed-jobs.json").read_text())
    for done in completed:
        if done["job"]["directory"] == directory:
            done["rank_sha256"][f"rank{rank}.json"] = p.sha(file)
    p.write(out / "completed-jobs.json", completed)


@pytest.mark.parametrize("tamper", ["row_bytes", "gate", "wire_bytes", "schedule", "library", "source",
                                    "calibration_time", "missing_rank", "diagnostic", "environment", "call_count",
                                    "calibration_seed", "operator_time"])
def test_replay_rejects_tampering(tmp_path, tamper):
    out = _fixture(tmp_path)
    op_dir = next(d for d in json.loads((out / "plan.json").read_text())["jobs"] if d["stage"] == "operator")["directory"]
    arrival_dir = next(d["directory"] for d in json.loads((out / "plan.json").read_text())["jobs"]
                       if d["stage"] == "operator" and d["arm"] == p.ARRIVAL)
    if tamper == "row_bytes":
        file = out / "results" / op_dir / "rank0.json"
        file.write_text(file.read_text().replace('"passed": true', '"passed":  true'))
    elif tamper == "gate":
        _retamper(out, op_dir, 0, lambda r: r["operator_results"][0].update(bf16_relative_l2=0.9))
    elif tamper == "wire_bytes":
        _retamper(out, op_dir, 1, lambda r: r["operator_results"][1]["execution"].update(
            remote_wire_bytes_per_source=1))
    elif tamper == "schedule":
        _retamper(out, op_dir, 0, lambda r: r["operator_results"][0]["execution"]["production_schedule"].reverse())
    elif tamper == "library":
        (out / "build" / "libtdb.so").write_bytes(b"changed")
    elif tamper == "source":
        file = out / "sources" / "tempname_dcu_b200" / "planning.py"
        file.write_text(file.read_text() + "\n# changed\n")
    elif tamper == "calibration_time":
        def mutate(row):
            row["calibration_results"]["raw_samples"][0]["max_rank_elapsed_seconds"] *= 2
        _retamper(out, "calibrate", 0, mutate)
    elif tamper == "missing_rank":
        (out / "results" / op_dir / "rank1.json").unlink()
    elif tamper == "diagnostic":
        _retamper(out, arrival_dir, 0, lambda r: r["operator_results"][0]["arrival_diagnostic"].update(
            ready_bypass_observed=False))
    elif tamper == "environment":  # hardware identity drifts between workers
        _retamper(out, op_dir, 1, lambda r: r["environment_identity"].update(device_name="H100"))
    elif tamper == "call_count":  # an operator reports calls it did not make
        _retamper(out, op_dir, 0, lambda r: r["operator_results"][0]["execution"].update(
            calls=r["operator_results"][0]["execution"]["calls"] + 1))
    elif tamper == "calibration_seed":
        def mutate(row):
            row["calibration_results"]["raw_samples"][0]["seed"] += 1
        _retamper(out, "calibrate", 0, mutate)
    elif tamper == "operator_time":  # a rank's time that is not a positive finite number
        _retamper(out, op_dir, 1, lambda r: r["operator_results"][0].update(elapsed_seconds=-1.0))
    with pytest.raises((ValueError, FileNotFoundError, KeyError)):
        R.replay(out)
