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
from _fake_batch import _diag, _sha, _state, fake_rows  # noqa: E402


def _fixture(tmp_path, extra=(), train=False):
    """A complete batch directory built by the real planner (calibration
    replays from synthetic timings): operator scope, or (``train``) the full
    scope with training windows whose order-only TACO arms trained
    identically."""
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
    p.write(out / "source-manifest.json", manifest)
    p.write(out / "plan.json", plan)
    config, world, model = plan["config"], 2, plan["config"]["model"]
    completed, execution_plan = [], None
    for job in plan["jobs"]:
        directory = out / "results" / job["directory"]
        directory.mkdir(parents=True)
        job_config = p.config_for_job(config, job, execution_plan)
        p.write(directory / "config.json", job_config)
        p.write(directory / "command.json", dict(job=job, command=["x"], environment={}))
        rows, bundle = fake_rows(job, job_config, directory, _sha(library), world)
        if bundle is not None:
            execution_plan = bundle
            p.write(out / "selection-plan.json", bundle)
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


def test_replay_reproduces_an_error_budget_selection(tmp_path):
    out = _fixture(tmp_path, ["--selection", "error-budget", "--error-budget", "0.01"])
    report = R.replay(out)
    assert report["completed"]
    plan = json.loads((out / "selection-plan.json").read_text())
    for role in ("attn", "mlp"):
        sel = plan["roles"][role]["diagnostics"]["selective"]
        assert sel["method"] == "error_budget" and sel["predicted_relative_l2"] <= 0.01
        assert sum(plan["roles"][role]["selective_mask"]) == len(sel["selected_physical_blocks"]) > 0
    assert C.arguments(["--selection", "error-budget", "--error-budget", "0.02"]).calibration["error_budget"] == 0.02
    with pytest.raises(ValueError):
        C.arguments(["--selection", "error-budget", "--error-budget", "0"])


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


FAKE_WORKER = r'''
import sys
from pathlib import Path
sys.path.insert(0, sys.argv[3])
from _fake_batch import fake_rows
from tempname_dcu_b200.experiment import protocol as p
directory, out = Path(sys.argv[1]), Path(sys.argv[2])
cfg = p.read(directory / "config.json")
rows, _ = fake_rows(cfg["job"], cfg, directory, p.sha(out / "build" / "libtdb.so"), cfg["world_size"])
for row in rows:
    p.write(directory / f"rank{row['rank']}.json", row)
'''


@pytest.mark.parametrize("scope", [["--operator-only"], ["--steps", "2", "--warmup-steps", "1"]])
def test_execute_runs_the_job_sequence_and_writes_an_auditable_report(tmp_path, monkeypatch, scope):
    """controller.execute end to end with a stand-in worker per job: snapshot,
    frozen plan, calibration freeze, per-job validation, trajectory checks,
    report, batch state -- and the result passes the read-only replay."""
    tests_dir = str(Path(__file__).resolve().parent)

    def command(python, source_root, directory, job, world):
        return [python, "-c", FAKE_WORKER, str(directory), str(out), tests_dir]
    monkeypatch.setattr(C, "command_for", command)
    args = C.arguments(["--execute", "--out", str(tmp_path / "run"), "--small-model", "--world-size", "2",
                        "--blocks", "1", *scope, "--operator-warmup", "1", "--operator-iters", "2",
                        "--calibration-pairs", "1"])
    out = args.out
    C.execute(args)
    state = json.loads((out / "batch-state.json").read_text())
    assert state["completed"] and state["status"] in ("completed", "operator_completed")
    report = R.replay(out)
    assert report["completed"] and json.loads((out / "report.json").read_text())["run_id"] == report["run_id"]
    assert (out / "report.md").read_text().startswith("# B200 five-arm experiment")
    assert (out / "selection-plan.json").is_file() and (out / "sources" / "tempname_dcu_b200").is_dir()
