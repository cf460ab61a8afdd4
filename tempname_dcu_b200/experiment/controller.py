"""Prepare, run and audit an isolated single-node B200 five-arm comparison.

    tempname_dcu_b200/experiment/run_init.sh [--execute] [--out DIR] [--world-size N] ...

Without ``--execute`` the controller only prints the plan (no torch import,
no files written).  With it: freeze a snapshot of the sources (+ manifest
sha256) and the native library, then run one ``torchrun`` per job
(preflight -> calibrate -> operator windows -> training windows) in its own
process group with a timeout, validate every job's rank rows, freeze the
calibrated plan after the calibrate job, check that the TACO arms trained
bitwise identically, and write ``report.json`` / ``report.md``.  SIGTERM
stops only this controller's worker process group.  ``--report`` audits a
finished directory read-only.

Reference parity: tools/dcu/phase6/init.py:1-279 and run_init.sh (CLI,
preview, snapshot, job loop, stop_process, batch-state.json).
"""
from __future__ import annotations

import argparse
import contextlib
from datetime import datetime, timezone
import os
from pathlib import Path
import shutil
import signal
import subprocess
import sys
import uuid

from . import protocol as p

REPO = Path(__file__).resolve().parents[2]
PACKAGE = REPO / "tempname_dcu_b200"


def arguments(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--trials", type=int, default=1)
    ap.add_argument("--blocks", type=int, default=10,
                    help="five-arm blocks per trial; 1 is a short test, multiples of 10 are balanced")
    ap.add_argument("--execute", action="store_true", help="without this flag only print the plan")
    ap.add_argument("--out", type=Path)
    ap.add_argument("--python", default=sys.executable)
    ap.add_argument("--world-size", type=int, choices=(1, 2, 4, 8), default=8,
                    help="1 runs the flux arm alone (no collective to compare)")
    ap.add_argument("--arm", action="append", choices=p.ARMS, dest="arms",
                    help="compare only these arms (repeatable; default all five)")
    ap.add_argument("--vocab", type=int, help="override the preset's vocabulary size")
    ap.add_argument("--vocab-pad", action="store_true",
                    help="pad the vocabulary up to a multiple of 128 x world_size (e.g. GPT-2's 50257)")
    ap.add_argument("--accum", type=int, help="micro-batches accumulated per optimizer step")
    ap.add_argument("--selective-mode", choices=("wire", "fp8-mma"), default="wire",
                    help="wire: selected blocks cross NVLink as TACO E4M3 packets (the reference's mode); "
                         "fp8-mma: their GEMM tiles run as block-scaled FP8 tcgen05 MMAs, BF16 on the wire")
    ap.add_argument("--chunk-rows", type=int)
    ap.add_argument("--warmup-steps", type=int, default=10)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--operator-warmup", type=int, default=100)
    ap.add_argument("--operator-iters", type=int, default=200)
    ap.add_argument("--quant-budget", type=float, default=0.25)
    ap.add_argument("--calibration-iters", type=int, default=5)
    ap.add_argument("--calibration-pairs", type=int, default=3)
    ap.add_argument("--calibration-warmup", type=int, default=2)
    ap.add_argument("--calibration-min-gain", type=float, default=0.002)
    ap.add_argument("--selection", choices=("timing", "error-budget"), default="timing",
                    help="how the selective arm picks its blocks: paired timing (the reference) or the codec error "
                         "measured on a calibration batch, within --error-budget")
    ap.add_argument("--error-budget", type=float, default=0.01,
                    help="relative L2 error of a projection output the selected blocks may add (error-budget mode)")
    scopes = ap.add_mutually_exclusive_group()
    scopes.add_argument("--operator-only", action="store_true")
    scopes.add_argument("--preflight-only", action="store_true")
    ap.add_argument("--profile", action="store_true", help="separate per-block timeline profile after timing")
    ap.add_argument("--small-model", action="store_true", help="diagnostic 2-layer model, not GPT-6.7B results")
    ap.add_argument("--bench-model", action="store_true", help="GPT-6.7B with vocab 50257 (padded) and 8 micro-batches")
    ap.add_argument("--worker-timeout", type=int, default=7200)
    ap.add_argument("--report", action="store_true", help="read-only audit of a completed --out directory")
    args = ap.parse_args(argv)
    args.arms = p.select_arms(args.arms)
    p.orders(args.trials, args.blocks, args.arms)
    p.require(args.world_size > 1 or args.arms == ("flux",),
              "--world-size 1 has no reduce-scatter to compare: use --arm flux")
    p.require(args.warmup_steps >= 0 and args.operator_warmup >= 0, "warm-up counts must be non-negative")
    p.require(args.steps > 0 and args.operator_iters > 0 and args.worker_timeout > 0,
              "timing counts and timeout must be positive")
    args.calibration = dict(warmup=args.calibration_warmup, iterations=args.calibration_iters,
                            training_pairs=args.calibration_pairs, confirmation_pairs=args.calibration_pairs,
                            min_gain=args.calibration_min_gain, quant_budget=args.quant_budget)
    if args.selection == "error-budget":
        args.calibration.update(selection_mode="error_budget", error_budget=args.error_budget)
    p.validate_calibration_options(args.calibration)
    p.require(not args.report or (args.out is not None and not args.execute and not args.operator_only
                                  and not args.preflight_only), "--report needs --out and cannot execute a stage")
    p.require(not (args.small_model and args.bench_model), "choose one model preset")
    model = dict(p.SMALL_MODEL if args.small_model else p.BENCH_MODEL if args.bench_model else p.MODEL)
    if args.chunk_rows is not None:
        model["chunk_rows"] = args.chunk_rows
    if args.vocab is not None:
        model["vocab"] = args.vocab
    if args.vocab_pad:
        model["pad_vocab"] = True
    if args.accum is not None:
        p.require(args.accum > 0, "--accum must be positive")
        model["accumulation_steps"] = args.accum
    p.validate_model(model, args.world_size)
    p.require(model["sequence"] * model["micro_batch"] // args.world_size // model["chunk_rows"] >= 2,
              "at least two blocks per destination are needed to distinguish the schedules")
    args.model = model
    if args.out is None:
        stamp = datetime.now(timezone.utc).strftime("%Y%m%d-%H%M%S-%f")
        args.out = REPO / "logs" / "experiment" / f"five-arm-{stamp}"
    args.out = args.out.expanduser().resolve()
    args.scope = "preflight" if args.preflight_only else "operator" if args.operator_only else "train"
    p.jobs(args.trials, args.blocks, args.scope, args.arms, args.world_size)
    p.require(args.report or args.scope != "train" or args.warmup_steps >= 1,
              "full training needs at least one warm-up step for the per-operator checks")
    return args


def source_files():
    files = []
    for path in PACKAGE.rglob("*"):
        if not path.is_file() or "__pycache__" in path.parts or "_native" in path.parts:
            continue
        if path.suffix in (".pyc", ".so", ".o"):
            continue
        files.append(path)
    for name in ("bench.py", "__graft_entry__.py", "README.md"):
        if (REPO / name).is_file():
            files.append(REPO / name)
    return sorted(set(files))


def plan_for(args, manifest=None, run_id=None):
    config = dict(protocol=p.PROTOCOL, run_id=run_id or "PREVIEW", world_size=args.world_size, model=args.model,
                  arms=list(args.arms), selective_mode=args.selective_mode,
                  timing=dict(warmup_steps=args.warmup_steps, timed_steps=args.steps,
                              operator_warmup=args.operator_warmup, operator_iterations=args.operator_iters),
                  seed=1234, token_seed=4321, build_dir=str(args.out / "build"), profile=args.profile,
                  source_manifest_sha256=p.digest(manifest) if manifest is not None else "PREVIEW",
                  recommended_image=p.RECOMMENDED_IMAGE, backend=p.BACKEND, calibration=args.calibration,
                  execution_plan=None, execution_plan_sha256=None)
    return dict(config=config, scope=args.scope, trials=args.trials, blocks=args.blocks,
                arms=list(args.arms), counterbalanced=p.balanced(args.blocks, args.arms),
                schedule=p.orders(args.trials, args.blocks, args.arms),
                jobs=p.jobs(args.trials, args.blocks, args.scope, args.arms, args.world_size))


def command_for(python, source_root, directory, job, world):
    return [python, "-m", "torch.distributed.run", "--standalone", "--nnodes=1", f"--nproc_per_node={world}",
            "--local-addr", "127.0.0.1", "-m", "tempname_dcu_b200.worker", "--config", str(directory / "config.json"),
            "--out", str(directory), "--stage", job["stage"], "--arm", job["arm"]]


# --------------------------------------------------------------- workers
#
# A job is one torchrun launch.  It runs in a session of its own, so the whole
# tree it spawns (torchrun, its rank processes) forms one process group that
# this controller can signal without touching anything else on the machine.

_ESCALATION = ((signal.SIGTERM, 10.0), (signal.SIGKILL, 10.0))


def stop_process(process):
    """Stop the worker group led by ``process``: each signal of the escalation
    goes to that group only, and the next one is sent if the leader has not
    exited within its grace period."""
    for number, grace in _ESCALATION:
        if process.poll() is not None:
            return
        try:
            os.killpg(process.pid, number)
        except ProcessLookupError:
            return
        try:
            process.wait(timeout=grace)
            return
        except subprocess.TimeoutExpired:
            continue


class WorkerGroup:
    """One worker job: started in its own session with its output in
    ``process.log``; ``run`` waits for it within the timeout and stops its
    process group on any way out (timeout, interrupt, error)."""

    PASSED_ENV = {"PYTHONDONTWRITEBYTECODE": "1", "PYTHONUNBUFFERED": "1"}
    TAIL_LINES = 40

    def __init__(self, command, directory, source_root):
        self.command = command
        self.log_path = directory / "process.log"
        self.source_root = source_root

    def environment(self):
        env = dict(os.environ, PYTHONPATH=str(self.source_root), **self.PASSED_ENV)
        env.setdefault("OMP_NUM_THREADS", "1")
        return env

    def run(self, timeout):
        with self.log_path.open("w") as log:
            process = subprocess.Popen(self.command, cwd=self.source_root, env=self.environment(), stdout=log,
                                       stderr=subprocess.STDOUT, start_new_session=True)
            try:
                code = process.wait(timeout=timeout)
            finally:
                stop_process(process)  # no-op once the leader has exited
        if code != 0:
            lines = self.log_path.read_text(errors="replace").splitlines()[-self.TAIL_LINES:]
            raise RuntimeError("worker exited %d (log: %s)\n%s" % (code, self.log_path, "\n".join(lines)))


def launch(command, directory, source_root, timeout):
    WorkerGroup(command, directory, source_root).run(timeout)


# --------------------------------------------------------------- batch bookkeeping

class BatchRecord:
    """The batch directory's bookkeeping files: ``batch-state.json`` (status
    and progress, rewritten on every transition) and ``completed-jobs.json``
    (one entry per validated job, with the hashes of what it left behind)."""

    def __init__(self, out, run_id, scope):
        self.out = out
        self.state = dict(protocol=p.PROTOCOL, run_id=run_id, status="preparing", completed=False, scope=scope,
                          finished_jobs=0)
        self.completed = []

    def save_state(self, **changes):
        self.state.update(changes)
        p.write(self.out / "batch-state.json", self.state)

    def start_ledger(self):
        p.write(self.out / "completed-jobs.json", self.completed)

    def finish_job(self, job, directory, world, plan_digest=None):
        entry = dict(job=job, command_sha256=p.sha(directory / "command.json"),
                     rank_sha256={name: p.sha(directory / name) for name in (f"rank{r}.json" for r in range(world))})
        if plan_digest is not None:
            entry["execution_plan_sha256"] = plan_digest
            entry["selection_plan_file_sha256"] = p.sha(self.out / "selection-plan.json")
        self.completed.append(entry)
        p.write(self.out / "completed-jobs.json", self.completed)
        self.save_state(finished_jobs=len(self.completed))


class Invariants:
    """Facts that must not change from one job of a batch to the next: the
    rank environment, the native library the ranks loaded, the initial
    weights/input of every training window, and -- within one five-arm block
    -- the trajectories of the TACO arms that differ only in production
    order."""

    def __init__(self):
        self.first = {}
        self.windows = {}

    def same_as_before(self, key, value, message):
        expected = self.first.setdefault(key, value)
        p.require(expected == value, message)

    def rows(self, rows):
        self.same_as_before("environment", [r["environment_identity"] for r in rows],
                            "hardware/software changed between workers")
        self.same_as_before("native", [r["codec_build"] for r in rows], "native library changed between workers")

    def training(self, job, rows):
        self.same_as_before("training", p.training_identity(rows), "initial weights/input differ across windows")
        block = self.windows.setdefault((job["trial"], job["block"]), {})
        block[job["arm"]] = rows
        present = [arm for arm in p.FULL_TACO_ARMS if arm in block]
        for arm in present[1:]:
            p.compare_taco_trajectories(block[present[0]], block[arm])


def freeze_sources(files, manifest, out):
    """Copy the sources into ``out/sources`` (verifying every copy against
    the manifest) and place this tree's native library beside them and under
    ``out/build``.  Returns the snapshot root the workers run from."""
    root = out / "sources"
    for f in files:
        rel = str(f.relative_to(REPO))
        dest = root / rel
        dest.parent.mkdir(parents=True, exist_ok=True)
        shutil.copyfile(f, dest)
        p.require(p.sha(dest) == manifest[rel], "source changed while freezing")
    from ..ops import _build
    library = _build.build()
    native_dir = root / "tempname_dcu_b200" / "_native"
    native_dir.mkdir(parents=True, exist_ok=True)
    for src, name in ((library, "libtdb.so"), (_build.paths(_build.debug_requested())[1], "manifest.json")):
        shutil.copyfile(src, native_dir / name)
    (out / "build").mkdir()
    shutil.copyfile(library, out / "build" / "libtdb.so")
    return root


_RECORDED_ENV_PREFIXES = ("NCCL_", "TORCH_NCCL_")
_RECORDED_ENV_NAMES = ("CUDA_VISIBLE_DEVICES", "OMP_NUM_THREADS")


def _recorded_environment():
    return {k: v for k, v in os.environ.items() if k.startswith(_RECORDED_ENV_PREFIXES) or k in _RECORDED_ENV_NAMES}


def execute(args):
    """Run every job of the plan in order (see the module docstring) and
    write the replayed report."""
    from . import report as reporting
    p.require(not args.out.exists(), "output directory exists; use a fresh --out")
    python = shutil.which(args.python)
    p.require(python is not None, f"python executable not found: {args.python}")
    files = source_files()
    manifest = {str(f.relative_to(REPO)): p.sha(f) for f in files}
    plan = plan_for(args, manifest=manifest, run_id=uuid.uuid4().hex)
    args.out.mkdir(parents=True, exist_ok=False)
    record = BatchRecord(args.out, plan["config"]["run_id"], args.scope)
    record.save_state()
    try:
        source_root = freeze_sources(files, manifest, args.out)
        p.write(args.out / "source-manifest.json", manifest)
        p.write(args.out / "plan.json", plan)
        record.start_ledger()
        invariants = Invariants()
        frozen_plan = None
        total = len(plan["jobs"])
        for job in plan["jobs"]:
            directory = args.out / "results" / job["directory"]
            directory.mkdir(parents=True, exist_ok=False)
            job_config = p.config_for_job(plan["config"], job, frozen_plan)
            p.write(directory / "config.json", job_config)
            command = command_for(python, source_root, directory, job, args.world_size)
            p.write(directory / "command.json", dict(job=job, command=command, environment=_recorded_environment()))
            record.save_state(status="running", active_job=job)
            print(f"[{job['index'] + 1}/{total}] {job['directory']}", flush=True)
            launch(command, directory, source_root, args.worker_timeout)
            rows = [p.read(directory / f"rank{r}.json") for r in range(args.world_size)]
            rows = p.validate_rows(rows, job, job_config)
            invariants.rows(rows)
            reporting.validate_artifacts(args.out, directory, rows, job_config)
            digest = None
            if job["stage"] == "calibrate":
                p.require(frozen_plan is None, "calibration runs once per fresh experiment")
                frozen_plan = p.calibration_from_rows(rows, job_config)
                reporting.validate_calibration_evidence(args.out, directory, rows, job_config)
                p.write(args.out / "selection-plan.json", frozen_plan)
                digest = p.digest(frozen_plan)
                record.save_state(execution_plan_sha256=digest)
            elif job["stage"] == "train":
                invariants.training(job, rows)
            record.finish_job(job, directory, args.world_size, digest)
        report = reporting.replay(args.out)
        p.write(args.out / "report.json", report)
        (args.out / "report.md").write_text(reporting.markdown(report))
        record.save_state(status="completed" if args.scope == "train" else f"{args.scope}_completed", completed=True,
                          active_job=None, report_sha256=p.sha(args.out / "report.json"),
                          formal_optimizer_steps=report["formal_optimizer_steps"])
        print(f"completed scope: {args.scope}\nreport: {args.out / 'report.md'}", flush=True)
    except KeyboardInterrupt as exc:
        record.save_state(status="interrupted", completed=False, error=f"KeyboardInterrupt: {exc}")
        raise
    except Exception as exc:
        record.save_state(status="failed", completed=False, error=f"{type(exc).__name__}: {exc}")
        raise


@contextlib.contextmanager
def _sigterm_interrupts():
    """While active, SIGTERM raises KeyboardInterrupt in the main thread, so
    a scheduler's stop unwinds ``execute`` (which stops the running worker
    group and marks the batch interrupted) instead of orphaning torchrun."""
    def interrupt(_number, _frame):
        raise KeyboardInterrupt("received SIGTERM")
    previous = signal.signal(signal.SIGTERM, interrupt)
    try:
        yield
    finally:
        signal.signal(signal.SIGTERM, previous)


def main(argv=None):
    args = arguments(argv)
    if args.report:
        from . import report as reporting
        print(reporting.markdown(reporting.replay(args.out)))
        return
    if args.execute:
        with _sigterm_interrupts():
            execute(args)
        return
    import json
    preview = dict(preview=True, writes_files=False, uses_gpu=False, output=str(args.out),
                   operator_rooflines=operator_rooflines(args), **plan_for(args))
    print(json.dumps(preview, ensure_ascii=False, indent=2))


def operator_rooflines(args):
    """Per role, the fused operator's roofline at the measured (or fallback)
    peaks with BF16 and with TACO bytes on the link (preview only; no GPU)."""
    if args.world_size < 2:
        return None
    from ..ops import roofline as rf
    tflops, nvlink, source = rf.peaks()
    out = dict(peaks=dict(bf16_tflops=tflops, nvlink_gbs=nvlink, source=source))
    for taco in (False, True):
        for path in rf.fused_paths(args.model, args.world_size, taco):
            if path["name"] in ("attn_out.fwd", "fc2.fwd"):
                us, bound = rf.roofline_us(path, tflops, nvlink)
                role = "attn" if path["name"].startswith("attn") else "mlp"
                out[f"{role}.{'taco' if taco else 'bf16'}"] = dict(us=round(us, 2), bound=bound,
                                                                     link_bytes=int(path["link_bytes"]))
    return out


# exit status of the command line per failure class (first match wins)
_EXIT_CODES = ((KeyboardInterrupt, 130, "interrupted; only this controller's worker process group was stopped"),
               ((ValueError, RuntimeError, OSError, subprocess.TimeoutExpired), 1, None))


def _cli():
    try:
        main()
    except BaseException as error:  # noqa: BLE001 - mapped to an exit status below
        for kinds, code, text in _EXIT_CODES:
            if isinstance(error, kinds):
                print(text or f"ERROR: {error}", file=sys.stderr)
                raise SystemExit(code) from None
        raise


if __name__ == "__main__":
    _cli()
