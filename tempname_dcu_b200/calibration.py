"""Calibrate-then-freeze on the target: measure complete fused operators and
let the planner (``planning.fit_role``) choose the arrival order and the
selective mask of each role, identically on every rank.

Every candidate is first checked against the independent references
(plain BF16 <= 5%, codec reference <= 1%) outside timing; then it is warmed
up and timed with CUDA events, and the elapsed time reduced with MAX over
ranks is what the planner sees.  Raw per-rank samples are written
atomically after every measurement so the controller can replay the planner
on the CPU and require the same plan.

With ``selection_mode="error_budget"`` (not in the reference) each role's
selective mask is instead chosen from codec error statistics of one
calibration batch (``block_statistics``); the arrival order is timed as
before.

Reference parity: python/flux_dcu/calibration.py:10-127.
"""
from __future__ import annotations

import json
import math
from pathlib import Path

from .planning import SCHEMA, fit_role, role_digest, settings

SAMPLES_SCHEMA = "b200-calibration-samples-v1"


def _write(path, value):
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(".tmp")
    tmp.write_text(json.dumps(value, indent=2, allow_nan=False) + "\n")
    tmp.replace(path)


def block_statistics(x, w, rank, world, group, chunk_rows):
    """Codec statistics of one projection on a calibration batch, per
    physical output block (the planner's error-budget input): ``error_sq``
    sums, over the block's remote sources, the squared TACO round-trip error
    of their partial products (tdb_taco_block_stats on this rank's partial,
    SUM over ranks); ``output_sq`` is the squared norm of the reduced output
    block.  Identical on every rank."""
    import torch
    import torch.distributed as dist
    from .ops import gemm as G
    from .ops.codec import codec
    partial = G.linear(x, w)
    stats = codec().block_stats(partial, chunk_rows)
    per = stats.shape[0] // world
    error_sq = stats[:, 2].clone()
    error_sq[rank * per:(rank + 1) * per] = 0  # a rank's own blocks never cross the link
    dist.all_reduce(error_sq, group=group)
    reduced = torch.empty((partial.shape[0] // world, partial.shape[1]), dtype=partial.dtype, device=partial.device)
    dist.reduce_scatter_tensor(reduced, partial, group=group)
    mine = codec().block_stats(reduced, chunk_rows)[:, 0].contiguous()
    output_sq = torch.empty(world * per, dtype=torch.float64, device=partial.device)
    dist.all_gather_into_tensor(output_sq, mine, group=group)
    return dict(error_sq=[float(v) for v in error_sq.cpu().tolist()],
                output_sq=[float(v) for v in output_sq.cpu().tolist()])


def calibrate(config, group, out):
    """Return {calibration_plan, calibration_results}; the plan is identical
    on all ranks (checked by digest consensus)."""
    import torch
    import torch.distributed as dist
    from .runtime import FluxB200
    from .worker import mx_projection_reference, projection_reference, relative_error, require_all
    cfg = settings(config.get("calibration"))
    model = config["model"]
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    if world != config["world_size"]:
        raise ValueError("calibration TP width differs from the frozen config")
    m, n, chunk = model["sequence"] * model["micro_batch"], model["hidden"], model["chunk_rows"]
    samples = []
    destination = Path(out) / f"calibration-rank{rank}-samples.json"
    roles = {}
    for role_index, (role, k) in enumerate((("attn", model["hidden"] // world), ("mlp", model["ffn"] // world))):
        def evaluate(plan, seed, arm, label):
            gen = torch.Generator(device="cuda").manual_seed(seed + 173 * rank + 7919 * role_index)
            x = torch.randn((m, k), generator=gen, device="cuda").to(torch.bfloat16)
            w = (torch.randn((n, k), generator=gen, device="cuda") / math.sqrt(k)).to(torch.bfloat16)
            mode = config.get("selective_mode", "wire") if arm.endswith("_selective") else "wire"
            op = FluxB200(m, n, k, group, arm, chunk_rows=chunk, plan=plan, selective_mode=mode)
            op.validate_next_call = True
            actual = op.forward(x, w)
            mask = plan["selective_mask"] if arm.endswith("_selective") else None
            plain, coded = projection_reference(x, w, rank, world, group, True, mask, chunk)
            if mode == "fp8-mma":  # candidates time the FP8 MMA blocks; the gate is the FP8 reference
                coded = mx_projection_reference(x, w, rank, world, group, op.mx["mask"])
            errors = torch.tensor([relative_error(actual, plain), relative_error(actual, coded)],
                                  dtype=torch.float64, device="cuda")
            dist.all_reduce(errors, op=dist.ReduceOp.MAX, group=group)
            plain_error, codec_error = (float(v) for v in errors.cpu().tolist())
            require_all(math.isfinite(plain_error) and math.isfinite(codec_error) and plain_error <= 0.05
                        and codec_error <= 0.01, f"calibration {role}/{label} failed its numerical gate", group)
            for _ in range(cfg["warmup"]):
                op.forward(x, w)
            torch.cuda.synchronize()
            dist.barrier(group=group)
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            for _ in range(cfg["iterations"]):
                op.forward(x, w)
            end.record()
            torch.cuda.synchronize()
            local = start.elapsed_time(end) / 1000.0
            peak = torch.tensor(local, dtype=torch.float64, device="cuda")
            dist.all_reduce(peak, op=dist.ReduceOp.MAX, group=group)
            elapsed = float(peak.item())
            samples.append(dict(role=role, label=label, seed=seed, arm=arm, plan_digest=role_digest(plan),
                                arrival_order=plan["arrival_order"], selective_mask=plan["selective_mask"],
                                local_elapsed_seconds=local, max_rank_elapsed_seconds=elapsed,
                                iterations=cfg["iterations"], warmup=cfg["warmup"], bf16_relative_l2=plain_error,
                                codec_reference_relative_l2=codec_error, correctness_passed=True))
            _write(destination, dict(schema=SAMPLES_SCHEMA, rank=rank, samples=samples))
            return elapsed

        stats = None
        if cfg.get("selection_mode") == "error_budget":  # one calibration batch per role
            gen = torch.Generator(device="cuda").manual_seed(9_000_000 + 173 * rank + 7919 * role_index)
            x = torch.randn((m, k), generator=gen, device="cuda").to(torch.bfloat16)
            w = (torch.randn((n, k), generator=gen, device="cuda") / math.sqrt(k)).to(torch.bfloat16)
            stats = block_statistics(x, w, rank, world, group, chunk)
        roles[role] = fit_role(m, n, k, world, chunk, evaluate, config=cfg,
                               seed=8_000_000 + 10_000_000 * role_index + int(config.get("seed", 1234)),
                               block_stats=stats)
    bundle = dict(schema=SCHEMA, world_size=world, transport_lanes=2, roles=roles)
    digest = role_digest(bundle)
    gathered = [None] * world
    dist.all_gather_object(gathered, digest, group=group)
    if len(set(gathered)) != 1:
        raise RuntimeError("calibration produced different plans on different ranks")
    return dict(calibration_plan=bundle,
                calibration_results=dict(plan_sha256=digest, raw_samples=samples, raw_samples_file=destination.name,
                                         selection_timing="max-rank complete fused operator (CUDA events); "
                                                          "references and validation excluded",
                                         training_and_confirmation_inputs_disjoint=True, no_fullstep_claim=True))
