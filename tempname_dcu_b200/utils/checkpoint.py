"""Sharded training checkpoint: save / resume of one tensor-parallel job.

The reference keeps no model or optimizer checkpoint (every window starts from
name-derived seeds, python/flux_dcu/model.py:197-201, and only records
digests, :327-336); its persisted artifacts are the frozen plan and the batch
directory.  Resuming a long run needs the optimizer state too, so this module
adds a per-rank checkpoint:

    <dir>/rank<r>.pt       this rank's flat fp32 master weights, Adam moments,
                           optimizer step, layout digest, RNG states
    <dir>/manifest.json    written by rank 0 after every rank has finished:
                           format, world size, step, config, plan digest and
                           the sha256 of every rank file

bf16 parameters are not stored: they are the round-to-nearest-even image of
the fp32 masters, exactly what the AdamW kernel writes after every step, and
are rebuilt on load.  Every file is written to a temporary name and renamed,
so a checkpoint directory never holds a half-written file under its final
name; the manifest appears last, so a directory without one is incomplete.
"""
from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path

FORMAT = "tempname-dcu-b200-checkpoint-v1"


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1 << 24), b""):
            h.update(block)
    return h.hexdigest()


def layout_digest(params) -> str:
    """sha256 over the flat layout (name, shape, offset, region flags)."""
    rows = [[s.name, list(s.shape), params.offsets[s.name], bool(s.replicated), bool(s.decay)]
            for s in params.specs]
    text = json.dumps(dict(total=params.total, rows=rows), sort_keys=True, separators=(",", ":"))
    return hashlib.sha256(text.encode()).hexdigest()


def _config_text(config) -> str:
    return json.dumps(config, sort_keys=True, separators=(",", ":"), allow_nan=False)


def _atomic_save(obj, path: Path):
    import torch
    tmp = path.with_name(path.name + ".tmp")
    torch.save(obj, tmp)
    os.replace(tmp, path)


def _barrier(model):
    if model.world > 1:
        model.tp.barrier()


def save(trainer, directory, *, plan_sha256=None) -> Path:
    """Write this rank's shard; rank 0 then writes the manifest.  Collective
    over the model's group (every rank must call it)."""
    import torch
    model, opt = trainer.model, trainer.optimizer
    P = model.params
    out = Path(directory)
    out.mkdir(parents=True, exist_ok=True)
    state = dict(format=FORMAT, rank=model.rank, world=model.world, step=int(opt.step_count),
                 layout=layout_digest(P), config=_config_text(model.config), plan_sha256=plan_sha256,
                 master=P.master.detach().cpu(), exp_avg=P.exp_avg.detach().cpu(),
                 exp_avg_sq=P.exp_avg_sq.detach().cpu(), cpu_rng=torch.get_rng_state(),
                 cuda_rng=torch.cuda.get_rng_state(P.device) if P.device.type == "cuda" else None)
    path = out / f"rank{model.rank}.pt"
    _atomic_save(state, path)
    _barrier(model)
    if model.rank == 0:
        files = {f"rank{r}.pt": _sha256(out / f"rank{r}.pt") for r in range(model.world)}
        manifest = dict(format=FORMAT, world=model.world, step=int(opt.step_count), config=model.config,
                        plan_sha256=plan_sha256, layout=state["layout"], files=files)
        tmp = out / "manifest.json.tmp"
        tmp.write_text(json.dumps(manifest, indent=2, sort_keys=True, allow_nan=False))
        os.replace(tmp, out / "manifest.json")
    _barrier(model)
    return out


def load(trainer, directory, *, plan_sha256=None) -> int:
    """Restore this rank's shard into the trainer; returns the optimizer step.

    Refuses a checkpoint whose manifest is missing, whose world size, config,
    layout or plan digest differ from the running job, or whose rank file does
    not match the sha256 recorded in the manifest."""
    import torch
    model, opt = trainer.model, trainer.optimizer
    P = model.params
    src = Path(directory)
    mpath = src / "manifest.json"
    if not mpath.is_file():
        raise ValueError(f"{src}: no manifest.json (incomplete checkpoint)")
    manifest = json.loads(mpath.read_text())
    if manifest.get("format") != FORMAT:
        raise ValueError(f"{src}: unknown checkpoint format {manifest.get('format')!r}")
    if manifest["world"] != model.world:
        raise ValueError(f"{src}: saved with world size {manifest['world']}, running {model.world}")
    if _config_text(manifest["config"]) != _config_text(model.config):
        raise ValueError(f"{src}: model/optimizer config differs from the running job")
    if manifest["layout"] != layout_digest(P):
        raise ValueError(f"{src}: flat parameter layout differs from the running job")
    if manifest.get("plan_sha256") != plan_sha256:
        raise ValueError(f"{src}: execution plan digest differs from the running job")
    name = f"rank{model.rank}.pt"
    path = src / name
    if _sha256(path) != manifest["files"].get(name):
        raise ValueError(f"{src}/{name}: sha256 does not match the manifest")
    state = torch.load(path, map_location="cpu", weights_only=False)
    if state["rank"] != model.rank or state["step"] != manifest["step"]:
        raise ValueError(f"{src}/{name}: rank or step inconsistent with the manifest")
    for key in ("master", "exp_avg", "exp_avg_sq"):
        src_t, dst_t = state[key], getattr(P, key)
        if src_t.shape != dst_t.shape or src_t.dtype != dst_t.dtype:
            raise ValueError(f"{src}/{name}: {key} has shape {tuple(src_t.shape)}/{src_t.dtype}")
        dst_t.copy_(src_t)
    P.param.copy_(P.master.to(torch.bfloat16))
    P.grad.zero_()
    opt.step_count = int(state["step"])
    if getattr(opt, "step_dev", None) is not None:  # device step counter read by the AdamW kernel
        opt.step_dev.fill_(opt.step_count)
    torch.set_rng_state(state["cpu_rng"])
    if state.get("cuda_rng") is not None and P.device.type == "cuda":
        torch.cuda.set_rng_state(state["cuda_rng"], P.device)
    _barrier(model)
    return opt.step_count
