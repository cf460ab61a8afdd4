"""Warm-up codec calibration on 2 GPUs (child processes over NCCL, NVLS off):
two TACO arms that differ only in production order train a small GPT with
``codec_calibration_steps=2``; both must freeze the same per-role masks
within the error budget, put them into their fused operators, and keep
training bitwise identically (losses and gradient norms) afterwards.
Skipped with fewer than two GPUs."""
import os

import pytest

pytestmark = pytest.mark.gpu


def _worker(rank, world, init_file, result_path):
    import json
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120), device_id=torch.device("cuda", rank))
    from tempname_dcu_b200.models.config import SMALL_CONFIG
    from tempname_dcu_b200.ops import native
    from tempname_dcu_b200.runtime import operator_factory_for, shutdown_context
    from tempname_dcu_b200.train import Trainer, synthetic_batches
    out = {}
    try:
        config = dict(SMALL_CONFIG, layers=2, accumulation_steps=2)
        for arm in ("flux_taco", "flux_taco_interleaved"):
            trainer = Trainer(config, arm, dist.group.WORLD, operator_factory=operator_factory_for(arm),
                              codec_calibration_steps=2, error_budget=0.02)
            (tokens, labels), = synthetic_batches(trainer.config, 1, seed=99)
            losses, norms = [], []
            for step in range(4):
                loss, norm = trainer.step(tokens, labels)
                losses.append(float(loss.item()))
                norms.append(float(norm.item()))
            torch.cuda.synchronize()
            native.raise_on_status()
            plan = trainer.codec_plan
            ops = trainer.model.operators
            out[arm] = dict(
                losses=losses, norms=norms,
                masks={r: plan["roles"][r]["selective_mask"] for r in ("attn", "mlp")},
                predicted={r: plan["roles"][r]["diagnostics"]["selective"]["predicted_relative_l2"]
                           for r in ("attn", "mlp")},
                applied=all(op.qmask.tolist() == [int(v) for v in plan["roles"][("attn", "mlp")[i % 2]]["selective_mask"]]
                            for i, op in enumerate(ops)),
                quantization=sorted({op.state()["quantization"] for op in ops}))
            del trainer
    finally:
        shutdown_context(dist.group.WORLD)
        if rank == 0:
            with open(result_path, "w") as fh:
                json.dump(out, fh)
        dist.destroy_process_group()


def test_warmup_calibration_freezes_identical_masks_for_order_only_arms(tmp_path):
    import json
    import math
    import torch
    import torch.multiprocessing as mp
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs at least two GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    path = str(tmp_path / "result.json")
    mp.spawn(_worker, args=(2, str(tmp_path / "rendezvous"), path), nprocs=2, join=True)
    res = json.load(open(path))
    a, b = res["flux_taco"], res["flux_taco_interleaved"]
    assert a["masks"] == b["masks"]
    assert a["losses"] == b["losses"] and a["norms"] == b["norms"]
    for arm in (a, b):
        assert arm["applied"] and arm["quantization"] == ["warmup_calibrated_remote_h128_e4m3"]
        assert all(0 <= v <= 0.02 for v in arm["predicted"].values())
        assert all(math.isfinite(x) for x in arm["losses"])
