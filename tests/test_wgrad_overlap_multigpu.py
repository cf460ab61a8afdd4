"""Backward weight-gradient overlap on 2 GPUs (child processes over NCCL,
NVLS off): a small GPT whose fused all-gather GEMMs and reduce-scatters are
active trains three steps with the weight-gradient GEMMs on a second stream
(``wgrad_sms``: their grids and the fused kernels' grids split the SMs), both
eagerly and replayed from a captured CUDA graph, and must match the
single-stream run bit for bit: losses, gradient norms and the fp32 master
weights (each weight's gradient accumulates in the same micro-batch order).
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
    from tempname_dcu_b200.ops import native
    from tempname_dcu_b200.runtime import operator_factory_for, shutdown_context
    from tempname_dcu_b200.train import Trainer, synthetic_batches
    out = {}
    try:
        # rows per rank (512) a multiple of 256, so the fused all-gather GEMMs run
        config = dict(layers=2, hidden=512, ffn=2048, heads=4, sequence=1024, micro_batch=1,
                      accumulation_steps=2, vocab=1024, chunk_rows=128)
        runs = {}
        for name, sms, graph in (("plain", 0, False), ("overlap", 40, False), ("plain_graph", 0, True),
                                 ("overlap_graph", 40, True)):
            trainer = Trainer(config, "flux", dist.group.WORLD, operator_factory=operator_factory_for("flux"),
                              cuda_graph=graph, graph_warmup=1, wgrad_sms=sms)
            assert (trainer.model._overlap is not None) == (sms > 0)
            (tokens, labels), = synthetic_batches(trainer.config, 1, seed=7)
            tokens, labels = tokens.cuda(), labels.cuda()
            losses, norms = [], []
            for _ in range(3):
                loss, norm = trainer.step(tokens, labels)
                losses.append(float(loss.item()))
                norms.append(float(norm.item()))
            torch.cuda.synchronize()
            native.raise_on_status()
            runs[name] = (losses, norms, trainer.model.params.master.clone())
            if graph:
                trainer.release_graph()
            del trainer
        base = runs["plain"]
        for name, (losses, norms, master) in runs.items():
            out[name] = dict(losses=losses, norms=norms, same=losses == base[0] and norms == base[1]
                             and bool(torch.equal(master, base[2])))
    finally:
        shutdown_context(dist.group.WORLD)
        if rank == 0:
            with open(result_path, "w") as fh:
                json.dump(out, fh)
        dist.destroy_process_group()


def test_weight_gradient_overlap_is_bitwise_neutral(tmp_path):
    import json
    import torch
    import torch.multiprocessing as mp
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs at least two GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    path = str(tmp_path / "result.json")
    mp.spawn(_worker, args=(2, str(tmp_path / "rendezvous"), path), nprocs=2, join=True)
    res = json.load(open(path))
    assert set(res) == {"plain", "overlap", "plain_graph", "overlap_graph"}, res
    for name, run in res.items():
        assert run["same"], (name, res)
