"""Sharded checkpoint save/resume (utils/checkpoint.py) on CPU: exact restore,
refusals (missing manifest, tampered shard, other config / world / plan),
and a 2-rank gloo save + load."""
import json
import os
import types

import pytest


def _trainer(rank=0, world=1, seed=3, layers=2, tp=None):
    import torch
    from tempname_dcu_b200.models.config import validate_config
    from tempname_dcu_b200.models.params import FlatParams, gpt_param_specs
    c = validate_config(dict(layers=layers, hidden=256, ffn=1024, heads=2, sequence=256, vocab=1024,
                             chunk_rows=128), world)
    P = FlatParams(gpt_param_specs(c, world), "cpu", rank=rank, seed=seed)
    P.master.copy_(P.param.float())
    g = torch.Generator().manual_seed(100 + rank)
    P.exp_avg.copy_(torch.randn(P.total, generator=g))
    P.exp_avg_sq.copy_(torch.rand(P.total, generator=g))
    model = types.SimpleNamespace(params=P, config=c, world=world, rank=rank, tp=tp)
    return types.SimpleNamespace(model=model, optimizer=types.SimpleNamespace(step_count=7))


def test_save_load_roundtrip_exact(tmp_path):
    import torch
    from tempname_dcu_b200.utils import checkpoint as ck
    a = _trainer(seed=3)
    a.model.params.master.add_(1e-3)          # masters not equal to the initial bf16 image
    a.model.params.param.copy_(a.model.params.master.to(torch.bfloat16))
    ck.save(a, tmp_path / "ck", plan_sha256="abc")
    b = _trainer(seed=9)
    b.optimizer.step_count = 0
    assert ck.load(b, tmp_path / "ck", plan_sha256="abc") == 7
    for key in ("master", "exp_avg", "exp_avg_sq", "param"):
        assert torch.equal(getattr(a.model.params, key), getattr(b.model.params, key)), key
    assert torch.count_nonzero(b.model.params.grad) == 0
    manifest = json.loads((tmp_path / "ck" / "manifest.json").read_text())
    assert manifest["world"] == 1 and manifest["step"] == 7 and set(manifest["files"]) == {"rank0.pt"}


def test_refusals(tmp_path):
    from tempname_dcu_b200.utils import checkpoint as ck
    a = _trainer()
    d = tmp_path / "ck"
    ck.save(a, d)
    with pytest.raises(ValueError, match="plan digest"):
        ck.load(_trainer(), d, plan_sha256="other")
    with pytest.raises(ValueError, match="config"):
        ck.load(_trainer(layers=3), d)
    (tmp_path / "empty").mkdir()
    with pytest.raises(ValueError, match="manifest"):
        ck.load(_trainer(), tmp_path / "empty")
    with open(d / "rank0.pt", "r+b") as f:     # flip one byte of the shard
        f.seek(200)
        byte = f.read(1)
        f.seek(200)
        f.write(bytes([byte[0] ^ 0xFF]))
    with pytest.raises(ValueError, match="sha256"):
        ck.load(_trainer(), d)




def _worker(rank, world, init_file, path, queue):
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    try:
        from tempname_dcu_b200.parallel.tp import TPGroup
        from tempname_dcu_b200.utils import checkpoint as ck
        tp = TPGroup(dist.group.WORLD)
        a = _trainer(rank=rank, world=world, tp=tp)
        ck.save(a, path)
        b = _trainer(rank=rank, world=world, seed=11, tp=tp)
        step = ck.load(b, path)
        same = all(torch.equal(getattr(a.model.params, k), getattr(b.model.params, k))
                   for k in ("master", "exp_avg", "exp_avg_sq", "param"))
        queue.put((rank, step, same))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks(tmp_path):
    import json as _json
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = str(tmp_path / "rendezvous")  # file rendezvous path (no TCP port race)
    path = str(tmp_path / "ck2")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, path, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=180) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert results == [(0, 7, True), (1, 7, True)]
    manifest = _json.loads((tmp_path / "ck2" / "manifest.json").read_text())
    assert manifest["world"] == 2 and sorted(manifest["files"]) == ["rank0.pt", "rank1.pt"]
