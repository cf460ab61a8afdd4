"""Model configuration, parameter accounting and flat storage on CPU, and the
tensor-parallel collectives over 2 gloo ranks (reference:
tests/test_model_contract.py)."""
import math
import os

import pytest

from tempname_dcu_b200.models.config import (BENCH_CONFIG, DEFAULT_CONFIG, padded_vocab, parameter_counts,
                                             train_flops_per_step, validate_config)


def test_default_is_full_gpt67b():
    c = validate_config({})
    assert (c["layers"], c["hidden"], c["ffn"], c["heads"], c["sequence"]) == (32, 4096, 16384, 32, 2048)
    assert c["sequence"] * c["micro_batch"] * c["accumulation_steps"] == 8192
    counts = parameter_counts(c)
    assert counts["logical_parameters"] == 6590963712
    assert (counts["parameters_per_rank"] - counts["replicated_parameters"]) * 8 + counts["replicated_parameters"] \
        == counts["logical_parameters"]
    assert counts["parameters_per_rank"] == 831905792
    assert counts["replicated_parameters"] == 9183232


def test_bench_config_pads_vocab_for_every_tp_width():
    for world in (1, 2, 4, 8):
        c = validate_config(BENCH_CONFIG, world)
        assert c["vocab"] == 50257 and c["padded_vocab"] == 50304
        assert c["padded_vocab"] % (8 * world) == 0
        assert c["sequence"] * c["micro_batch"] * c["accumulation_steps"] == 16384
    assert padded_vocab(dict(vocab=33792), 8) == 33792


@pytest.mark.parametrize("changes", [{"heads": 31}, {"vocab": 33791}, {"hidden": 4097}, {"sequence": 2047},
                                     {"chunk_rows": 192}, {"layers": 0}, {"micro_batch": True},
                                     {"learning_rate": math.nan}, {"pad_vocab": 1}])
def test_partition_validation(changes):
    with pytest.raises(ValueError):
        validate_config(changes)


def test_flops_per_step_matches_6nd_plus_attention():
    c = validate_config(BENCH_CONFIG, 1)
    flops = train_flops_per_step(BENCH_CONFIG)
    tokens = 16384
    matmul = 32 * (4 * 4096 ** 2 + 2 * 4096 * 16384) + 50304 * 4096
    assert flops == pytest.approx(6 * tokens * matmul + 3 * tokens * 32 * 2 * 2048 * 4096, rel=1e-12)
    assert c["padded_vocab"] == 50304


def test_flat_parameter_layout_regions_and_alignment():
    import torch
    from tempname_dcu_b200.models.params import ALIGN, FlatParams, gpt_param_specs
    c = validate_config(dict(layers=2, hidden=256, ffn=1024, heads=2, sequence=256, vocab=1024, chunk_rows=128), 2)
    specs = gpt_param_specs(c, 2)
    flat = FlatParams(specs, "cpu", rank=1, seed=3)
    assert flat.numel_logical() == parameter_counts(c, 2)["parameters_per_rank"]
    for name, off in flat.offsets.items():
        assert off % ALIGN == 0
    lo, hi = flat.replicated_range
    for s in specs:
        off = flat.offsets[s.name]
        assert (lo <= off < hi) == s.replicated
        in_decay = any(a <= off < b for a, b in flat.decay_ranges)
        assert in_decay == s.decay
    assert torch.equal(flat.p("layers.0.ln1_weight"), torch.ones(256, dtype=torch.bfloat16))
    assert torch.count_nonzero(flat.p("layers.1.fc2_bias")) == 0
    assert torch.equal(flat.master.bfloat16(), flat.param)
    std = flat.p("layers.0.fc2_weight").float().std().item()
    assert abs(std - 0.02 / math.sqrt(4)) < 0.003
    other = FlatParams(specs, "cpu", rank=0, seed=3)
    assert torch.equal(flat.p("position"), other.p("position"))          # replicated: same on every rank
    assert not torch.equal(flat.p("embedding"), other.p("embedding"))    # sharded: rank-specific




def _gloo_worker(rank, world, init_file, queue):
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    try:
        from tempname_dcu_b200.parallel.tp import TPGroup
        tp = TPGroup(dist.group.WORLD)
        local = torch.arange(6, dtype=torch.float32).reshape(3, 2) + 10 * rank
        full = tp.gather(local)
        expect = torch.cat([torch.arange(6, dtype=torch.float32).reshape(3, 2) + 10 * r for r in range(world)])
        ok_gather = torch.equal(full, expect)
        big = torch.arange(world * 4, dtype=torch.float32).reshape(world * 2, 2) * (rank + 1)
        part = tp.scatter_sum(big)
        total = sum(r + 1 for r in range(world))
        ok_scatter = torch.equal(part, (torch.arange(world * 4, dtype=torch.float32).reshape(world * 2, 2)
                                        * total).chunk(world)[rank])
        stats = tp.all_gather_stacked(torch.full((3,), float(rank)))
        ok_stack = torch.equal(stats, torch.stack([torch.full((3,), float(r)) for r in range(world)]))
        t = torch.tensor([float(rank)])
        tp.all_reduce_(t)
        queue.put((rank, ok_gather, ok_scatter, ok_stack, float(t.item())))
    finally:
        dist.destroy_process_group()


def test_tp_collectives_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    world = 2
    init_file = str(tmp_path / "rendezvous")  # file rendezvous: no TCP port to race for
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, init_file, queue)) for r in range(world)]
    for proc in procs:
        proc.start()
    results = [queue.get(timeout=120) for _ in range(world)]
    for proc in procs:
        proc.join(timeout=60)
    for rank, g, s, st, total in results:
        assert g and s and st, rank
        assert total == 1.0


def test_default_config_untouched():
    assert DEFAULT_CONFIG["vocab"] == 33792 and DEFAULT_CONFIG["accumulation_steps"] == 4


def test_layer_ranges_are_named_only_when_enabled():
    import torch
    from types import SimpleNamespace
    from tempname_dcu_b200.models.gpt import GPT
    with torch.profiler.profile() as prof:
        with GPT._range(SimpleNamespace(trace_ranges=False), "tdb/layer0/fwd"):
            torch.ones(3).sum()
        with GPT._range(SimpleNamespace(trace_ranges=True), "tdb/layer1/bwd"):
            torch.ones(3).sum()
    names = [e.name for e in prof.events() if e.name.startswith("tdb/")]
    assert names == ["tdb/layer1/bwd"]


def test_native_shape_limits():
    from tempname_dcu_b200.models.config import BENCH_CONFIG, native_shape_ok, validate_config
    c = validate_config(dict(BENCH_CONFIG), 8)
    assert native_shape_ok(c, 8)
    assert not native_shape_ok(validate_config(dict(BENCH_CONFIG, micro_batch=16), 8), 8)  # 32768 tokens
    assert not native_shape_ok(validate_config(dict(BENCH_CONFIG, heads=64), 8), 8)  # head_dim 64
