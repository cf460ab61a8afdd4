"""Schedules, selection, byte accounting and the measured planner (reference:
tests/test_mapping.py and tests/test_planning.py), plus the fused operator's
device tables (tile order, consumption order, signal counts)."""
import copy
import json
import math

import pytest

from tempname_dcu_b200 import planning as P
from tempname_dcu_b200.mapping import (ARMS, block_selection, schedule, selection_statistics, split_sizes,
                                       tile_table, wire_bytes)
from tempname_dcu_b200.runtime import operator_layout


# ------------------------------------------------------------------ mapping
def test_common_interleave_and_local_spacing():
    for world in (2, 4, 8):
        base = schedule(256 * world, 4096, 512, world, 128, "flux_taco")
        mixed = schedule(256 * world, 4096, 512, world, 128, "flux_taco_interleaved")
        assert sorted(x["physical"] for x in mixed) == list(range(2 * world))
        assert {(x["destination"], x["row"]) for x in base} == {(x["destination"], x["row"]) for x in mixed}
        for rank in range(world):
            assert [x["slot"] for x in mixed if x["destination"] == rank] == [rank, rank + world]
        assert base != mixed


def test_exchange_splits_pair_up():
    for world in (2, 4, 8):
        for dest in range(world):
            pairs = [split_sizes(world, rank, dest, 136) for rank in range(world)]
            for s in range(world):
                for t in range(world):
                    assert pairs[s][0][t] == pairs[t][1][s]
            assert sum(sum(send) for send, _ in pairs) == (world - 1) * 136


def test_exact_wire_bytes():
    assert wire_bytes(2048, 4096, 8, False) == 14680064
    assert wire_bytes(2048, 4096, 8, True) == 7798784


@pytest.mark.parametrize("args", [(2049, 4096, 512, 8, 128), (2048, 130, 512, 8, 128), (2048, 4096, 0, 8, 128),
                                  (2048, 4096, 512, 8, 512), (2048, 4096, 512, 1, 128)])
def test_invalid_shapes(args):
    with pytest.raises(ValueError):
        schedule(*args, "flux")


def test_arrival_plan_keeps_destinations_and_physical_lanes():
    for world in (2, 4, 8):
        shape = (256 * world, 4096, 512)
        original = schedule(*shape, world, 128, ARMS[2])
        reverse = [d * 2 + (1 - w) for w in range(2) for d in range(world)]
        plan = P.make_role(*shape, world, 128, order=reverse)
        changed = schedule(*shape, world, 128, ARMS[3], plan)
        assert [r["destination"] for r in changed] == [i % world for i in range(2 * world)]
        assert {r["physical"]: r["lane"] for r in original} == {r["physical"]: r["lane"] for r in changed}
        assert [r["lane"] for r in original] != [r["lane"] for r in changed]


def test_only_selective_arm_uses_mask_and_plans_are_arm_specific():
    shape = (512, 128, 64)
    plan = P.make_role(*shape, 2, 128, mask=[False, True, False, False])
    assert block_selection(*shape, 2, 128, ARMS[3], plan) == [True] * 4
    assert block_selection(*shape, 2, 128, ARMS[4], plan) == plan["selective_mask"]
    assert block_selection(*shape, 2, 128, ARMS[0]) == [False] * 4
    for arm in ARMS[3:]:
        with pytest.raises(ValueError):
            schedule(*shape, 2, 128, arm)
    for arm in ARMS[:3]:
        with pytest.raises(ValueError):
            schedule(*shape, 2, 128, arm, plan)


@pytest.mark.parametrize("field,value", [("arrival_order", [0, 0, 1, 3]), ("arrival_order", [2, 0, 1, 3]),
                                         ("arrival_order", [False, 2, 1, 3]), ("selective_mask", [1, 0, 0, 0]),
                                         ("shape", [1024, 128, 64]), ("chunk_rows", 64), ("diagnostics", None)])
def test_plan_mutation_rejected(field, value):
    shape = (512, 128, 64)
    plan = copy.deepcopy(P.make_role(*shape, 2, 128))
    plan[field] = value
    with pytest.raises(ValueError):
        schedule(*shape, 2, 128, ARMS[4], plan)


def test_block_bytes_match_planner_accounting():
    for world in (2, 4, 8):
        m, n, k, chunk = 256 * world, 4096, 512, 128
        for mask in ([False] * (2 * world), [True] * (2 * world), [i % 3 == 0 for i in range(2 * world)]):
            plan = P.make_role(m, n, k, world, chunk, mask=mask)
            actual = selection_statistics(m, n, world, chunk, mask)
            expected = P.quantization_statistics(plan, world)
            assert actual["remote_wire_bytes_by_source"] == expected["remote_wire_bytes_per_source"]
            assert actual["selected_remote_blocks_by_source"] == expected["selected_per_source"]
            assert sum(actual["selected_remote_blocks_by_source"]) == sum(mask) * (world - 1)
            if all(mask):
                assert actual["remote_wire_bytes_by_source"] == [wire_bytes(m, n, world, True)] * world
            if not any(mask):
                assert actual["remote_wire_bytes_by_source"] == [wire_bytes(m, n, world, False)] * world


def test_tile_table_follows_the_schedule():
    for arm in ARMS[:3]:
        order = schedule(2048, 4096, 512, 8, 128, arm)
        table = tile_table(2048, 4096, 8, 128, arm, block_m=128, block_n=256)
        assert len(table) == 16 * 16 and sorted(table) == list(range(256))
        assert [t // 16 for t in table[::16]] == [item["row"] // 128 for item in order]


def test_operator_layout_per_rank_tables():
    for world in (2, 8):
        m = 2048
        for rank in range(world):
            lay = operator_layout(m, 4096, 512, world, rank, "flux_taco_interleaved")
            per = m // world // 128
            assert sorted(lay["consume"]) == list(range(per))
            assert lay["signals"] == (4096 // 256) * 4
            assert lay["consumer_policy"] == "ordered"
        plan = P.make_role(m, 4096, 512, world, 128)
        lay = operator_layout(m, 4096, 512, world, 0, ARMS[3], plan)
        assert lay["consumer_policy"] == "per_lane_ready"
        first0 = next(it for it in lay["order"] if it["lane"] == 0)
        assert lay["delay_tile"] == (first0["row"] // 128, 0)


# ----------------------------------------------------------------- planner
def test_candidates_legal_rank_independent_deduplicated():
    for world in (2, 4, 8):
        shape = (4 * world, 128, 16, world, 2)
        cands = P.candidates(*shape)
        assert cands[0]["arrival_order"] == P.base_order(*shape)
        assert len({tuple(c["arrival_order"]) for c in cands}) == len(cands)
        for c in cands:
            plan = P.make_role(*shape, order=c["arrival_order"])
            assert P.validate_role_plan(plan, *shape) is plan
            assert [b // 2 for b in plan["arrival_order"]] == [s % world for s in range(2 * world)]


def test_keyword_signature_and_invalid_plans():
    shape = (8, 128, 16, 2, 2)
    plan = P.make_role(*shape)
    assert P.validate_role_plan(plan, shape=[8, 128, 16], world_size=2, chunk_rows=2) is plan
    for key, value in [("shape", [8, 128, 17]), ("chunk_rows", 4), ("arrival_order", [0, 1, 2, 3]),
                       ("arrival_order", [0, 2, 0, 3]), ("selective_mask", [1, 0, 1, 0])]:
        with pytest.raises(ValueError):
            P.validate_role_plan(dict(plan, **{key: value}), *shape)


def test_closure_and_source_byte_accounting():
    plan = P.make_role(8, 128, 16, 2, 2, mask=[True, False, False, False])
    stats = P.quantization_statistics(plan, 2)
    assert P.quantized_blocks(plan) == [0]
    assert stats["actual_remote_fraction"] == 0.25
    assert stats["quantized_remote_contributions"] == 1
    assert stats["selected_per_source"] == [0, 1]
    assert stats["remote_wire_bytes_per_source"] == [1024, 784]
    assert stats["mixed_source_blocks"] == 0


def test_default_h128_counts():
    plan = P.make_role(2048, 4096, 512, 8, 128)
    assert P.quantization_statistics(plan, 8)["remote_wire_bytes_per_source"] == [7798784] * 8
    plan["selective_mask"] = [False] * 16
    assert P.quantization_statistics(plan, 8)["remote_wire_bytes_per_source"] == [14680064] * 8


def test_digest_stable_and_rejects_nan():
    plan = P.make_role(8, 128, 16, 2, 2)
    assert P.role_digest(plan) == P.role_digest(json.loads(json.dumps(plan)))
    assert P.role_digest(plan) != P.role_digest(dict(plan, selective_mask=[False] * 4))
    with pytest.raises(ValueError):
        P.role_digest(dict(plan, diagnostics={"t": float("nan")}))


SHAPE = (8, 128, 16, 2, 2)
CFG = dict(warmup=0, iterations=1, training_pairs=3, confirmation_pairs=3, min_gain=0.002, quant_budget=0.5)


def evaluator(reject_arrival=False, reject_mask=False, noise=False):
    calls = []
    reverse = P.candidates(*SHAPE)[1]["arrival_order"]

    def measure(plan, seed, arm, label):
        calls.append(dict(plan=json.loads(json.dumps(plan)), seed=seed, arm=arm, label=label))
        if arm == P.ARRIVAL_ARM:
            t = 90.0 if plan["arrival_order"] == reverse else 100.0
            if reject_arrival and label.startswith("arrival_confirmation") and "/candidate" in label:
                t = 110.0
        else:
            t = 100.0 - 3.0 * sum(plan["selective_mask"])
            if reject_mask and label.startswith("selective_confirmation") and "/candidate" in label:
                t = 101.0
        if noise and "confirmation" in label and "/pair1/candidate" in label:
            t = 101.0
        return t
    return measure, calls


def test_fit_selects_order_and_budgeted_mask():
    evaluate, calls = evaluator()
    plan = P.fit_role(*SHAPE, evaluate, config=CFG)
    assert plan["diagnostics"]["arrival"]["accepted"] and plan["diagnostics"]["selective"]["accepted"]
    assert sum(plan["selective_mask"]) == 2 and plan["selective_mask"] == [True, True, False, False]
    sel = plan["diagnostics"]["selective"]
    assert sel["full_control"]["fractional_gain"] > sel["confirmation"]["fractional_gain"]


def test_confirmation_never_reselects_and_uses_disjoint_seeds():
    evaluate, calls = evaluator(reject_arrival=True, reject_mask=True)
    plan = P.fit_role(*SHAPE, evaluate, config=CFG)
    assert plan["arrival_order"] == P.base_order(*SHAPE)
    assert plan["selective_mask"] == [False] * 4
    train = {c["seed"] for c in calls if "training" in c["label"]}
    confirm = {c["seed"] for c in calls if "confirmation" in c["label"]}
    assert train and confirm and not train & confirm


def test_one_unstable_confirmation_pair_rejects():
    evaluate, _ = evaluator(noise=True)
    plan = P.fit_role(*SHAPE, evaluate, config=CFG)
    assert not plan["diagnostics"]["arrival"]["accepted"]
    assert plan["arrival_order"] == P.base_order(*SHAPE)


def test_zero_budget_still_measures_full_control():
    evaluate, calls = evaluator()
    plan = P.fit_role(*SHAPE, evaluate, config=dict(CFG, quant_budget=0.0))
    assert plan["selective_mask"] == [False] * 4
    assert any("selective_full_control" in c["label"] for c in calls)
    assert not any("singleton" in c["label"] for c in calls)


def test_full_budget_allows_full_quantization():
    evaluate, _ = evaluator()
    plan = P.fit_role(*SHAPE, evaluate, config=dict(CFG, quant_budget=1.0))
    assert plan["selective_mask"] == [True] * 4


@pytest.mark.parametrize("bad", [0.0, -1.0, float("nan"), dict(correctness_passed=False, elapsed_seconds=1.0)])
def test_invalid_or_failed_measurements_are_fatal(bad):
    with pytest.raises(ValueError):
        P.fit_role(*SHAPE, lambda *a: bad, config=CFG)


def test_error_budget_mode_selects_cheapest_blocks_within_budget():
    """selection_mode="error_budget": blocks are taken in ascending codec
    error while sqrt(sum error_sq / sum output_sq) <= error_budget and the
    count <= floor(blocks * quant_budget); no mask timing is measured."""
    evaluate, calls = evaluator()
    stats = dict(error_sq=[4e-4, 1e-4, 9e-4, 2e-4], output_sq=[1.0, 1.0, 1.0, 1.0])
    cfg = dict(CFG, quant_budget=1.0, selection_mode="error_budget", error_budget=0.01)
    plan = P.fit_role(*SHAPE, evaluate, config=cfg, block_stats=stats)
    # 1e-4 (block 1) + 2e-4 (block 3) -> sqrt(3e-4 / 4) = 0.0087 <= 0.01; adding 4e-4 -> 0.0132 > 0.01
    assert plan["selective_mask"] == [False, True, False, True]
    sel = plan["diagnostics"]["selective"]
    assert sel["method"] == "error_budget" and sel["ranked_blocks"] == [1, 3, 0, 2]
    assert math.isclose(sel["predicted_relative_l2"], math.sqrt(3e-4 / 4))
    assert sel["block_statistics"] == stats
    assert not any(c["arm"] == P.SELECTIVE_ARM for c in calls)  # the mask was not timed
    # the block budget still caps the count
    capped = P.fit_role(*SHAPE, evaluate, config=dict(cfg, quant_budget=0.25, error_budget=1.0), block_stats=stats)
    assert capped["selective_mask"] == [False, True, False, False]
    # replay from the frozen statistics reproduces the plan exactly
    again = P.fit_role(*SHAPE, evaluator()[0], config=cfg, block_stats=sel["block_statistics"])
    assert again == plan


def test_error_budget_settings_and_statistics_are_checked():
    assert "selection_mode" not in P.settings(CFG)  # timing plans keep the reference's settings exactly
    with pytest.raises(ValueError):
        P.settings(dict(CFG, error_budget=0.01))  # a budget without the mode
    with pytest.raises(ValueError):
        P.settings(dict(CFG, selection_mode="error_budget", error_budget=0.0))
    with pytest.raises(ValueError):
        P.settings(dict(CFG, selection_mode="fastest"))
    cfg = dict(CFG, selection_mode="error_budget")
    with pytest.raises(ValueError):
        P.fit_role(*SHAPE, evaluator()[0], config=cfg)  # statistics required
    for bad in (dict(error_sq=[0.1] * 3, output_sq=[1.0] * 4), dict(error_sq=[0.1] * 4, output_sq=[0.0] * 4),
                dict(error_sq=[float("nan")] * 4, output_sq=[1.0] * 4), dict(error_sq=[0.1] * 4)):
        with pytest.raises(ValueError):
            P.fit_role(*SHAPE, evaluator()[0], config=cfg, block_stats=bad)


def test_gemm_tile_picker_prefers_full_waves():
    """The tcgen05 GEMM's tile choice (pure host function of the library)."""
    import ctypes
    from tempname_dcu_b200.ops import native
    fn = native.lib().tdb_gemm_pick_tile
    fn.argtypes = [ctypes.c_int] * 4
    fn.restype = ctypes.c_int
    assert fn(2048, 16384, 4096, 148) == 512   # large: 2-CTA 256 x 256
    assert fn(2048, 1536, 4096, 148) == 192    # TP8 QKV: 128 x 192 fills one wave
    assert fn(2048, 2048, 4096, 148) == 512    # TP8 FC1: 64 SM pairs in one wave
    assert fn(128, 128, 64, 148) == 128
    assert fn(64, 96, 64, 148) == 128          # N <= 128 keeps the narrow tile


def test_remote_first_order_rotates_destinations():
    from tempname_dcu_b200.mapping import remote_first_order, schedule, tiles_for_order
    m, n, k, world, chunk = 4096, 512, 256, 4, 128
    order = schedule(m, n, k, world, chunk, "flux")
    for rank in range(world):
        rf = remote_first_order(order, world, rank)
        dests = [item["destination"] for item in rf]
        per = m // world // chunk
        expect = [(rank + 1 + i) % world for i in range(world) for _ in range(per)]
        assert dests == expect
        for d in range(world):  # block order inside a destination is unchanged
            assert [x["within"] for x in rf if x["destination"] == d] == list(range(per))
        tiles = tiles_for_order(rf, n, chunk, block_m=128, block_n=256)
        assert sorted(tiles) == list(range((m // 128) * (n // 256)))


def test_ag_tile_table_local_rows_first():
    from tempname_dcu_b200.parallel.allgather import ag_tile_table
    world, rows, n = 4, 512, 1000
    for bn in (128, 192, 256, 512):
        tm, tn = (256, 256) if bn == 512 else (128, bn)
        n_tiles = -(-n // tn)
        for rank in range(world):
            t = ag_tile_table(world, rank, rows, n, bn)
            assert sorted(t) == list(range(world * rows // tm * n_tiles))
            first_rows = {x // n_tiles * tm for x in t[: rows // tm * n_tiles]}
            assert all(rank * rows <= r < (rank + 1) * rows for r in first_rows)


def test_mma_row_blocks_follow_the_selected_physical_blocks():
    from tempname_dcu_b200.mapping import mma_row_blocks
    m, n, k, world, chunk = 2048, 4096, 512, 8, 256
    plan = P.make_role(m, n, k, world, chunk, mask=[i % 3 == 0 for i in range(m // chunk)])
    order = schedule(m, n, k, world, chunk, ARMS[4], plan)
    rows = mma_row_blocks(order, plan["selective_mask"], m, chunk)
    assert len(rows) == m // 128
    for p, selected in enumerate(plan["selective_mask"]):
        assert rows[2 * p] == rows[2 * p + 1] == int(selected)  # two 128-row blocks per 256-row chunk
