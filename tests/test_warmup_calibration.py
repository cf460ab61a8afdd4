"""Warm-up codec calibration (warmup_calibration.py), host logic on CPU:
the frozen masks follow the planner's error-budget rule per role, the bundle
has the calibrated-plan schema, and the Trainer refuses the option where it
cannot apply (one rank, the BF16 arm)."""
import math
import types

import pytest

from tempname_dcu_b200 import planning as P
from tempname_dcu_b200.warmup_calibration import METHOD, CodecObserver


def _observer(world=2, blocks=8, stats=None):
    model = types.SimpleNamespace(world=world, rank=0, m=blocks * 128, h=1024, f=4096, device="cpu",
                                  config=dict(chunk_rows=128))
    obs = CodecObserver.__new__(CodecObserver)
    obs.model, obs.world, obs.rank, obs.chunk_rows = model, world, 0, 128
    obs.blocks, obs.per = blocks, blocks // world
    obs.observations = {"attn": 3, "mlp": 3}
    obs.statistics = lambda: stats
    return obs


def test_freeze_picks_cheapest_blocks_per_role_within_budget():
    stats = dict(attn=dict(error_sq=[4e-4, 1e-4, 9e-4, 2e-4, 5e-4, 3e-4, 8e-4, 6e-4], output_sq=[1.0] * 8),
                 mlp=dict(error_sq=[1e-6] * 8, output_sq=[1.0] * 8))
    bundle = _observer(stats=stats).freeze(error_budget=0.01)
    assert bundle["schema"] == P.SCHEMA and bundle["world_size"] == 2 and bundle["transport_lanes"] == 2
    attn, mlp = bundle["roles"]["attn"], bundle["roles"]["mlp"]
    # ascending error: 1e-4 (1), 2e-4 (3), 3e-4 (5) -> sqrt(6e-4 / 8) = 0.0087; + 4e-4 -> 0.0112 > 0.01
    assert attn["selective_mask"] == [False, True, False, True, False, True, False, False]
    assert mlp["selective_mask"] == [True] * 8  # tiny errors: every block fits the budget
    for role in (attn, mlp):
        diag = role["diagnostics"]
        assert diag["method"] == METHOD and diag["observations"] == 3
        assert diag["selective"]["predicted_relative_l2"] <= 0.01
        assert role["arrival_order"] == P.base_order(*role["shape"], 2, 128)
    assert math.isclose(attn["diagnostics"]["selective"]["predicted_relative_l2"], math.sqrt(6e-4 / 8))


def test_trainer_refuses_calibration_without_taco_operators():
    from tempname_dcu_b200.models.config import SMALL_CONFIG
    from tempname_dcu_b200.train import Trainer
    with pytest.raises(ValueError, match="codec calibration"):
        Trainer(dict(SMALL_CONFIG, layers=1), "flux_taco", None, device="cpu", codec_calibration_steps=2)
