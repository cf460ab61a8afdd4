"""The same-box torch baseline trainer (models/torch_baseline.py) steps on CPU."""
import math


def test_baseline_trainer_steps_and_learns_on_cpu():
    from tempname_dcu_b200.models.config import SMALL_CONFIG
    from tempname_dcu_b200.models.torch_baseline import BaselineTrainer
    from tempname_dcu_b200.train import synthetic_batches
    cfg = dict(SMALL_CONFIG, layers=1, accumulation_steps=2)
    t = BaselineTrainer(cfg, None, device="cpu")
    (tok, lab), = synthetic_batches(t.config, 1, pin=False)
    losses = []
    for _ in range(3):
        loss, norm = t.step(tok, lab)
        assert math.isfinite(float(norm)) and float(norm) > 0
        losses.append(float(loss))
    assert abs(losses[0] - math.log(t.config["vocab"])) < 0.5
    assert losses[-1] < losses[0]
    assert sum(t.replicated) == 3 + 6      # position and the final LN pair, plus LN pairs and row biases
