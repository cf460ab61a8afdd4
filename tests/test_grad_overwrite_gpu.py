"""The first micro-batch of a step writes the gradients (one GPU).

``Trainer`` runs the first micro-batch of every step with
``overwrite_grads=True`` and the AdamW update then leaves the gradient buffer
as it is (no zeroing pass).  This checks that

* one micro-batch with ``overwrite_grads`` writes every parameter's gradient
  (the buffer is pre-filled with NaN) and gives bit for bit what accumulating
  onto a zeroed buffer gives, also for the second, accumulating micro-batch;
* two optimizer steps of the Trainer end in the same fp32 master weights as
  the zero-then-accumulate schedule, eagerly and replayed from a CUDA graph.
"""
import pytest

pytestmark = pytest.mark.gpu

CONFIG = dict(layers=2, hidden=256, ffn=1024, heads=2, sequence=256, micro_batch=1, accumulation_steps=2,
              vocab=1024, chunk_rows=128)


def _grads(model):
    return {name: model.Gr(name).clone() for name in model.params.order}


def test_first_micro_batch_writes_every_gradient(cuda):
    import torch
    from tempname_dcu_b200.models.gpt import GPT
    from tempname_dcu_b200.train import synthetic_batches
    model = GPT(dict(CONFIG), "flux", None, device="cuda")
    (tokens, labels), = synthetic_batches(model.config, 1, seed=3)
    tokens, labels = tokens.cuda(), labels.cuda()
    model.params.grad.zero_()
    model.forward_backward(tokens[0], labels[0])
    first = _grads(model)
    model.forward_backward(tokens[1], labels[1])
    both = _grads(model)
    model.params.grad.fill_(float("nan"))
    model.forward_backward(tokens[0], labels[0], overwrite_grads=True)
    for name, ref in first.items():
        got = model.Gr(name)
        assert torch.isfinite(got).all(), name
        assert torch.equal(got, ref), name
    model.forward_backward(tokens[1], labels[1])
    for name, ref in both.items():
        assert torch.equal(model.Gr(name), ref), name


@pytest.mark.parametrize("graph", [False, True])
def test_trainer_matches_zero_then_accumulate(cuda, graph):
    import torch
    from tempname_dcu_b200.train import Trainer, synthetic_batches
    new = Trainer(dict(CONFIG), "flux", None, device="cuda", cuda_graph=graph, graph_warmup=1)
    assert new.optimizer.zero_grad is False
    old = Trainer(dict(CONFIG), "flux", None, device="cuda")
    old.optimizer.zero_grad = True
    (tokens, labels), = synthetic_batches(new.config, 1, seed=5)
    tokens, labels = tokens.cuda(), labels.cuda()
    for _ in range(3):
        new.step(tokens, labels)
        old.loss.zero_()
        for micro in range(CONFIG["accumulation_steps"]):
            old.model.forward_backward(tokens[micro], labels[micro], old.loss)
        old.optimizer.step(old.loss)
    torch.cuda.synchronize()
    assert torch.equal(new.model.params.master, old.model.params.master)
    assert torch.equal(new.loss, old.loss)
    if graph:
        new.release_graph()
