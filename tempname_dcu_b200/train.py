"""Training loop: the public training API of the framework.

``Trainer(config, arm, group, ...)`` owns one rank's model and optimizer;
``Trainer.step(tokens, targets)`` runs one optimizer step over
``accumulation_steps`` micro-batches and returns the step's (loss, grad norm)
as device scalars.  Token tensors may live in pinned host memory: each
micro-batch is copied to the device asynchronously inside the step.

``train_window`` reproduces the reference's timed window record (warm-up
steps, timed steps, losses, grad norms, parameter digests, memory peaks,
operator counters): python/flux_dcu/model.py:339-476, with device-side
timing (CUDA events, max over ranks) instead of host wall clock.
"""
from __future__ import annotations

import hashlib

from .models.config import parameter_counts, validate_config
from .models.gpt import GPT, Optimizer


def tensor_digest(named_tensors):
    """sha256 over (name, shape, dtype, raw bytes) of each tensor, in order."""
    import torch
    digest = hashlib.sha256()
    for name, tensor in named_tensors:
        value = tensor.detach().cpu().contiguous()
        digest.update(name.encode())
        digest.update(str(tuple(value.shape)).encode())
        digest.update(str(value.dtype).encode())
        digest.update(value.view(torch.uint8).numpy().tobytes())
    return digest.hexdigest()


def synthetic_batches(config, steps=1, seed=4321, pin=True):
    """Uniform random tokens in [0, vocab): a list of (tokens, labels) of
    shape [accumulation_steps, micro_batch*sequence] per step (CPU, pinned)."""
    import torch
    c = validate_config(config, 1)
    gen = torch.Generator(device="cpu").manual_seed(seed)
    out = []
    for _ in range(steps):
        stream = torch.randint(0, c["vocab"], (c["accumulation_steps"], c["micro_batch"], c["sequence"] + 1),
                               generator=gen)
        tokens = stream[:, :, :-1].reshape(c["accumulation_steps"], -1).contiguous()
        labels = stream[:, :, 1:].reshape(c["accumulation_steps"], -1).contiguous()
        if pin and torch.cuda.is_available():
            tokens, labels = tokens.pin_memory(), labels.pin_memory()
        out.append((tokens, labels))
    return out


class Trainer:
    """One tensor-parallel rank's trainer: model, fused AdamW, static inputs.

    ``cuda_graph=True`` captures the whole optimizer step (every micro-batch's
    forward and backward, the gradient collectives, clipping and AdamW) into
    one CUDA graph after ``graph_warmup`` eager steps and replays it from then
    on, so the host issues one launch per step instead of thousands.  Every
    per-step quantity that a replay must refresh lives on the device (the
    AdamW step number, the fused operators' call epochs); inputs are copied
    into fixed device buffers before each replay."""

    def __init__(self, config, arm="flux", group=None, *, device="cuda", seed=1234, operator_factory=None,
                 execution_plan=None, cuda_graph=False, graph_warmup=2, taco_allgather=False,
                 codec_calibration_steps=0, error_budget=0.01, wgrad_sms=None):
        """``codec_calibration_steps`` > 0 (TACO arms on two or more ranks):
        observe the codec error of every forward reduce-scatter input during
        that many first steps, then freeze one block mask per role within
        ``error_budget`` (warmup_calibration) and keep it; ``codec_plan``
        holds the frozen bundle afterwards.  Those steps run eagerly.
        ``wgrad_sms`` > 0 overlaps the backward's weight-gradient GEMMs with
        the fused collectives (``GPT.set_wgrad_overlap``); None: the default
        for the world size (``models.gpt.default_wgrad_sms``)."""
        import torch
        self.model = GPT(config, arm, group, device=device, seed=seed, operator_factory=operator_factory,
                         execution_plan=execution_plan, taco_allgather=taco_allgather, wgrad_sms=wgrad_sms)
        c = self.config = self.model.config
        self.optimizer = Optimizer(self.model, c["learning_rate"], c["weight_decay"], c["max_grad_norm"])
        self.optimizer.zero_grad = False  # _body's first micro-batch overwrites every gradient
        for op in self.model.operators:  # block-scaled FP8 operators re-quantize weights once per step
            if getattr(op, "mx", None) is not None:
                op.weight_version = self.optimizer.step_dev
        self.device = self.model.device
        self.loss = torch.zeros((), dtype=torch.float32, device=self.device)
        accum, m = c["accumulation_steps"], self.model.m
        self._tokens = torch.empty((accum, m), dtype=torch.int64, device=self.device)
        self._labels = torch.empty((accum, m), dtype=torch.int64, device=self.device)
        self.cuda_graph = bool(cuda_graph)
        self.graph_warmup = int(graph_warmup)
        self._graph = None
        self._eager_steps = 0
        self.graph_kernels = 0   # library kernels recorded in the captured step
        self.graph_replays = 0
        self.codec_calibration_steps = int(codec_calibration_steps)
        self.error_budget = float(error_budget)
        self.codec_plan = None
        self._steps_done = 0
        if self.codec_calibration_steps:
            if self.model.world < 2 or arm == "flux" or operator_factory is None:
                raise ValueError("codec calibration needs a TACO arm's fused operators on two or more ranks")
            if not 0 < self.error_budget <= 1:
                raise ValueError("error_budget must be in (0, 1]")
            self.graph_warmup = max(self.graph_warmup, self.codec_calibration_steps)

    def save_checkpoint(self, directory, plan_sha256=None):
        """Sharded checkpoint of masters + Adam state (utils/checkpoint.py);
        collective over the tensor-parallel group."""
        from .utils import checkpoint
        return checkpoint.save(self, directory, plan_sha256=plan_sha256)

    def load_checkpoint(self, directory, plan_sha256=None):
        """Resume from ``save_checkpoint``; returns the restored optimizer step."""
        from .utils import checkpoint
        return checkpoint.load(self, directory, plan_sha256=plan_sha256)

    def _body(self, tokens, labels):
        c = self.config
        calibrating = self._steps_done < self.codec_calibration_steps
        if calibrating and self.model.codec_observer is None:
            from .warmup_calibration import CodecObserver
            self.model.codec_observer = CodecObserver(self.model)
        self.loss.zero_()
        for micro in range(c["accumulation_steps"]):
            # the first micro-batch writes the gradients: no zeroing pass in the update
            self.model.forward_backward(tokens[micro], labels[micro], self.loss, overwrite_grads=micro == 0)
        norm = self.optimizer.step(self.loss)
        self._steps_done += 1
        if calibrating and self._steps_done == self.codec_calibration_steps:
            from . import warmup_calibration
            self.codec_plan = self.model.codec_observer.freeze(self.error_budget)
            self.model.codec_observer = None
            warmup_calibration.apply(self.model, self.codec_plan)
        return norm

    def step(self, tokens, labels):
        """One optimizer step over ``accumulation_steps`` micro-batches.

        tokens/labels: int64 [accumulation_steps, micro_batch*sequence] on the
        host (pinned, copied asynchronously here) or on the device."""
        import torch
        if not self.cuda_graph:
            if tokens.device.type != "cuda":
                self._tokens.copy_(tokens, non_blocking=True)
                self._labels.copy_(labels, non_blocking=True)
                tokens, labels = self._tokens, self._labels
            norm = self._body(tokens, labels)
            return self.loss, norm
        if tokens.data_ptr() != self._tokens.data_ptr():
            self._tokens.copy_(tokens, non_blocking=True)
        if labels.data_ptr() != self._labels.data_ptr():
            self._labels.copy_(labels, non_blocking=True)
        if self._graph is None and self._eager_steps < self.graph_warmup:
            self._eager_steps += 1
            norm = self._body(self._tokens, self._labels)
            return self.loss, norm
        if self._graph is None:
            from .ops import native
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            before = native.launch_count()
            with torch.cuda.graph(graph):
                self._graph_norm = self._body(self._tokens, self._labels)
            self.graph_kernels = native.launch_count() - before
            self._graph = graph  # capture recorded one step (host step count included); run it
        else:
            self.optimizer.step_count += 1
        self._graph.replay()
        self.graph_replays += 1
        return self.loss, self._graph_norm

    def release_graph(self):
        """Drop the captured graph (before tearing down process groups)."""
        self._graph = None


def train_window(config, arm, group, warmup_steps, timed_steps, *, seed=1234, token_seed=4321, operator_factory=None,
                 execution_plan=None):
    """Train a fresh model for warm-up + timed steps; returns the reference
    window record plus device-timed ``elapsed_seconds`` (max over ranks)."""
    import torch
    import torch.distributed as dist
    for name, value in (("warmup_steps", warmup_steps), ("timed_steps", timed_steps)):
        if type(value) is not int or value < 1:
            raise ValueError(f"invalid {name}")
    trainer = Trainer(config, arm, group, seed=seed, operator_factory=operator_factory,
                      execution_plan=execution_plan)
    model = trainer.model
    c = trainer.config
    world = model.world
    counts = parameter_counts(c, world)
    actual = model.parameter_count()
    if actual != counts["parameters_per_rank"]:
        raise RuntimeError("actual parameter count differs from the configuration")
    initial = tensor_digest(model.named_parameters())
    (tokens, labels), = synthetic_batches(c, 1, token_seed)
    input_hash = tensor_digest([(f"tokens.{i}", tokens[i]) for i in range(len(tokens))] +
                               [(f"labels.{i}", labels[i]) for i in range(len(labels))])
    tokens, labels = tokens.to(trainer.device), labels.to(trainer.device)
    # the first warm-up call of every fused operator validates its buffers
    # (untimed, rank-coordinated; python/flux_dcu/model.py:366-367)
    for op in model.operators:
        if hasattr(op, "validate_next_call"):
            op.validate_next_call = True
    for _ in range(warmup_steps):
        trainer.step(tokens, labels)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(group=group)
    torch.cuda.reset_peak_memory_stats()
    calls_before = model.forward_calls
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    losses, norms = [], []
    start.record()
    for _ in range(timed_steps):
        loss, norm = trainer.step(tokens, labels)
        losses.append(loss.clone())
        norms.append(norm.clone())
    end.record()
    torch.cuda.synchronize()
    local = start.elapsed_time(end) / 1000.0
    elapsed = torch.tensor(local, dtype=torch.float64, device=trainer.device)
    if world > 1:
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX, group=group)
    forwards = model.forward_calls - calls_before
    if forwards != timed_steps * c["accumulation_steps"]:
        raise RuntimeError("wrong formal forward count")
    return dict(elapsed_seconds=float(elapsed.item()), local_elapsed_seconds=local, timed_steps=timed_steps,
                warmup_steps=warmup_steps, losses=[float(x.item()) for x in losses],
                grad_norms=[float(x.item()) for x in norms],
                tokens_per_step=c["sequence"] * c["micro_batch"] * c["accumulation_steps"],
                initialization_sha256=initial, input_sha256=input_hash,
                final_parameters_sha256=tensor_digest(model.named_parameters()),
                actual_model_config={k: v for k, v in c.items()}, parameter_counts=counts,
                actual_parameters_per_rank=actual, dtype="bfloat16", optimizer="AdamW-fp32-master",
                deterministic_algorithms=True,
                gradient_policy="fp32 gradient accumulation in the GEMM epilogue; replicated gradients summed; "
                                "replicated norm counted once",
                optimizer_weight_decay_policy="matrix parameters only; biases and LayerNorm vectors excluded",
                model_implementation="tempname_dcu_b200-tp-sp-gpt-sm100a-v1",
                attention_implementation="hand-written causal flash attention (sm_100a)",
                timing="CUDA events on the compute stream, max over ranks", rank=model.rank,
                operator_counters=dict(model_forwards=forwards, target_modules=2 * c["layers"],
                                       actual_calls_per_instance=[getattr(op, "calls", 0) for op in model.operators]),
                operator_states=[op.state() for op in model.operators if hasattr(op, "state")],
                memory=dict(peak_allocated_bytes=torch.cuda.max_memory_allocated(),
                            peak_reserved_bytes=torch.cuda.max_memory_reserved()))
