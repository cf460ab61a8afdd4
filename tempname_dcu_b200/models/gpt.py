"""Sequence/tensor-parallel GPT on the sm_100a kernels.

The training micro-step is an explicit forward/backward schedule over the
native kernels (no per-op autograd graph):

forward, per layer (x: SP rows [m/W, h])::

    ln1 = LN(x); ln1f = AG(ln1); qkv = ln1f Wqkv^T + b       (column-parallel)
    a = causal_flash_attention(qkv)                           (local heads)
    x1 = x + RS(a Wo^T) + bo                                  (row-parallel, operator)
    ln2 = LN(x1); ln2f = AG(ln2); z = ln2f W1^T + b1; h = gelu(z)
    x2 = x1 + RS(h W2^T) + b2                                 (row-parallel, operator)

backward mirrors it: data gradients through the transposed GEMMs (the
collective order reversed), weight gradients accumulated directly into the
fp32 gradient buffer by the GEMM epilogue, bias gradients by deterministic
column sums, GELU backward fused into the FC2 data-gradient epilogue.
With fused operators on 2..8 ranks the embedding's reduce-scatter and its
backward gather become a sparse exchange (parallel/embedding_exchange.py):
each token row moves only from its vocabulary shard's owner, bit for bit the
same result.  The LM head is the tied vocabulary-sharded embedding; the vocab-parallel
cross-entropy writes its gradient over the logits in place, so the backward
starts inside the loss.

Everything is deterministic (no floating-point atomics), so arms that only
reorder production produce bitwise-identical losses, norms and weights.

Reference parity: python/flux_dcu/model.py:178-292 (GPT, SumScatter,
ColumnLinear, RowLinear, VocabCrossEntropy, replicated-gradient all-reduce,
global grad norm) and :339-476 (train_window).
"""
from __future__ import annotations

from .config import native_shape_ok, validate_config
from .params import FlatParams, gpt_param_specs

ARMS = ("flux", "flux_taco", "flux_taco_interleaved", "flux_taco_interleaved_arrival",
        "flux_taco_interleaved_arrival_selective")


class NcclRowOperator:
    """Row-parallel output projection without fusion: GEMM, NCCL
    reduce-scatter, bias + residual.  (With one rank: one fused GEMM.)"""

    calls = 0

    def __init__(self, tp):
        self.tp = tp

    def forward(self, a_full, weight, bias, residual):
        from ..ops import gemm as G
        from ..ops import kernels as K
        self.calls += 1
        if self.tp.world == 1:
            return G.linear_residual(a_full, weight, bias, residual)
        partial = G.linear(a_full, weight)
        out = self.tp.scatter_sum(partial)
        return K.bias_residual(out, bias, residual, out=out)

    def state(self):
        return dict(backend="nccl-reduce-scatter", calls=self.calls)


def default_wgrad_sms(world):
    """SMs given to the backward's weight-gradient stream by default at this
    tensor-parallel world size (0: no overlap).  Measured on 8 B200s (GPT-6.7B
    step, ms): 0 -> 258.7, 24 -> 243.6, 40 -> 242.4, 56 -> 243.3, 72 -> 247.1;
    on 4: 0 -> 297.6, 40 -> 275.7; on 2 (where the fused kernels are
    compute-bound): 0 -> 453.7, 32 -> 509.9, 48 -> 453.2, so no overlap there."""
    return 40 if world >= 4 else 0


class GPT:
    """One rank's shard of the TP/SP GPT with flat parameter storage."""

    def __init__(self, config, arm="flux", group=None, *, device="cuda", seed=1234, operator_factory=None,
                 execution_plan=None, materialize=True, taco_allgather=False, wgrad_sms=None):
        """``wgrad_sms`` > 0 (two or more ranks): in the backward, every
        layer's weight-gradient GEMMs run on a second stream, each on at most
        that many SMs, while the communication-bound fused all-gather and
        reduce-scatter kernels on the compute stream keep the other SMs
        (``set_wgrad_overlap``); None takes ``default_wgrad_sms(world)``."""
        import torch
        from ..parallel.tp import TPGroup
        self.tp = TPGroup(group)
        self.world, self.rank = self.tp.world, self.tp.rank
        self.config = c = validate_config(config, self.world)
        if not native_shape_ok(c, self.world):
            raise ValueError("the sm_100a kernels need head_dim 128, 8-aligned shard widths and at most "
                             "16384 tokens per micro-batch")
        if arm not in ARMS and arm != "nccl":
            raise ValueError(f"unknown arm {arm}")
        self.arm = arm
        self.device = torch.device(device)
        self.seed = seed
        self.h, self.f = c["hidden"], c["ffn"]
        self.heads_local = c["heads"] // self.world
        self.m = c["sequence"] * c["micro_batch"]
        self.ml = self.m // self.world
        self.vocab_local = c["padded_vocab"] // self.world
        self.vocab_start = self.rank * self.vocab_local
        self.valid_vocab_local = max(0, min(self.vocab_local, c["vocab"] - self.vocab_start))
        self.params = FlatParams(gpt_param_specs(c, self.world), self.device, rank=self.rank, seed=seed,
                                 materialize=materialize)
        self.forward_calls = 0
        # warm-up codec calibration (warmup_calibration.CodecObserver) while attached
        self.codec_observer = None
        self.trace_ranges = False  # per-layer profiler / NVTX ranges (utils.trace --ranges)
        self.operators = []
        factory = operator_factory
        for index in range(c["layers"]):
            for role, k in (("attn", self.h // self.world), ("mlp", self.f // self.world)):
                if factory is None:
                    self.operators.append(NcclRowOperator(self.tp))
                else:
                    plan = execution_plan["roles"][role] if (execution_plan and arm in ARMS[3:]) else None
                    self.operators.append(factory(m=self.m, n=self.h, k=k, group=group, arm=arm,
                                                  chunk_rows=c["chunk_rows"], plan=plan))
        self._scratch = {}
        self._overlap = None   # (fused-kernel CTAs, weight-gradient CTAs) when the backward overlaps them
        self._wgrad_stream = None
        self._wgrad_pending = None
        self.set_wgrad_overlap(default_wgrad_sms(self.world) if wgrad_sms is None else wgrad_sms)
        # Backward reduce-scatters of the column-parallel data gradients
        # (dX = RS(dY W)) run through the same fused kernel (BF16, ordered)
        # whenever the forward projections do.
        self._bwd_rs = {}
        self.agg = None
        self.embx = None
        from ..parallel import embedding_exchange as embx
        if factory is not None and 1 < self.world <= 8 and embx.enabled():
            # sparse embedding exchange instead of the dense reduce-scatter / gather
            self.embx = embx.EmbeddingExchange(self.tp, self.ml, self.h, self.vocab_local)
        if factory is not None and self.world > 1:
            # sequence-parallel all-gathers over NVLink (same rows/cols everywhere)
            self.tp.enable_symmetric_gather(self.ml, self.h)
            if self.ml % 256 == 0:
                # ... and, where a GEMM consumes the gathered rows, fused into it
                from ..parallel.allgather import SymmAgGemm
                # taco_allgather: the gathered rows of peers cross NVLink as TACO packets
                self.agg = SymmAgGemm(self.tp, self.ml, self.h, taco=taco_allgather)
            from ..runtime import FluxB200
            for k in (3 * self.h // self.world, self.f // self.world, self.vocab_local):
                if k not in self._bwd_rs:
                    self._bwd_rs[k] = FluxB200(self.m, self.h, k, group, "flux", chunk_rows=c["chunk_rows"],
                                               b_mn=True, remote_first=True)

    def _dgrad_rs(self, dy, weight):
        """RS(dy @ weight) -> [m/W, h]: fused kernel when available, else
        GEMM + NCCL reduce-scatter."""
        from ..ops import gemm as G
        op = self._bwd_rs.get(dy.shape[1])
        if op is not None:
            with self._fused_share():
                return op.forward(dy, weight)
        return self.tp.scatter_sum(G.matmul_nt(dy, weight))

    # ------------------------------------------------ backward overlap
    def set_wgrad_overlap(self, wgrad_sms):
        """Run the per-layer weight-gradient GEMMs of the backward on a
        second stream, on at most ``wgrad_sms`` SMs, beside the fused
        collective kernels, which are then limited to the remaining SMs (0:
        off, everything on one stream).  With tensor parallelism the fused
        kernels wait on NVLink for most of their time, so the GEMMs fill SMs
        that would idle.  Each weight's gradient still accumulates in
        micro-batch order, so the result is bitwise the same.  Takes effect
        for the next backward (and the next captured graph)."""
        import torch
        wgrad_sms = int(wgrad_sms)
        if wgrad_sms <= 0 or self.world < 2:
            self._overlap = None
            return
        from ..ops import native
        sms = int(native.lib().tdb_sm_count(torch.cuda.current_device()))
        wgrad_sms = min(max(2, wgrad_sms - wgrad_sms % 2), sms - 2)
        self._overlap = (sms - wgrad_sms, wgrad_sms)
        if self._wgrad_stream is None:
            self._wgrad_stream = torch.cuda.Stream(device=self.device)

    def _fused_share(self):
        import contextlib
        from ..ops import native
        return native.grid_limit(self._overlap[0]) if self._overlap else contextlib.nullcontext()

    def _wgrad(self, dy, x, name, keep, acc=True):
        """Gr(name) (+)= dy^T x: on the weight-gradient stream when
        overlapping (``keep`` holds the operands until the compute stream has
        waited for it), else in line."""
        import torch
        from ..ops import gemm as G
        from ..ops import native
        if self._overlap is None:
            G.weight_grad(dy, x, self.Gr(name), accumulate=acc)
            return
        side = self._wgrad_stream
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side), native.grid_limit(self._overlap[1]):
            G.weight_grad(dy, x, self.Gr(name), accumulate=acc)
        keep.extend((dy, x))

    def _wgrad_layer_done(self, keep):
        """After a layer's backward: the compute stream waits for the PREVIOUS
        layer's weight gradients (so they overlap this layer's collectives)
        and releases their operands; this layer's stay pending."""
        import torch
        if self._overlap is None:
            return
        done = torch.cuda.Event()
        done.record(self._wgrad_stream)
        if self._wgrad_pending is not None:
            torch.cuda.current_stream().wait_event(self._wgrad_pending[0])
        self._wgrad_pending = (done, keep)

    def _wgrad_join(self):
        import torch
        if self._overlap is None:
            return
        torch.cuda.current_stream().wait_stream(self._wgrad_stream)
        self._wgrad_pending = None

    # ------------------------------------------------------------ helpers
    def _buf(self, key, numel, dtype):
        import torch
        t = self._scratch.get(key)
        if t is None or t.numel() < numel or t.dtype != dtype:
            t = torch.empty(numel, dtype=dtype, device=self.device)
            self._scratch[key] = t
        return t[:numel]

    def P(self, name):
        return self.params.p(name)

    def Gr(self, name):
        return self.params.g(name)

    # ------------------------------------------------------------ forward
    def _embed(self, tokens):
        import torch
        from ..ops import kernels as K
        c = self.config
        if self.embx is not None:
            return self.embx.forward(tokens, self.P("embedding"), self.vocab_start, self.P("position"),
                                     self.rank * self.ml, c["sequence"])
        out = torch.empty((self.m, self.h), dtype=torch.bfloat16, device=self.device)
        if self.world == 1:
            K.embedding_fwd(tokens, self.P("embedding"), 0, out, self.P("position"), 0, c["sequence"])
            return out
        K.embedding_fwd(tokens, self.P("embedding"), self.vocab_start, out)
        x = self.tp.scatter_sum(out)
        K.add_positions(x, self.P("position"), self.rank * self.ml, c["sequence"])
        return x

    def _layer_fwd(self, i, x):
        from ..ops import gemm as G
        from ..ops import kernels as K
        c, p = self.config, f"layers.{i}."
        eps = c["layer_norm_epsilon"]
        ln1, mean1, rstd1 = K.layernorm_fwd(x, self.P(p + "ln1_weight"), self.P(p + "ln1_bias"), eps)
        if self.agg is not None:
            qkv, ln1f = self.agg(ln1, self.P(p + "qkv_weight"), mode=self.agg.BIAS, bias=self.P(p + "qkv_bias"))
        else:
            ln1f = self.tp.gather(ln1)
            qkv = G.linear(ln1f, self.P(p + "qkv_weight"), self.P(p + "qkv_bias"))
        attn, lse = K.attention_fwd(qkv, c["micro_batch"], c["sequence"], self.heads_local)
        if self.codec_observer is not None:
            self.codec_observer.observe("attn", attn, self.P(p + "attn_weight"))
        x1 = self.operators[2 * i].forward(attn, self.P(p + "attn_weight"), self.P(p + "attn_bias"), x)
        ln2, mean2, rstd2 = K.layernorm_fwd(x1, self.P(p + "ln2_weight"), self.P(p + "ln2_bias"), eps)
        if self.agg is not None:
            h1, ln2f, z = self.agg(ln2, self.P(p + "fc1_weight"), mode=self.agg.BIAS_GELU,
                                   bias=self.P(p + "fc1_bias"))
        else:
            ln2f = self.tp.gather(ln2)
            h1, z = G.linear_gelu(ln2f, self.P(p + "fc1_weight"), self.P(p + "fc1_bias"))
        if self.codec_observer is not None:
            self.codec_observer.observe("mlp", h1, self.P(p + "fc2_weight"))
        x2 = self.operators[2 * i + 1].forward(h1, self.P(p + "fc2_weight"), self.P(p + "fc2_bias"), x1)
        return x2, (x, mean1, rstd1, ln1f, qkv, attn, lse, x1, mean2, rstd2, ln2f, z, h1)

    def forward_backward(self, tokens, targets, loss_acc=None, *, grad_scale=None, loss_scale=None,
                         overwrite_grads=False):
        """One micro-batch: forward, loss (added into ``loss_acc``) and the
        full backward, accumulating fp32 gradients -- or, with
        ``overwrite_grads`` (the first micro-batch of a step), writing them, so
        that the gradient buffer needs no zeroing between steps (every
        parameter receives a gradient in every micro-batch; x written equals
        0 + x accumulated, bit for bit).  ``tokens``/``targets`` are the
        flattened micro-batch [micro_batch*sequence] (int64, device)."""
        import torch
        from ..ops import gemm as G
        from ..ops import kernels as K
        c = self.config
        if tokens.shape != (self.m,) or targets.shape != (self.m,):
            raise ValueError("tokens/targets must hold the full flattened micro-batch")
        accum = c["accumulation_steps"]
        grad_scale = 1.0 / (self.m * accum) if grad_scale is None else grad_scale
        loss_scale = 1.0 / (self.m * accum) if loss_scale is None else loss_scale
        if loss_acc is None:
            loss_acc = torch.zeros((), dtype=torch.float32, device=self.device)
        self.forward_calls += 1
        # ---- forward
        x = self._embed(tokens)
        saved = []
        for i in range(c["layers"]):
            with self._range(f"tdb/layer{i}/fwd"):
                x, s = self._layer_fwd(i, x)
            saved.append(s)
        xl = x
        eps = c["layer_norm_epsilon"]
        lnf, meanf, rstdf = K.layernorm_fwd(xl, self.P("final_weight"), self.P("final_bias"), eps)
        if self.agg is not None:
            logits, lnff = self.agg(lnf, self.P("embedding"))  # [m, V/W]
        else:
            lnff = self.tp.gather(lnf)
            logits = G.linear(lnff, self.P("embedding"))  # [m, V/W]
        stats = K.xent_stats(logits, targets, self.vocab_start, self.valid_vocab_local)
        all_stats = self.tp.all_gather_stacked(stats)
        gstats = self._buf("gstats", self.m * 2, torch.float32).view(self.m, 2)
        row_loss = self._buf("row_loss", self.m, torch.float32)
        K.xent_combine(all_stats, self.world, self.m, gstats, row_loss, loss_acc, loss_scale, accumulate=True)
        # ---- backward (starts inside the loss: logits <- dlogits)
        K.xent_grad(logits, targets, self.vocab_start, self.valid_vocab_local, gstats, grad_scale)
        acc = not overwrite_grads
        dlnf = self._dgrad_rs(logits, self.P("embedding"))
        # the LM-head weight gradient comes first: the embedding backward adds onto it below
        G.weight_grad(logits, lnff, self.Gr("embedding"), accumulate=acc)
        del logits
        ln_scratch = self._buf("ln_scratch", K.layernorm_scratch_floats(self.ml, self.h), torch.float32)
        dx = K.layernorm_bwd(xl, self.P("final_weight"), meanf, rstdf, dlnf, self.Gr("final_weight"),
                             self.Gr("final_bias"), ln_scratch, accumulate=acc)
        for i in reversed(range(c["layers"])):
            with self._range(f"tdb/layer{i}/bwd"):
                dx = self._layer_bwd(i, dx, saved[i], ln_scratch, acc)
            saved[i] = None
        self._wgrad_join()
        # ---- embedding / positions
        if overwrite_grads:
            self.Gr("position").zero_()
        K.position_bwd(dx, self.rank * self.ml if self.world > 1 else 0, c["sequence"], self.Gr("position"))
        if self.embx is not None:  # only the rows of tokens in this rank's shard, from their holders
            dfull = self.embx.backward(tokens, dx, self.vocab_start,
                                       self._buf("emb_dfull", self.m * self.h, torch.bfloat16).view(self.m, self.h))
        else:
            dfull = self.tp.gather(dx)
        sorted_tokens, order = K.sort_tokens(tokens, self._buf("sorted_tokens", self.m, torch.int64),
                                             self._buf("token_order", self.m, torch.int64))
        K.embedding_bwd(sorted_tokens, order, dfull, self.vocab_start, self.vocab_local, self.Gr("embedding"))
        return loss_acc

    def _range(self, name):
        """Named range (torch.profiler record_function + NVTX) around a layer's
        forward or backward when ``trace_ranges`` is set; a no-op otherwise."""
        import contextlib
        if not self.trace_ranges:
            return contextlib.nullcontext()
        import torch
        stack = contextlib.ExitStack()
        stack.enter_context(torch.profiler.record_function(name))
        torch.cuda.nvtx.range_push(name)
        stack.callback(torch.cuda.nvtx.range_pop)
        return stack

    def _colsum(self, x, name, acc=True, keep=None):
        """Gr(name) (+)= column sums of x (a bias gradient).  With the
        backward overlap and a ``keep`` list it runs on the weight-gradient
        stream too (off the compute stream's critical path; same order per
        bias, so the same bits).  One scratch buffer per shape, allocated on
        first use and kept, so no buffer is shared across streams."""
        import torch
        from ..ops import kernels as K
        rows, cols = x.shape
        scratch = self._buf(f"colsum{rows}x{cols}", K.colsum_scratch_floats(rows, cols), torch.float32)
        if self._overlap is None or keep is None:
            K.colsum(x, self.Gr(name), scratch, accumulate=acc)
            return
        side = self._wgrad_stream
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            K.colsum(x, self.Gr(name), scratch, accumulate=acc)
        keep.append(x)

    def _layer_bwd(self, i, dx2, saved, ln_scratch, acc=True):
        from ..ops import gemm as G
        from ..ops import kernels as K
        c, p = self.config, f"layers.{i}."
        x, mean1, rstd1, ln1f, qkv, attn, lse, x1, mean2, rstd2, ln2f, z, h1 = saved
        keep = []  # operands of weight / bias gradients still running on the overlap stream
        # FC2 (row-parallel): x2 = x1 + RS(h1 W2^T) + b2
        self._colsum(dx2, p + "fc2_bias", acc, keep)
        if self.agg is not None:
            with self._fused_share():
                dz, dyf = self.agg(dx2, self.P(p + "fc2_weight"), b_mn=True, mode=self.agg.GELU_BWD, aux=z)
        else:
            dyf = self.tp.gather(dx2)
            dz = G.matmul_nt(dyf, self.P(p + "fc2_weight"), gelu_pre=z)
        self._wgrad(dyf, h1, p + "fc2_weight", keep, acc)
        # FC1 (column-parallel)
        self._colsum(dz, p + "fc1_bias", acc, keep)
        self._wgrad(dz, ln2f, p + "fc1_weight", keep, acc)
        dln2 = self._dgrad_rs(dz, self.P(p + "fc1_weight"))
        dx1 = K.layernorm_bwd(x1, self.P(p + "ln2_weight"), mean2, rstd2, dln2, self.Gr(p + "ln2_weight"),
                              self.Gr(p + "ln2_bias"), ln_scratch, dres=dx2, accumulate=acc)
        # attention out (row-parallel)
        self._colsum(dx1, p + "attn_bias", acc, keep)
        if self.agg is not None:
            with self._fused_share():
                dattn, dyf = self.agg(dx1, self.P(p + "attn_weight"), b_mn=True)
        else:
            dyf = self.tp.gather(dx1)
            dattn = G.matmul_nt(dyf, self.P(p + "attn_weight"))
        self._wgrad(dyf, attn, p + "attn_weight", keep, acc)
        dqkv = K.attention_bwd(qkv, attn, dattn, lse, c["micro_batch"], c["sequence"], self.heads_local)
        # QKV (column-parallel)
        self._colsum(dqkv, p + "qkv_bias", acc, keep)
        self._wgrad(dqkv, ln1f, p + "qkv_weight", keep, acc)
        dln1 = self._dgrad_rs(dqkv, self.P(p + "qkv_weight"))
        dx = K.layernorm_bwd(x, self.P(p + "ln1_weight"), mean1, rstd1, dln1, self.Gr(p + "ln1_weight"),
                             self.Gr(p + "ln1_bias"), ln_scratch, dres=dx1, accumulate=acc)
        self._wgrad_layer_done(keep)
        return dx

    # ------------------------------------------------------------ gradients
    def reduce_replicated_gradients(self):
        lo, hi = self.params.replicated_range
        if self.world > 1 and hi > lo:
            self.tp.all_reduce_(self.params.grad[lo:hi])

    def global_grad_norm_sq(self, out):
        """fp64 sum of squares over this rank's sharded gradients plus (rank 0
        only) the replicated ones, all-reduced over the group."""
        import torch
        from ..ops import kernels as K
        partial = self._buf("sumsq_partial", K.sumsq_partials_count(), torch.float64)
        lo, hi = self.params.sharded_range
        K.sumsq(self.params.grad[lo:hi], partial, out, accumulate=False)
        if self.rank == 0:
            rlo, rhi = self.params.replicated_range
            K.sumsq(self.params.grad[rlo:rhi], partial, out, accumulate=True)
        self.tp.all_reduce_(out)
        return out

    def named_parameters(self):
        return self.params.named_parameters()

    def parameter_count(self):
        return self.params.numel_logical()


class Optimizer:
    """Fused AdamW over the flat buffers with global-norm clipping computed on
    the device (betas (0.9, 0.95), eps 1e-8, decoupled decay on matrices)."""

    def __init__(self, model, lr, weight_decay, max_grad_norm, betas=(0.9, 0.95), eps=1e-8):
        import torch
        self.model, self.lr, self.wd, self.max_norm = model, lr, weight_decay, max_grad_norm
        self.betas, self.eps = betas, eps
        self.step_count = 0
        dev = model.device
        self.norm_sq = torch.zeros((), dtype=torch.float64, device=dev)
        self.norm = torch.zeros((), dtype=torch.float64, device=dev)
        self.coef = torch.ones((), dtype=torch.float32, device=dev)
        self.finite = torch.ones((), dtype=torch.int32, device=dev)
        self.step_dev = torch.zeros((), dtype=torch.int32, device=dev)  # advanced by the clip kernel
        # False when every step's first micro-batch overwrites the gradients
        # (Trainer): the update then does not zero them
        self.zero_grad = True

    def step(self, loss=None):
        from ..ops import kernels as K
        m = self.model
        m.reduce_replicated_gradients()
        m.global_grad_norm_sq(self.norm_sq)
        self.finite.fill_(1)
        K.clip_coef(self.norm_sq, self.max_norm, self.norm, self.coef, loss, self.finite, step_counter=self.step_dev)
        self.step_count += 1
        P = m.params
        K.adamw(P.master, P.grad, P.exp_avg, P.exp_avg_sq, P.param, wd_ranges=P.decay_ranges, lr=self.lr,
                beta1=self.betas[0], beta2=self.betas[1], eps=self.eps, weight_decay=self.wd,
                step_dev=self.step_dev, coef=self.coef, finite=self.finite, zero_grad=self.zero_grad)
        return self.norm


def build_model(config, arm="flux", group=None, codec=None, *, device="cuda", seed=1234, operator_factory=None,
                execution_plan=None):
    """Build one rank's model.  ``operator_factory(m, n, k, group, arm,
    chunk_rows, plan)`` builds the row-parallel operators (the fused
    GEMM+reduce-scatter of ``runtime.FluxB200`` for the five arms); None
    uses plain NCCL."""
    if arm in ARMS[3:] and operator_factory is not None and execution_plan is None:
        raise ValueError("arrival/selective arms need a frozen execution plan")
    return GPT(config, arm, group, device=device, seed=seed, operator_factory=operator_factory,
               execution_plan=execution_plan)
