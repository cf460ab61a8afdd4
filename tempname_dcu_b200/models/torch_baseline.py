"""Same-box baseline: the reference design expressed with stock PyTorch on CUDA.

Torch BF16 GEMMs (cuBLAS via ``F.linear``), ``scaled_dot_product_attention``,
``F.layer_norm``, NCCL all-gather / reduce-scatter for sequence parallelism,
autograd, FP32-master AdamW from ``torch.optim`` -- none of this framework's
kernels.  It is what ``bench.py --impl baseline`` times: the same-box
"torch BF16 GEMM + NCCL" comparison point for the fused kernels.

Reference parity: python/flux_dcu/model.py:65-476 (the same model and
training-step semantics, with plain NCCL reduce-scatter in place of the
operator).
"""
from __future__ import annotations

import math

from .config import validate_config


def _impl():
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    def world(group):
        return dist.get_world_size(group) if dist.is_initialized() else 1

    def gather(x, group):
        if world(group) == 1:
            return x
        out = torch.empty((x.shape[0] * world(group), *x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x.contiguous(), group=group)
        return out

    def scatter(x, group):
        if world(group) == 1:
            return x
        out = torch.empty((x.shape[0] // world(group), *x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.reduce_scatter_tensor(out, x.contiguous(), group=group)
        return out

    class Gather(torch.autograd.Function):
        @staticmethod
        def forward(ctx, x, group):
            ctx.group = group
            return gather(x, group)

        @staticmethod
        def backward(ctx, g):
            return scatter(g, ctx.group), None

    class Scatter(torch.autograd.Function):
        @staticmethod
        def forward(ctx, x, group):
            ctx.group = group
            return scatter(x, group)

        @staticmethod
        def backward(ctx, g):
            return gather(g, ctx.group), None

    class VocabCE(torch.autograd.Function):
        @staticmethod
        def forward(ctx, logits, targets, start, valid, group):
            work = logits.float()
            if valid < work.shape[1]:
                work[:, valid:] = -float("inf")
            m = work.max(-1).values
            if world(group) > 1:
                dist.all_reduce(m, op=dist.ReduceOp.MAX, group=group)
            e = (work - m.unsqueeze(-1)).exp()
            s = e.sum(-1)
            if world(group) > 1:
                dist.all_reduce(s, group=group)
            mask = (targets >= start) & (targets < start + valid)
            idx = (targets - start).clamp(0, work.shape[1] - 1)
            t = work.gather(-1, idx.unsqueeze(-1)).squeeze(-1) * mask
            if world(group) > 1:
                dist.all_reduce(t, group=group)
            ctx.save_for_backward(e / s.unsqueeze(-1), idx, mask)
            return s.log() + m - t

        @staticmethod
        def backward(ctx, g):
            p, idx, mask = ctx.saved_tensors
            grad = p.clone()
            grad[torch.arange(grad.shape[0], device=grad.device), idx] -= mask.to(grad.dtype)
            return (grad * g.unsqueeze(-1)).to(torch.bfloat16), None, None, None, None

    return torch, dist, F, Gather, Scatter, VocabCE


class BaselineTrainer:
    def __init__(self, config, group=None, seed=1234, device="cuda"):
        torch, dist, F, Gather, Scatter, VocabCE = _impl()
        self.torch, self.dist, self.F = torch, dist, F
        self.Gather, self.Scatter, self.CE = Gather, Scatter, VocabCE
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        c = self.config = validate_config(config, self.world)
        self.device = torch.device("cpu") if device == "cpu" else torch.device(device, torch.cuda.current_device())
        h, f, L, W = c["hidden"], c["ffn"], c["layers"], self.world
        gen = torch.Generator(device=self.device).manual_seed(seed + 1000003 * self.rank)

        def p(shape, std=0.02, fill=None):
            t = torch.empty(shape, dtype=torch.bfloat16, device=self.device)
            if fill is None:
                t.normal_(0, std, generator=gen)
            else:
                t.fill_(fill)
            return torch.nn.Parameter(t)
        self.vocab_local = c["padded_vocab"] // W
        self.params = dict(embedding=p((self.vocab_local, h)), position=p((c["sequence"], h)),
                           final_w=p((h,), fill=1.0), final_b=p((h,), fill=0.0))
        self.layers = []
        for _ in range(L):
            self.layers.append(dict(ln1_w=p((h,), fill=1.0), ln1_b=p((h,), fill=0.0), ln2_w=p((h,), fill=1.0),
                                    ln2_b=p((h,), fill=0.0), qkv_w=p((3 * h // W, h)), qkv_b=p((3 * h // W,), fill=0.0),
                                    attn_w=p((h, h // W), 0.02 / math.sqrt(2 * L)), attn_b=p((h,), fill=0.0),
                                    fc1_w=p((f // W, h)), fc1_b=p((f // W,), fill=0.0),
                                    fc2_w=p((h, f // W), 0.02 / math.sqrt(2 * L)), fc2_b=p((h,), fill=0.0)))
        self.all = list(self.params.values()) + [v for layer in self.layers for v in layer.values()]
        replicated = {"position", "final_w", "final_b", "ln1_w", "ln1_b", "ln2_w", "ln2_b", "attn_b", "fc2_b"}
        names = list(self.params) + [k for layer in self.layers for k in layer]
        self.replicated = [n in replicated for n in names]
        self.masters = [torch.nn.Parameter(q.detach().float().clone()) for q in self.all]
        decay = [m for q, m in zip(self.all, self.masters) if q.ndim >= 2]
        no_decay = [m for q, m in zip(self.all, self.masters) if q.ndim < 2]
        self.opt = torch.optim.AdamW([dict(params=decay, weight_decay=c["weight_decay"]),
                                      dict(params=no_decay, weight_decay=0.0)], lr=c["learning_rate"],
                                     betas=(0.9, 0.95), eps=1e-8, fused=self.device.type == "cuda")

    def _forward(self, tokens, targets):
        torch, F, c, W, g = self.torch, self.F, self.config, self.world, self.group
        m = c["sequence"] * c["micro_batch"]
        start = self.rank * self.vocab_local
        valid = max(0, min(self.vocab_local, c["vocab"] - start))
        mine = (tokens >= start) & (tokens < start + self.vocab_local)
        x = F.embedding((tokens - start).clamp(0, self.vocab_local - 1), self.params["embedding"]) * mine.unsqueeze(-1)
        x = self.Scatter.apply(x, g) if W > 1 else x
        rows = m // W
        pos = torch.arange(self.rank * rows, (self.rank + 1) * rows, device=tokens.device) % c["sequence"]
        x = x + F.embedding(pos, self.params["position"])
        Hl, hd = c["heads"] // W, c["hidden"] // c["heads"]
        for layer in self.layers:
            n = F.layer_norm(x, (c["hidden"],), layer["ln1_w"], layer["ln1_b"], c["layer_norm_epsilon"])
            n = self.Gather.apply(n, g) if W > 1 else n
            qkv = F.linear(n, layer["qkv_w"], layer["qkv_b"])
            q, k, v = qkv.reshape(c["micro_batch"], c["sequence"], 3, Hl, hd).permute(2, 0, 3, 1, 4).unbind(0)
            a = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(m, Hl * hd)
            o = F.linear(a, layer["attn_w"])
            o = self.Scatter.apply(o, g) if W > 1 else o
            x = x + o + layer["attn_b"]
            n = F.layer_norm(x, (c["hidden"],), layer["ln2_w"], layer["ln2_b"], c["layer_norm_epsilon"])
            n = self.Gather.apply(n, g) if W > 1 else n
            hmid = F.gelu(F.linear(n, layer["fc1_w"], layer["fc1_b"]))
            o = F.linear(hmid, layer["fc2_w"])
            o = self.Scatter.apply(o, g) if W > 1 else o
            x = x + o + layer["fc2_b"]
        x = F.layer_norm(x, (c["hidden"],), self.params["final_w"], self.params["final_b"], c["layer_norm_epsilon"])
        x = self.Gather.apply(x, g) if W > 1 else x
        logits = F.linear(x, self.params["embedding"])
        return self.CE.apply(logits, targets, start, valid, g).mean()

    def step(self, tokens, labels):
        torch, c = self.torch, self.config
        if tokens.device != self.device:
            tokens, labels = tokens.to(self.device, non_blocking=True), labels.to(self.device, non_blocking=True)
        accum = c["accumulation_steps"]
        loss_sum = torch.zeros((), device=self.device)
        for mstr in self.masters:
            mstr.grad = None
        for i in range(accum):
            loss = self._forward(tokens[i], labels[i])
            (loss / accum).backward()
            loss_sum += loss.detach() / accum
            for q, mstr in zip(self.all, self.masters):
                if mstr.grad is None:
                    mstr.grad = q.grad.float()
                else:
                    mstr.grad.add_(q.grad.float())
                q.grad = None
        grads = [mstr.grad for mstr in self.masters]
        rep = [g for g, r in zip(grads, self.replicated) if r]
        shard = [g for g, r in zip(grads, self.replicated) if not r]
        if self.world > 1:
            flat = torch.cat([g.reshape(-1) for g in rep])
            self.dist.all_reduce(flat, group=self.group)
            torch._foreach_copy_(rep, [x.view_as(g) for x, g in zip(flat.split([g.numel() for g in rep]), rep)])
        sq = torch.stack([torch.linalg.vector_norm(x).double() ** 2 for x in shard]).sum()
        if self.world > 1:
            self.dist.all_reduce(sq, group=self.group)
        sq = sq + torch.stack([torch.linalg.vector_norm(x).double() ** 2 for x in rep]).sum()
        norm = sq.sqrt()
        coef = (c["max_grad_norm"] / (norm + 1e-6)).clamp(max=1.0).float()
        torch._foreach_mul_(grads, coef)
        self.opt.step()
        with torch.no_grad():
            torch._foreach_copy_(self.all, self.masters)
        return loss_sum, norm
