"""Flat parameter storage for the tensor-parallel GPT.

All parameters of one rank live in a few flat buffers -- fp32 masters, bf16
model weights, fp32 gradient accumulators and the two AdamW moments -- and
every named parameter is a view into them.  The layout groups parameters into
four regions::

    [sharded, weight-decay][sharded, no-decay][replicated, no-decay][replicated, decay]

so that the fused AdamW applies decay to two ranges, the replicated
gradients are one contiguous all-reduce, and the global gradient norm counts
replicated parameters once (rank 0) with two sum-of-squares launches.
Every view starts on a 128-element boundary (TMA needs 16-byte aligned bases).

Initialisation follows the reference (python/flux_dcu/model.py:187-227):
normal(0, 0.02) from a generator seeded by the parameter name (plus a
per-rank offset for sharded tensors), std 0.02/sqrt(2L) for the two
row-parallel output projections, ones/zeros for LayerNorm, zero biases; the
bf16 values are the masters' initial contents.
"""
from __future__ import annotations

from dataclasses import dataclass
import hashlib
import math

ALIGN = 128


@dataclass(frozen=True)
class ParamSpec:
    name: str
    shape: tuple
    replicated: bool
    decay: bool
    init: str  # "normal" | "ones" | "zeros"
    std: float = 0.02

    @property
    def numel(self) -> int:
        return math.prod(self.shape)


def gpt_param_specs(c, world):
    h, f, L = c["hidden"], c["ffn"], c["layers"]
    out_std = 0.02 / math.sqrt(2 * L)
    specs = [ParamSpec("embedding", (c["padded_vocab"] // world, h), False, True, "normal"),
             ParamSpec("position", (c["sequence"], h), True, True, "normal")]
    for i in range(L):
        p = f"layers.{i}."
        specs += [
            ParamSpec(p + "ln1_weight", (h,), True, False, "ones"),
            ParamSpec(p + "ln1_bias", (h,), True, False, "zeros"),
            ParamSpec(p + "ln2_weight", (h,), True, False, "ones"),
            ParamSpec(p + "ln2_bias", (h,), True, False, "zeros"),
            ParamSpec(p + "qkv_weight", (3 * h // world, h), False, True, "normal"),
            ParamSpec(p + "qkv_bias", (3 * h // world,), False, False, "zeros"),
            ParamSpec(p + "attn_weight", (h, h // world), False, True, "normal", out_std),
            ParamSpec(p + "attn_bias", (h,), True, False, "zeros"),
            ParamSpec(p + "fc1_weight", (f // world, h), False, True, "normal"),
            ParamSpec(p + "fc1_bias", (f // world,), False, False, "zeros"),
            ParamSpec(p + "fc2_weight", (h, f // world), False, True, "normal", out_std),
            ParamSpec(p + "fc2_bias", (h,), True, False, "zeros"),
        ]
    specs += [ParamSpec("final_weight", (h,), True, False, "ones"),
              ParamSpec("final_bias", (h,), True, False, "zeros")]
    return specs


def _region(spec):
    return (0 if spec.decay else 1) if not spec.replicated else (2 if not spec.decay else 3)


def name_seed(name: str, seed: int, rank: int, replicated: bool) -> int:
    salt = int.from_bytes(hashlib.sha256(name.encode()).digest()[:8], "little")
    return (seed + salt + (0 if replicated else 1000003 * rank)) % (2 ** 63 - 1)


class FlatParams:
    """Flat master/param/grad/moment buffers with named views."""

    def __init__(self, specs, device, *, rank=0, seed=1234, materialize=True):
        import torch
        self.specs = sorted(specs, key=lambda s: (_region(s), specs.index(s)))
        self.order = [s.name for s in specs]  # canonical (construction) order
        self.offsets = {}
        cursor = 0
        bounds = [0, 0, 0, 0, 0]
        for region in range(4):
            bounds[region] = cursor
            for spec in self.specs:
                if _region(spec) != region:
                    continue
                self.offsets[spec.name] = cursor
                cursor += -(-spec.numel // ALIGN) * ALIGN
        bounds[4] = cursor
        self.total = cursor
        self.region_bounds = bounds
        self.sharded_range = (0, bounds[2])
        self.replicated_range = (bounds[2], bounds[4])
        self.decay_ranges = [(bounds[0], bounds[1]), (bounds[3], bounds[4])]
        self.device = torch.device(device)
        self.spec_by_name = {s.name: s for s in self.specs}
        self.rank = rank
        self.seed = seed
        if materialize:
            self.allocate()
            self.initialize()

    def allocate(self):
        import torch
        n, dev = self.total, self.device
        self.master = torch.zeros(n, dtype=torch.float32, device=dev)
        self.param = torch.zeros(n, dtype=torch.bfloat16, device=dev)
        self.grad = torch.zeros(n, dtype=torch.float32, device=dev)
        self.exp_avg = torch.zeros(n, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros(n, dtype=torch.float32, device=dev)

    def _view(self, flat, name):
        spec = self.spec_by_name[name]
        off = self.offsets[name]
        return flat[off:off + spec.numel].view(spec.shape)

    def p(self, name):
        return self._view(self.param, name)

    def g(self, name):
        return self._view(self.grad, name)

    def m(self, name):
        return self._view(self.master, name)

    def initialize(self):
        import torch
        for spec in self.specs:
            view = self.p(spec.name)
            if spec.init == "ones":
                view.fill_(1)
            elif spec.init == "zeros":
                view.zero_()
            else:
                gen = torch.Generator(device=self.device)
                gen.manual_seed(name_seed(spec.name, self.seed, self.rank, spec.replicated))
                view.normal_(0.0, spec.std, generator=gen)
        self.master.copy_(self.param.float())

    def named_parameters(self):
        """(name, bf16 view) in canonical construction order."""
        return [(name, self.p(name)) for name in self.order]

    def numel_logical(self):
        return sum(s.numel for s in self.specs)
