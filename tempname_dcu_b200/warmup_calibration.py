"""Codec calibration on the first training steps, then frozen.

``Trainer(codec_calibration_steps=N, error_budget=e)`` runs its first N steps
with a ``CodecObserver`` attached to the model.  In every forward pass the
observer takes the input of each row-parallel output projection (attention
out and FC2) with its weight, forms this rank's partial product (the tensor
the fused operator would send), and accumulates per physical output block

* ``error_sq``: the squared TACO round-trip error of the partial, for the
  blocks this rank sends to other ranks (``tdb_taco_block_stats``), and
* ``output_sq``: the squared norm of the reduced block (after the
  reduce-scatter, on the owning rank),

summed over layers, micro-batches and steps.  ``freeze`` sums the error over
ranks, gathers the owners' output norms, and chooses one mask per role with
the planner's error-budget rule (``planning._fit_mask_error``): blocks in
ascending order of codec error while the predicted relative L2 error of the
projection output stays within the budget (and the count within the block
budget).  The masks are frozen into a plan bundle of the calibrated-plan
schema and applied to the TACO operators (``FluxB200.freeze_selection``);
blocks outside the mask then cross NVLink as BF16.  Every rank derives the
same masks from the same reduced statistics, and arms that differ only in
production order observe identical partials, so they freeze identical masks.

This realises the benchmark's "TACO calibrated on 10 warm-up steps then
frozen"; the reference calibrates the operator in isolation instead
(python/flux_dcu/calibration.py:44-127), which ``calibration.calibrate``
keeps.  The observation costs one extra GEMM and reduce-scatter per
projection and is only active during the calibration steps.
"""
from __future__ import annotations

ROLES = ("attn", "mlp")
METHOD = "training-warmup-codec-error-budget-v1"


class CodecObserver:
    def __init__(self, model):
        import torch
        self.model = model
        self.world, self.rank = model.world, model.rank
        self.chunk_rows = model.config["chunk_rows"]
        self.blocks = model.m // self.chunk_rows
        self.per = self.blocks // self.world
        dev = model.device
        self.error_sq = {r: torch.zeros(self.blocks, dtype=torch.float64, device=dev) for r in ROLES}
        self.output_sq = {r: torch.zeros(self.per, dtype=torch.float64, device=dev) for r in ROLES}
        self.observations = {r: 0 for r in ROLES}

    def observe(self, role, a_full, weight):
        """Accumulate the statistics of one projection call (a_full [m, k]
        on this rank, weight [n, k])."""
        from .ops import gemm as G
        from .ops.codec import codec
        partial = G.linear(a_full, weight)
        stats = codec().block_stats(partial, self.chunk_rows)
        err = stats[:, 2].clone()
        err[self.rank * self.per:(self.rank + 1) * self.per] = 0  # own blocks never cross the link
        self.error_sq[role] += err
        reduced = self.model.tp.scatter_sum(partial)
        self.output_sq[role] += codec().block_stats(reduced, self.chunk_rows)[:, 0]
        self.observations[role] += 1

    def statistics(self):
        """Rank-combined statistics per role (collective)."""
        import torch
        out = {}
        for role in ROLES:
            err = self.error_sq[role].clone()
            self.model.tp.all_reduce_(err)
            mine = self.output_sq[role].contiguous()
            gathered = self.model.tp.all_gather_stacked(mine).reshape(-1) if self.world > 1 else mine
            out[role] = dict(error_sq=[float(v) for v in err.cpu().tolist()],
                             output_sq=[float(v) for v in gathered.to(torch.float64).cpu().tolist()])
        return out

    def freeze(self, error_budget, quant_budget=1.0):
        """Choose and return the frozen plan bundle (collective)."""
        from . import planning as P
        stats = self.statistics()
        cfg = P.settings(dict(quant_budget=quant_budget, selection_mode="error_budget", error_budget=error_budget))
        m, n = self.model.m, self.model.h
        roles = {}
        for role, k in (("attn", self.model.h // self.world), ("mlp", self.model.f // self.world)):
            base = P.base_order(m, n, k, self.world, self.chunk_rows)
            mask, diag = P._fit_mask_error((m, n, k, self.world, self.chunk_rows), base, stats[role], cfg)
            plan = P.make_role(m, n, k, self.world, self.chunk_rows, order=base, mask=mask)
            plan["diagnostics"] = dict(method=METHOD, settings=cfg, selective=diag,
                                       observations=self.observations[role],
                                       actual_selection=P.quantization_statistics(plan, self.world))
            roles[role] = P.validate_role_plan(plan, m, n, k, self.world, self.chunk_rows)
        return dict(schema=P.SCHEMA, world_size=self.world, transport_lanes=2, roles=roles)


def apply(model, bundle):
    """Give every TACO-format fused operator of ``model`` its role's frozen mask."""
    for index, op in enumerate(model.operators):
        if hasattr(op, "freeze_selection") and getattr(op, "arm", "flux") != "flux":
            op.freeze_selection(bundle["roles"][ROLES[index % 2]]["selective_mask"])
