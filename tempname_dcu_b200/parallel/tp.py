"""Tensor/sequence-parallel group plumbing.

``TPGroup`` wraps the torch.distributed process group of one tensor-parallel
group and provides the collectives the model needs:

* ``gather(x_local)`` -- all-gather of sequence-parallel rows (SP -> full);
* ``scatter_sum(x_full)`` -- reduce-scatter back to SP rows;
* ``all_reduce_(t)`` / ``all_gather_stats`` -- small control-plane reductions.

With world size 1 every collective is the identity.  These NCCL paths are the
plumbing and the baseline; the fused GEMM+collective kernels replace them on
the hot paths through ``runtime.FluxB200``.

Reference parity: ``python/flux_dcu/model.py:65-98`` (gather_rows,
scatter_sum, including the gloo special case used by CPU tests).
"""
from __future__ import annotations


class TPGroup:
    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.world = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
            self.backend = str(dist.get_backend(group))
        else:
            self.world, self.rank, self.backend = 1, 0, "none"
        self.symm_gather = None

    def enable_symmetric_gather(self, rows, cols):
        """Route gathers of [rows, cols] bf16 blocks through the NVLink pull
        kernel (parallel/allgather.py) instead of NCCL.  Collective."""
        if self.world > 1 and self.backend == "nccl" and self.symm_gather is None:
            from .allgather import SymmAllGather
            self.symm_gather = SymmAllGather(self, rows, cols)
        return self.symm_gather

    # ------------------------------------------------------------------ rows
    def gather(self, x_local, out=None):
        import torch
        if self.world == 1:
            return x_local
        x_local = x_local.contiguous()
        if self.symm_gather is not None and self.symm_gather.matches(x_local):
            return self.symm_gather(x_local, out)
        rows = x_local.shape[0]
        if out is None:
            out = torch.empty((rows * self.world, *x_local.shape[1:]), dtype=x_local.dtype, device=x_local.device)
        if self.backend == "gloo":
            pieces = list(out.chunk(self.world, 0))
            self.dist.all_gather(pieces, x_local, group=self.group)
        else:
            self.dist.all_gather_into_tensor(out, x_local, group=self.group)
        return out

    def scatter_sum(self, x_full, out=None):
        import torch
        if self.world == 1:
            return x_full
        if x_full.shape[0] % self.world:
            raise ValueError("reduce-scatter rows do not divide the tensor-parallel group")
        if self.backend == "gloo":
            # gloo lacks reduce_scatter_tensor in some releases: all-reduce then take our rows
            copy = x_full.contiguous().clone()
            self.dist.all_reduce(copy, group=self.group)
            res = copy.chunk(self.world, 0)[self.rank].contiguous()
            if out is not None:
                out.copy_(res)
                return out
            return res
        if out is None:
            out = torch.empty((x_full.shape[0] // self.world, *x_full.shape[1:]), dtype=x_full.dtype,
                              device=x_full.device)
        self.dist.reduce_scatter_tensor(out, x_full.contiguous(), group=self.group)
        return out

    # ------------------------------------------------------------ small ops
    def all_reduce_(self, t, op=None):
        if self.world > 1:
            self.dist.all_reduce(t, op=op or self.dist.ReduceOp.SUM, group=self.group)
        return t

    def all_gather_stacked(self, t, out=None):
        """[world, *t.shape] stacked all-gather (rank order)."""
        import torch
        if self.world == 1:
            return t.unsqueeze(0)
        if out is None:
            out = torch.empty((self.world, *t.shape), dtype=t.dtype, device=t.device)
        if self.backend == "gloo":
            self.dist.all_gather(list(out.unbind(0)), t.contiguous(), group=self.group)
        else:
            self.dist.all_gather_into_tensor(out.view(-1), t.contiguous().view(-1), group=self.group)
        return out

    def barrier(self):
        if self.world > 1:
            self.dist.barrier(group=self.group)


class LoopbackGroup:
    """A stand-in tensor-parallel group of ``world`` ranks on ONE GPU: this
    process is rank 0 and every peer's symmetric heap is this GPU's own heap,
    so no data is exchanged and nothing ever signals on behalf of the missing
    ranks.  It exists to drive the fused kernels' bounded waits to expiry on
    a single device (failure-detection tests): a wait for another rank's flag
    runs out, the kernel records the status and returns, and the host raises.
    It is not a way to compute anything."""

    loopback = True
    backend = "loopback"

    def __init__(self, world=2):
        if world < 2:
            raise ValueError("a loopback group stands in for at least two ranks")
        self.world, self.rank, self.group = int(world), 0, None
        self.symm_gather = None

    def all_gather_stacked(self, t, out=None):
        stacked = t.unsqueeze(0).expand(self.world, *t.shape)
        if out is None:
            return stacked.clone()
        out.copy_(stacked)
        return out

    def all_reduce_(self, t, op=None):
        return t

    def barrier(self):
        pass

