"""Sequence-parallel all-gather over NVLink peer memory (``csrc/allgather.cu``).

``SymmAllGather(tp, rows, cols)`` owns a small symmetric region (two send
slots of [rows, cols] bf16 and one flag word per source) and gathers the
[rows, cols] block of every rank into a [world * rows, cols] tensor with the
library's own pull kernel -- the NCCL all-gather is not on the data path.
Epochs and slot parity live on the device, so calls can be captured in a
CUDA graph.  Creation is collective (every rank, same order).

Reference parity: python/flux_dcu/model.py:75-81 (gather_rows).
"""
from __future__ import annotations

import ctypes

from ..ops import native

native.register("tdb_ag_region_bytes", [ctypes.c_longlong, ctypes.c_longlong], ctypes.c_longlong)
native.register("tdb_allgather", [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_longlong, ctypes.c_longlong,
                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_ulonglong,
                                  ctypes.c_void_p, ctypes.c_double, ctypes.c_void_p])

PEER_WAIT_SECONDS = 20.0


class SymmAllGather:
    def __init__(self, tp, rows, cols):
        import torch
        from .symmetric import SymmetricHeap
        if cols % 8:
            raise ValueError("columns must be a multiple of 8")
        self.tp, self.rows, self.cols = tp, int(rows), int(cols)
        self.heap = SymmetricHeap(tp, int(native.lib().tdb_ag_region_bytes(self.rows, self.cols)))
        self.state = torch.zeros(2, dtype=torch.int32, device=self.heap.device)
        self.calls = 0

    def matches(self, x):
        import torch
        return (x.dim() == 2 and tuple(x.shape) == (self.rows, self.cols) and x.dtype == torch.bfloat16
                and x.is_cuda and x.stride(1) == 1 and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0)

    def __call__(self, x, out=None):
        import torch
        if not self.matches(x):
            raise ValueError(f"expected a 16-byte aligned bf16 [{self.rows}, {self.cols}] block")
        if out is None:
            out = torch.empty((self.tp.world * self.rows, self.cols), dtype=torch.bfloat16, device=x.device)
        native.check(native.lib().tdb_allgather(x.data_ptr(), x.stride(0), self.rows, self.cols, out.data_ptr(),
                                                self.heap.peers.data_ptr(), self.tp.world, self.tp.rank, 0,
                                                self.state.data_ptr(), PEER_WAIT_SECONDS, native.stream_ptr()),
                     "symmetric all-gather")
        self.calls += 1
        return out

    def close(self):
        self.heap.close()
