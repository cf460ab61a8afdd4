"""Sequence-parallel all-gather over NVLink peer memory (``csrc/allgather.cu``).

``SymmAllGather(tp, rows, cols)`` owns a small symmetric region (two send
slots of [rows, cols] bf16 and one flag word per source) and gathers the
[rows, cols] block of every rank into a [world * rows, cols] tensor with the
library's own pull kernel -- the NCCL all-gather is not on the data path.
Epochs and slot parity live on the device, so calls can be captured in a
CUDA graph.  Creation is collective (every rank, same order).

``SymmAgGemm`` fuses the gather into the tcgen05 GEMM that consumes it
(``csrc/ag_gemm.cu``), optionally TACO-compressed (``taco=True``);
``set_ag_variant`` chooses how the rows move (pulled by the consuming GEMM,
or pushed by their owner into every peer's receive buffer).

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


native.register("tdb_ag_gemm", [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int,
                                ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_longlong,
                                ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong,
                                ctypes.c_void_p, ctypes.c_float, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                ctypes.c_int, ctypes.c_int, ctypes.c_ulonglong, ctypes.c_ulonglong, ctypes.c_void_p,
                                ctypes.c_void_p, ctypes.c_double, ctypes.c_int, ctypes.c_void_p])
native.register("tdb_ag_gemm_region_bytes", [ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int], ctypes.c_longlong)
native.register("tdb_gemm_pick_tile", [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int])
native.register("tdb_ag_set_variant", [ctypes.c_int])


def ag_variant():
    """The current ``set_ag_variant`` setting (-1 = automatic)."""
    return int(native.lib().tdb_ag_set_variant(-100))


def set_ag_variant(variant):
    """How the fused all-gather GEMM moves the gathered rows on this process:
    0 = the epilogue warps pull them before their first tile, 1 = four
    auxiliary warps pull concurrently with the pipeline, 2 = the same
    auxiliary warps with sixteen 16-byte loads in flight per thread, 3 = the
    auxiliary warps push this rank's rows into every peer's receive buffer
    and copy the received rows locally (the compressed gather keeps 2);
    -1 = automatic (the default): 2 from four ranks up, else 0 -- the faster
    one measured on 8 and on 2 B200s.  Results are bitwise the same; all
    ranks must use the same variant.  Returns the previous one."""
    if variant not in (-1, 0, 1, 2, 3):
        raise ValueError("variant must be -1 (automatic), 0, 1, 2 or 3")
    return int(native.lib().tdb_ag_set_variant(int(variant)))


def ag_tile_table(world, rank, rows, n, bn):
    """Tile order of the fused all-gather GEMM: this rank's rows first, then
    rank+1, rank+2, ...; all N tiles of a row block consecutively.  ``bn`` is
    the GEMM tile code (128/192/256: 128-row tiles of that width; 512: 2-CTA
    256 x 256 tiles).  Values are ``m_tile * n_tiles + n_tile``."""
    tm, tn = (256, 256) if bn == 512 else (128, bn)
    if rows % tm:
        raise ValueError("rows per rank must be a multiple of the tile height")
    n_tiles = -(-n // tn)
    per = rows // tm
    table = []
    for k in range(world):
        s = (rank + k) % world
        for mb in range(s * per, (s + 1) * per):
            table.extend(mb * n_tiles + nb for nb in range(n_tiles))
    return table


class SymmAgGemm:
    """All-gather fused into the tcgen05 GEMM (``csrc/ag_gemm.cu``):
    ``out, full = agg(x_local, weight, ...)`` computes
    ``out = epilogue(AG(x_local) @ weight^T)`` (weight [N, K], or [K, N] with
    ``b_mn``) and returns the gathered rows ``full`` [world * rows, K] too.
    Every call of an instance gathers the same [rows, K] block shape; creation
    is collective.  ``wait_seconds`` bounds the wait for each peer's rows (on
    expiry the kernel records a peer-flag timeout and returns).

    ``taco=True`` compresses the gather: each rank stages its rows as TACO
    H128/E4M3 packets (136 bytes per 128 values, 0.53 of BF16 on the link)
    and the pulling CTAs decode peers' packets into the gathered buffer; a
    rank's own rows stay exact.  All ranks must agree on ``taco``."""

    STORE, BIAS, BIAS_GELU, GELU_BWD = 0, 1, 2, 3

    def __init__(self, tp, rows, cols, taco=False, wait_seconds=PEER_WAIT_SECONDS):
        import torch
        from .symmetric import SymmetricHeap
        if not 0 < wait_seconds <= 600:
            raise ValueError("wait_seconds must be in (0, 600]")
        self.wait_seconds = float(wait_seconds)
        if rows % 256 or cols % 64 or (taco and cols % 128):
            raise ValueError("the fused all-gather GEMM needs rows % 256 == 0 and K % 64 == 0 (K % 128 compressed)")
        self.tp, self.rows, self.cols = tp, int(rows), int(cols)
        self.taco = bool(taco)
        self.region_bytes = int(native.lib().tdb_ag_gemm_region_bytes(self.rows, self.cols, tp.world))
        self.heap = SymmetricHeap(tp, self.region_bytes)
        dev = self.heap.device
        self.state = torch.zeros(2, dtype=torch.int32, device=dev)
        self.ready = torch.zeros(tp.world * self.rows // 128, dtype=torch.int32, device=dev)
        self.sms = int(native.lib().tdb_sm_count(torch.cuda.current_device()))
        self.tables = {}
        self.calls = 0

    def _table(self, n, bn):
        import torch
        key = (n, bn)
        if key not in self.tables:
            self.tables[key] = torch.tensor(ag_tile_table(self.tp.world, self.tp.rank, self.rows, n, bn),
                                            dtype=torch.int32, device=self.heap.device)
        return self.tables[key]

    def __call__(self, x, weight, *, b_mn=False, mode=0, bias=None, aux=None, aux_out=None, alpha=1.0, out=None,
                 full=None):
        import torch
        if (tuple(x.shape) != (self.rows, self.cols) or x.dtype != torch.bfloat16 or x.stride(1) != 1
                or x.stride(0) % 8):
            raise ValueError(f"expected bf16 [{self.rows}, {self.cols}] rows")
        M, K = self.tp.world * self.rows, self.cols
        N = weight.shape[1] if b_mn else weight.shape[0]
        if (weight.shape[0] if b_mn else weight.shape[1]) != K:
            raise ValueError("weight inner dimension does not match the gathered rows")
        bn = int(native.lib().tdb_gemm_pick_tile(M, N, K, self.sms))
        if out is None:
            out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
        if full is None:
            full = torch.empty((M, K), dtype=torch.bfloat16, device=x.device)
        if mode == self.BIAS_GELU and aux_out is None:
            aux_out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
        aux_t = aux_out if mode == self.BIAS_GELU else aux
        native.check(native.lib().tdb_ag_gemm(
            x.data_ptr(), x.stride(0), full.data_ptr(), self.rows, K, weight.data_ptr(), int(bool(b_mn)),
            weight.stride(0), out.data_ptr(), out.stride(0), N, int(mode), 0 if bias is None else bias.data_ptr(),
            0 if aux is None else aux.data_ptr(), 0 if aux_t is None else aux_t.stride(0),
            0 if aux_out is None else aux_out.data_ptr(), float(alpha), bn, self._table(N, bn).data_ptr(),
            self.heap.peers.data_ptr(), self.tp.world, self.tp.rank, 0, self.region_bytes, self.state.data_ptr(),
            self.ready.data_ptr(), self.wait_seconds, int(self.taco), native.stream_ptr()), "fused all-gather GEMM")
        self.calls += 1
        if mode == self.BIAS_GELU:
            return out, full, aux_out
        return out, full

    def close(self):
        self.heap.close()
