"""Sparse vocabulary-parallel embedding exchange over NVLink (``csrc/embed_exchange.cu``).

``EmbeddingExchange(tp, ml, H, local_vocab)`` replaces the dense collectives
around the vocabulary-sharded embedding of a tensor/sequence-parallel GPT:

* ``forward(tokens, table, vocab_start, positions, pos_offset, seq, out)``
  writes this rank's sequence-parallel rows ``x`` [ml, H] = embedding rows +
  learned positions.  The owner of each token's vocabulary shard writes the
  row straight into the receiving rank's double-buffered slot, so about
  ``m * H * 2 / W`` bytes leave a rank instead of the dense reduce-scatter's
  ``(W-1)/W`` of ``m * H * 2``; the result is bit for bit the
  reduce-scatter's (one nonzero source per row).
* ``backward(tokens, dy, vocab_start, out)`` sends each of this rank's row
  gradients ``dy`` [ml, H] only to the owner of its token and fills, in
  ``out`` [W * ml, H], every row whose token this rank owns -- exactly the
  rows the table backward reads -- so ``embedding_bwd`` runs on it unchanged.

Slot parities are chosen on the device, so calls can be captured in a CUDA
graph.

Creation is collective.  Reference parity: python/flux_dcu/model.py:236-249
(masked lookup, SumScatter) and its backward.
"""
from __future__ import annotations

import ctypes

from ..ops import native

native.register("tdb_embx_region_bytes", [ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int], ctypes.c_longlong)
native.register("tdb_embx_forward", [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_longlong,
                                     ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                     ctypes.c_int, ctypes.c_int, ctypes.c_longlong, ctypes.c_longlong,
                                     ctypes.c_ulonglong, ctypes.c_void_p, ctypes.c_double, ctypes.c_void_p])
native.register("tdb_embx_backward", [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_longlong,
                                      ctypes.c_longlong, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_longlong, ctypes.c_longlong, ctypes.c_ulonglong, ctypes.c_void_p,
                                      ctypes.c_double, ctypes.c_void_p])

PEER_WAIT_SECONDS = 20.0
_HEADER = 256
# Whether models built from now on use the exchange (True, the default) or
# the dense reduce-scatter / all-gather; a process-wide switch for A/B runs.
_ENABLED = True


def set_embedding_exchange(on):
    """Enable or disable the sparse exchange for models created afterwards;
    returns the previous setting.  Both forms give bitwise the same rows."""
    global _ENABLED
    old, _ENABLED = _ENABLED, bool(on)
    return old


def enabled():
    return _ENABLED


class EmbeddingExchange:
    def __init__(self, tp, ml, H, local_vocab, wait_seconds=PEER_WAIT_SECONDS):
        import torch
        from .symmetric import SymmetricHeap
        if tp.world < 2 or tp.world > 8 or H % 8:
            raise ValueError("the embedding exchange needs 2..8 ranks and H % 8 == 0")
        self.tp, self.ml, self.H, self.local_vocab = tp, int(ml), int(H), int(local_vocab)
        self.wait_seconds = float(wait_seconds)
        self.heap = SymmetricHeap(tp, int(native.lib().tdb_embx_region_bytes(self.ml, self.H, tp.world)))
        dev = self.heap.device
        self.fwd_state = torch.zeros(2, dtype=torch.int32, device=dev)
        self.bwd_state = torch.zeros(2, dtype=torch.int32, device=dev)

    def forward(self, tokens, table, vocab_start, positions, pos_offset, seq, out=None):
        import torch
        tp = self.tp
        if tokens.numel() != tp.world * self.ml or table.shape[1] != self.H or positions.shape[1] != self.H:
            raise ValueError("tokens must cover all W * ml rows; table and positions [*, H]")
        if out is None:
            out = torch.empty((self.ml, self.H), dtype=torch.bfloat16, device=table.device)
        native.check(native.lib().tdb_embx_forward(
            tokens.data_ptr(), table.data_ptr(), int(vocab_start), table.shape[0], positions.data_ptr(),
            int(pos_offset), int(seq), out.data_ptr(), self.heap.peers.data_ptr(), tp.world, tp.rank, self.ml,
            self.H, 0, self.fwd_state.data_ptr(), self.wait_seconds, native.stream_ptr()),
            "embedding exchange forward")
        return out

    def backward(self, tokens, dy, vocab_start, out):
        """Fill, in ``out`` [W * ml, H], the gradient rows of the tokens in
        this rank's vocabulary shard (starting at ``vocab_start``)."""
        tp = self.tp
        if tokens.numel() != tp.world * self.ml or tuple(dy.shape) != (self.ml, self.H) or dy.stride(1) != 1:
            raise ValueError("dy must be this rank's [ml, H] rows")
        if tuple(out.shape) != (tp.world * self.ml, self.H) or not out.is_contiguous():
            raise ValueError("out must be a contiguous [W * ml, H] buffer")
        native.check(native.lib().tdb_embx_backward(
            tokens.data_ptr(), dy.data_ptr(), dy.stride(0), int(vocab_start), self.local_vocab, out.data_ptr(),
            self.heap.peers.data_ptr(), tp.world, tp.rank, self.ml, self.H, 0, self.bwd_state.data_ptr(),
            self.wait_seconds, native.stream_ptr()), "embedding exchange backward")
        return out

    def close(self):
        self.heap.close()
