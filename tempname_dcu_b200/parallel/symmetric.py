"""Symmetric device heap over a tensor-parallel group (CUDA IPC).

``SymmetricHeap(tp, nbytes)`` allocates ``nbytes`` on every rank, exchanges the
IPC handles over the process group and maps all peers.  ``peers`` is a device
int64 tensor of the W base addresses (rank order), which the fused kernels
take as their peer table; ``view(offset, shape, dtype)`` aliases a region of
the local heap as a torch tensor (for validation and tests).

Creation and ``close()`` are collective: every rank of the group must call
them in the same order.

A 256-byte canary of 0xA5 bytes follows the usable ``nbytes`` of every heap;
``canaries_intact()`` checks it (an overrun by any writer -- local or peer --
shows up there).
"""
from __future__ import annotations

import ctypes

from ..ops import native

native.register("tdb_symm_handle_bytes", [])
native.register("tdb_symm_alloc", [ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p])
native.register("tdb_symm_open", [ctypes.c_void_p, ctypes.c_void_p])
native.register("tdb_symm_close", [ctypes.c_void_p])
native.register("tdb_symm_free", [ctypes.c_void_p])
native.register("tdb_memset_async", [ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p])
native.register("tdb_memcpy_async", [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p])
native.register("tdb_can_access_peer", [ctypes.c_int, ctypes.c_int])

_DTYPE_STR = {"torch.uint8": "|u1", "torch.bfloat16": "<V2", "torch.float32": "<f4", "torch.int32": "<i4",
              "torch.int64": "<i8"}


class _CudaArray:
    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = dict(shape=tuple(shape), typestr=typestr, data=(ptr, False), version=3,
                                             strides=None)


def alias(ptr, shape, dtype, device):
    """A torch tensor aliasing device memory at ``ptr`` (no copy)."""
    import torch
    if dtype == torch.bfloat16:
        raw = torch.as_tensor(_CudaArray(ptr, tuple(shape), "<i2"), device=device)
        return raw.view(torch.bfloat16)
    return torch.as_tensor(_CudaArray(ptr, tuple(shape), _DTYPE_STR[str(dtype)]), device=device)


CANARY_BYTES = 256
CANARY_VALUE = 0xA5


class SymmetricHeap:
    def __init__(self, tp, nbytes):
        import torch
        self.tp = tp
        self.nbytes = int(nbytes)
        self.device = torch.device("cuda", torch.cuda.current_device())
        lib = native.lib()
        hbytes = int(lib.tdb_symm_handle_bytes())
        handle = (ctypes.c_uint8 * hbytes)()
        base = ctypes.c_void_p()
        native.check(lib.tdb_symm_alloc(self.nbytes + CANARY_BYTES, ctypes.byref(base), ctypes.addressof(handle)),
                     "symm alloc")
        self.base = int(base.value)
        native.check(lib.tdb_memset_async(self.base + self.nbytes, CANARY_VALUE, CANARY_BYTES, native.stream_ptr()),
                     "symm canary")
        self.opened = []
        if getattr(tp, "loopback", False):  # every peer is this GPU's own heap (one-GPU wait tests)
            addrs = [self.base] * tp.world
        else:
            addrs = self._map_peers(tp, handle, hbytes)
        self.addrs = addrs
        self.peers = torch.tensor(addrs, dtype=torch.int64, device=self.device)
        torch.cuda.synchronize()
        tp.barrier()
        self.closed = False

    def _map_peers(self, tp, handle, hbytes):
        """Exchange IPC handles over the group and open every peer's heap."""
        import torch
        lib = native.lib()
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
        everyone = tp.all_gather_stacked(mine).cpu()
        addrs = []
        for r in range(tp.world):
            if r == tp.rank:
                addrs.append(self.base)
                continue
            buf = (ctypes.c_uint8 * hbytes)(*everyone[r].tolist())
            ptr = ctypes.c_void_p()
            native.check(lib.tdb_symm_open(ctypes.addressof(buf), ctypes.byref(ptr)), f"symm open rank {r}")
            addrs.append(int(ptr.value))
            self.opened.append(int(ptr.value))
        return addrs

    def canaries_intact(self):
        """True when the guard bytes after this rank's heap still hold the canary."""
        import torch
        guard = alias(self.base + self.nbytes, (CANARY_BYTES,), torch.uint8, self.device)
        return bool((guard == CANARY_VALUE).all().item())

    def view(self, offset, shape, dtype):
        return alias(self.base + int(offset), shape, dtype, self.device)

    def zero_(self, offset=0, nbytes=None, stream=None):
        nbytes = self.nbytes - offset if nbytes is None else nbytes
        native.check(native.lib().tdb_memset_async(self.base + offset, 0, nbytes, native.stream_ptr(stream)),
                     "symm memset")

    def close(self):
        """Collective: unmap peers and free the local heap."""
        import torch
        if self.closed:
            return
        torch.cuda.synchronize()
        self.tp.barrier()
        lib = native.lib()
        for ptr in self.opened:
            lib.tdb_symm_close(ptr)
        lib.tdb_symm_free(self.base)
        self.closed = True
