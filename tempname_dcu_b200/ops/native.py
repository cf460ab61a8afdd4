"""ctypes binding of ``libtdb.so`` (the native sm_100a library).

Every kernel of the framework is reached through a plain ``extern "C"`` entry
point that takes raw device pointers plus a ``cudaStream_t`` and returns a CUDA
error code (0 on success); the text of the last host-side validation error is
available from ``tdb_last_error``.  There is no fallback: if the library
cannot be built or loaded the call raises.

Reference parity: ``python/flux_dcu/codec.py:112-226`` (ctypes signatures,
tensor contract checks, error text from the library).
"""
from __future__ import annotations

import ctypes
import threading

from . import _build

ABI_VERSION = 5

c_void_p, c_int, c_int64, c_float, c_uint64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_uint64

# name -> argtypes (all return c_int status unless listed in _RESTYPE)
SIGNATURES = {
    "tdb_abi_version": [],
    "tdb_launch_count": [],
    "tdb_last_error": [],
    "tdb_error_string": [c_int],
    "tdb_read_status": [c_void_p],
    "tdb_clear_status": [],
    "tdb_sm_count": [c_int],
    "tdb_set_grid_limit": [c_int],
    "tdb_diagnostic_delay": [ctypes.c_ulonglong, c_void_p],
    "tdb_taco_encode": [c_void_p, c_void_p, c_int64, c_void_p],
    "tdb_taco_decode": [c_void_p, c_void_p, c_int64, c_void_p],
    "tdb_taco_reduce": [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_void_p],
    "tdb_taco_block_stats": [c_void_p, c_int64, c_int, c_void_p, c_void_p],
    "tdb_e4m3_probe": [c_void_p, c_void_p, c_void_p, c_int64, c_void_p],
}
_RESTYPE = {"tdb_last_error": ctypes.c_char_p, "tdb_error_string": ctypes.c_char_p,
            "tdb_launch_count": ctypes.c_longlong}

_LOCK = threading.Lock()
_LIB = None
LOADED_PATH = None


def register(name: str, argtypes: list, restype=c_int) -> None:
    """Declare an additional entry point (used by op modules at import)."""
    SIGNATURES[name] = argtypes
    if restype is not c_int:
        _RESTYPE[name] = restype
    if _LIB is not None:
        _bind(_LIB, name)


def _bind(lib, name):
    fn = getattr(lib, name)
    fn.argtypes = SIGNATURES[name]
    fn.restype = _RESTYPE.get(name, c_int)


def lib():
    """Build (if needed) and load the native library exactly once."""
    global _LIB, LOADED_PATH
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            path = _build.build()
            handle = ctypes.CDLL(str(path), mode=ctypes.RTLD_GLOBAL)
            for name in SIGNATURES:
                _bind(handle, name)
            if handle.tdb_abi_version() != ABI_VERSION:
                raise RuntimeError("libtdb.so ABI mismatch; rebuild the native library")
            _LIB, LOADED_PATH = handle, path
    return _LIB


class NativeError(RuntimeError):
    pass


def check(status: int, what: str = "") -> None:
    if status:
        handle = lib()
        detail = handle.tdb_last_error()
        detail = detail.decode(errors="replace") if detail else ""
        cuda = handle.tdb_error_string(status)
        cuda = cuda.decode(errors="replace") if cuda else "unknown"
        raise NativeError(f"{what or 'native call'} failed ({status}: {cuda}){': ' + detail if detail else ''}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def stream_ptr(stream=None) -> int:
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return int(stream.cuda_stream)


def read_status() -> list[int]:
    """Synchronously read the device status word [code, where, d0, d1]."""
    buf = (ctypes.c_int * 4)()
    check(lib().tdb_read_status(ctypes.addressof(buf)), "tdb_read_status")
    return list(buf)


def clear_status() -> None:
    check(lib().tdb_clear_status(), "tdb_clear_status")


STATUS_NAMES = {0: "ok", 1: "pipeline wait timeout", 2: "peer flag timeout", 3: "local flag timeout",
                4: "bad argument"}


def raise_on_status() -> None:
    """Raise if any kernel recorded a bounded-wait expiry or argument error."""
    code, where, d0, d1 = read_status()
    if code:
        clear_status()
        raise NativeError(f"device status {code} ({STATUS_NAMES.get(code, 'unknown')}) at site {where} "
                          f"detail=({d0},{d1})")


def launch_count() -> int:
    """Kernels launched through libtdb.so in this process so far."""
    return int(lib().tdb_launch_count())


class grid_limit:
    """``with grid_limit(n):`` -- the persistent GEMM-shaped kernels (plain
    GEMMs, fused collectives) launched inside, from this thread, use at most
    ``n`` CTAs (0: no cap), so that two of them on different streams share the
    SMs instead of queueing.  Launch geometry is fixed when a CUDA graph is
    captured, so the cap also holds on replay."""

    def __init__(self, ctas):
        self.ctas = int(ctas)
        self.previous = 0

    def __enter__(self):
        self.previous = int(lib().tdb_set_grid_limit(self.ctas))
        return self

    def __exit__(self, *exc):
        lib().tdb_set_grid_limit(self.previous)
        return False
