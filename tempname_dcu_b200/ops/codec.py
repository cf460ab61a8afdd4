"""TACO codec on the GPU: encode / decode / ordered reduce / diagnostic delay.

Reference parity: ``python/flux_dcu/codec.py`` (``NativeCodec.encode``,
``decode``, ``reduce``, ``delay`` and ``packet_bytes``) with the same tensor
contracts: contiguous BF16 inputs, a uint8 SoA packet of exactly
``elements/128*136`` bytes aligned to 4 bytes, no overlapping buffers.  The
kernels are ``csrc/codec.cu``.
"""
from __future__ import annotations

from . import native

GROUP_SIZE = 128
GROUP_BYTES = 136


def packet_bytes(elements: int) -> int:
    if type(elements) is not int or elements <= 0 or elements % GROUP_SIZE:
        raise ValueError("TACO packets need a positive multiple of 128 elements")
    return elements // GROUP_SIZE * GROUP_BYTES


def _torch():
    import torch
    return torch


def _check(tensor, dtype, name):
    torch = _torch()
    if not isinstance(tensor, torch.Tensor) or tensor.dtype != dtype:
        raise TypeError(f"{name} must be a {dtype} tensor")
    if tensor.device.type != "cuda" or not tensor.is_contiguous() or tensor.numel() <= 0:
        raise ValueError(f"{name} must be a non-empty contiguous CUDA tensor")
    if tensor.device.index != torch.cuda.current_device():
        raise ValueError(f"{name} must live on the current CUDA device")


def _disjoint(a, b):
    a0, b0 = a.data_ptr(), b.data_ptr()
    a1, b1 = a0 + a.numel() * a.element_size(), b0 + b.numel() * b.element_size()
    if max(a0, b0) < min(a1, b1):
        raise ValueError("codec buffers must not overlap")


class Codec:
    """GPU TACO codec bound to the native library (one instance per process)."""

    def __init__(self):
        self.lib = native.lib()
        self.library_path = str(native.LOADED_PATH)
        from . import _build
        self.manifest = _build.manifest()

    def encode(self, source, packet, stream=None):
        torch = _torch()
        _check(source, torch.bfloat16, "input")
        _check(packet, torch.uint8, "packet")
        if packet.numel() != packet_bytes(source.numel()):
            raise ValueError("packet must hold exactly input.numel()/128*136 bytes")
        if packet.data_ptr() % 4:
            raise ValueError("packet storage must be 4-byte aligned")
        _disjoint(source, packet)
        native.check(self.lib.tdb_taco_encode(source.data_ptr(), packet.data_ptr(), source.numel(),
                                              native.stream_ptr(stream)), "taco encode")
        return packet

    def decode(self, packet, output, stream=None):
        torch = _torch()
        _check(packet, torch.uint8, "packet")
        _check(output, torch.bfloat16, "output")
        if packet.numel() != packet_bytes(output.numel()):
            raise ValueError("packet must hold exactly output.numel()/128*136 bytes")
        if packet.data_ptr() % 4:
            raise ValueError("packet storage must be 4-byte aligned")
        _disjoint(packet, output)
        native.check(self.lib.tdb_taco_decode(packet.data_ptr(), output.data_ptr(), output.numel(),
                                              native.stream_ptr(stream)), "taco decode")
        return output

    def reduce(self, local, remote, output, rank: int, world: int, stream=None):
        torch = _torch()
        for tensor, name in ((local, "local"), (remote, "remote"), (output, "output")):
            _check(tensor, torch.bfloat16, name)
        if type(rank) is not int or type(world) is not int or not 2 <= world <= 128 or not 0 <= rank < world:
            raise ValueError("need 2 <= world <= 128 and 0 <= rank < world")
        if local.ndim != 2 or output.shape != local.shape or tuple(remote.shape) != (world - 1, *local.shape):
            raise ValueError("expected local/output [rows, n] and remote [world-1, rows, n]")
        _disjoint(local, output)
        _disjoint(remote, output)
        native.check(self.lib.tdb_taco_reduce(local.data_ptr(), remote.data_ptr(), output.data_ptr(),
                                              local.numel(), rank, world, native.stream_ptr(stream)),
                     "ordered reduce")
        return output

    def delay(self, cycles: int, stream=None):
        """Bounded single-thread device delay (profiling diagnostic only)."""
        if type(cycles) is not int or not 0 < cycles <= 100_000_000:
            raise ValueError("diagnostic delay needs 0 < cycles <= 100000000")
        native.check(self.lib.tdb_diagnostic_delay(cycles, native.stream_ptr(stream)), "diagnostic delay")

    def block_stats(self, source, block_rows: int, stream=None):
        """Per block of ``block_rows`` rows of a [rows, n] bf16 tensor: fp64
        [blocks, 3] = (sum x^2, max |x|, sum (roundtrip(x) - x)^2), where
        roundtrip is encode -> decode -> bf16.  Used for the selective arm's
        error budget; deterministic."""
        torch = _torch()
        _check(source, torch.bfloat16, "input")
        if source.ndim != 2 or type(block_rows) is not int or block_rows <= 0 or source.shape[0] % block_rows:
            raise ValueError("expected [rows, n] with rows a multiple of block_rows")
        blocks = source.shape[0] // block_rows
        out = torch.empty((blocks, 3), dtype=torch.float64, device=source.device)
        native.check(self.lib.tdb_taco_block_stats(source.data_ptr(), block_rows * source.shape[1], blocks,
                                                   out.data_ptr(), native.stream_ptr(stream)), "codec block stats")
        return out

    def e4m3_probe(self, values):
        """Hardware E4M3 conversion of fp32 values (test hook): (codes, decode(index))."""
        torch = _torch()
        values = values.contiguous().float()
        codes = torch.empty(values.numel(), dtype=torch.uint8, device=values.device)
        decoded = torch.empty(values.numel(), dtype=torch.float32, device=values.device)
        native.check(self.lib.tdb_e4m3_probe(values.data_ptr(), codes.data_ptr(), decoded.data_ptr(),
                                             values.numel(), native.stream_ptr()), "e4m3 probe")
        return codes, decoded


_CODEC = None


def codec() -> Codec:
    global _CODEC
    if _CODEC is None:
        _CODEC = Codec()
    return _CODEC
