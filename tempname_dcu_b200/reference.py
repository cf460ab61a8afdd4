"""Standard-library FP64 oracle for the TACO H128/E4M3FN codec and the ordered
BF16 source reduction.

This module imports neither torch nor the native library, so it can check the
device kernels independently: the transform is an explicit dense Walsh matrix
product in FP64 (not a butterfly), E4M3FN encoding searches the finite code
table with round-half-to-even on the code's low bit, and BF16 rounding is done
on the FP32 bit pattern.

Reference parity: ``python/flux_dcu/reference.py`` (the same oracle contract:
``fp32``, ``bf16_bits``/``bf16_round``, ``e4m3_decode``/``e4m3_encode``,
``hadamard_fp64``, ``encode_group``/``decode_group``, ``encode``/``decode``,
``reduce_sources``, ``relative_l2``).  The wire format and the group math are
a protocol and are reproduced exactly; the implementation is independent.
"""
from __future__ import annotations

import bisect
import math
import struct

GROUP_SIZE = 128
GROUP_BYTES = 136
E4M3_MAX = 448.0
QUANT_RANGE = (1e-12, 1e6)
ADAPTIVE_RANGE = (1e-3, 1e3)

_F32 = struct.Struct("<f")
_U32 = struct.Struct("<I")


def fp32(value: float) -> float:
    """Round a Python float to the nearest FP32 value (overflow -> +-inf)."""
    try:
        return _F32.unpack(_F32.pack(float(value)))[0]
    except OverflowError:
        return math.copysign(math.inf, value)


def _bits(value: float) -> int:
    return _U32.unpack(_F32.pack(fp32(value)))[0]


def bf16_bits(value: float) -> int:
    """FP32 -> BF16 bit pattern, round half to even; NaN becomes a quiet NaN."""
    bits = _bits(value)
    if bits & 0x7FFFFFFF > 0x7F800000:
        return ((bits >> 16) | 0x40) & 0xFFFF
    lsb = (bits >> 16) & 1
    return ((bits + 0x7FFF + lsb) >> 16) & 0xFFFF


def bf16_round(value: float) -> float:
    return _F32.unpack(_U32.pack(bf16_bits(value) << 16))[0]


def e4m3_decode(code: int) -> float:
    """Exact value of an E4M3FN byte (bias 7, 0x7f/0xff are NaN)."""
    if type(code) is not int or not 0 <= code < 256:
        raise ValueError("E4M3FN codes are integers in [0, 255]")
    sign = -1.0 if code & 0x80 else 1.0
    exponent, mantissa = (code >> 3) & 0xF, code & 0x7
    if exponent == 0xF and mantissa == 0x7:
        return math.nan
    if exponent == 0:
        return sign * mantissa * 2.0 ** -9
    return sign * (1.0 + mantissa / 8.0) * 2.0 ** (exponent - 7)


# Ascending magnitudes of the 127 finite non-negative codes (code == index).
_MAGNITUDES = [e4m3_decode(code) for code in range(127)]


def e4m3_encode(value: float) -> int:
    """FP32 -> E4M3FN, round to nearest with ties to the even code, saturating
    at +-448.  Signed zero is kept; non-finite inputs are rejected."""
    value = fp32(value)
    if not math.isfinite(value):
        raise ValueError("the oracle encodes finite values only")
    sign = 0x80 if math.copysign(1.0, value) < 0 else 0
    magnitude = min(abs(value), E4M3_MAX)
    upper = bisect.bisect_left(_MAGNITUDES, magnitude)
    if upper == 0:
        return sign
    if upper >= len(_MAGNITUDES):
        return sign | 126
    lower = upper - 1
    below, above = magnitude - _MAGNITUDES[lower], _MAGNITUDES[upper] - magnitude
    if below < above:
        code = lower
    elif above < below:
        code = upper
    else:
        code = lower if lower % 2 == 0 else upper
    return sign | code


def _walsh_sign(row: int, col: int) -> float:
    return -1.0 if bin(row & col).count("1") & 1 else 1.0


_WALSH = [[_walsh_sign(r, c) for c in range(GROUP_SIZE)] for r in range(GROUP_SIZE)]


def hadamard_fp64(values) -> list[float]:
    """Orthonormal Sylvester Walsh-Hadamard transform of exactly 128 values as
    a dense FP64 matrix-vector product (self-inverse)."""
    data = [float(v) for v in values]
    if len(data) != GROUP_SIZE or not all(math.isfinite(v) for v in data):
        raise ValueError("the transform needs exactly 128 finite values")
    scale = 1.0 / math.sqrt(GROUP_SIZE)
    return [math.fsum(s * v for s, v in zip(row, data)) * scale for row in _WALSH]


def _clamp(x: float, lo: float, hi: float) -> float:
    return min(max(x, lo), hi)


def encode_group(values):
    """One 128-value group -> (payload bytes, FP32 quant scale, FP32 adaptive scale).

    Inputs are treated as BF16 storage.  The math is FP64, so bytes that sit
    exactly on an FP32 rounding boundary may legitimately differ from a device
    encoder that accumulates in FP32."""
    data = [bf16_round(v) for v in values]
    if len(data) != GROUP_SIZE or not all(math.isfinite(v) for v in data):
        raise ValueError("a group is exactly 128 finite BF16 values")
    mean_square = math.fsum(v * v for v in data) / GROUP_SIZE
    variance = max(mean_square + 1e-6, 1e-12)
    adaptive = fp32(_clamp(E4M3_MAX / math.sqrt(variance), *ADAPTIVE_RANGE))
    coefficients = hadamard_fp64([v * adaptive for v in data])
    peak = max(abs(c) for c in coefficients)
    quant = fp32(_clamp(max(peak, 1e-12) / E4M3_MAX, *QUANT_RANGE))
    payload = bytes(e4m3_encode(_clamp(c / quant, -E4M3_MAX, E4M3_MAX)) for c in coefficients)
    return payload, quant, adaptive


def _check_scales(quant: float, adaptive: float) -> None:
    ok_q = math.isfinite(quant) and fp32(QUANT_RANGE[0]) <= quant <= QUANT_RANGE[1]
    ok_a = math.isfinite(adaptive) and fp32(ADAPTIVE_RANGE[0]) <= adaptive <= ADAPTIVE_RANGE[1]
    if not (ok_q and ok_a):
        raise ValueError("corrupt TACO scales")


def decode_group(payload, quant: float, adaptive: float) -> list[float]:
    payload = bytes(payload)
    if len(payload) != GROUP_SIZE:
        raise ValueError("a group payload is exactly 128 bytes")
    quant, adaptive = float(quant), float(adaptive)
    _check_scales(quant, adaptive)
    coefficients = [e4m3_decode(code) for code in payload]
    if any(math.isnan(c) for c in coefficients):
        raise ValueError("NaN E4M3FN payload is not a valid finite TACO packet")
    restored = hadamard_fp64([c * quant for c in coefficients])
    return [bf16_round(v / adaptive) for v in restored]


def encode(values) -> bytes:
    """Encode a multiple of 128 values into the SoA packet
    ``[payload][fp32 quant scales][fp32 adaptive scales]``."""
    data = list(values)
    if not data or len(data) % GROUP_SIZE:
        raise ValueError("encode needs a positive multiple of 128 values")
    groups = [encode_group(data[i:i + GROUP_SIZE]) for i in range(0, len(data), GROUP_SIZE)]
    count = len(groups)
    return (b"".join(g[0] for g in groups)
            + struct.pack(f"<{count}f", *(g[1] for g in groups))
            + struct.pack(f"<{count}f", *(g[2] for g in groups)))


def decode(packet) -> list[float]:
    raw = bytes(packet)
    if not raw or len(raw) % GROUP_BYTES:
        raise ValueError("a packet holds exactly 136 bytes per group")
    count = len(raw) // GROUP_BYTES
    elements = count * GROUP_SIZE
    quants = struct.unpack_from(f"<{count}f", raw, elements)
    adaptives = struct.unpack_from(f"<{count}f", raw, elements + 4 * count)
    out: list[float] = []
    for g in range(count):
        out.extend(decode_group(raw[g * GROUP_SIZE:(g + 1) * GROUP_SIZE], quants[g], adaptives[g]))
    return out


def reduce_sources(local, remote, rank: int, world: int) -> list[float]:
    """Sum world sources in rank order 0..world-1 with BF16 rounding after each
    addition; ``remote`` lists the world-1 other sources in ascending rank
    order and ``local`` is placed at position ``rank``."""
    if type(rank) is not int or type(world) is not int or not 2 <= world <= 128 or not 0 <= rank < world:
        raise ValueError("invalid rank/world")
    mine = [bf16_round(v) for v in local]
    others = [[bf16_round(v) for v in row] for row in remote]
    if not mine or len(others) != world - 1 or any(len(row) != len(mine) for row in others):
        raise ValueError("need world-1 remote sources shaped like the local one")
    if not all(math.isfinite(v) for row in [mine, *others] for v in row):
        raise ValueError("the reduction oracle needs finite inputs")
    ordered = others[:rank] + [mine] + others[rank:]
    total = [0.0] * len(mine)
    for source in ordered:
        total = [bf16_round(fp32(a + b)) for a, b in zip(total, source)]
    return total


def relative_l2(actual, expected) -> float:
    a, e = list(actual), list(expected)
    if not a or len(a) != len(e):
        raise ValueError("relative_l2 needs equal non-empty vectors")
    if not all(math.isfinite(float(v)) for v in a + e):
        return math.inf
    num = math.fsum((x - y) ** 2 for x, y in zip(a, e))
    den = math.fsum(y * y for y in e)
    if den == 0:
        return 0.0 if num == 0 else math.inf
    return math.sqrt(num / den)
