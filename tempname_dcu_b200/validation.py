"""Untimed wire-format and buffer gates for the fused operators.

``validate_packet_bytes`` is a stdlib check of one SoA TACO packet;
``packet_tensor_valid`` computes the same predicate on a device tensor and
returns a 0-d bool without copying the packet to the host; and
``validate_operator_buffers`` checks every buffer an operator call touched and
combines the verdict across ranks with one MIN all-reduce so that all ranks
raise (or pass) together.

Reference parity: ``python/flux_dcu/validation.py:14-109``.  Gates: no NaN
E4M3 payload byte (``code & 0x7f == 0x7f``), quant scales finite in
``[fp32(1e-12), 1e6]``, adaptive scales finite in ``[fp32(1e-3), 1e3]``.
"""
from __future__ import annotations

import math
import struct

_F32 = struct.Struct("<f")


def _fp32(value: float) -> float:
    return _F32.unpack(_F32.pack(value))[0]


QUANT_MIN, QUANT_MAX = _fp32(1e-12), _fp32(1e6)
ADAPT_MIN, ADAPT_MAX = _fp32(1e-3), _fp32(1e3)


def _groups(elements) -> int:
    if type(elements) is not int or elements <= 0 or elements % 128:
        raise ValueError("packet element count must be a positive multiple of 128")
    return elements // 128


def validate_packet_bytes(packet, elements):
    """Raise ValueError unless ``packet`` is a well-formed finite TACO packet."""
    raw = bytes(packet)
    groups = _groups(elements)
    if len(raw) != groups * 136:
        raise ValueError("wrong TACO packet size")
    if any((byte & 0x7F) == 0x7F for byte in raw[:elements]):
        raise ValueError("non-finite E4M3FN payload byte")
    quant = struct.unpack_from(f"<{groups}f", raw, elements)
    adapt = struct.unpack_from(f"<{groups}f", raw, elements + 4 * groups)
    if not all(math.isfinite(q) and QUANT_MIN <= q <= QUANT_MAX for q in quant):
        raise ValueError("invalid quantization scales")
    if not all(math.isfinite(a) and ADAPT_MIN <= a <= ADAPT_MAX for a in adapt):
        raise ValueError("invalid adaptive scales")
    return dict(passed=True, elements=elements, groups=groups, bytes=len(raw))


def packet_tensor_valid(packet, elements):
    """0-d bool tensor: the packet tensor passes the wire gates.

    Structural problems (dtype, size, alignment) raise ValueError; numeric
    problems return False so that ranks can combine verdicts collectively."""
    import torch
    groups = _groups(elements)
    if (not isinstance(packet, torch.Tensor) or packet.dtype != torch.uint8 or not packet.is_contiguous()
            or packet.numel() != groups * 136 or packet.data_ptr() % 4):
        raise ValueError("expected an aligned contiguous uint8 TACO packet of the exact size")
    flat = packet.view(-1)
    payload_ok = torch.bitwise_and(flat[:elements], 0x7F).ne(0x7F).all()
    quant = flat[elements:elements + 4 * groups].view(torch.float32)
    adapt = flat[elements + 4 * groups:].view(torch.float32)
    quant_ok = (torch.isfinite(quant) & (quant >= QUANT_MIN) & (quant <= QUANT_MAX)).all()
    adapt_ok = (torch.isfinite(adapt) & (adapt >= ADAPT_MIN) & (adapt <= ADAPT_MAX)).all()
    return payload_ok & quant_ok & adapt_ok


def validate_operator_buffers(op, input_, weight, output):
    """Synchronise, check every finite BF16 buffer and every packet the
    operator owns, then agree across ranks (MIN all-reduce).  Must be called
    by all ranks of ``op.group`` at the same call boundary, outside timing."""
    import torch
    import torch.distributed as dist
    torch.cuda.synchronize()
    device = output.device
    good = torch.ones((), dtype=torch.bool, device=device)
    details = []
    finite_checked = packets_checked = 0
    verdicts = []
    try:
        for name, tensor in [("input", input_), ("weight", weight), ("output", output),
                             *op.validation_tensors()]:
            if not isinstance(tensor, torch.Tensor) or tensor.dtype != torch.bfloat16 or not tensor.is_cuda:
                raise ValueError(f"invalid BF16 tensor in validation: {name}")
            ok = torch.isfinite(tensor).all()
            verdicts.append((name, ok))
            good = good & ok
            finite_checked += 1
        for name, packet, elements in op.validation_packets():
            ok = packet_tensor_valid(packet, elements)
            verdicts.append((name, ok))
            good = good & ok
            packets_checked += 1
    except (ValueError, TypeError, KeyError, IndexError) as exc:
        good = torch.zeros((), dtype=torch.bool, device=device)
        details.append(str(exc))
    flag = good.to(torch.int32)
    if dist.is_initialized() and op.world > 1:
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=op.group)
    if int(flag.item()) != 1:
        bad = [name for name, ok in verdicts if not bool(ok.item())]
        if bad:
            details.append("failing here: " + ", ".join(bad[:8]))
            import sys
            print(f"[validation rank {dist.get_rank() if dist.is_initialized() else 0}] non-finite or invalid: "
                  f"{bad[:8]}", file=sys.stderr, flush=True)
        raise RuntimeError("full-buffer finite/packet validation failed on at least one rank"
                           + (": " + "; ".join(details) if details else ""))
    return dict(passed=True, finite_tensors_checked=finite_checked, packets_checked=packets_checked,
                scales="finite qscale in [FP32(1e-12),1e6], adaptive in [FP32(1e-3),1e3]",
                scope="untimed; every buffer of the call", rank_coordinated=True)
