"""GPU codec kernels (csrc/codec.cu) against the stdlib FP64 oracle.

Gates follow the reference worker: actual-packet decode vs FP64 decode of the
same bytes <= 1% relative L2, independent encode+decode <= 2%
(python/flux_dcu/worker.py:58-83).
"""
import math
import random
import struct

import pytest

from tempname_dcu_b200 import reference as ref

pytestmark = pytest.mark.gpu


def _adjacent(value, direction):
    bits = struct.unpack("<I", struct.pack("<f", value))[0]
    return struct.unpack("<f", struct.pack("<I", bits + direction))[0]


def test_hardware_e4m3_matches_oracle_on_every_midpoint(cuda):
    import torch
    from tempname_dcu_b200.ops.codec import codec
    values = [0.0, -0.0, 448.0, -448.0, 1e20, -1e20, 500.0, -460.0]
    for low in range(126):
        mid = (ref.e4m3_decode(low) + ref.e4m3_decode(low + 1)) / 2
        for x in (_adjacent(mid, -1), mid, _adjacent(mid, 1)):
            values += [x, -x]
    rng = random.Random(71)
    values += [rng.uniform(-500, 500) for _ in range(2000)]
    values += [rng.uniform(-0.02, 0.02) for _ in range(2000)]
    pad = max(0, 256 - len(values))
    values += [0.0] * pad
    tensor = torch.tensor(values, dtype=torch.float32, device=cuda)
    codes, decoded = codec().e4m3_probe(tensor)
    codes = codes.cpu().tolist()
    for value, code in zip(values, codes):
        assert code == ref.e4m3_encode(value), (value, code)
    decoded = decoded.cpu().tolist()
    for code in range(256):
        expected = ref.e4m3_decode(code)
        if math.isnan(expected):
            assert math.isnan(decoded[code])
        else:
            assert decoded[code] == expected, code


def _cases(torch, device):
    gen = torch.Generator(device="cpu").manual_seed(9871)
    zero = torch.zeros(256)
    gauss = torch.randn(1024, generator=gen)
    outlier = torch.randn(256, generator=gen)
    outlier[0], outlier[128] = 128.0, -96.0
    tiny = torch.full((128,), 1e-8) * torch.tensor([(-1) ** i for i in range(128)])
    return [x.to(torch.bfloat16).to(device) for x in (zero, gauss, outlier, tiny)]


def test_encode_decode_against_fp64_oracle(cuda):
    import torch
    from tempname_dcu_b200.ops.codec import codec, packet_bytes
    c = codec()
    for x in _cases(torch, cuda):
        packet = torch.empty(packet_bytes(x.numel()), dtype=torch.uint8, device=cuda)
        out = torch.empty_like(x)
        c.encode(x, packet)
        c.decode(packet, out)
        torch.cuda.synchronize()
        raw = bytes(packet.cpu().tolist())
        from tempname_dcu_b200.validation import validate_packet_bytes
        validate_packet_bytes(raw, x.numel())
        byte_ref = ref.decode(raw)
        independent = ref.decode(ref.encode(x.float().cpu().tolist()))
        actual = out.float().cpu().tolist()
        assert ref.relative_l2(actual, byte_ref) <= 0.01
        assert ref.relative_l2(actual, independent) <= 0.02
        # scales agree with the oracle closely (FP32 vs FP64 accumulation)
        groups = x.numel() // 128
        quant = struct.unpack_from(f"<{groups}f", raw, x.numel())
        oracle = ref.encode(x.float().cpu().tolist())
        oq = struct.unpack_from(f"<{groups}f", oracle, x.numel())
        for a, b in zip(quant, oq):
            assert abs(a - b) <= 1e-5 * max(abs(b), 1e-30) + 1e-30


def test_ordered_reduce_matches_oracle_bitwise(cuda):
    import torch
    from tempname_dcu_b200.ops.codec import codec
    gen = torch.Generator(device="cpu").manual_seed(5)
    for world in (2, 4, 8):
        for rank in (0, world - 1):
            rows, n = 3, 136
            local = torch.randn(rows, n, generator=gen).to(torch.bfloat16)
            remote = torch.randn(world - 1, rows, n, generator=gen).to(torch.bfloat16) * 64
            out = torch.empty(rows, n, dtype=torch.bfloat16, device=cuda)
            codec().reduce(local.to(cuda), remote.to(cuda), out, rank, world)
            expected = ref.reduce_sources(local.flatten().float().tolist(),
                                          [r.flatten().float().tolist() for r in remote], rank, world)
            assert out.float().cpu().flatten().tolist() == expected


def test_placement_changes_result_like_reference(cuda):
    import torch
    from tempname_dcu_b200.ops.codec import codec
    sources = [256.0, 1.0, -256.0, 1.0]
    for rank in range(4):
        local = torch.full((1, 8), sources[rank], dtype=torch.bfloat16, device=cuda)
        remote = torch.tensor([[[s] * 8] for i, s in enumerate(sources) if i != rank],
                              dtype=torch.bfloat16, device=cuda)
        out = torch.empty_like(local)
        codec().reduce(local, remote, out, rank, 4)
        assert out.float().unique().tolist() == [1.0]


def test_diagnostic_delay_bounds(cuda):
    from tempname_dcu_b200.ops.codec import codec
    import torch
    codec().delay(1000)
    torch.cuda.synchronize()
    with pytest.raises(ValueError):
        codec().delay(0)
    with pytest.raises(ValueError):
        codec().delay(100_000_001)


def test_block_stats_against_fp64_oracle(cuda):
    """Per-block codec statistics (sumsq, amax, roundtrip error) vs the oracle."""
    import torch
    from tempname_dcu_b200.ops.codec import codec
    torch.manual_seed(5)
    rows, cols, block_rows = 8, 256, 2
    x = (torch.randn(rows, cols, device=cuda) * torch.linspace(0.01, 30, rows, device=cuda)[:, None]).to(torch.bfloat16)
    stats = codec().block_stats(x, block_rows).cpu()
    assert stats.shape == (rows // block_rows, 3) and stats.dtype == torch.float64
    for b in range(rows // block_rows):
        part = x[b * block_rows:(b + 1) * block_rows].float().cpu().reshape(-1).tolist()
        rt = [ref.bf16_round(v) for v in ref.decode(ref.encode(part))]
        sumsq = sum(v * v for v in part)
        err = sum((a - v) ** 2 for a, v in zip(rt, part))
        assert abs(stats[b, 0].item() - sumsq) <= 1e-5 * sumsq
        assert stats[b, 1].item() == max(abs(v) for v in part)
        assert abs(stats[b, 2].item() - err) <= 0.05 * err + 1e-12 * sumsq
    again = codec().block_stats(x, block_rows).cpu()
    assert torch.equal(stats, again)
