"""CPU checks of the FP64 oracle, the wire contract and the device scalar
helpers compiled for the host (reference: tests/test_codec_reference.py)."""
import ctypes
import math
from pathlib import Path
import random
import shutil
import struct
import subprocess
import sys
import tempfile

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
from tempname_dcu_b200 import reference as ref  # noqa: E402
from tempname_dcu_b200.ops.codec import packet_bytes  # noqa: E402


def adjacent(value, direction):
    bits = struct.unpack("<I", struct.pack("<f", value))[0]
    return struct.unpack("<f", struct.pack("<I", bits + direction))[0]


def _host_helpers():
    """Compile the host branches of the device helpers (common.cuh's BF16
    rounding, codec.cuh's E4M3 decode) with nvcc (no GPU needed)."""
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).is_file():
        pytest.skip("nvcc unavailable")
    src = ('#include "codec.cuh"\n'
           'extern "C" unsigned short bf16_host(float x) { return tdb::float_to_bf16_bits(x); }\n'
           'extern "C" float e4m3_host(unsigned x) { return tdb::taco::e4m3_to_float(x); }\n')
    folder = tempfile.mkdtemp(prefix="tdb-host-")
    cu, lib = Path(folder) / "h.cu", Path(folder) / "h.so"
    cu.write_text(src)
    subprocess.run([nvcc, "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "-I", str(ROOT / "tempname_dcu_b200/csrc"),
                    str(cu), "-o", str(lib)], check=True, capture_output=True, text=True)
    native = ctypes.CDLL(str(lib))
    native.bf16_host.argtypes, native.bf16_host.restype = [ctypes.c_float], ctypes.c_ushort
    native.e4m3_host.argtypes, native.e4m3_host.restype = [ctypes.c_uint], ctypes.c_float
    return native


def test_host_compiled_scalar_helpers_match_oracle():
    native = _host_helpers()
    values = [0.0, -0.0, 448.0, -448.0, 1e20, -1e20, 1 + 2 ** -8, 1 + 3 * 2 ** -8]
    for low in range(126):
        mid = (ref.e4m3_decode(low) + ref.e4m3_decode(low + 1)) / 2
        for x in (adjacent(mid, -1), mid, adjacent(mid, 1)):
            values += [x, -x]
    rng = random.Random(71)
    values += [rng.uniform(-500, 500) for _ in range(2000)]
    for v in values:
        assert native.bf16_host(v) == ref.bf16_bits(v), v
    for code in range(256):
        expected = ref.e4m3_decode(code)
        got = native.e4m3_host(code)
        assert (math.isnan(got) and math.isnan(expected)) or got == expected, code


def test_all_finite_codes_roundtrip():
    for code in range(256):
        if code & 127 != 127:
            assert ref.e4m3_encode(ref.e4m3_decode(code)) == code


def test_signed_zero_and_bf16_signs():
    assert ref.e4m3_encode(0.0) == 0
    assert ref.e4m3_encode(-0.0) == 128
    assert math.copysign(1, ref.e4m3_decode(128)) == -1
    assert ref.bf16_bits(-0.0) == 0x8000


def test_midpoints_round_half_to_even_code():
    for low in range(126):
        mid = (ref.e4m3_decode(low) + ref.e4m3_decode(low + 1)) / 2
        even = low if low % 2 == 0 else low + 1
        assert ref.e4m3_encode(mid) == even
        assert ref.e4m3_encode(-mid) == even | 128
        assert ref.e4m3_encode(adjacent(mid, -1)) == low
        assert ref.e4m3_encode(adjacent(mid, 1)) == low + 1


def test_subnormals_max_and_saturation():
    assert ref.e4m3_decode(1) == 2 ** -9
    assert ref.e4m3_decode(8) == 2 ** -6
    assert ref.e4m3_decode(126) == 448
    assert ref.e4m3_encode(1e20) == 126
    assert ref.e4m3_encode(-1e20) == 254


def test_nonfinite_rejected():
    for value in (math.nan, math.inf, -math.inf):
        with pytest.raises(ValueError):
            ref.e4m3_encode(value)
    assert math.isnan(ref.e4m3_decode(127))


def test_bf16_known_ties():
    assert ref.bf16_round(1 + 2 ** -8) == 1
    assert ref.bf16_round(1 + 3 * 2 ** -8) == 1 + 2 ** -6
    assert ref.bf16_round(-(1 + 2 ** -8)) == -1


def test_dense_transform_orthonormal_and_self_inverse():
    rng = random.Random(7321)
    values = [rng.uniform(-1, 1) for _ in range(128)]
    back = ref.hadamard_fp64(ref.hadamard_fp64(values))
    assert max(abs(a - b) for a, b in zip(values, back)) < 1e-12
    assert abs(math.fsum(x * x for x in values) - math.fsum(x * x for x in ref.hadamard_fp64(values))) < 1e-10


def test_constant_and_impulse():
    const = ref.hadamard_fp64([1.0] * 128)
    assert abs(const[0] - math.sqrt(128)) < 1e-12 and all(v == 0 for v in const[1:])
    imp = ref.hadamard_fp64([1.0] + [0.0] * 127)
    assert all(abs(v - 1 / math.sqrt(128)) < 1e-15 for v in imp)


def test_zero_packet_exact_layout():
    packet = ref.encode([0.0] * 256)
    assert len(packet) == 272
    assert packet[:256] == bytes(256)
    assert struct.unpack_from("<ff", packet, 256) == (ref.fp32(1e-12),) * 2
    assert struct.unpack_from("<ff", packet, 264) == (1000.0,) * 2
    assert ref.decode(packet) == [0.0] * 256


def test_structure_of_arrays_not_interleaved():
    first = [1.0] * 128
    second = [(-1.0 if i % 2 else 1.0) * 9 for i in range(128)]
    q0, s0, a0 = ref.encode_group(first)
    q1, s1, a1 = ref.encode_group(second)
    assert ref.encode(first + second) == q0 + q1 + struct.pack("<ffff", s0, s1, a0, a1)


def test_roundtrip_error_small():
    rng = random.Random(99)
    cases = [[rng.gauss(0, 1) for _ in range(128)],
             [1000.0] + [rng.uniform(-0.01, 0.01) for _ in range(127)],
             [1e-8 * (-1 if i % 2 else 1) for i in range(128)]]
    for values in cases:
        expected = [ref.bf16_round(v) for v in values]
        assert ref.relative_l2(ref.decode(ref.encode(values)), expected) < 0.05


def test_invalid_shapes_and_corrupt_packets():
    for values in ([], [0.0] * 127, [0.0] * 129, [math.inf] * 128):
        with pytest.raises(ValueError):
            ref.encode(values)
    good = bytearray(ref.encode([1.0] * 128))
    for offset, value in ((128, math.nan), (128, -1.0), (132, 0.0)):
        bad = good.copy()
        struct.pack_into("<f", bad, offset, value)
        with pytest.raises(ValueError):
            ref.decode(bad)
    bad = good.copy()
    bad[0] = 127
    with pytest.raises(ValueError):
        ref.decode(bad)


def test_ordered_reduction_depends_on_source_order():
    sources = [[256.0], [1.0], [-256.0], [1.0]]
    for rank in range(4):
        remote = sources[:rank] + sources[rank + 1:]
        assert ref.reduce_sources(sources[rank], remote, rank, 4) == [1.0]
    reordered = [sources[0], sources[2], sources[1], sources[3]]
    assert ref.reduce_sources(reordered[0], reordered[1:], 0, 4) == [2.0]


def test_packet_bytes_contract():
    assert packet_bytes(128) == 136
    assert packet_bytes(256 * 4096) == 1114112
    for elements in (0, -128, 129, 128.0, True):
        with pytest.raises(ValueError):
            packet_bytes(elements)


def test_oracle_and_codec_import_without_torch():
    script = ("import sys; sys.path.insert(0, %r); import tempname_dcu_b200.reference, tempname_dcu_b200.ops.codec, "
              "tempname_dcu_b200.mapping, tempname_dcu_b200.planning; assert 'torch' not in sys.modules" % str(ROOT))
    subprocess.run([sys.executable, "-c", script], check=True)


def test_packet_validators_bytes_and_tensor():
    import torch
    from tempname_dcu_b200.validation import packet_tensor_valid, validate_packet_bytes
    packet = ref.encode([0.0] * 256)
    result = validate_packet_bytes(packet, 256)
    assert result["passed"] and result["groups"] == 2 and result["bytes"] == 272
    good = bytearray(ref.encode([1.0] * 256))
    for index, byte in ((0, 127), (255, 255)):
        bad = good.copy()
        bad[index] = byte
        with pytest.raises(ValueError, match="payload"):
            validate_packet_bytes(bad, 256)
    for index, value in ((256, math.nan), (260, math.inf), (260, 0.0), (264, -1.0), (268, 1001.0)):
        bad = good.copy()
        struct.pack_into("<f", bad, index, value)
        with pytest.raises(ValueError, match="scales"):
            validate_packet_bytes(bad, 256)
    for raw, elements in ((bytes(135), 128), (bytes(272), 128), (bytes(136), 129)):
        with pytest.raises(ValueError):
            validate_packet_bytes(raw, elements)
    t = torch.tensor(list(packet), dtype=torch.uint8)
    assert packet_tensor_valid(t, 256).item()
    t[255] = 255
    assert not packet_tensor_valid(t, 256).item()
