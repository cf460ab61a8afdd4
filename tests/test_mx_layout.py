"""Block-scaled FP8 scale-atom layout and the quantizer's torch restatement
(CPU): the atom byte order, the no-saturation scale rule and round trips."""
import torch

from tempname_dcu_b200.ops import mx


def test_atom_layout_round_trip_and_byte_positions():
    torch.manual_seed(0)
    e = torch.randint(-127, 128, (256, 12), dtype=torch.int32)  # every row and block distinct
    sf = mx.pack_scales(e, 256, 384)
    assert sf.numel() == mx.scale_bytes(256, 384) == 2 * 3 * 512
    assert torch.equal(mx.scales_dense(sf, 256, 384).long(), (e + 127).long())
    for r in range(256):
        for kb in range(12):
            kc, j = kb // 4, kb % 4
            off = (kc * 2 + r // 128) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + j
            assert sf[off].item() == e[r, kb].item() + 127


def test_scale_rule_never_saturates_and_is_tight():
    torch.manual_seed(1)
    x = (torch.randn(128, 256) * torch.logspace(-6, 6, 256)).to(torch.bfloat16)
    values, e = mx.quantize_reference(x)
    amax = x.float().view(128, 8, 32).abs().amax(-1)
    scaled_max = amax / torch.exp2(e.float())
    assert (scaled_max <= mx.E4M3_MAX).all()
    assert (scaled_max > mx.E4M3_MAX / 2).all()  # one smaller exponent would overflow
    assert (values.abs() <= mx.E4M3_MAX).all()


def test_zero_blocks_and_dequantize_error():
    x = torch.randn(128, 128).to(torch.bfloat16)
    x[:, :32] = 0
    values, e = mx.quantize_reference(x)
    assert (e[:, 0] == -127).all() and (values[:, :32] == 0).all()
    q = values.to(torch.float8_e4m3fn).view(torch.uint8)
    d = mx.dequantize(q, mx.pack_scales(e, 128, 128))
    rel = ((d - x.float()).norm() / x.float().norm()).item()
    assert rel < 0.04


def _host_scale_rule():
    """The device scale rule (csrc/mx_scale.cuh) compiled for the host."""
    import ctypes
    import shutil
    import subprocess
    import tempfile
    from pathlib import Path
    import pytest
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).is_file():
        pytest.skip("nvcc unavailable")
    csrc = Path(__file__).resolve().parents[1] / "tempname_dcu_b200" / "csrc"
    folder = Path(tempfile.mkdtemp(prefix="tdb-mx-"))
    (folder / "h.cu").write_text('#include "mx_scale.cuh"\n'
                                 'extern "C" int mx_exp(float a) { return tdb::mx_scale::block_exponent(a); }\n')
    subprocess.run([nvcc, "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "-I", str(csrc), str(folder / "h.cu"),
                    "-o", str(folder / "h.so")], check=True, capture_output=True, text=True)
    lib = ctypes.CDLL(str(folder / "h.so"))
    lib.mx_exp.argtypes, lib.mx_exp.restype = [ctypes.c_float], ctypes.c_int
    return lib


def test_device_scale_rule_matches_the_torch_restatement_on_every_bf16():
    lib = _host_scale_rule()
    bits = torch.arange(0, 0x7F80, dtype=torch.int32).to(torch.int16)  # every finite non-negative bf16
    values = bits.view(torch.bfloat16)
    block = torch.zeros(values.numel(), 32, dtype=torch.bfloat16)
    block[:, 5] = values  # a one-value block: amax is the value
    _, ref = mx.quantize_reference(block)
    got = torch.tensor([lib.mx_exp(v) for v in values.float().tolist()], dtype=ref.dtype)
    assert torch.equal(got, ref[:, 0])
