"""tcgen05 descriptors built by csrc/common.cuh (compiled for the host)
against the bit-field layouts of the public CUTLASS sm100 headers
(cute/arch/mma_sm100_desc.hpp): the kind::f16 and kind::mxf8f6f4 instruction
descriptors and the 128B-swizzled / unswizzled shared-memory matrix
descriptors.  Skipped when the CUTLASS headers are not installed."""
import importlib.util
import shutil
import subprocess
import tempfile
from pathlib import Path

import pytest

CSRC = Path(__file__).resolve().parents[1] / "tempname_dcu_b200" / "csrc"


def _cutlass_include():
    spec = importlib.util.find_spec("flashinfer")
    if spec is None or not spec.submodule_search_locations:
        return None
    inc = Path(list(spec.submodule_search_locations)[0]) / "data" / "cutlass" / "include"
    return inc if (inc / "cute" / "arch" / "mma_sm100_desc.hpp").is_file() else None


PROGRAM = r'''
#include "common.cuh"
#include <cute/arch/mma_sm100_desc.hpp>
#include <cstdio>
int main() {
  int bad = 0;
  for (int m : {64, 128}) for (int n = 8; n <= 256; n += 8) {
    cute::UMMA::InstrDescriptorBlockScaled d = {};
    d.scale_format_ = 1; d.m_dim_ = m >> 4; d.n_dim_ = n >> 3;   // e4m3 x e4m3, ue8m0, K-major
    bad += uint32_t(d) != tdb::idesc_mxf8(m, n);
    for (int amn = 0; amn < 2; ++amn) for (int bmn = 0; bmn < 2; ++bmn) {
      cute::UMMA::InstrDescriptor e = {};
      e.c_format_ = 1; e.a_format_ = 1; e.b_format_ = 1;          // f32 += bf16 x bf16
      e.m_dim_ = m >> 4; e.n_dim_ = n >> 3; e.a_major_ = amn; e.b_major_ = bmn;
      bad += uint32_t(e) != tdb::idesc_bf16(m, n, amn, bmn);
    }
  }
  for (uint32_t addr = 0; addr < (1u << 18); addr += 1040) for (uint32_t lbo : {0u, 16u, 8192u}) {
    for (uint32_t sbo : {128u, 1024u, 2048u}) {
      cute::UMMA::SmemDescriptor s = {};
      s.start_address_ = (addr >> 4) & 0x3FFF; s.leading_byte_offset_ = lbo >> 4; s.stride_byte_offset_ = sbo >> 4;
      s.version_ = 1; s.base_offset_ = 0; s.lbo_mode_ = 0;
      s.layout_type_ = uint8_t(cute::UMMA::LayoutType::SWIZZLE_128B);
      bad += uint64_t(s) != tdb::smem_desc_sw128(addr, lbo, sbo);
      s.layout_type_ = uint8_t(cute::UMMA::LayoutType::SWIZZLE_NONE);
      bad += uint64_t(s) != tdb::smem_desc_plain(addr, lbo, sbo);
    }
  }
  printf("%d\n", bad);
  return bad != 0;
}
'''


def test_descriptors_match_the_cutlass_bit_fields(tmp_path):
    inc = _cutlass_include()
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if inc is None or not Path(nvcc).is_file():
        pytest.skip("CUTLASS headers or nvcc unavailable")
    (tmp_path / "d.cu").write_text(PROGRAM)
    build = subprocess.run([nvcc, "-std=c++17", "-I", str(CSRC), "-I", str(inc), str(tmp_path / "d.cu"), "-o",
                            str(tmp_path / "d")], capture_output=True, text=True, timeout=600)
    assert build.returncode == 0, build.stderr[-3000:]
    run = subprocess.run([str(tmp_path / "d")], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and run.stdout.strip() == "0", run.stdout


SF_PROGRAM = r'''
#include <cute/tensor.hpp>
#include <cutlass/detail/sm100_blockscaled_layout.hpp>
#include <cstdio>
int main() {
  using Atom = cutlass::detail::Sm1xxBlockScaledBasicChunk<32>::SfKMajorAtom;
  Atom a;
  int bad = 0;
  for (int r = 0; r < 128; ++r)
    for (int k = 0; k < 128; ++k) bad += int(a(r, k)) != (r % 32) * 16 + (r / 32) * 4 + k / 32;
  printf("%d %d\n", bad, int(cute::cosize(a)));
  return bad != 0;
}
'''


def test_scale_atom_matches_the_cutlass_sf_atom(tmp_path):
    """Inside a 512-byte atom (128 rows x 128 K values, one ue8m0 per 32) the
    byte of row r and K value k is (r % 32) * 16 + (r / 32) * 4 + k / 32 --
    the order quantize_kernel writes and tcgen05.cp 32x128b.warpx4 expects."""
    inc = _cutlass_include()
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if inc is None or not Path(nvcc).is_file():
        pytest.skip("CUTLASS headers or nvcc unavailable")
    (tmp_path / "sf.cu").write_text(SF_PROGRAM)
    build = subprocess.run([nvcc, "-std=c++17", "-I", str(inc), str(tmp_path / "sf.cu"), "-o", str(tmp_path / "sf")],
                           capture_output=True, text=True, timeout=600)
    assert build.returncode == 0, build.stderr[-3000:]
    run = subprocess.run([str(tmp_path / "sf")], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and run.stdout.split() == ["0", "512"], run.stdout
