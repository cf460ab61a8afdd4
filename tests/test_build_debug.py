"""The TDB_DEBUG build variant (CPU): its own library, objects and manifest,
the -DTDB_DEBUG flag in the content key, and device code using the
TDB_DEBUG_OK index check compiles in both variants."""
import subprocess

import pytest

from tempname_dcu_b200.ops import _build


def test_debug_variant_is_a_separate_build(monkeypatch):
    release, debug = _build.paths(False), _build.paths(True)
    assert all(a != b for a, b in zip(release, debug))
    assert "-DTDB_DEBUG=1" in _build.flags(True) and "-DTDB_DEBUG=1" not in _build.flags(False)
    monkeypatch.setenv("TDB_DEBUG", "1")
    assert _build.debug_requested()
    monkeypatch.setenv("TDB_DEBUG", "0")
    assert not _build.debug_requested()


@pytest.mark.parametrize("debug", [False, True])
def test_debug_check_macro_compiles(tmp_path, debug):
    src = tmp_path / "probe.cu"
    src.write_text('''#include "common.cuh"
__global__ void probe(const int* idx, int n, float* out, int* status) {
  const int i = idx[threadIdx.x];
  if (TDB_DEBUG_OK(status, i >= 0 && i < n, 7, threadIdx.x, i)) out[i] = 1.f;
}
''')
    cmd = [_build.nvcc_path(), *_build.flags(debug), "-I", str(_build.CSRC), "-c", str(src),
           "-o", str(tmp_path / "probe.o")]
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-3000:]
