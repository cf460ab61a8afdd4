"""The special-function-free 2^x of the attention softmax
(csrc/exp2_fma.cuh), compiled for the host and checked against exp2 on a
dense grid of the softmax range: relative error <= 1.1e-4 on [-125, 0] (the
Chebyshev cubic's bound on [-0.5, 0.5]), exact-within-bound at the integers
and half-integers (where the rounding of n switches), and 2^-125 at or
below the clamp."""
import ctypes
import shutil
import subprocess
import tempfile
from pathlib import Path

import numpy as np
import pytest


def _lib():
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).is_file():
        pytest.skip("nvcc unavailable")
    csrc = Path(__file__).resolve().parents[1] / "tempname_dcu_b200" / "csrc"
    folder = Path(tempfile.mkdtemp(prefix="tdb-exp2-"))
    (folder / "h.cu").write_text(
        '#include "exp2_fma.cuh"\n'
        'extern "C" void run(const float* x, float* y, long n) {\n'
        '  for (long i = 0; i < n; ++i) y[i] = tdb::exp2_fma(x[i]);\n'
        '}\n')
    subprocess.run([nvcc, "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "-I", str(csrc), str(folder / "h.cu"),
                    "-o", str(folder / "h.so")], check=True, capture_output=True, text=True)
    lib = ctypes.CDLL(str(folder / "h.so"))
    lib.run.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_long]
    return lib


def _eval(lib, x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib.run(x.ctypes.data, y.ctypes.data, x.size)
    return y


def test_exp2_fma_error_bound():
    lib = _lib()
    x = np.linspace(-125.0, 0.0, 2_000_001, dtype=np.float32)
    y = _eval(lib, x).astype(np.float64)
    assert np.max(np.abs(y / np.exp2(x.astype(np.float64)) - 1)) <= 1.1e-4
    edges = np.concatenate([np.arange(-125, 1), np.arange(-124.5, 0, 1.0)]).astype(np.float32)
    edges = np.concatenate([edges, np.nextafter(edges, np.float32(-np.inf)), np.nextafter(edges, np.float32(1))])
    edges = edges[(edges >= -125) & (edges <= 0)]
    assert np.max(np.abs(_eval(lib, edges) / np.exp2(edges.astype(np.float64)) - 1)) <= 1.1e-4
    tiny = _eval(lib, np.array([-125.5, -200.0, -np.inf], dtype=np.float32))
    assert np.all(np.abs(tiny / 2.0 ** -125 - 1) <= 1.1e-4)
