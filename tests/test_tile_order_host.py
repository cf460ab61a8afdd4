"""The GEMM tile scheduler's tile decode (``TileOrder::tile`` in
csrc/gemm.cuh) compiled for the host: the grouped raster visits every output
tile exactly once, keeps ``group_m`` m-blocks per band, and an explicit tile
table is followed verbatim -- a skipped or repeated tile would silently drop
or double part of a GEMM."""
import ctypes
import random
import shutil
import subprocess
import tempfile
from pathlib import Path

import pytest

CSRC = Path(__file__).resolve().parents[1] / "tempname_dcu_b200" / "csrc"


@pytest.fixture(scope="module")
def lib():
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).is_file():
        pytest.skip("nvcc unavailable")
    folder = Path(tempfile.mkdtemp(prefix="tdb-tiles-"))
    (folder / "t.cu").write_text('''#include "gemm.cuh"
extern "C" void decode(int num_m, int num_n, int group_m, const int* table, int count, int* mb, int* nb) {
  tdb::gemm::TileOrder o;
  o.num_m = num_m; o.num_n = num_n; o.group_m = group_m; o.table = table; o.num_tiles = count;
  for (int i = 0; i < count; ++i) o.tile(i, mb[i], nb[i]);
}
''')
    subprocess.run([nvcc, "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "-I", str(CSRC), str(folder / "t.cu"),
                    "-o", str(folder / "t.so")], check=True, capture_output=True, text=True)
    handle = ctypes.CDLL(str(folder / "t.so"))
    handle.decode.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                              ctypes.c_void_p, ctypes.c_void_p]
    return handle


def _decode(lib, num_m, num_n, group_m, table=None):
    count = len(table) if table is not None else num_m * num_n
    mb, nb = (ctypes.c_int * count)(), (ctypes.c_int * count)()
    tab = (ctypes.c_int * count)(*table) if table is not None else None
    lib.decode(num_m, num_n, group_m, tab, count, mb, nb)
    return list(zip(mb, nb))


@pytest.mark.parametrize("num_m,num_n,group_m", [(1, 1, 16), (16, 16, 16), (17, 5, 16), (64, 12, 16),
                                                 (3, 40, 8), (33, 33, 8), (128, 2, 1)])
def test_grouped_raster_is_a_bijection_in_bands(lib, num_m, num_n, group_m):
    tiles = _decode(lib, num_m, num_n, group_m)
    assert sorted(tiles) == [(m, n) for m in range(num_m) for n in range(num_n)]
    for i, (m, n) in enumerate(tiles):  # band b holds m-blocks [b*group_m, (b+1)*group_m)
        assert m // group_m == i // (group_m * num_n)


def test_explicit_table_is_followed(lib):
    rng = random.Random(5)
    num_m, num_n = 16, 8
    table = list(range(num_m * num_n))
    rng.shuffle(table)
    tiles = _decode(lib, num_m, num_n, 1, table)
    assert tiles == [(t // num_n, t % num_n) for t in table]
