"""The exported C ABI (csrc/tdb.h) against the library and the Python bindings.

* every prototype in ``tdb.h`` names a symbol that ``libtdb.so`` exports, and
  every ``TDB_API`` definition in the sources has a prototype (the sources
  include the header, so nvcc already rejects a definition whose types differ);
* every ctypes signature the Python side registers (``native.SIGNATURES``)
  has the same number of arguments as the prototype and, per argument, the
  same kind: pointer, signed / unsigned integer of the same width, or float of
  the same width;
* the LayerNorm entry points refuse misaligned bf16 pointers with an error
  code before touching the GPU (checked here with fake addresses, no device).

CPU only: the library loads without a GPU and the checks run before any CUDA
call.
"""
import ctypes
import re
from pathlib import Path

import pytest

CSRC = Path(__file__).resolve().parents[1] / "tempname_dcu_b200" / "csrc"

_C_KINDS = {
    "int": "i4", "unsigned int": "u4", "unsigned": "u4", "long long": "i8", "unsigned long long": "u8",
    "int64_t": "i8", "uint64_t": "u8", "size_t": "u8", "float": "f4", "double": "f8", "int32_t": "i4",
    "uint32_t": "u4",
}


def _prototypes():
    text = (CSRC / "tdb.h").read_text()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    protos = {}
    for m in re.finditer(r"([A-Za-z_][\w\s\*]*?)\b(tdb_\w+)\s*\(([^)]*)\)\s*;", text):
        name, args = m.group(2), m.group(3).strip()
        kinds = []
        if args and args != "void":
            for arg in args.split(","):
                arg = " ".join(arg.split())
                if "*" in arg:
                    kinds.append("p")
                    continue
                base = re.sub(r"\b(const)\b", "", arg).split()
                base = " ".join(base[:-1])  # drop the parameter name
                assert base in _C_KINDS, (name, arg)
                kinds.append(_C_KINDS[base])
        protos[name] = kinds
    return protos


def _ctypes_kind(t):
    if t in (ctypes.c_void_p, ctypes.c_char_p) or (isinstance(t, type) and issubclass(t, ctypes._Pointer)):
        return "p"
    if t in (ctypes.c_float, ctypes.c_double):
        return "f%d" % ctypes.sizeof(t)
    signed = t(-1).value < 0
    return ("i" if signed else "u") + str(ctypes.sizeof(t))


def _all_signatures():
    # importing the op modules registers their entry points
    import tempname_dcu_b200.ops.gemm  # noqa: F401
    import tempname_dcu_b200.ops.kernels  # noqa: F401
    import tempname_dcu_b200.ops.mx  # noqa: F401
    import tempname_dcu_b200.parallel.allgather  # noqa: F401
    import tempname_dcu_b200.parallel.symmetric  # noqa: F401
    import tempname_dcu_b200.runtime  # noqa: F401
    from tempname_dcu_b200.ops import native
    return native.SIGNATURES


def test_every_definition_has_a_prototype():
    protos = _prototypes()
    defined = set()
    for src in CSRC.glob("*.cu"):
        for m in re.finditer(r"TDB_API\s+[^{;]*?\b(tdb_\w+)\s*\([^)]*\)\s*\{", src.read_text(), re.S):
            defined.add(m.group(1))
    assert defined, "no TDB_API definitions found"
    assert defined - set(protos) == set(), sorted(defined - set(protos))
    assert set(protos) - defined == set(), sorted(set(protos) - defined)


def test_library_exports_every_prototype():
    from tempname_dcu_b200.ops import native
    lib = native.lib()
    missing = [name for name in _prototypes() if not hasattr(lib, name)]
    assert not missing, missing


def test_ctypes_signatures_match_the_header():
    protos = _prototypes()
    sigs = _all_signatures()
    for name, argtypes in sigs.items():
        assert name in protos, f"{name} is bound in Python but not declared in tdb.h"
        got = [_ctypes_kind(t) for t in argtypes]
        assert got == protos[name], (name, got, protos[name])


@pytest.mark.parametrize("entry", ["fwd", "bwd", "noalloc"])
def test_layernorm_refuses_misaligned_rows(entry):
    from tempname_dcu_b200.ops import native
    lib = native.lib()
    aligned, odd = 0x10000, 0x10002  # fake device addresses: the check runs before any CUDA call
    rows, H = 32, 768
    v = ctypes.c_void_p
    if entry == "fwd":
        fn = lib.tdb_layernorm_fwd
        fn.argtypes = [v, v, v, v, v, v, ctypes.c_int, ctypes.c_int, ctypes.c_float, v]
        rc = fn(odd, aligned, aligned, aligned, aligned, aligned, rows, H, 1e-5, None)
    elif entry == "bwd":
        fn = lib.tdb_layernorm_bwd
        fn.argtypes = [v] * 10 + [ctypes.c_int] * 3 + [v]
        rc = fn(aligned, aligned, aligned, aligned, aligned, odd, aligned, aligned, aligned, aligned, rows, H, 0, None)
    else:
        fn = lib.tdb_layernorm_bwd_noalloc
        fn.argtypes = [v] * 9 + [ctypes.c_int] * 3 + [v]
        rc = fn(aligned, aligned, aligned, aligned, odd, None, aligned, aligned, aligned, rows, H, 0, None)
    assert rc == 1  # cudaErrorInvalidValue
    assert b"16-byte aligned" in lib.tdb_last_error()
