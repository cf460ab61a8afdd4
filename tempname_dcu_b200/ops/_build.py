"""In-tree build of the native sm_100a library ``libtdb.so``.

Every ``csrc/*.cu`` file is compiled by nvcc for ``sm_100a`` only
(``-gencode arch=compute_100a,code=sm_100a``) into an object whose name carries
a content key (sha256 of the source, every shared header, the flags and the
nvcc version), and the objects are linked into
``tempname_dcu_b200/_native/libtdb.so``.  A manifest next to the library
records the key of every object and of the link, so an unchanged tree is
never rebuilt and a changed header rebuilds everything that includes it.
The build holds an ``flock`` so concurrent ranks or test workers build once.

``TDB_DEBUG=1`` selects a separate debug library (``libtdb_debug.so``, its
own objects and manifest) compiled with ``-DTDB_DEBUG``: kernels then check
tile, block and rank indices (``TDB_DEBUG_OK`` in ``csrc/common.cuh``),
record a failed check in the status word and skip the access -- a
sanitizer substitute that never traps.

Reference parity: ``python/flux_dcu/codec.py:58-109`` (content-addressed build
cache under an flock with a manifest).  Here the library is built in the
source tree so that it travels with the repository to the GPU host.
"""
from __future__ import annotations

import concurrent.futures
import fcntl
import hashlib
import json
import os
from pathlib import Path
import shutil
import subprocess
import uuid

PACKAGE = Path(__file__).resolve().parents[1]
CSRC = PACKAGE / "csrc"
NATIVE = PACKAGE / "_native"
OBJ = NATIVE / "obj"
LIBRARY = NATIVE / "libtdb.so"
MANIFEST = NATIVE / "manifest.json"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]
DEBUG_FLAGS = ["-DTDB_DEBUG=1"]


def debug_requested() -> bool:
    return os.environ.get("TDB_DEBUG", "") not in ("", "0")


def paths(debug: bool) -> tuple[Path, Path, Path]:
    """(library, manifest, object directory) of the release or debug build."""
    if debug:
        return NATIVE / "libtdb_debug.so", NATIVE / "manifest_debug.json", NATIVE / "obj_debug"
    return LIBRARY, MANIFEST, OBJ


def flags(debug: bool) -> list[str]:
    return ARCH_FLAGS + NVCC_FLAGS + (DEBUG_FLAGS if debug else [])


def nvcc_path() -> str:
    for candidate in (os.environ.get("TDB_NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).is_file():
            return candidate
    raise RuntimeError("nvcc not found: the native sm_100a library cannot be built")


def _sha(data: bytes) -> str:
    return hashlib.sha256(data).hexdigest()


def _nvcc_version(nvcc: str) -> str:
    return subprocess.run([nvcc, "--version"], check=True, capture_output=True, text=True, timeout=60).stdout


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")))


def _keys(nvcc: str, debug: bool = False) -> dict:
    version = _nvcc_version(nvcc)
    header_blob = b"".join(p.name.encode() + p.read_bytes() for p in headers())
    flags = globals()["flags"](debug)
    result = {}
    for src in sources():
        identity = json.dumps(dict(source=src.name, flags=flags, nvcc=version), sort_keys=True).encode()
        result[src.name] = _sha(identity + src.read_bytes() + header_blob)[:20]
    link = _sha(json.dumps(result, sort_keys=True).encode())[:20]
    return dict(objects=result, link=link, flags=flags, nvcc_version=version.strip().splitlines()[-1])


def _compile(nvcc: str, src: Path, obj: Path, flags: list[str]) -> tuple[Path, str]:
    tmp = obj.with_name(obj.stem + "." + uuid.uuid4().hex[:8] + ".tmp.o")
    cmd = [nvcc, *flags, "-I", str(CSRC), "-c", str(src), "-o", str(tmp)]
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=1800)
    if proc.returncode:
        tmp.unlink(missing_ok=True)
        raise RuntimeError(f"nvcc failed for {src.name} (exit {proc.returncode}):\n{proc.stderr[-6000:]}")
    os.replace(tmp, obj)
    return obj, proc.stderr


def up_to_date(debug: bool | None = None) -> bool:
    debug = debug_requested() if debug is None else debug
    LIBRARY, MANIFEST, _ = paths(debug)
    if not LIBRARY.is_file() or not MANIFEST.is_file():
        return False
    try:
        manifest = json.loads(MANIFEST.read_text())
        keys = _keys(nvcc_path(), debug)
    except (OSError, ValueError, RuntimeError, subprocess.SubprocessError):
        return False
    return manifest.get("link") == keys["link"] and manifest.get("library_sha256") == _sha(LIBRARY.read_bytes())


def build(verbose: bool = False, jobs: int | None = None, debug: bool | None = None) -> Path:
    """Compile and link ``libtdb.so`` (or, with ``debug`` / ``TDB_DEBUG=1``,
    ``libtdb_debug.so``) if anything changed; return its path."""
    debug = debug_requested() if debug is None else debug
    LIBRARY, MANIFEST, OBJ = paths(debug)
    nvcc = nvcc_path()
    NATIVE.mkdir(parents=True, exist_ok=True)
    OBJ.mkdir(parents=True, exist_ok=True)
    with open(NATIVE / ".build.lock", "a") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        keys = _keys(nvcc, debug)
        if LIBRARY.is_file() and MANIFEST.is_file():
            try:
                old = json.loads(MANIFEST.read_text())
                if old.get("link") == keys["link"] and old.get("library_sha256") == _sha(LIBRARY.read_bytes()):
                    return LIBRARY
            except ValueError:
                pass
        todo = []
        objects = []
        for src in sources():
            obj = OBJ / f"{src.stem}.{keys['objects'][src.name]}.o"
            objects.append(obj)
            if not obj.is_file():
                todo.append((src, obj))
        logs = {}
        if todo:
            workers = jobs or max(1, min(len(todo), os.cpu_count() or 4))
            with concurrent.futures.ThreadPoolExecutor(workers) as pool:
                futures = {pool.submit(_compile, nvcc, src, obj, keys["flags"]): src for src, obj in todo}
                for future in concurrent.futures.as_completed(futures):
                    obj, log = future.result()
                    logs[futures[future].name] = log
                    if verbose:
                        print(f"[tdb build] compiled {futures[future].name}", flush=True)
        tmp = NATIVE / f".{LIBRARY.stem}.{uuid.uuid4().hex[:8]}.so"
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objects)]
        proc = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
        if proc.returncode:
            tmp.unlink(missing_ok=True)
            raise RuntimeError(f"link of {LIBRARY.name} failed:\n{proc.stderr[-4000:]}")
        os.replace(tmp, LIBRARY)
        manifest = dict(keys, library_sha256=_sha(LIBRARY.read_bytes()), objects_built=sorted(logs),
                        ptxas_log={k: v[-2000:] for k, v in logs.items() if v.strip()})
        MANIFEST.write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n")
        # Drop objects that no longer belong to any source revision.
        keep = {p.name for p in objects}
        for stale in OBJ.glob("*.o"):
            if stale.name not in keep:
                stale.unlink(missing_ok=True)
        return LIBRARY


def manifest() -> dict:
    path = paths(debug_requested())[1]
    return json.loads(path.read_text()) if path.is_file() else {}


def manifest_for_rows() -> dict:
    """Build identity recorded in rank rows: library bytes hash and a source
    hash over every csrc file (the analogue of the reference's codec build
    manifest, python/flux_dcu/codec.py:72-109)."""
    blob = b"".join(p.name.encode() + p.read_bytes() for p in sorted(sources() + headers()))
    m = manifest()
    debug = debug_requested()
    library = paths(debug)[0]
    return dict(library=str(library), library_sha256=_sha(library.read_bytes()) if library.is_file() else None,
                identity=dict(source_sha256=_sha(blob), flags=flags(debug),
                              nvcc_version=m.get("nvcc_version")),
                link_key=m.get("link"))


if __name__ == "__main__":
    print(build(verbose=True))
