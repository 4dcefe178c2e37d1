"""Build libcsn_b200.so in-tree with nvcc for sm_100a.

    python -m csn_b200._build          (with clifford-space-network_b200/ on sys.path)

Each ``csrc/*.cu`` is compiled to an object in ``csrc/_build/`` (in parallel) and the
objects are linked into ``csn_b200/libcsn_b200.so`` with the CUDA runtime linked
statically, so the library depends only on the driver.

The build is content-addressed: a SHA-256 over every source, header and the build flags is
compiled into the library (``csn_version()`` ends in ``src <hash>``) and recorded beside it,
so a library whose sources changed since it was linked is rebuilt whatever the file times
say, and a caller can check that the library it loaded is the one these sources make.
"""
from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = ROOT / "csrc"
OBJ = CSRC / "_build"
LIB = PKG / "libcsn_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build csn_b200")


def sources() -> list:
    return sorted(CSRC.glob("*.cu"))


HASH_FILE = LIB.with_name(LIB.name + ".srchash")
# what the last build() call did: "built" or "reused"
last_action = None


def source_hash() -> str:
    """SHA-256 (first 16 hex digits) over the build flags and every source and header."""
    deps = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h"))
    deps.append(ROOT.parent / "include" / "csn_b200.h")
    h = hashlib.sha256(" ".join(ARCH + FLAGS).encode())
    for p in deps:
        if p.exists():
            h.update(p.name.encode())
            h.update(p.read_bytes())
    return h.hexdigest()[:16]


def _stale(digest: str) -> bool:
    if not LIB.exists() or not HASH_FILE.exists():
        return True
    return HASH_FILE.read_text().strip() != digest


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every CUDA source and link the shared library (skipped when the library was
    built from exactly these sources)."""
    global last_action
    digest = source_hash()
    if not force and not _stale(digest):
        last_action = "reused"
        return LIB
    nvcc = _nvcc()
    OBJ.mkdir(parents=True, exist_ok=True)

    def compile_one(src: Path) -> Path:
        obj = OBJ / (src.stem + ".o")
        cmd = [nvcc, *ARCH, *FLAGS, f"-DCSN_SOURCE_HASH=\"{digest}\"", "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    HASH_FILE.write_text(digest + "\n")
    last_action = "built"
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
