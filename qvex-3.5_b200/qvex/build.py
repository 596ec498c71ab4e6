"""Build libqvex.so (the C-ABI CUDA library) in-tree for sm_100a.

    python -m qvex.build            # from qvex-3.5_b200/, or via __graft_entry__.build()

Each csrc/*.cu is compiled by nvcc (-gencode arch=compute_100a,code=sm_100a, -O3,
-lineinfo) into _build/, then linked into qvex/libqvex.so with the CUDA runtime
linked statically.  The library has no torch dependency: Python reaches it through
ctypes (qvex/_lib.py).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parents[1]          # qvex-3.5_b200/
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
BUILD = PKG_ROOT / "_build"
INCLUDE = REPO_ROOT / "include"
LIB = Path(__file__).resolve().parent / "libqvex.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills", "-I", str(INCLUDE), "-I", str(CSRC)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise FileNotFoundError("nvcc not found")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return _sources() + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _deps())


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    if not force and up_to_date():
        return LIB
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()
    flags = NVCC_FLAGS + (extra_flags or [])

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        cmd = [cc, *ARCH, *flags, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}")
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-cudart", "static"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("link of libqvex.so failed")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
