"""Builds the in-tree CUDA library ``libnnb.so`` for sm_100a with nvcc.

Each ``csrc/*.cu`` file is compiled to an object in parallel, then linked with the static CUDA
runtime into ``nnb/libnnb.so`` next to this file, so the library travels with the source tree and
needs no JIT cache. nvcc cross-compiles, so this runs on a machine without a GPU.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess

PKG_DIR = pathlib.Path(__file__).resolve().parent
CSRC = PKG_DIR.parent / "csrc"
INCLUDE = PKG_DIR.parent.parent / "include"
LIB = PKG_DIR / "libnnb.so"
OBJ_DIR = PKG_DIR.parent / "_build"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "--fmad=false",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I", str(INCLUDE),
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _compile(nvcc: str, src: pathlib.Path, extra: list[str]) -> pathlib.Path:
    obj = OBJ_DIR / (src.stem + ".o")
    cmd = [nvcc, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj


def sources() -> list[pathlib.Path]:
    return sorted(CSRC.glob("*.cu"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*")) + list(INCLUDE.glob("*.h"))
    return all(p.stat().st_mtime <= t for p in deps)


def build(force: bool = False, verbose_ptxas: bool = False) -> pathlib.Path:
    """Compiles every csrc/*.cu for sm_100a and links nnb/libnnb.so; returns its path."""
    if not force and up_to_date():
        return LIB
    nvcc = _nvcc()
    OBJ_DIR.mkdir(exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(nvcc, s, extra), sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, "-shared", "-cudart", "static", "-gencode", "arch=compute_100a,code=sm_100a",
           *map(str, objs), "-o", str(tmp), "-lrt", "-ldl", "-lpthread"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    import sys
    print(build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv))
