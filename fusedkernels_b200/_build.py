"""Build recipe for libfkb200.so (all CUDA sources under csrc/, sm_100a only).

Each ``csrc/*.cu`` is compiled to an object with nvcc in parallel, then linked into one
shared library with a static CUDA runtime, so the library depends on nothing but the
NVIDIA driver at run time and can be loaded (for symbol checks) on a machine without a
GPU.  Objects are rebuilt only when a source or header is newer.

    python -m fusedkernels_b200._build           # build (incremental)
    python -m fusedkernels_b200._build --clean   # rebuild everything
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
OUT_DIR = PKG / "_lib"
LIB_NAME = "libfkb200.so"
LIB_PATH = OUT_DIR / LIB_NAME
OBJ_DIR = PKG.parent / "_build" / "obj"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-Xptxas", "-warn-spills",
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists() and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libfkb200.so")
    return cand


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _newest(paths) -> float:
    return max((p.stat().st_mtime for p in paths), default=0.0)


def _compile(src: Path, obj: Path, verbose: bool) -> tuple[Path, str]:
    cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(clean: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile and link libfkb200.so in-tree; returns its path."""
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    srcs = _sources()
    hdr_time = _newest(_headers())
    todo = []
    objs = []
    for s in srcs:
        o = OBJ_DIR / (s.stem + ".o")
        objs.append(o)
        if clean or not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime, hdr_time):
            todo.append((s, o))
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            for obj, log in ex.map(lambda so: _compile(so[0], so[1], verbose), todo):
                if log.strip():
                    logs.append(f"--- {obj.name}\n{log}")
    if todo or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < _newest(objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp),
               *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB_PATH)
    if verbose and logs:
        print("\n".join(logs), file=sys.stderr)
    return LIB_PATH


if __name__ == "__main__":
    build(clean="--clean" in sys.argv, verbose="-v" in sys.argv)
    print(LIB_PATH)
