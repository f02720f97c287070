"""Builds the in-tree CUDA library ``libtorchbvh_b200.so`` for sm_100a.

Each ``csrc/*.cu`` file is compiled to an object in parallel, then linked
into one shared library next to this file (CUDA runtime linked statically).
Used by ``__graft_entry__.build()`` and by developers; rebuilding is skipped
when the library is newer than every source file.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = PACKAGE_DIR.parent / "include"
LIB_NAME = "libtorchbvh_b200.so"
LIB_PATH = PACKAGE_DIR / LIB_NAME

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    # Same floating-point mode as the reference extension (torchbvh/_extension.py:36):
    # flush-to-zero, approximate division in the Morton normalisation, FMA contraction.
    "--use_fast_math",
    "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-Wall",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return _sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    lib_mtime = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > lib_mtime for p in _deps())


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    if not force and not is_stale():
        return LIB_PATH
    nvcc = _nvcc()
    obj_dir = PACKAGE_DIR / "_build"
    obj_dir.mkdir(exist_ok=True)
    flags = NVCC_FLAGS + list(extra_flags or [])

    def compile_one(src: Path) -> Path:
        obj = obj_dir / (src.stem + ".o")
        cmd = [nvcc, *flags, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
        if verbose and (proc.stdout or proc.stderr):
            print(proc.stdout, proc.stderr, flush=True)
        return obj

    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, os.cpu_count() or 1)) as pool:
        objs = list(pool.map(compile_one, _sources()))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static",
           *[str(o) for o in objs], "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{proc.stdout}\n{proc.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    import sys

    print(build(force="--force" in sys.argv, verbose=True))
