"""Test infrastructure only: build and load the reference k-NN harness.

``oracle/ref_knn_harness.cu`` includes the unmodified reference
``torchbvh/csrc/knn_query.cu`` and instantiates its traversal launcher at
K in {9, 17, 32, 33}. It is compiled here (with the reference's own CUDA
flags, ``torchbvh/_extension.py:36``) into ``oracle/_ref/knn_harness/`` and
loaded from there by the golden-vector generator; nothing in
``torchbvh_b200`` imports this module or the library it builds.

    python oracle/ref_harness.py <reference root>     # build (CPU is enough)

The reference root is the directory holding the reference's ``torchbvh``
package (its ``csrc`` sources are compiled in place, never copied). Set
``TORCH_CUDA_ARCH_LIST=10.0`` when no GPU is visible; the build script does
that by default.
"""

from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
BUILD_DIR = ORACLE_DIR / "_ref" / "knn_harness"
NAME = "tbvh_ref_knn_harness"
CUDA_FLAGS = ["-O3", "--use_fast_math", "-lineinfo"]


def library_path() -> Path:
    return BUILD_DIR / f"{NAME}.so"


def build(ref_root: str | os.PathLike) -> Path:
    csrc = Path(ref_root) / "torchbvh" / "csrc"
    if not (csrc / "knn_query.cu").exists():
        raise FileNotFoundError(f"reference sources not found under {csrc}")
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils import cpp_extension

    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    cpp_extension.load(name=NAME, sources=[str(ORACLE_DIR / "ref_knn_harness.cu")],
                       extra_cflags=["-O2"], extra_cuda_cflags=CUDA_FLAGS,
                       extra_include_paths=[str(csrc)], build_directory=str(BUILD_DIR),
                       with_cuda=True, verbose=False)
    return library_path()


def load():
    """Imports the prebuilt harness (no rebuild: the reference tree is absent on the GPU box)."""
    path = library_path()
    if not path.exists():
        raise FileNotFoundError(f"{path} not built; run python oracle/ref_harness.py <reference root>")
    import torch  # noqa: F401  (the extension links against libtorch)

    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python oracle/ref_harness.py <reference root>")
    print(build(sys.argv[1]))
