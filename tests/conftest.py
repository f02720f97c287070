"""Shared pytest setup.

Tests marked ``gpu`` need a CUDA device (a B200 on the GPU box). Without one
they are skipped, unless the run selected them explicitly with ``-m gpu``:
then a missing GPU is a failure, so a GPU run can never pass by skipping.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU; run on the GPU box with -m gpu")


def _gpu_explicitly_selected(config) -> bool:
    expr = (config.getoption("markexpr") or "").replace(" ", "")
    return "gpu" in expr and "notgpu" not in expr


_NO_GPU_FAILS = False


def pytest_collection_modifyitems(config, items):
    global _NO_GPU_FAILS
    import torch

    if torch.cuda.is_available():
        return
    if _gpu_explicitly_selected(config):
        _NO_GPU_FAILS = True  # _gpu_required() fails every selected GPU test
        return
    skip = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _gpu_required(request):
    """With ``-m gpu`` and no CUDA device, every GPU test fails (never skips or xfails)."""
    if _NO_GPU_FAILS and request.node.get_closest_marker("gpu") is not None:
        pytest.fail("no CUDA device: a -m gpu run needs one")


@pytest.fixture(scope="session")
def oracle():
    from oracle import pyoracle

    pyoracle.lib()
    return pyoracle


@pytest.fixture(scope="session")
def native_lib():
    from torchbvh_b200 import _build_lib, _native

    if _build_lib.is_stale():
        _build_lib.build()
    return _native.load_library()
