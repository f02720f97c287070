"""Failure handling on the GPU without a GPU fault: a bounded device wait is made
to run out and must come back as a status bit, with the device still usable.

The radix sort's decoupled look-back is the one place where a block waits for
another. The library's self-test runs one real sort pass in which tile 0 is
never claimed (its ticket counter starts at 1), so the wait of tile 1 can only
end by its bound. Nothing here traps, asserts on the device or spins without
a limit.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import torchbvh_b200 as torchbvh
from torchbvh_b200 import _native

pytestmark = pytest.mark.gpu


def _selftest() -> int:
    lib = _native.load_library()
    ws = torch.empty(lib.tbvh_selftest_workspace_size(), dtype=torch.uint8, device="cuda")
    bits = ctypes.c_uint(0)
    rc = lib.tbvh_selftest_lookback_timeout(0, ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream,
                                            ctypes.byref(bits))
    assert rc == 0, lib.tbvh_last_error()
    return int(bits.value)


def test_lookback_wait_gives_up_and_reports():
    assert torchbvh.device_status() == 0
    bits = _selftest()
    assert bits & _native.TBVH_DEVICE_LOOKBACK_TIMEOUT, bits
    # The status word was cleared by the self-test's read.
    assert torchbvh.device_status() == 0


def test_device_is_usable_after_a_timed_out_wait(oracle):
    assert _selftest() & _native.TBVH_DEVICE_LOOKBACK_TIMEOUT
    rng = np.random.default_rng(5)
    pts = rng.random((30_000, 3), dtype=np.float32)
    q = rng.random((999, 3), dtype=np.float32)
    with torchbvh.BVH(torch.from_numpy(pts).cuda()) as bvh:
        idx, dist = bvh.knn(torch.from_numpy(q).cuda(), 16)
    bi, bd = oracle.knn_bruteforce(pts, q, 16)
    np.testing.assert_array_equal(dist.cpu().numpy().view(np.uint32), bd.view(np.uint32))
    np.testing.assert_array_equal(idx.cpu().numpy(), bi)
    assert torchbvh.device_status() == 0
