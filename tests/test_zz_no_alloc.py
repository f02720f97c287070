"""The allocation-free query sort (tbvh_sort_queries_noalloc) against the
workspace version (tbvh_sort_queries), both called through the C ABI.

It exists for callers that cannot allocate device memory (a plugin or FFI
binding holding only the buffers it was handed; a service that reserves its
memory at start-up). Its scratch is a fixed array inside the library, shared
by every call, so the test makes two calls in a row with different inputs:
each must equal the workspace version's output exactly (integer
permutation), which also shows nothing left over from the first call leaks
into the second. A second test checks consecutive calls against the
reference's own query permutation stored in the golden vectors. Collected
last so a first-failure stop has run the rest.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from torchbvh_b200 import _native

pytestmark = pytest.mark.gpu

MAX_QUERIES = 262_144


def _lib():
    lib = _native.load_library()
    fn = lib.tbvh_sort_queries_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                   ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return lib


def _workspace_sort(lib, q, clouds, per_cloud, offsets, total, dim, smin, smax):
    out = torch.empty((total,), dtype=torch.int64, device=q.device)
    ws_bytes = lib.tbvh_sort_queries_workspace_size(clouds, total, dim)
    ws = torch.empty((ws_bytes,), dtype=torch.uint8, device=q.device)
    rc = lib.tbvh_sort_queries(q.device.index, q.data_ptr(), clouds, per_cloud,
                               offsets.data_ptr() if offsets is not None else None, total, dim,
                               smin.data_ptr(), smax.data_ptr(), out.data_ptr(), ws.data_ptr(), ws_bytes,
                               torch.cuda.current_stream(q.device).cuda_stream)
    assert rc == 0, lib.tbvh_last_error()
    return out


def _noalloc_sort(lib, q, clouds, per_cloud, offsets, total, dim, smin, smax):
    out = torch.full((total,), -7, dtype=torch.int64, device=q.device)
    rc = lib.tbvh_sort_queries_noalloc(q.device.index, q.data_ptr(), clouds, per_cloud,
                                       offsets.data_ptr() if offsets is not None else None, total, dim,
                                       smin.data_ptr(), smax.data_ptr(), out.data_ptr(),
                                       torch.cuda.current_stream(q.device).cuda_stream)
    assert rc == 0, lib.tbvh_last_error()
    return out


def _case_fixed(seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.rand((4, 50_000, 3), generator=g).cuda()
    smin = q.amin(dim=1).contiguous()
    smax = q.amax(dim=1).contiguous()
    return q, 4, 50_000, None, 200_000, 3, smin, smax


def _case_ragged(seed):
    rng = np.random.default_rng(seed)
    sizes = [1, 4097, 90_000, 33, 165_000]
    total = sum(sizes)
    q = torch.from_numpy(rng.random((total, 2), dtype=np.float32)).cuda()
    offsets = torch.tensor(np.concatenate([[0], np.cumsum(sizes)]), dtype=torch.int64, device="cuda")
    smin = torch.zeros((len(sizes), 2), device="cuda")
    smax = torch.ones((len(sizes), 2), device="cuda")
    return q, len(sizes), 0, offsets, total, 2, smin, smax


def test_noalloc_sort_matches_workspace_sort_twice_in_a_row():
    lib = _lib()
    first = _case_fixed(31)
    second = _case_ragged(32)
    assert second[4] <= MAX_QUERIES
    got_first = _noalloc_sort(lib, *first)
    got_second = _noalloc_sort(lib, *second)
    want_first = _workspace_sort(lib, *first)
    want_second = _workspace_sort(lib, *second)
    torch.cuda.synchronize()
    assert torch.equal(got_first, want_first)
    assert torch.equal(got_second, want_second)
    # And again on the first input, after the array held the second call's data.
    assert torch.equal(_noalloc_sort(lib, *first), want_first)
    assert _native.device_status() == 0


def test_noalloc_sort_rejects_more_than_its_capacity():
    lib = _lib()
    q = torch.zeros((MAX_QUERIES + 1, 3), device="cuda")
    smin = torch.zeros((1, 3), device="cuda")
    smax = torch.ones((1, 3), device="cuda")
    out = torch.empty((MAX_QUERIES + 1,), dtype=torch.int64, device="cuda")
    rc = lib.tbvh_sort_queries_noalloc(0, q.data_ptr(), 1, MAX_QUERIES + 1, None, MAX_QUERIES + 1, 3,
                                       smin.data_ptr(), smax.data_ptr(), out.data_ptr(),
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == _native.TBVH_ERR_BAD_ARG
    assert b"static scratch capacity" in lib.tbvh_last_error()


def test_noalloc_sort_matches_reference_permutation():
    """Two calls in a row on golden cases: each output must equal the reference's own
    query permutation (its morton_sort_queries_narrow, stored by the golden generator)."""
    from pathlib import Path

    golden = Path(__file__).resolve().parent / "golden" / "reference_cuda.npz"
    data = np.load(golden)
    if "c1/query_order" not in data.files:
        pytest.skip("golden file predates the stored reference query permutation")
    lib = _lib()
    for name in ("c1", "rand_d2_n20000_k8", "batched_3x3000_k8", "rand_d3_n20000_k16"):
        if name == "c1":
            from torchbvh_b200 import workloads

            q = workloads.c1_single_uniform().queries.numpy()
        else:
            q = data[f"{name}/queries"]
        want = data[f"{name}/query_order"]
        qt = torch.from_numpy(np.ascontiguousarray(q)).cuda()
        lo = torch.from_numpy(np.ascontiguousarray(data[f"{name}/scene_min"])).cuda().reshape(-1, q.shape[-1])
        hi = torch.from_numpy(np.ascontiguousarray(data[f"{name}/scene_max"])).cuda().reshape(-1, q.shape[-1])
        clouds = lo.shape[0]
        per_cloud = q.shape[-2]
        got = _noalloc_sort(lib, qt, clouds, per_cloud, None, clouds * per_cloud, q.shape[-1], lo, hi)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(got.cpu().numpy().reshape(want.shape), want)
    assert _native.device_status() == 0
