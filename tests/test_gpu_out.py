"""``knn(..., out=(indices, squared_distances))``: results written into
caller-owned tensors, on the device (by the traversal) or in pinned host memory
(by a copy). Rows must equal the allocating call bit for bit on every layout
(single, batched, ragged) and both top-k forms. The C ABI's direct stores into
page-locked host memory are checked through the raw entry point."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import torchbvh_b200 as torchbvh
from torchbvh_b200 import _native

pytestmark = pytest.mark.gpu


def _rand(seed, shape):
    g = torch.Generator().manual_seed(seed)
    return torch.rand(shape, generator=g)


def _outs(shape, where):
    if where == "pinned":
        return (torch.full(shape, -3, dtype=torch.int64).pin_memory(),
                torch.full(shape, -3.0, dtype=torch.float32).pin_memory())
    return (torch.full(shape, -3, dtype=torch.int64, device="cuda"),
            torch.full(shape, -3.0, dtype=torch.float32, device="cuda"))


@pytest.mark.parametrize("where", ["pinned", "device"])
@pytest.mark.parametrize("k", [4, 32])
def test_single_cloud_out(where, k):
    points = _rand(1, (20_000, 3)).cuda()
    queries = _rand(2, (9_999, 3)).cuda()
    with torchbvh.BVH(points) as bvh:
        want_i, want_d = bvh.knn(queries, k)
        out = _outs((9_999, k), where)
        got = bvh.knn(queries, k, out=out)
        torch.cuda.current_stream().synchronize()
    assert got[0] is out[0] and got[1] is out[1]
    assert torch.equal(out[0].cuda(), want_i) and torch.equal(out[1].cuda(), want_d)
    assert torchbvh.device_status() == 0


@pytest.mark.parametrize("sort_queries", [True, False])
def test_batched_out_pinned(sort_queries):
    points = _rand(3, (4, 5_000, 2)).cuda()
    queries = _rand(4, (4, 3_000, 2)).cuda()
    with torchbvh.BVH(points) as bvh:
        want_i, want_d = bvh.knn(queries, 8, sort_queries=sort_queries)
        out = _outs((4, 3_000, 8), "pinned")
        bvh.knn(queries, 8, sort_queries=sort_queries, out=out)
        torch.cuda.current_stream().synchronize()
    assert torch.equal(out[0].cuda(), want_i) and torch.equal(out[1].cuda(), want_d)


def test_ragged_out_pinned():
    sizes = [700, 64, 3_000, 1_200]
    qsizes = [50, 900, 7, 1_333]
    points = _rand(5, (sum(sizes), 3)).cuda()
    queries = _rand(6, (sum(qsizes), 3)).cuda()
    offs = torch.tensor(np.concatenate([[0], np.cumsum(sizes)]), dtype=torch.int64, device="cuda")
    qoffs = torch.tensor(np.concatenate([[0], np.cumsum(qsizes)]), dtype=torch.int64, device="cuda")
    with torchbvh.BVH(points, batch_offsets=offs) as bvh:
        want_i, want_d = bvh.knn(queries, 16, query_offsets=qoffs)
        out = _outs((sum(qsizes), 16), "pinned")
        bvh.knn(queries, 16, query_offsets=qoffs, out=out)
        torch.cuda.current_stream().synchronize()
    assert torch.equal(out[0].cuda(), want_i) and torch.equal(out[1].cuda(), want_d)


def test_out_rejects_pageable_host_and_wrong_shapes():
    points = _rand(7, (2_000, 3)).cuda()
    queries = _rand(8, (100, 3)).cuda()
    with torchbvh.BVH(points) as bvh:
        with pytest.raises(ValueError, match="pinned host memory"):
            bvh.knn(queries, 8, out=(torch.empty((100, 8), dtype=torch.int64), torch.empty((100, 8))))
        with pytest.raises(ValueError, match="shape"):
            bvh.knn(queries, 8, out=_outs((100, 4), "device"))
        with pytest.raises(ValueError, match="int64"):
            bvh.knn(queries, 8, out=(torch.empty((100, 8), device="cuda"), torch.empty((100, 8), device="cuda")))
        with pytest.raises(ValueError, match="source_points"):
            bvh.knn(queries, 8, source_points=points, out=_outs((100, 8), "device"))


def test_c_abi_refuses_pageable_output_before_launch():
    """The library checks every output pointer with cudaPointerGetAttributes and
    returns TBVH_ERR_BAD_ARG for pageable host memory: nothing is launched."""
    points = _rand(9, (2_000, 3)).cuda()
    queries = _rand(10, (64, 3)).cuda()
    with torchbvh.BVH(points) as bvh:
        h = bvh._handle
        lib = _native.load_library()
        launches = lib.tbvh_kernel_launch_count()
        host_idx = np.zeros((64, 8), dtype=np.int64)   # pageable
        dev_dist = torch.empty((64, 8), device="cuda")
        rc = lib.tbvh_query_knn(0, h["node_aabbs"].data_ptr(), h["sorted_indices"].data_ptr(), 1, 2_000, None, None,
                                queries.data_ptr(), 64, None, 64, None, 3, 8,
                                host_idx.ctypes.data, dev_dist.data_ptr(), None, 0, _native._stream(queries.device))
        assert rc == _native.TBVH_ERR_BAD_ARG
        assert b"page-locked" in lib.tbvh_last_error()
        assert lib.tbvh_kernel_launch_count() == launches
    assert not host_idx.any()


@pytest.mark.parametrize("k", [8, 32])
def test_c_abi_stores_rows_into_page_locked_host_memory(k):
    """Outputs in page-locked host memory (mapped at the same address) are
    written by the traversal itself, row for row equal to a device result."""
    points = _rand(11, (30_000, 3)).cuda()
    queries = _rand(12, (5_000, 3)).cuda()
    with torchbvh.BVH(points) as bvh:
        want_i, want_d = bvh.knn(queries, k)
        h = bvh._handle
        order = _native._C.morton_sort_queries_narrow(queries.unsqueeze(0), h["scene_min"].unsqueeze(0),
                                                      h["scene_max"].unsqueeze(0)).contiguous()
        host_i, host_d = _outs((5_000, k), "pinned")
        lib = _native.load_library()
        rc = lib.tbvh_query_knn(0, h["node_aabbs"].data_ptr(), h["sorted_indices"].data_ptr(), 1, 30_000, None, None,
                                queries.data_ptr(), 5_000, None, 5_000, order.data_ptr(), 3, k,
                                host_i.data_ptr(), host_d.data_ptr(), None, 0, _native._stream(queries.device))
        assert rc == 0
        torch.cuda.current_stream().synchronize()
    assert torch.equal(host_i, want_i.cpu()) and torch.equal(host_d, want_d.cpu())
    assert torchbvh.device_status() == 0
