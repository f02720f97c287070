"""tbvh_query_knn_share on one GPU: a share of the queries of one cloud, each
result row written at the query's own row of every destination buffer.

On one GPU the destinations are local buffers; the multi-GPU form (peer-mapped
destinations) is covered by tests/test_gpu_distributed.py.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import torchbvh_b200 as torchbvh
from torchbvh_b200 import _native
from torchbvh_b200._native import _C

pytestmark = pytest.mark.gpu


def _cloud(seed, shape):
    g = torch.Generator().manual_seed(seed)
    return torch.rand(shape, generator=g).cuda()


@pytest.mark.parametrize("dim", [2, 3])
@pytest.mark.parametrize("k", [4, 8, 16, 32])
def test_shares_fill_their_rows_of_every_destination(dim, k):
    points = _cloud(300 + dim + k, (5000, dim))
    queries = _cloud(301 + dim + k, (2999, dim))
    with torchbvh.BVH(points) as bvh:
        h = bvh._handle
        ref_idx, ref_dist = bvh.knn(queries, k)
        order = _C.morton_sort_queries_narrow(queries.unsqueeze(0), h["scene_min"].unsqueeze(0),
                                              h["scene_max"].unsqueeze(0))[0]
        dests = [(torch.full((2999, k), -7, dtype=torch.int64, device="cuda"),
                  torch.full((2999, k), -7.0, device="cuda")) for _ in range(2)]
        cuts = [0, 1000, 2100, 2999]
        for a, b in zip(cuts, cuts[1:]):
            _native.query_knn_share(h["node_aabbs"], h["sorted_indices"], 5000, queries, order[a:b].contiguous(), k,
                                    [d[0].data_ptr() for d in dests], [d[1].data_ptr() for d in dests])
            torch.cuda.synchronize()
            rows = order[b:]  # not served yet: untouched
            for di, dd in dests:
                assert bool((di[rows] == -7).all()) and bool((dd[rows] == -7.0).all())
    for di, dd in dests:
        assert torch.equal(di, ref_idx) and torch.equal(dd, ref_dist)
    assert torchbvh.device_status() == 0


def test_share_in_given_order_matches_too():
    points = _cloud(7, (4096, 3))
    queries = _cloud(8, (1500, 3))
    with torchbvh.BVH(points) as bvh:
        h = bvh._handle
        ref_idx, ref_dist = bvh.knn(queries, 16)
        di = torch.empty((1500, 16), dtype=torch.int64, device="cuda")
        dd = torch.empty((1500, 16), device="cuda")
        share = torch.arange(1500, dtype=torch.int64, device="cuda")
        _native.query_knn_share(h["node_aabbs"], h["sorted_indices"], 4096, queries, share, 16,
                                [di.data_ptr()], [dd.data_ptr()])
    assert torch.equal(di, ref_idx) and torch.equal(dd, ref_dist)
    assert torchbvh.device_status() == 0


def test_share_with_an_out_of_range_index_sets_the_status_bit():
    """A share entry outside [0, num_queries) is clamped to query 0 (so every read and
    write stays in bounds) and raises TBVH_DEVICE_BAD_INDEX; the valid rows are exact."""
    points = _cloud(9, (4096, 3))
    queries = _cloud(10, (1500, 3))
    assert torchbvh.device_status() == 0
    with torchbvh.BVH(points) as bvh:
        h = bvh._handle
        ref_idx, ref_dist = bvh.knn(queries, 8)
        di = torch.full((1500, 8), -7, dtype=torch.int64, device="cuda")
        dd = torch.full((1500, 8), -7.0, device="cuda")
        share = torch.tensor([5, 1500, 7, -3], dtype=torch.int64, device="cuda")
        _native.query_knn_share(h["node_aabbs"], h["sorted_indices"], 4096, queries, share, 8,
                                [di.data_ptr()], [dd.data_ptr()])
        torch.cuda.synchronize()
    assert torchbvh.device_status() == _native.TBVH_DEVICE_BAD_INDEX
    for row in (0, 5, 7):
        assert torch.equal(di[row], ref_idx[row]) and torch.equal(dd[row], ref_dist[row])
    untouched = torch.ones(1500, dtype=torch.bool, device="cuda")
    untouched[[0, 5, 7]] = False
    assert bool((di[untouched] == -7).all()) and bool((dd[untouched] == -7.0).all())


def test_peer_buffer_round_trip_on_one_device():
    ptr, handle = _native.peer_alloc(0, 1024 * 8)
    try:
        t = _native.device_tensor(ptr, (1024,), torch.int64, torch.device("cuda", 0))
        t.copy_(torch.arange(1024, device="cuda"))
        torch.cuda.synchronize()
        assert len(handle) == 64
        assert int(t.sum()) == 1023 * 1024 // 2
    finally:
        _native.peer_free(0, ptr)


@pytest.mark.parametrize("world,split", [(1, "morton"), (2, "morton"), (3, "morton"), (8, "morton"),
                                         (4, "interleaved"), (8, "interleaved")])
def test_query_shares_partition_the_queries_in_morton_order(oracle, world, split):
    """tbvh_share_queries on one GPU, every rank's share in turn: the shares
    partition the queries, each share is in ascending Morton order (codes against
    the BVH's scene box), and the share sizes are balanced to the cell size."""
    from torchbvh_b200 import distributed as tdist

    g = torch.Generator().manual_seed(40 + world)
    points = torch.rand((60_000, 3), generator=g).cuda()
    queries = torch.rand((50_001, 3), generator=g).cuda()
    m = queries.shape[0]
    with torchbvh.BVH(points) as bvh:
        h = bvh._handle
        shares = [tdist._owned_queries_cuda(h, queries, r, world, split) for r in range(world)]
        lo, hi = h["scene_min"].cpu().numpy(), h["scene_max"].cpu().numpy()
    torch.cuda.synchronize()
    allq = torch.cat(shares).cpu()
    assert torch.equal(torch.sort(allq).values, torch.arange(m))
    # The oracle's Morton codes divide with IEEE division where the kernels use
    # the fast-math quotient, so a query within an ulp of a cell boundary may
    # differ by one cell: allow a handful of inversions.
    codes = oracle.morton_codes(queries.cpu().numpy(), lo, hi).astype(np.int64)
    for s in shares:
        c = codes[s.cpu().numpy()]
        assert np.count_nonzero(np.diff(c) < 0) <= 4
    sizes = [s.numel() for s in shares]
    # A 15-bit cell of this uniform cloud holds about m / 32768 queries.
    runs = 1 if split == "morton" else 32
    assert max(sizes) - min(sizes) <= 2 * runs * (4 * m // 32768 + 8)
    assert torchbvh.device_status() == 0


def test_interleaved_share_matches_single_gpu_results():
    points = _cloud(60, (40_000, 3))
    queries = _cloud(61, (20_000, 3))
    from torchbvh_b200 import distributed as tdist

    with torchbvh.BVH(points) as bvh:
        want_i, want_d = bvh.knn(queries, 16)
        h = bvh._handle
        di = torch.full((20_000, 16), -1, dtype=torch.int64, device="cuda")
        dd = torch.full((20_000, 16), -1.0, device="cuda")
        for r in range(4):
            share = tdist._owned_queries_cuda(h, queries, r, 4, "interleaved")
            _native.query_knn_share(h["node_aabbs"], h["sorted_indices"], 40_000, queries, share, 16,
                                    [di.data_ptr()], [dd.data_ptr()])
    torch.cuda.synchronize()
    assert torch.equal(di, want_i) and torch.equal(dd, want_d)
    assert torchbvh.device_status() == 0


@pytest.mark.parametrize("k", [8, 32])
def test_int32_destinations_widen_to_the_int64_result(k):
    """tbvh_query_knn_share_i32 + tbvh_widen_indices (the NVLink-thrifty form of the
    fused all-gather) give the same rows as the int64 path (register and heap top-k)."""
    points = _cloud(70, (30_000, 3))
    queries = _cloud(71, (7_001, 3))
    with torchbvh.BVH(points) as bvh:
        want_i, want_d = bvh.knn(queries, k)
        h = bvh._handle
        order = _C.morton_sort_queries_narrow(queries.unsqueeze(0), h["scene_min"].unsqueeze(0),
                                              h["scene_max"].unsqueeze(0))[0].contiguous()
        wire = [torch.full((7_001, k), -5, dtype=torch.int32, device="cuda") for _ in range(2)]
        dd = [torch.full((7_001, k), -5.0, device="cuda") for _ in range(2)]
        _native.query_knn_share(h["node_aabbs"], h["sorted_indices"], 30_000, queries, order, k,
                                [w.data_ptr() for w in wire], [d.data_ptr() for d in dd], index_bits=32)
        wide = torch.empty((7_001, k), dtype=torch.int64, device="cuda")
        _native.widen_indices(wire[1], wide)
    torch.cuda.synchronize()
    assert torch.equal(wide, want_i) and torch.equal(dd[0], want_d) and torch.equal(dd[1], want_d)
    assert torch.equal(wire[0].long(), want_i)
    assert torchbvh.device_status() == 0


def test_two_and_three_dimensional_shares_in_one_process():
    """The share-cells kernel opts in to 128 KB of shared memory separately for
    its 2-D and 3-D forms: selecting shares of a 3-D cloud and then of a 2-D one
    (and back) in one process must work for both."""
    from torchbvh_b200 import distributed as tdist

    for dim in (3, 2, 3):
        g = torch.Generator().manual_seed(80 + dim)
        points = torch.rand((20_000, dim), generator=g).cuda()
        queries = torch.rand((10_003, dim), generator=g).cuda()
        with torchbvh.BVH(points) as bvh:
            shares = [tdist._owned_queries_cuda(bvh._handle, queries, r, 3, "morton") for r in range(3)]
        torch.cuda.synchronize()
        assert torch.equal(torch.sort(torch.cat(shares).cpu()).values, torch.arange(10_003))
    assert torchbvh.device_status() == 0


def test_unaligned_queries_give_the_same_shares():
    """The share-cells kernel reads queries in 128-bit quads only from a 16-byte
    aligned array: a view one query into its storage must select the same shares."""
    from torchbvh_b200 import distributed as tdist

    g = torch.Generator().manual_seed(90)
    points = torch.rand((30_000, 3), generator=g).cuda()
    qbase = torch.rand((20_002, 3), generator=g).cuda()
    view, copy = qbase[1:], qbase[1:].clone()
    assert view.data_ptr() % 16 != 0 and copy.data_ptr() % 16 == 0
    with torchbvh.BVH(points) as bvh:
        for r in range(4):
            a = tdist._owned_queries_cuda(bvh._handle, view, r, 4, "morton")
            b = tdist._owned_queries_cuda(bvh._handle, copy, r, 4, "morton")
            assert torch.equal(a, b)
    assert torchbvh.device_status() == 0
