"""BVH build parity on the GPU (ports tests/test_bvh_build.py of the reference
and adds exact comparisons with the oracle).

node_aabbs, scene bounds and traversal arrays must equal the oracle's exactly
(min/max involve no rounding). sorted_indices must be a stable Morton order;
against the oracle's IEEE-division Morton codes only points within a few ulp
of a quantisation boundary may land in a neighbouring cell (see
oracle/tbvh_oracle.h); bit equality with the reference CUDA build is pinned
by tests/test_golden.py.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import torchbvh_b200 as torchbvh
from tests import clouds

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().cpu().numpy()


def check_build(oracle, pts: np.ndarray, bvh) -> None:
    n, d = pts.shape
    nodes = _np(bvh["node_aabbs"])
    sidx = _np(bvh["sorted_indices"])
    assert bvh["num_leaves"] == n
    assert bvh["dim"] == d
    assert bvh["num_real_nodes"] == oracle.real_node_count(n)
    assert bvh["leaf_level"] == oracle.leaf_level(n)
    assert bvh["virtual_leaves"] == (1 << bvh["leaf_level"]) - n
    assert nodes.shape == (oracle.real_node_count(n), 2 * d)
    assert bvh["sorted_indices"].dtype == torch.int64
    np.testing.assert_array_equal(np.sort(sidx), np.arange(n))
    lo, hi = oracle.scene_bounds(pts)
    np.testing.assert_array_equal(_np(bvh["scene_min"]), lo)
    np.testing.assert_array_equal(_np(bvh["scene_max"]), hi)
    ref = oracle.build_tree(pts, sidx)
    np.testing.assert_array_equal(nodes, ref["node_aabbs"])
    for key in ("left_child_mem", "right_child_mem", "mem_to_leaf"):
        assert bvh[key].dtype == torch.int32
        np.testing.assert_array_equal(_np(bvh[key]), ref[key])
    codes = oracle.morton_codes(pts, lo, hi).astype(np.int64)
    sc = codes[sidx]
    # Stable: equal codes keep ascending original index.
    same = sc[1:] == sc[:-1]
    assert np.all(sidx[1:][same] > sidx[:-1][same])
    # Morton order up to boundary-adjacent cells (approximate division on the GPU).
    assert np.count_nonzero(sc[1:] < sc[:-1]) <= max(2, n // 500)


@pytest.mark.parametrize("case", clouds.BUILD_CASES, ids=lambda c: c[0])
def test_build_cases(oracle, case):
    _, pts = case
    bvh = torchbvh.build_bvh(torch.from_numpy(pts).cuda())
    check_build(oracle, pts, bvh)
    assert torchbvh.device_status() == 0


@pytest.mark.parametrize("d", [2, 3])
@pytest.mark.parametrize("n", [1023, 1024, 1025, 2048, 5000, 70_000, 300_001])
def test_random_builds_multi_block(oracle, d, n):
    rng = np.random.default_rng(n + d)
    pts = rng.random((n, d), dtype=np.float32) * np.float32(7) - np.float32(3)
    bvh = torchbvh.build_bvh(torch.from_numpy(pts).cuda())
    check_build(oracle, pts, bvh)
    assert torchbvh.device_status() == 0


def test_build_matches_oracle_sort_on_snapped_grid(oracle):
    # Points on a coarse grid well inside their Morton cells: no division
    # rounding can move them, so the GPU order must equal the oracle's exactly.
    rng = np.random.default_rng(3)
    cells = rng.integers(0, 1000, size=(20000, 3))
    pts = ((cells.astype(np.float32) + np.float32(0.5)) / np.float32(1024)).astype(np.float32)
    pts[0] = 0.0
    pts[1] = 1.0
    bvh = torchbvh.build_bvh(torch.from_numpy(pts).cuda())
    ref = oracle.build(pts)
    np.testing.assert_array_equal(_np(bvh["sorted_indices"]), ref["sorted_indices"])
    np.testing.assert_array_equal(_np(bvh["node_aabbs"]), ref["node_aabbs"])


def test_degenerate_2d_extent():
    pts = torch.tensor([[7.0, -3.0]] * 3, device="cuda")
    bvh = torchbvh.build_bvh(pts)
    expected = pts[0].expand_as(bvh["node_aabbs"][:, :2])
    assert torch.equal(bvh["node_aabbs"][:, :2], expected)
    assert torch.equal(bvh["node_aabbs"][:, 2:], bvh["node_aabbs"][:, :2])


def test_batched_build_equals_single_builds(oracle):
    rng = np.random.default_rng(17)
    pts = rng.random((5, 3001, 3), dtype=np.float32)
    pts[2] *= 100.0
    batched = torchbvh.build_bvh(torch.from_numpy(pts).cuda())
    for b in range(5):
        single = torchbvh.build_bvh(torch.from_numpy(pts[b]).cuda())
        for key in ("node_aabbs", "sorted_indices", "scene_min", "scene_max"):
            assert torch.equal(batched[key][b], single[key]), key
        for key in ("left_child_mem", "right_child_mem", "mem_to_leaf"):
            assert torch.equal(batched[key], single[key]), key


def test_ragged_build_equals_single_builds():
    rng = np.random.default_rng(23)
    sizes = [1, 2, 33, 1024, 1025, 4099, 7, 70_000]
    pts = rng.random((sum(sizes), 3), dtype=np.float32)
    offsets = torch.tensor(np.concatenate([[0], np.cumsum(sizes)]), dtype=torch.int64, device="cuda")
    pts_t = torch.from_numpy(pts).cuda()
    ragged = torchbvh.build_bvh(pts_t, batch_offsets=offsets)
    for b, handle in enumerate(ragged._handles):
        lo, hi = int(offsets[b]), int(offsets[b + 1])
        single = torchbvh.build_bvh(pts_t[lo:hi].contiguous())
        for key in ("node_aabbs", "sorted_indices", "scene_min", "scene_max", "left_child_mem", "right_child_mem",
                    "mem_to_leaf"):
            assert torch.equal(handle[key], single[key]), (b, key)
        for key in ("num_leaves", "num_real_nodes", "leaf_level", "virtual_leaves", "dim"):
            assert handle[key] == single[key]
    assert torchbvh.device_status() == 0


def test_build_rejects_unsupported_inputs():
    with pytest.raises(ValueError, match="D must be 2 or 3"):
        torchbvh.build_bvh(torch.zeros((4, 4), device="cuda"))
    with pytest.raises(ValueError, match="float32"):
        torchbvh.build_bvh(torch.zeros((4, 2), device="cuda", dtype=torch.float64))


@pytest.mark.parametrize("d", [2, 3])
@pytest.mark.parametrize("n", [1, 5, 4097, 300_001])
def test_unaligned_points_build_the_same_tree(d, n):
    """The bounds and key kernels read points in 128-bit quads when the array
    is 16-byte aligned and point by point otherwise: a view that starts one
    point into its storage (4·D bytes, never 16-byte aligned) must give the
    same tree, box and query order as an aligned copy."""
    g = torch.Generator().manual_seed(500 + d + n)
    base = torch.rand((n + 1, d), generator=g).cuda()
    view = base[1:]
    assert view.data_ptr() % 16 != 0 and view.is_contiguous()
    copy = view.clone()
    assert copy.data_ptr() % 16 == 0
    qbase = torch.rand((n + 1, d), generator=g).cuda()
    a = torchbvh.build_bvh(view)
    b = torchbvh.build_bvh(copy)
    for key in ("node_aabbs", "sorted_indices", "scene_min", "scene_max"):
        assert torch.equal(a[key], b[key]), key
    if n >= 4:
        ia, da = torchbvh.query_knn(a, qbase[1:], 4)
        ib, db = torchbvh.query_knn(b, qbase[1:].clone(), 4)
        assert torch.equal(ia, ib) and torch.equal(da, db)
    assert torchbvh.device_status() == 0


@pytest.mark.parametrize("d", [2, 3])
@pytest.mark.parametrize("n", [1, 7, 100_003])
def test_scene_bounds_alone_equal_the_builds(d, n):
    """tbvh_scene_bounds gives the build's scene box bit for bit (aligned and
    unaligned point arrays)."""
    from torchbvh_b200 import _native

    g = torch.Generator().manual_seed(600 + d + n)
    base = (torch.randn((n + 1, d), generator=g) * 50.0 + 3.0).cuda()
    for pts in (base[1:], base[1:].clone()):
        lo, hi = _native.scene_bounds(pts)
        h = torchbvh.build_bvh(pts)
        assert torch.equal(lo, h["scene_min"]) and torch.equal(hi, h["scene_max"])
