"""k-NN parity on the GPU: the CUDA path through the C ABI against the CPU
oracle on the same seeded inputs.

Bar: distances bit-identical to the oracle (same float32 arithmetic as the
reference kernel); indices identical to the canonical brute force, which
orders exact ties by source index; identical to the reference's own traversal
(restated in the oracle) except for the order among exactly tied distances.
Case list follows tests/test_knn.py of the reference.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import torchbvh_b200 as torchbvh
from tests import clouds

pytestmark = pytest.mark.gpu


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def _gpu_knn(points: np.ndarray, queries: np.ndarray, k: int, **kw):
    p = torch.from_numpy(np.ascontiguousarray(points, np.float32)).cuda()
    q = torch.from_numpy(np.ascontiguousarray(queries, np.float32)).cuda()
    bvh = torchbvh.build_bvh(p)
    idx, dist = torchbvh.query_knn(bvh, q, k, **kw)
    assert torchbvh.device_status() == 0
    return bvh, _np(idx), _np(dist)


def _assert_exact(oracle, points, queries, k, idx, dist, tree=None):
    bi, bd = oracle.knn_bruteforce(points, queries, k)
    np.testing.assert_array_equal(dist.view(np.uint32), bd.view(np.uint32))
    np.testing.assert_array_equal(idx, bi)
    np.testing.assert_array_equal(oracle.pair_distances(points, queries, idx).view(np.uint32), dist.view(np.uint32))
    if tree is not None:
        ri, rd = oracle.knn_reference(tree, queries, k)
        ok, msg = oracle.tie_equivalent(idx, dist, ri, rd)
        assert ok, msg


def _tree_np(bvh) -> dict:
    return {"node_aabbs": _np(bvh["node_aabbs"]), "sorted_indices": _np(bvh["sorted_indices"])}


@pytest.mark.parametrize("d", [2, 3])
@pytest.mark.parametrize("k", [4, 8, 16, 32])
@pytest.mark.parametrize("n", [32, 33, 64, 1000, 4097])
def test_random_clouds_match_oracle(oracle, d, k, n):
    rng = np.random.default_rng(1000 + 100 * d + k + n)
    pts = rng.random((n, d), dtype=np.float32)
    q = rng.random((257, d), dtype=np.float32)
    bvh, idx, dist = _gpu_knn(pts, q, k)
    _assert_exact(oracle, pts, q, k, idx, dist, _tree_np(bvh))


@pytest.mark.parametrize("d", [2, 3])
@pytest.mark.parametrize("k", [4, 8, 16])
def test_self_query_returns_self_first(oracle, d, k):
    rng = np.random.default_rng(2000 + d * 10 + k)
    pts = rng.random((48, d), dtype=np.float32)
    _, idx, dist = _gpu_knn(pts, pts, k)
    _assert_exact(oracle, pts, pts, k, idx, dist)
    assert np.all(dist[:, 0] == 0.0)
    np.testing.assert_array_equal(idx[:, 0], np.arange(48))


@pytest.mark.parametrize("n", [4, 5, 8, 17, 31])
@pytest.mark.parametrize("k", [4])
def test_tiny_clouds(oracle, n, k):
    rng = np.random.default_rng(n)
    pts = rng.random((n, 3), dtype=np.float32)
    q = rng.random((40, 3), dtype=np.float32)
    _, idx, dist = _gpu_knn(pts, q, k)
    _assert_exact(oracle, pts, q, k, idx, dist)


@pytest.mark.parametrize("case", clouds.knn_pathological_cases(), ids=lambda c: c[0])
def test_pathological_clouds(oracle, case):
    _, pts, k = case
    q = pts[: min(7, pts.shape[0])] + np.float32(0.125)
    bvh, idx, dist = _gpu_knn(pts, q, k)
    _assert_exact(oracle, pts, q, k, idx, dist, _tree_np(bvh))


@pytest.mark.parametrize("d", [2, 3])
@pytest.mark.parametrize("k", [4, 8, 16])
def test_true_ties_are_canonical_and_tie_equivalent_to_reference(oracle, d, k):
    pts, q, expected = clouds.symmetric_tie_cloud(d)
    bvh, idx, dist = _gpu_knn(pts, q, k)
    _assert_exact(oracle, pts, q, k, idx, dist, _tree_np(bvh))
    assert np.all(dist == np.float32(expected))


@pytest.mark.parametrize("d", [2, 3])
@pytest.mark.parametrize("k", [4, 8, 16])
def test_all_duplicate_cloud(oracle, d, k):
    pts = np.full((20, d), 3.5, np.float32)
    q = np.full((3, d), 3.5, np.float32)
    _, idx, dist = _gpu_knn(pts, q, k)
    _assert_exact(oracle, pts, q, k, idx, dist)
    assert np.all(dist == 0.0)


@pytest.mark.parametrize("d", [2, 3])
@pytest.mark.parametrize("k", [4, 8, 16, 32])
def test_robust_matrix_with_ties_duplicates_outliers(oracle, d, k):
    rng = np.random.default_rng(2400 + d * 100 + k)
    random_points = rng.random((96, d), dtype=np.float32) * 2 - 1
    tie_block = np.zeros((k + 2, d), np.float32)
    dup = np.full((2, d), 0.25, np.float32)
    out = np.zeros((2, d), np.float32)
    out[0, 0], out[1, 0] = 50.0, -50.0
    out[:, 1] = [30.0, -30.0]
    pts = np.concatenate([random_points, tie_block, dup, out])
    disp = np.linspace(0.015, 0.045, d, dtype=np.float32)
    q = np.concatenate([pts[:19], pts[19:38] + disp, np.zeros((5, d), np.float32), out + 0.1 * disp,
                        rng.random((17, d), dtype=np.float32) * 2 - 1])
    bvh, idx, dist = _gpu_knn(pts, q, k)
    _assert_exact(oracle, pts, q, k, idx, dist, _tree_np(bvh))


def test_far_points_keep_reference_sentinels(oracle):
    pts = np.array([[0.0, 0.0], [1.0, 0.0], [0.0, 1.0], [1.0e20, 1.0e20]], np.float32)
    q = np.array([[0.25, 0.25]], np.float32)
    _, idx, dist = _gpu_knn(pts, q, 4)
    assert idx[0, 3] == -1 and dist[0, 3] == np.finfo(np.float32).max
    _assert_exact(oracle, pts, q, 4, idx, dist)


@pytest.mark.parametrize("d", [2, 3])
@pytest.mark.parametrize("k", [4, 8, 16, 32])
def test_sorted_and_unsorted_paths_agree(d, k):
    rng = np.random.default_rng(3100 + d * 10 + k)
    pts = torch.from_numpy(rng.random((257, d), dtype=np.float32)).cuda()
    q = torch.from_numpy(rng.random((123, d), dtype=np.float32)).cuda()
    bvh = torchbvh.build_bvh(pts)
    i0, d0 = torchbvh.query_knn(bvh, q, k, sort_queries=False)
    i1, d1 = torchbvh.query_knn(bvh, q, k, sort_queries=True)
    i2, d2 = torchbvh.query_knn(bvh, q, k)
    assert torch.equal(i0, i1) and torch.equal(i1, i2)
    assert torch.equal(d0, d1) and torch.equal(d1, d2)


def test_queries_far_outside_the_scene(oracle):
    rng = np.random.default_rng(9)
    pts = rng.random((3000, 3), dtype=np.float32)
    q = np.concatenate([rng.random((50, 3), dtype=np.float32) * 40 - 20, np.array([[1e6, -1e6, 3e5]], np.float32)])
    _, idx, dist = _gpu_knn(pts, q, 16)
    _assert_exact(oracle, pts, q, 16, idx, dist)


def test_many_queries_multiple_blocks(oracle):
    rng = np.random.default_rng(11)
    pts = rng.random((20000, 3), dtype=np.float32)
    q = rng.random((5000, 3), dtype=np.float32)
    bvh, idx, dist = _gpu_knn(pts, q, 8)
    _assert_exact(oracle, pts, q, 8, idx, dist, _tree_np(bvh))
