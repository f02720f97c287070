"""CPU checks of the oracle itself: pinned against the reference's own headers
(compiled for the host into oracle/_ref) and against the reference's build
invariants and k-NN contracts. No GPU needed."""

from __future__ import annotations

import numpy as np
import pytest

from tests import clouds


@pytest.fixture(scope="module")
def ref(oracle):
    lib = oracle.ref_lib()
    if lib is None:
        try:
            oracle.compile_libs(ref=True)
        except Exception as exc:  # the reference sources are not present on every machine
            pytest.skip(f"reference header shim unavailable: {exc}")
        lib = oracle.ref_lib()
    if lib is None:
        pytest.skip("reference header shim unavailable")
    return lib


def _edge_points(rng, d):
    lo = rng.uniform(-3, 1, size=d).astype(np.float32)
    hi = (lo + rng.uniform(0.5, 4, size=d)).astype(np.float32)
    pts = rng.uniform(lo - 0.5, hi + 0.5, size=(4000, d)).astype(np.float32)
    # exact corners, quantisation boundaries and outside-the-box clamping
    pts[:8] = lo
    pts[8:16] = hi
    bins = 1024 if d == 3 else 65536
    for i in range(16, 400):
        t = (i % bins) / bins
        pts[i] = lo + (hi - lo) * np.float32(t)
    return pts, lo, hi


@pytest.mark.parametrize("d", [2, 3])
def test_oracle_morton_matches_reference_headers(oracle, ref, d):
    rng = np.random.default_rng(100 + d)
    pts, lo, hi = _edge_points(rng, d)
    ours = oracle.morton_codes(pts, lo, hi)
    lo_c = lo.ctypes.data
    hi_c = hi.ctypes.data
    if d == 3:
        theirs = np.array([ref.tbr_morton_encode_3d(*map(float, p), lo_c, hi_c) for p in pts], dtype=np.uint32)
    else:
        theirs = np.array([ref.tbr_morton_encode_2d(*map(float, p), lo_c, hi_c) for p in pts], dtype=np.uint32)
    np.testing.assert_array_equal(ours, theirs)


def test_oracle_morton_degenerate_extent_matches_reference(oracle, ref):
    lo = np.array([1.0, 2.0, 3.0], np.float32)
    hi = np.array([1.0, 5.0, 3.0], np.float32)  # zero extent on x and z
    pts = np.array([[1.0, 2.0, 3.0], [7.0, 4.0, -1.0], [0.0, 5.0, 3.0]], np.float32)
    ours = oracle.morton_codes(pts, lo, hi)
    theirs = [ref.tbr_morton_encode_3d(*map(float, p), lo.ctypes.data, hi.ctypes.data) for p in pts]
    np.testing.assert_array_equal(ours, np.array(theirs, np.uint32))


@pytest.mark.parametrize("n", list(range(1, 140)) + [255, 256, 257, 1000, 1023, 1024, 1025, 4097])
def test_oracle_tree_layout_matches_reference_headers(oracle, ref, n):
    leaf = oracle.leaf_level(n)
    assert leaf == ref.tbr_leaf_level(n)
    assert oracle.real_node_count(n) == ref.tbr_real_node_count(n)
    # Row of (level l, position j) is rowoff(l) + j with rowoff the running sum of
    # ceil(n / 2^(L-l)); it must equal the reference's memory_index of the
    # implicit node 2^l - 1 + j for every real node.
    row = 0
    for level in range(leaf + 1):
        count = ((n - 1) >> (leaf - level)) + 1
        for j in range(1 << level):
            implicit = (1 << level) - 1 + j
            virtual = bool(ref.tbr_is_virtual(n, implicit))
            assert virtual == (j >= count)
            if not virtual:
                assert ref.tbr_memory_index(n, implicit) == row + j
        row += count
    assert row == oracle.real_node_count(n)


def test_oracle_stable_argsort_is_stable(oracle):
    rng = np.random.default_rng(5)
    keys = rng.integers(0, 50, size=10000, dtype=np.uint32)
    np.testing.assert_array_equal(oracle.stable_argsort(keys), np.argsort(keys, kind="stable"))


def _assert_tree_invariants(oracle, pts, tree):
    n, d = pts.shape
    nodes = tree["node_aabbs"]
    sidx = tree["sorted_indices"]
    leaf = tree["leaf_level"]
    assert nodes.shape == (oracle.real_node_count(n), 2 * d)
    np.testing.assert_array_equal(np.sort(sidx), np.arange(n))
    assert np.all(nodes[:, :d] <= nodes[:, d:])
    counts = [((n - 1) >> (leaf - l)) + 1 for l in range(leaf + 1)]
    rowoff = np.concatenate([[0], np.cumsum(counts)])
    np.testing.assert_array_equal(nodes[rowoff[leaf]:rowoff[leaf] + n, :d], pts[sidx])
    np.testing.assert_array_equal(nodes[0, :d], pts.min(axis=0))
    np.testing.assert_array_equal(nodes[0, d:], pts.max(axis=0))
    for level in range(leaf):
        for j in range(counts[level]):
            parent = nodes[rowoff[level] + j]
            kids = [nodes[rowoff[level + 1] + 2 * j]]
            if 2 * j + 1 < counts[level + 1]:
                kids.append(nodes[rowoff[level + 1] + 2 * j + 1])
            kids = np.stack(kids)
            np.testing.assert_array_equal(parent[:d], kids[:, :d].min(axis=0))
            np.testing.assert_array_equal(parent[d:], kids[:, d:].max(axis=0))


@pytest.mark.parametrize("case", clouds.BUILD_CASES, ids=lambda c: c[0])
def test_oracle_build_invariants(oracle, case):
    _, pts = case
    pts = np.asarray(pts, np.float32)
    tree = oracle.build(pts)
    _assert_tree_invariants(oracle, pts, tree)
    lo, hi = oracle.scene_bounds(pts)
    np.testing.assert_array_equal(tree["scene_min"], lo)
    np.testing.assert_array_equal(tree["scene_max"], hi)
    codes = oracle.morton_codes(pts, lo, hi)
    np.testing.assert_array_equal(tree["sorted_indices"], np.argsort(codes, kind="stable"))


@pytest.mark.parametrize("d", [2, 3])
@pytest.mark.parametrize("k", [4, 8, 16, 32])
def test_oracle_reference_traversal_matches_bruteforce(oracle, d, k):
    rng = np.random.default_rng(200 + 10 * d + k)
    pts = rng.random((700, d), dtype=np.float32)
    q = rng.random((300, d), dtype=np.float32)
    tree = oracle.build(pts)
    ri, rd = oracle.knn_reference(tree, q, k)
    bi, bd = oracle.knn_bruteforce(pts, q, k)
    np.testing.assert_array_equal(rd.view(np.uint32), bd.view(np.uint32))
    np.testing.assert_array_equal(ri, bi)  # tie-free random cloud


@pytest.mark.parametrize("d", [2, 3])
@pytest.mark.parametrize("k", [4, 8, 16])
def test_oracle_tie_cases_are_tie_equivalent(oracle, d, k):
    pts, q, expected = clouds.symmetric_tie_cloud(d)
    tree = oracle.build(pts)
    ri, rd = oracle.knn_reference(tree, q, k)
    bi, bd = oracle.knn_bruteforce(pts, q, k)
    ok, msg = oracle.tie_equivalent(ri, rd, bi, bd)
    assert ok, msg
    assert np.all(rd == np.float32(expected))
    assert np.all(bi == np.sort(bi, axis=1))  # canonical order: ties by ascending index


def _fma32(a, b, c):
    # a*b is exact in float64 for float32 inputs; one rounding of the sum in
    # float64 and one to float32 reproduce fmaf for these magnitudes.
    return np.float32(np.float64(a) * np.float64(b) + np.float64(c))


def test_oracle_distance_is_fma_contracted(oracle):
    # d = fma(e2, e2, fma(e1, e1, e0*e0)); these inputs give a different float32
    # than the unfused sum of squares, so the test pins the contraction.
    q = np.array([[0.1244208812713623, 0.45349788665771484, 0.9769059419631958]], np.float32)
    p = np.array([[0.1340416669845581, 0.38331156969070435, 0.4031129479408264]], np.float32)
    _, dist = oracle.knn_bruteforce(np.repeat(p, 4, axis=0), q, 4)
    e = (p[0] - q[0]).astype(np.float32)
    fused = _fma32(e[2], e[2], _fma32(e[1], e[1], np.float32(e[0] * e[0])))
    unfused = np.float32(np.float32(np.float32(e[0] * e[0]) + np.float32(e[1] * e[1])) + np.float32(e[2] * e[2]))
    assert fused != unfused
    assert dist[0, 0] == fused


def test_oracle_far_points_are_never_reported(oracle):
    # A squared distance that overflows float32 never enters the top-k: the
    # reference keeps FLT_MAX / -1 in such slots (knn_query.cu:13,85-88,101).
    pts = np.array([[0.0, 0.0], [1.0, 0.0], [0.0, 1.0], [1.0e20, 1.0e20]], np.float32)
    q = np.array([[0.25, 0.25]], np.float32)
    tree = oracle.build(pts)
    ri, rd = oracle.knn_reference(tree, q, 4)
    bi, bd = oracle.knn_bruteforce(pts, q, 4)
    assert ri[0, 3] == -1 and rd[0, 3] == np.finfo(np.float32).max
    np.testing.assert_array_equal(ri, bi)
    np.testing.assert_array_equal(rd, bd)
