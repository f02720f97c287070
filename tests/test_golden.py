"""Golden vectors from the reference's own CUDA path (tests/golden/reference_cuda.npz,
made by tests/golden/make_golden.py on a B200 from the unmodified reference).

CPU tests pin the oracle: its tree build from the reference's sorted order,
its scene bounds and its restated DFS traversal must reproduce the reference
outputs exactly, ties included. GPU tests pin the B200 path: build outputs
bit-identical (values; -0.0 == +0.0), distances bit-identical, indices
identical except for the order among exactly tied distances.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_cuda.npz"

if not GOLDEN.exists():
    pytest.skip("golden vectors not generated yet (tests/golden/make_golden.py)", allow_module_level=True)

_data = np.load(GOLDEN, allow_pickle=False)
CASES = [str(c) for c in _data["_cases"]]


def _case(name: str) -> dict:
    prefix = f"{name}/"
    out = {key[len(prefix):]: _data[key] for key in _data.files if key.startswith(prefix)}
    if str(out["mode"]) == "workload_c1":
        from torchbvh_b200 import workloads

        w = workloads.c1_single_uniform()
        out["points"] = w.points.numpy()
        out["queries"] = w.queries.numpy()
    return out


def _per_cloud(case: dict):
    pts = case["points"]
    if pts.ndim == 2:
        yield pts, case["queries"], {k: case[k] for k in case}
        return
    for b in range(pts.shape[0]):
        sub = {k: (v[b] if isinstance(v, np.ndarray) and v.ndim >= 2 and v.shape[0] == pts.shape[0]
                   and k not in ("left_child_mem", "right_child_mem", "mem_to_leaf") else v)
               for k, v in case.items()}
        yield pts[b], case["queries"][b], sub


@pytest.mark.parametrize("name", CASES)
def test_oracle_reproduces_reference_build(oracle, name):
    case = _case(name)
    for pts, _, c in _per_cloud(case):
        lo, hi = oracle.scene_bounds(pts)
        np.testing.assert_array_equal(lo, c["scene_min"])
        np.testing.assert_array_equal(hi, c["scene_max"])
        tree = oracle.build_tree(pts, c["sorted_indices"])
        np.testing.assert_array_equal(tree["node_aabbs"], c["node_aabbs"])
        for key in ("left_child_mem", "right_child_mem", "mem_to_leaf"):
            np.testing.assert_array_equal(tree[key], c[key])


@pytest.mark.parametrize("name", CASES)
def test_oracle_morton_order_vs_reference(oracle, name):
    # The oracle divides with IEEE division, the reference with fast-math CUDA
    # division: only points within a few ulp of a cell boundary may differ.
    case = _case(name)
    for pts, _, c in _per_cloud(case):
        lo, hi = oracle.scene_bounds(pts)
        mine = oracle.stable_argsort(oracle.morton_codes(pts, lo, hi))
        mismatched = int(np.count_nonzero(mine != c["sorted_indices"]))
        assert mismatched <= max(4, pts.shape[0] // 200), mismatched


@pytest.mark.parametrize("name", CASES)
def test_oracle_traversal_reproduces_reference_exactly(oracle, name):
    case = _case(name)
    if "indices" not in case:
        pytest.skip("build-only case")
    k = int(case["k"])
    for pts, q, c in _per_cloud(case):
        tree = {"node_aabbs": c["node_aabbs"], "sorted_indices": c["sorted_indices"]}
        idx, dist = oracle.knn_reference(tree, q, k)
        np.testing.assert_array_equal(dist.view(np.uint32), c["distances"].view(np.uint32))
        np.testing.assert_array_equal(idx, c["indices"])
        np.testing.assert_array_equal(c["indices"], c["indices_unsorted"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_b200_build_matches_reference_cuda(name):
    import torchbvh_b200 as torchbvh

    case = _case(name)
    bvh = torchbvh.build_bvh(torch.from_numpy(np.ascontiguousarray(case["points"])).cuda())
    np.testing.assert_array_equal(bvh["sorted_indices"].cpu().numpy(), case["sorted_indices"])
    np.testing.assert_array_equal(bvh["node_aabbs"].cpu().numpy(), case["node_aabbs"])
    np.testing.assert_array_equal(bvh["scene_min"].cpu().numpy(), case["scene_min"])
    np.testing.assert_array_equal(bvh["scene_max"].cpu().numpy(), case["scene_max"])
    for key in ("left_child_mem", "right_child_mem", "mem_to_leaf"):
        np.testing.assert_array_equal(bvh[key].cpu().numpy(), case[key])


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_b200_knn_matches_reference_cuda(oracle, name):
    import torchbvh_b200 as torchbvh

    case = _case(name)
    if "indices" not in case:
        pytest.skip("build-only case")
    k = int(case["k"])
    bvh = torchbvh.build_bvh(torch.from_numpy(np.ascontiguousarray(case["points"])).cuda())
    q = torch.from_numpy(np.ascontiguousarray(case["queries"])).cuda()
    for sort in (True, False):
        idx, dist = torchbvh.query_knn(bvh, q, k, sort_queries=sort)
        ok, msg = oracle.tie_equivalent(idx.cpu().numpy(), dist.cpu().numpy(), case["indices"], case["distances"])
        assert ok, msg
    assert torchbvh.device_status() == 0


def _query_order_case(name: str) -> dict:
    case = _case(name)
    if "query_order" not in case:
        pytest.skip("golden file predates the stored reference query permutation")
    return case


@pytest.mark.parametrize("name", CASES)
def test_oracle_query_order_vs_reference(oracle, name):
    # The reference's own query permutation (_C.morton_sort_queries_narrow,
    # torchbvh/csrc/morton_sort.cu:212-287) against the oracle's stable sort of
    # Morton codes taken with the reference's scene bounds (same ulp caveat as
    # the point order above).
    case = _query_order_case(name)
    q_all = case["queries"]
    orders = case["query_order"]
    lo_all, hi_all = case["scene_min"], case["scene_max"]
    if q_all.ndim == 2:
        q_all, orders, lo_all, hi_all = q_all[None], orders[None], lo_all[None], hi_all[None]
    for q, order, lo, hi in zip(q_all, orders, lo_all, hi_all):
        mine = oracle.stable_argsort(oracle.morton_codes(q, lo, hi))
        mismatched = int(np.count_nonzero(mine != order))
        assert mismatched <= max(4, q.shape[0] // 200), mismatched


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_b200_query_order_matches_reference_cuda(name):
    from torchbvh_b200._native import _C

    case = _query_order_case(name)
    q = torch.from_numpy(np.ascontiguousarray(case["queries"])).cuda()
    lo = torch.from_numpy(case["scene_min"]).cuda()
    hi = torch.from_numpy(case["scene_max"]).cuda()
    if q.dim() == 2:
        got = _C.morton_sort_queries_narrow(q[None], lo[None], hi[None])[0]
    else:
        got = _C.morton_sort_queries_narrow(q, lo, hi)
    np.testing.assert_array_equal(got.cpu().numpy(), case["query_order"])
