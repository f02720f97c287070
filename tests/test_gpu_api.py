"""Public API contracts on the GPU (ports tests/test_python_api.py,
tests/test_bvh_class.py, tests/test_batched_python_api.py,
tests/test_ragged_python_api.py and tests/test_noncontiguous_public_api.py of
the reference, k-NN surface)."""

from __future__ import annotations

import pytest
import torch

import torchbvh_b200 as torchbvh
import torchbvh_b200._query as query_module
from torchbvh_b200 import BVH

pytestmark = pytest.mark.gpu


def _offsets(values):
    return torch.tensor(values, device="cuda", dtype=torch.int64)


def _make_points(n=20, dim=3):
    base = torch.linspace(-1.0, 1.0, n, device="cuda")
    if dim == 2:
        return torch.stack((base, base.square() - 0.25), dim=1).contiguous()
    return torch.stack((base, base.square() - 0.25, torch.sin(2.0 * base)), dim=1).contiguous()


@pytest.mark.parametrize("dim", [2, 3])
def test_build_query_destroy_lifecycle(dim):
    torch.manual_seed(7000 + dim)
    points = torch.rand((24, dim), device="cuda")
    queries = points[:6] + 0.01
    bvh = torchbvh.build_bvh(points)
    assert isinstance(bvh, torchbvh.BVHHandle) and not bvh.destroyed and bvh["dim"] == dim
    idx, dist = torchbvh.query_knn(bvh, queries, 4)
    expected = torch.cdist(queries, points, compute_mode="donot_use_mm_for_euclid_dist").square()
    torch.testing.assert_close(dist, expected.topk(4, largest=False).values, rtol=1e-5, atol=1e-5)
    torchbvh.destroy_bvh(bvh)
    assert bvh.destroyed
    with pytest.raises(RuntimeError, match="destroyed"):
        torchbvh.query_knn(bvh, queries, 4)
    with pytest.raises(RuntimeError, match="destroyed"):
        _ = bvh["dim"]


def test_rejects_unsupported_k_with_public_message():
    points = torch.rand((8, 2), device="cuda")
    bvh = torchbvh.build_bvh(points)
    with pytest.raises(ValueError, match="k must be 4, 8, or 16"):
        torchbvh.query_knn(bvh, points, 5)


def test_k32_is_supported():
    points = torch.rand((64, 3), device="cuda")
    idx, dist = torchbvh.query_knn(torchbvh.build_bvh(points), points, 32)
    assert idx.shape == (64, 32)
    assert torch.all(dist[:, :-1] <= dist[:, 1:])


def test_rejects_plain_mapping():
    points = torch.rand((16, 3), device="cuda")
    bvh = torchbvh.build_bvh(points)
    with pytest.raises(TypeError, match="BVHHandle"):
        torchbvh.query_knn(dict(bvh), points[:3].contiguous(), 4)
    with pytest.raises(TypeError, match="handle returned by build_bvh"):
        torchbvh.destroy_bvh(dict(bvh))
    assert not bvh.destroyed


def test_sort_queries_true_uses_ordered_traversal(monkeypatch):
    points = torch.rand((16, 3), device="cuda").contiguous()
    queries = points[:5].contiguous()
    bvh = torchbvh.build_bvh(points)
    calls = []

    def fake_sort(query_batch, scene_min, scene_max):
        calls.append(("sort", query_batch.shape, scene_min.shape, scene_max.shape))
        b, m, _ = query_batch.shape
        return torch.arange(m, device=query_batch.device, dtype=torch.int64).expand(b, m).contiguous()

    def fake_ordered(*args):
        calls.append(("ordered", args[2].shape, args[3].shape, args[-1]))
        b, m, _ = args[2].shape
        k = int(args[-1])
        return (torch.zeros((b, m, k), device="cuda", dtype=torch.int64),
                torch.zeros((b, m, k), device="cuda", dtype=torch.float32))

    def fake_unordered(*args):
        raise AssertionError("unordered route must not be used when sort_queries=True")

    monkeypatch.setattr(query_module._C, "morton_sort_queries_narrow", fake_sort)
    monkeypatch.setattr(query_module._C, "query_knn_batched_cached_bounds_ordered", fake_ordered)
    monkeypatch.setattr(query_module._C, "query_knn_batched_cached_bounds", fake_unordered)
    idx, dist = torchbvh.query_knn(bvh, queries, 4, sort_queries=True)
    assert idx.shape == (5, 4) and dist.shape == (5, 4)
    assert [c[0] for c in calls] == ["sort", "ordered"]
    assert calls[0][1] == (1, 5, 3) and calls[1][1] == (1, 5, 3) and calls[1][2] == (1, 5) and calls[1][3] == 4


def test_handles_have_traversal_fields():
    points = torch.rand((16, 3), device="cuda")
    for bvh in (torchbvh.build_bvh(points), torchbvh.build_bvh(torch.rand((2, 16, 3), device="cuda"))):
        for key in ("left_child_mem", "right_child_mem", "mem_to_leaf"):
            assert key in bvh and bvh[key].dtype == torch.int32


def test_bvh_class_lifecycle_and_delegation():
    points = _make_points(20, 3)
    queries = points[3:8] + 0.02
    with BVH(points) as bvh:
        assert not bvh.destroyed and not hasattr(bvh, "__getitem__")
        i_cls, d_cls, p_cls = bvh.knn(queries, 4, source_points=points)
    assert bvh.destroyed
    with pytest.raises(RuntimeError):
        bvh.knn(points[:3], k=4)
    bvh.destroy()  # idempotent
    handle = torchbvh.build_bvh(points)
    i_fn, d_fn, p_fn = torchbvh.query_knn(handle, queries, 4, source_points=points)
    assert torch.equal(i_cls, i_fn) and torch.equal(d_cls, d_fn) and torch.equal(p_cls, p_fn)


def test_batched_class_and_ragged_class():
    pts = _make_points().unsqueeze(0).expand(2, -1, -1).contiguous()
    with BVH(pts) as bvh:
        i_cls, d_cls = bvh.knn((pts[:, 3:8] + 0.02).contiguous(), 4)
    handle = torchbvh.build_bvh(pts)
    i_fn, d_fn = torchbvh.query_knn(handle, (pts[:, 3:8] + 0.02).contiguous(), 4)
    assert torch.equal(i_cls, i_fn) and torch.equal(d_cls, d_fn)
    ragged = BVH(_make_points(20), batch_offsets=_offsets([0, 10, 20]))
    idx, dist = ragged.knn(_make_points(20), 4, query_offsets=_offsets([0, 10, 20]))
    assert idx.shape == (20, 4) and torch.all(dist[:, 0] == 0)
    ragged.destroy()
    assert ragged.destroyed


def test_batched_lifecycle_and_validation():
    torch.manual_seed(13001)
    points = torch.rand((3, 17, 3), device="cuda")
    queries = torch.rand((3, 5, 3), device="cuda")
    bvh = torchbvh.build_bvh(points)
    assert isinstance(bvh, torchbvh.BatchedBVHHandle)
    assert bvh["batch_size"] == 3 and bvh["num_leaves"] == 17 and bvh["dim"] == 3
    assert bvh["node_aabbs"].shape == (3, bvh["num_real_nodes"], 6)
    assert bvh["sorted_indices"].shape == (3, 17) and bvh["scene_min"].shape == (3, 3)
    idx, dist, pos = torchbvh.query_knn(bvh, queries, 4, source_points=points)
    assert idx.shape == (3, 5, 4) and pos.shape == (3, 5, 4, 3)
    for bad, match in [(queries[0], "shape"), (queries[:1], "batch size"),
                       (torch.rand((3, 4, 2), device="cuda"), "last dimension"), (queries.double(), "float32")]:
        with pytest.raises((ValueError, RuntimeError), match=match):
            torchbvh.query_knn(bvh, bad, 4)
    with pytest.raises(ValueError, match="shape"):
        torchbvh.query_knn(torchbvh.build_bvh(points[0].contiguous()), queries, 4)
    with pytest.raises(ValueError, match="CUDA"):
        torchbvh.build_bvh(points.cpu())
    torchbvh.destroy_bvh(bvh)
    with pytest.raises(RuntimeError, match="destroyed"):
        torchbvh.query_knn(bvh, queries, 4)


def test_ragged_lifecycle_validation_and_cascade_destroy():
    torch.manual_seed(14001)
    counts, qcounts = [9, 17, 12], [4, 7, 5]
    points = torch.cat([torch.rand((c, 3), device="cuda") + 10.0 * b for b, c in enumerate(counts)])
    queries = torch.cat([torch.rand((c, 3), device="cuda") + 10.0 * b for b, c in enumerate(qcounts)])
    bo, qo = _offsets([0, 9, 26, 38]), _offsets([0, 4, 11, 16])
    bvh = torchbvh.build_bvh(points, batch_offsets=bo)
    assert isinstance(bvh, torchbvh.RaggedBVHHandle)
    assert bvh["batch_size"] == 3 and bvh["dim"] == 3
    assert torch.equal(bvh["batch_offsets"], bo)
    assert torch.equal(bvh["num_leaves_per_sample"], torch.tensor(counts, device="cuda"))
    idx, dist, pos = torchbvh.query_knn(bvh, queries, 4, query_offsets=qo, source_points=points)
    assert idx.shape == (16, 4) and pos.shape == (16, 4, 3)
    for b, c in enumerate(counts):
        q0, q1 = int(qo[b]), int(qo[b + 1])
        assert int(idx[q0:q1].min()) >= 0 and int(idx[q0:q1].max()) < c
    inner = list(bvh._handles)
    assert len(inner) == 3 and all(not h.destroyed for h in inner)
    assert inner[1]["num_leaves"] == 17
    torchbvh.destroy_bvh(bvh)
    assert bvh.destroyed and all(h.destroyed for h in inner)
    torchbvh.destroy_bvh(bvh)
    with pytest.raises(RuntimeError, match="destroyed"):
        torchbvh.query_knn(bvh, queries, 4, query_offsets=qo)


@pytest.mark.parametrize("bad,match", [
    (lambda o: o.view(1, -1), "shape"),
    (lambda o: o.to(torch.int32), "int64"),
    (lambda o: o.cpu(), "CUDA"),
    (lambda o: _offsets([1, 4, 8]), "start at 0"),
    (lambda o: _offsets([0, 4, 7]), "final offset"),
    (lambda o: _offsets([0, 8, 8]), "strictly increasing"),
])
def test_ragged_build_rejects_bad_offsets(bad, match):
    points = torch.rand((8, 2), device="cuda")
    with pytest.raises(ValueError, match=match):
        torchbvh.build_bvh(points, batch_offsets=bad(_offsets([0, 4, 8])))


def test_ragged_query_rejections():
    points = torch.rand((11, 2), device="cuda")
    queries = torch.rand((8, 2), device="cuda")
    bvh = torchbvh.build_bvh(points, batch_offsets=_offsets([0, 3, 11]))
    with pytest.raises(ValueError, match="k must be 4, 8, or 16"):
        torchbvh.query_knn(bvh, queries, 5, query_offsets=_offsets([0, 4, 8]))
    with pytest.raises(ValueError, match="batch size"):
        torchbvh.query_knn(bvh, queries, 4, query_offsets=_offsets([0, 2, 5, 8]))
    with pytest.raises(ValueError, match="at least k"):
        torchbvh.query_knn(bvh, queries, 4, query_offsets=_offsets([0, 4, 8]))
    with pytest.raises(ValueError, match="query_offsets is required"):
        torchbvh.query_knn(bvh, queries, 4)
    single = torchbvh.build_bvh(points)
    with pytest.raises(TypeError, match="RaggedBVHHandle"):
        torchbvh.query_knn(single, queries, 4, query_offsets=_offsets([0, 8]))


def _noncontiguous(shape, fill=None):
    storage = torch.empty((*shape[:-1], shape[-1] + 1), device="cuda")
    view = storage[..., : shape[-1]]
    view.copy_(torch.randn(shape, device="cuda") if fill is None else fill)
    assert not view.is_contiguous()
    return view


def test_noncontiguous_inputs_match_contiguous():
    points = _noncontiguous((32, 3))
    queries = _noncontiguous((7, 3), fill=points[:7] + 0.01)
    actual = torchbvh.query_knn(torchbvh.build_bvh(points), queries, 4, source_points=points)
    expected = torchbvh.query_knn(torchbvh.build_bvh(points.contiguous()), queries.contiguous(), 4,
                                  source_points=points.contiguous())
    for a, e in zip(actual, expected):
        assert torch.equal(a, e)
    bpoints = _noncontiguous((2, 32, 3))
    bqueries = _noncontiguous((2, 7, 3), fill=bpoints[:, :7] + 0.01)
    actual = torchbvh.query_knn(torchbvh.build_bvh(bpoints), bqueries, 4, source_points=bpoints)
    expected = torchbvh.query_knn(torchbvh.build_bvh(bpoints.contiguous()), bqueries.contiguous(), 4,
                                  source_points=bpoints.contiguous())
    for a, e in zip(actual, expected):
        assert torch.equal(a, e)


def test_native_functions_reject_bad_arguments():
    from torchbvh_b200._native import _C

    points = torch.rand((1, 16, 3), device="cuda")
    data = _C.build_bvh_batched_cooperative(points)
    with pytest.raises(RuntimeError, match="num_leaves must be >= k"):
        _C.query_knn_batched_cached_bounds(data["node_aabbs"], data["sorted_indices"], points, 16,
                                           data["num_real_nodes"], 3, 32)
    with pytest.raises(RuntimeError, match="node_aabbs has incompatible shape"):
        _C.query_knn_batched_cached_bounds(data["node_aabbs"][:, :-1].contiguous(), data["sorted_indices"], points,
                                           16, data["num_real_nodes"], 3, 4)
    with pytest.raises(RuntimeError, match="points must be contiguous CUDA float32"):
        _C.build_bvh_batched_cooperative(points.double())
