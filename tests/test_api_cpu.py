"""Host-side API logic that needs no GPU: constants, public surface, handle
lifecycle, dispatch errors and input validation raised before any native
call (messages as in the reference's _validation.py / _query.py)."""

from __future__ import annotations

import pytest
import torch

import torchbvh_b200 as torchbvh
from torchbvh_b200 import _handles, _validation


def test_constants_and_surface():
    assert torchbvh.SUPPORTED_K == (4, 8, 16, 32)
    assert torchbvh.SUPPORTED_DIMS == (2, 3)
    for name in ("BVH", "build_bvh", "query_knn", "destroy_bvh", "BVHHandle", "BatchedBVHHandle",
                 "RaggedBVHHandle", "SUPPORTED_K", "SUPPORTED_DIMS"):
        assert name in torchbvh.__all__ and hasattr(torchbvh, name)


def test_handle_mapping_and_destroy():
    h = torchbvh.BVHHandle({"dim": 3, "num_leaves": 5})
    assert h["dim"] == 3 and len(h) == 2 and set(h) == {"dim", "num_leaves"}
    torchbvh.destroy_bvh(h)
    assert h.destroyed
    torchbvh.destroy_bvh(h)
    with pytest.raises(RuntimeError, match="destroyed"):
        _ = h["dim"]


def test_batched_handle_marker_and_message():
    h = torchbvh.BatchedBVHHandle({"batch_size": 2})
    assert h["_batched"] is True
    h.destroy()
    with pytest.raises(RuntimeError, match="Batched BVH handle has been destroyed"):
        len(h)


def test_lazy_ragged_sample_handles_and_cascade():
    built = []

    def factory(b):
        def make():
            built.append(b)
            return {"num_leaves": 10 + b}
        return make

    inner = [_handles._LazyBVHHandle(factory(b)) for b in range(3)]
    ragged = torchbvh.RaggedBVHHandle({"batch_size": 3}, inner, {"dim": 3})
    assert built == []
    assert inner[2]["num_leaves"] == 12 and built == [2]
    assert ragged["_ragged"] is True
    torchbvh.destroy_bvh(ragged)
    assert ragged.destroyed and all(h.destroyed for h in inner)
    with pytest.raises(RuntimeError, match="Ragged BVH handle has been destroyed"):
        _ = ragged["batch_size"]


def test_query_knn_rejects_foreign_handles():
    with pytest.raises(TypeError, match="BVHHandle"):
        torchbvh.query_knn(object(), torch.empty((4, 2)), 4)
    with pytest.raises(TypeError, match="query_offsets requires a RaggedBVHHandle"):
        torchbvh.query_knn(torchbvh.BVHHandle({}), torch.empty((4, 2)), 4, query_offsets=torch.zeros(2))
    with pytest.raises(TypeError, match="handle returned by build_bvh"):
        torchbvh.destroy_bvh({"dim": 3})


def test_unsupported_k_message_keeps_reference_text():
    with pytest.raises(ValueError, match="k must be 4, 8, or 16"):
        _validation._validate_supported_k("query_knn", 5)
    _validation._validate_supported_k("query_knn", 32)


@pytest.mark.parametrize("points,match", [
    (torch.zeros((4, 4)), "D must be 2 or 3"),
    (torch.zeros((4, 2), dtype=torch.float64), "CUDA tensor"),
    (torch.zeros((4, 2)), "CUDA tensor"),
    (torch.zeros((2, 2, 2, 2)), "shape"),
])
def test_build_validation_before_native(points, match):
    with pytest.raises(ValueError, match=match):
        torchbvh.build_bvh(points)


def test_ragged_build_requires_2d_points():
    with pytest.raises(ValueError, match="ragged mode requires 2-D points"):
        torchbvh.build_bvh(torch.zeros((1, 8, 2)), batch_offsets=torch.tensor([0, 8]))


def test_offset_value_validation():
    with pytest.raises(ValueError, match="start at 0"):
        _validation._validate_offset_values("build_bvh", [1, 4, 8], 8)
    with pytest.raises(ValueError, match="final offset"):
        _validation._validate_offset_values("build_bvh", [0, 4, 7], 8)
    with pytest.raises(ValueError, match="strictly increasing"):
        _validation._validate_offset_values("build_bvh", [0, 8, 8], 8)
    assert _validation._validate_offset_values("build_bvh", [0, 4, 8], 8) == [0, 4, 8]


def test_offsets_validation_on_cpu_tensor():
    with pytest.raises(ValueError, match="must be a CUDA tensor"):
        _validation._validate_offsets("build_bvh", torch.tensor([0, 4, 8]), total_rows=8,
                                      device=torch.device("cpu"))
    with pytest.raises(ValueError, match="int64"):
        _validation._validate_offsets("build_bvh", torch.tensor([0, 4, 8], dtype=torch.int32), total_rows=8,
                                      device=torch.device("cpu"))


def test_workload_generators_are_seeded():
    from torchbvh_b200 import workloads

    a = workloads.make("c1")
    b = workloads.make("c1")
    assert torch.equal(a.points, b.points) and torch.equal(a.queries, b.queries)
    assert a.points.shape == (10_000, 3) and a.k == 4
    r = workloads.make("c5", clouds=8, lo=1024, hi=4096)
    sizes = r.cloud_sizes()
    assert len(sizes) == 8 and all(1024 <= s <= 4096 for s in sizes)
    assert torch.equal(r.points, r.queries)


@pytest.mark.parametrize(
    "pos_shape,q_shape,match",
    [
        ((24, 3), (2, 24, 3, 3), "pos.*shape"),
        ((2, 24, 3), (2, 72, 3), "q.*shape"),
        ((2, 24, 4), (2, 24, 3, 4), "D must be 2 or 3"),
        ((1, 24, 3), (2, 24, 3, 3), "batch size"),
        ((2, 24, 3), (2, 3, 3, 3), "point dimension"),
        ((2, 24, 3), (2, 24, 3, 2), "last dimension"),
        ((2, 24, 3), (2, 24, 0, 3), "at least one head"),
        ((2, 24, 3), (2, 24, 3, 3), "CUDA tensor"),
    ],
)
def test_displaced_validation_order_and_messages(pos_shape, q_shape, match):
    with pytest.raises(ValueError, match=match):
        torchbvh.query_displaced_knn(torch.zeros(pos_shape), torch.zeros(q_shape), 4)


def test_interpolate_displaced_rejects_unknown_reduction_first():
    with pytest.raises(ValueError, match="reduction must be 'weighted_mean'"):
        torchbvh.interpolate_displaced(torch.zeros(1), torch.zeros(1), torch.zeros(1), 4, reduction="mean")


def test_gather_neighbor_values_shape_checks_on_cpu():
    values = torch.zeros((2, 6, 3, 4))
    with pytest.raises(ValueError, match="values must have shape"):
        torchbvh.gather_neighbor_values(values[0], torch.zeros((2, 6, 3, 2), dtype=torch.int64))
    with pytest.raises(ValueError, match="head dimension"):
        torchbvh.gather_neighbor_values(values, torch.zeros((2, 6, 2, 2), dtype=torch.int64))
    with pytest.raises(ValueError, match="values must be a CUDA tensor"):
        torchbvh.gather_neighbor_values(values, torch.zeros((2, 6, 3, 2), dtype=torch.int64))


def test_package_surface_matches_the_reference_knn_exports():
    # torchbvh/__init__.py exports BVH but no BatchedBVH / RaggedBVH classes, and its
    # k-NN workflows and constants by these names.
    assert hasattr(torchbvh, "BVH") and "BVH" in torchbvh.__all__
    for absent in ("BatchedBVH", "RaggedBVH"):
        assert not hasattr(torchbvh, absent) and absent not in torchbvh.__all__
    for name in ("BVHHandle", "BatchedBVHHandle", "RaggedBVHHandle", "build_bvh", "destroy_bvh", "query_knn",
                 "query_displaced_knn", "gather_neighbor_values", "interpolate_displaced", "SUPPORTED_K",
                 "SUPPORTED_DIMS"):
        assert name in torchbvh.__all__ and hasattr(torchbvh, name)


def test_bvh_class_is_not_a_mapping():
    assert not hasattr(torchbvh.BVH, "__getitem__")
    for method in ("knn", "destroy", "__enter__", "__exit__"):
        assert callable(getattr(torchbvh.BVH, method))


def test_out_pair_checks_on_cpu():
    """``knn(..., out=...)`` argument rules (checked before any device work)."""
    from torchbvh_b200._query import _checked_out

    dev = torch.device("cuda", 0)
    assert _checked_out(None, (5, 4), dev, None) is None
    cpu_pair = (torch.empty((5, 4), dtype=torch.int64), torch.empty((5, 4)))
    with pytest.raises(ValueError, match="pinned host memory"):
        _checked_out(cpu_pair, (5, 4), dev, None)
    with pytest.raises(ValueError, match="must be a pair"):
        _checked_out(cpu_pair[0], (5, 4), dev, None)
    with pytest.raises(ValueError, match="shape"):
        _checked_out(cpu_pair, (5, 8), dev, None)
    with pytest.raises(ValueError, match="indices must be a torch.int64"):
        _checked_out((cpu_pair[1], cpu_pair[1]), (5, 4), dev, None)
    with pytest.raises(ValueError, match="contiguous"):
        _checked_out((torch.empty((4, 5), dtype=torch.int64).t(), cpu_pair[1]), (5, 4), dev, None)
    with pytest.raises(ValueError, match="source_points"):
        _checked_out(cpu_pair, (5, 4), dev, torch.zeros(1))


def test_shared_buffer_views_cover_every_wire_dtype():
    """PeerResults views its IPC buffers as int64 / int32 indices and float32
    distances; each needs an array-interface type string of the right width."""
    from torchbvh_b200 import _native

    for dtype in (torch.int64, torch.int32, torch.float32):
        typestr = _native._TYPESTR[dtype]
        assert int(typestr[2:]) == torch.empty((), dtype=dtype).element_size()


def test_peer_results_rejects_bad_options_before_any_collective():
    from torchbvh_b200 import distributed as tdist

    with pytest.raises(ValueError, match="index_bits"):
        tdist.PeerResults(10, 4, index_bits=16)
    with pytest.raises(ValueError, match="transport"):
        tdist.PeerResults(10, 4, transport="nvshmem")
    with pytest.raises(ValueError, match="int32 indices"):
        tdist.PeerResults(10, 4, index_bits=64, transport="multicast")
