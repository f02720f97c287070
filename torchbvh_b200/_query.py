"""Build and query orchestration (torchbvh/_query.py:29-405, same contracts).

Single and fixed-size batched calls go through the reference-named ``_C``
functions exactly like the reference (single = batched with B = 1, then the
batch dimension is squeezed). Ragged calls differ in mechanism only: the
reference loops over samples in Python (one build and one query per sample,
then ``torch.cat``); here every sample is built and queried in one native
launch sequence over the packed tensors. Public results, shapes, local
indices and error messages are unchanged.
"""

from __future__ import annotations

from collections.abc import Mapping

import torch

from ._constants import SUPPORTED_DIMS
from ._handles import (
    BVHHandle,
    BatchedBVHHandle,
    RaggedBVHHandle,
    _LazyBVHHandle,
    _batched_bvh_data,
    _bvh_data,
    _ragged_bvh_data,
)
from ._native import _C
from ._validation import (
    _as_contiguous,
    _as_contiguous_int64,
    _validate_cuda_float32,
    _validate_offsets,
    _validate_ragged_points,
    _validate_supported_k,
)

_INT32_MAX = 2**31 - 1


def _validate_narrow_build_extent(prefix: str, points: torch.Tensor) -> None:
    # Indices and sort values are 32-bit inside the native path (as in the reference).
    total = int(points.size(0)) if points.dim() == 2 else int(points.size(0)) * int(points.size(1))
    if total > _INT32_MAX:
        raise ValueError(f"{prefix}: total point count must fit in signed int32")


# ---------------------------------------------------------------------------
# Builders
# ---------------------------------------------------------------------------

def _build_bvh_single(points: torch.Tensor) -> BVHHandle:
    if points.dim() != 2:
        raise ValueError("build_bvh: points must have shape (N, D)")
    if points.size(1) not in SUPPORTED_DIMS:
        raise ValueError("build_bvh: D must be 2 or 3")
    _validate_cuda_float32("build_bvh", points, "points")
    points = _as_contiguous(points)
    _validate_narrow_build_extent("build_bvh", points)
    data = dict(_C.build_bvh_batched_cooperative(points.unsqueeze(0)))
    data.pop("batch_size")
    for key in ("node_aabbs", "sorted_indices", "scene_min", "scene_max"):
        data[key] = data[key].squeeze(0)
    return BVHHandle(data)


def _build_bvh_batched(points: torch.Tensor) -> BatchedBVHHandle:
    if points.dim() != 3:
        raise ValueError("build_bvh: batched points must have shape (B, N, D)")
    if points.size(2) not in SUPPORTED_DIMS:
        raise ValueError("build_bvh: D must be 2 or 3")
    _validate_cuda_float32("build_bvh", points, "points")
    points = _as_contiguous(points)
    _validate_narrow_build_extent("build_bvh", points)
    return BatchedBVHHandle(_C.build_bvh_batched_cooperative(points))


def _sample_payload(packed: Mapping, batch: int) -> dict:
    """Per-sample BVHHandle payload as views into the packed ragged build."""
    p0, p1 = packed["point_offsets"][batch], packed["point_offsets"][batch + 1]
    r0, r1 = packed["row_offsets"][batch], packed["row_offsets"][batch + 1]
    n = p1 - p0
    leaf_level = (n - 1).bit_length()
    return {
        "node_aabbs": packed["node_aabbs"][r0:r1],
        "sorted_indices": packed["sorted_indices"][p0:p1],
        "scene_min": packed["scene_min"][batch],
        "scene_max": packed["scene_max"][batch],
        "num_leaves": n,
        "num_real_nodes": r1 - r0,
        "leaf_level": leaf_level,
        "virtual_leaves": (1 << leaf_level) - n,
        "dim": packed["dim"],
        "left_child_mem": packed["left_child_mem"][r0:r1],
        "right_child_mem": packed["right_child_mem"][r0:r1],
        "mem_to_leaf": packed["mem_to_leaf"][r0:r1],
    }


def _build_bvh_ragged(points: torch.Tensor, batch_offsets: torch.Tensor) -> RaggedBVHHandle:
    points = _as_contiguous(points)
    batch_offsets = _as_contiguous_int64(batch_offsets)
    offsets = _validate_ragged_points("build_bvh", points, batch_offsets)
    packed = dict(_C.build_bvh_ragged(points, batch_offsets, offsets))
    # The handle owns its own copy of the offsets, like the reference's handle payload.
    packed["point_offsets_device"] = batch_offsets.clone()
    handles = [_LazyBVHHandle(lambda b=b: _sample_payload(packed, b)) for b in range(len(offsets) - 1)]
    counts = torch.diff(batch_offsets).clone()
    return RaggedBVHHandle(
        {
            "batch_offsets": packed["point_offsets_device"],
            "num_leaves_per_sample": counts,
            "batch_size": len(offsets) - 1,
            "dim": int(points.size(1)),
        },
        handles,
        packed,
    )


def build_bvh(
    points: torch.Tensor,
    *,
    batch_offsets: torch.Tensor | None = None,
) -> BVHHandle | BatchedBVHHandle | RaggedBVHHandle:
    """Build a BVH. Dispatches on points shape and batch_offsets.

    - ``(N, D)`` -> single BVH, returns ``BVHHandle``
    - ``(B, N, D)`` -> fixed-size batched BVHs, returns ``BatchedBVHHandle``
    - ``(total_N, D)`` + ``batch_offsets=(B+1,)`` -> ragged packed BVHs, returns ``RaggedBVHHandle``

    Ragged neighbor indices are local to each sample.
    """
    if batch_offsets is not None:
        if points.dim() != 2:
            raise ValueError("build_bvh: ragged mode requires 2-D points (total_N, D)")
        return _build_bvh_ragged(points, batch_offsets)
    if points.dim() == 3:
        return _build_bvh_batched(points)
    if points.dim() == 2:
        return _build_bvh_single(points)
    raise ValueError("build_bvh: points must have shape (N, D) or (B, N, D)")


# ---------------------------------------------------------------------------
# Queries
# ---------------------------------------------------------------------------

def _query_knn_single(
    bvh: BVHHandle,
    query_points: torch.Tensor,
    k: int,
    *,
    source_points: torch.Tensor | None = None,
    sort_queries: bool = True,
):
    _validate_supported_k("query_knn", k)
    data = _bvh_data(bvh, "query_knn")
    if query_points.dim() != 2:
        raise ValueError("query_knn: query_points must have shape (M, D)")
    if query_points.size(1) != data["dim"]:
        raise ValueError("query_knn: query_points second dimension must match BVH dim")
    _validate_cuda_float32("query_knn", query_points, "query_points")
    if query_points.device != data["sorted_indices"].device:
        raise ValueError("query_knn: query_points must be on the same device as the BVH")
    query_points = _as_contiguous(query_points)
    if source_points is not None:
        _validate_single_source_points("query_knn", data, source_points)
        source_points = _as_contiguous(source_points)
    batched_queries = query_points.unsqueeze(0)
    node_aabbs = data["node_aabbs"].unsqueeze(0)
    sorted_indices = data["sorted_indices"].unsqueeze(0)
    sort_perm = None
    if sort_queries:
        sort_perm = _C.morton_sort_queries_narrow(
            batched_queries,
            data["scene_min"].unsqueeze(0),
            data["scene_max"].unsqueeze(0),
        ).contiguous()
    if source_points is not None:
        indices, squared_distances, positions = _C.query_knn_gather_positions(
            node_aabbs, sorted_indices, batched_queries, sort_perm, source_points.detach().unsqueeze(0),
            data["num_leaves"], data["num_real_nodes"], data["dim"], k,
        )
        indices = indices.squeeze(0)
        positions = _with_source_grad(source_points, positions.squeeze(0), indices, int(data["num_leaves"]))
        return indices, squared_distances.squeeze(0), positions
    if sort_queries:
        indices, squared_distances = _C.query_knn_batched_cached_bounds_ordered(
            node_aabbs,
            sorted_indices,
            batched_queries,
            sort_perm,
            data["num_leaves"],
            data["num_real_nodes"],
            data["dim"],
            k,
        )
    else:
        indices, squared_distances = _C.query_knn_batched_cached_bounds(
            node_aabbs,
            sorted_indices,
            batched_queries,
            data["num_leaves"],
            data["num_real_nodes"],
            data["dim"],
            k,
        )
    return indices.squeeze(0), squared_distances.squeeze(0)


class _GatheredPositions(torch.autograd.Function):
    """Neighbour positions gathered inside the k-NN kernel, differentiable with
    respect to ``source_points`` like the reference's ``source_points[indices]``
    (torchbvh/_query.py:174,203-215): the backward pass scatter-adds each
    neighbour's gradient onto the source row it was read from."""

    @staticmethod
    def forward(ctx, source_points, positions, source_rows):
        ctx.save_for_backward(source_rows)
        ctx.source_shape = source_points.shape
        return positions

    @staticmethod
    def backward(ctx, grad_positions):
        (source_rows,) = ctx.saved_tensors
        shape = ctx.source_shape
        dim = shape[-1]
        grad = torch.zeros((_rows_of(shape), dim), dtype=grad_positions.dtype, device=grad_positions.device)
        grad.index_add_(0, source_rows.reshape(-1), grad_positions.reshape(-1, dim))
        return grad.reshape(shape), None, None


def _rows_of(shape) -> int:
    rows = 1
    for extent in shape[:-1]:
        rows *= int(extent)
    return rows


def _with_source_grad(source_points, positions, indices, cloud_size, row_base=None):
    """Attaches the gradient path to fused-gather positions when ``source_points``
    requires it. ``cloud_size`` is each row's cloud point count (an int, or a
    tensor broadcasting against ``indices``); ``row_base`` the first source row of
    each query's cloud. An empty slot (-1) read the cloud's last point in the
    kernel, so its gradient goes there too."""
    if not (torch.is_grad_enabled() and source_points.requires_grad):
        return positions
    if isinstance(cloud_size, torch.Tensor):
        last = cloud_size - 1
    else:
        last = torch.full_like(indices, cloud_size - 1)
    rows = torch.where(indices < 0, last, indices)
    if row_base is not None:
        rows = rows + row_base
    return _GatheredPositions.apply(source_points, positions, rows)


def _validate_single_source_points(prefix: str, data: Mapping, source_points: torch.Tensor) -> None:
    if source_points.dim() != 2:
        raise ValueError(f"{prefix}: source_points must have shape (N, D)")
    if source_points.size(0) != data["num_leaves"]:
        raise ValueError(f"{prefix}: source_points first dimension must match BVH num_leaves")
    if source_points.size(1) != data["dim"]:
        raise ValueError(f"{prefix}: source_points second dimension must match BVH dim")
    _validate_cuda_float32(prefix, source_points, "source_points")
    if source_points.device != data["sorted_indices"].device:
        raise ValueError(f"{prefix}: source_points must be on the same device as the BVH")


def _validate_batched_source_points(prefix: str, data: Mapping, source_points: torch.Tensor) -> None:
    if source_points.dim() != 3:
        raise ValueError(f"{prefix}: source_points must have shape (B, N, D)")
    if source_points.size(0) != data["batch_size"]:
        raise ValueError(f"{prefix}: source_points batch size must match BVH batch_size")
    if source_points.size(1) != data["num_leaves"]:
        raise ValueError(f"{prefix}: source_points second dimension must match BVH num_leaves")
    if source_points.size(2) != data["dim"]:
        raise ValueError(f"{prefix}: source_points last dimension must match BVH dim")
    _validate_cuda_float32(prefix, source_points, "source_points")
    if source_points.device != data["sorted_indices"].device:
        raise ValueError(f"{prefix}: source_points must be on the same device as the BVH")


def _query_knn_batched(
    bvh: BatchedBVHHandle,
    query_points: torch.Tensor,
    k: int,
    *,
    source_points: torch.Tensor | None = None,
    sort_queries: bool = True,
):
    _validate_supported_k("query_knn", k)
    data = _batched_bvh_data(bvh, "query_knn")
    if query_points.dim() != 3:
        raise ValueError("query_knn: batched query_points must have shape (B, M, D)")
    if query_points.size(0) != data["batch_size"]:
        raise ValueError("query_knn: query_points batch size must match BVH batch_size")
    if query_points.size(2) != data["dim"]:
        raise ValueError("query_knn: query_points last dimension must match BVH dim")
    _validate_cuda_float32("query_knn", query_points, "query_points")
    if query_points.device != data["sorted_indices"].device:
        raise ValueError("query_knn: query_points must be on the same device as the BVH")
    query_points = _as_contiguous(query_points)
    if source_points is not None:
        _validate_batched_source_points("query_knn", data, source_points)
        source_points = _as_contiguous(source_points)

    sort_perm = None
    if sort_queries:
        sort_perm = _C.morton_sort_queries_narrow(query_points, data["scene_min"], data["scene_max"]).contiguous()
    if source_points is not None:
        indices, squared_distances, positions = _C.query_knn_gather_positions(
            data["node_aabbs"], data["sorted_indices"], query_points, sort_perm, source_points.detach(),
            data["num_leaves"], data["num_real_nodes"], data["dim"], k,
        )
        n = int(data["num_leaves"])
        cloud_base = (torch.arange(indices.size(0), device=indices.device, dtype=torch.int64) * n).view(-1, 1, 1)
        positions = _with_source_grad(source_points, positions, indices, n, cloud_base)
        return indices, squared_distances, positions
    if sort_queries:
        indices, squared_distances = _C.query_knn_batched_cached_bounds_ordered(
            data["node_aabbs"],
            data["sorted_indices"],
            query_points,
            sort_perm,
            data["num_leaves"],
            data["num_real_nodes"],
            data["dim"],
            k,
        )
    else:
        indices, squared_distances = _C.query_knn_batched_cached_bounds(
            data["node_aabbs"],
            data["sorted_indices"],
            query_points,
            data["num_leaves"],
            data["num_real_nodes"],
            data["dim"],
            k,
        )
    return indices, squared_distances


def _validate_ragged_source_points(
    prefix: str,
    data: Mapping,
    source_points: torch.Tensor,
    *,
    total_rows: int,
    device: torch.device,
) -> None:
    if source_points.dim() != 2:
        raise ValueError(f"{prefix}: ragged source_points must have shape (total_N, D)")
    if source_points.size(0) != total_rows:
        raise ValueError(f"{prefix}: source_points first dimension must match BVH total_N")
    if source_points.size(1) != data["dim"]:
        raise ValueError(f"{prefix}: source_points second dimension must match BVH dim")
    _validate_cuda_float32(prefix, source_points, "source_points")
    if source_points.device != device:
        raise ValueError(f"{prefix}: source_points must be on the same device as the BVH")


def _query_knn_ragged(
    bvh: RaggedBVHHandle,
    query_points: torch.Tensor,
    query_offsets: torch.Tensor,
    k: int,
    *,
    source_points: torch.Tensor | None = None,
):
    _validate_supported_k("query_knn", k)

    data, packed = _ragged_bvh_data(bvh, "query_knn")
    if query_points.dim() != 2:
        raise ValueError("query_knn: ragged query_points must have shape (total_M, D)")
    if query_points.size(1) != data["dim"]:
        raise ValueError("query_knn: query_points second dimension must match BVH dim")
    _validate_cuda_float32("query_knn", query_points, "query_points")
    if query_points.device != data["batch_offsets"].device:
        raise ValueError("query_knn: query_points must be on the same device as the BVH")
    query_points = _as_contiguous(query_points)
    query_offsets = _as_contiguous_int64(query_offsets)

    q_offsets = _validate_offsets(
        "query_knn",
        query_offsets,
        total_rows=int(query_points.size(0)),
        device=query_points.device,
    )
    if len(q_offsets) - 1 != data["batch_size"]:
        raise ValueError("query_knn: query_offsets batch size must match BVH batch_size")

    batch_offsets = packed["point_offsets"]
    counts = [right - left for left, right in zip(batch_offsets, batch_offsets[1:])]
    if any(count < k for count in counts):
        raise ValueError("query_knn: each source sample must contain at least k points")

    if source_points is not None:
        _validate_ragged_source_points(
            "query_knn",
            data,
            source_points,
            total_rows=batch_offsets[-1],
            device=query_points.device,
        )
        source_points = _as_contiguous(source_points)

    total = q_offsets[-1]
    order = _C.morton_sort_queries_ragged(query_points, query_offsets, total, packed["scene_min"], packed["scene_max"])
    if source_points is None:
        return _C.query_knn_ragged(packed, query_points, query_offsets, total, order, k)
    indices, distances, positions = _C.query_knn_ragged(
        packed, query_points, query_offsets, total, order, k, source_points=source_points.detach()
    )
    if torch.is_grad_enabled() and source_points.requires_grad:
        query_counts = torch.diff(query_offsets)
        point_offsets = packed["point_offsets_device"]
        row_base = torch.repeat_interleave(point_offsets[:-1], query_counts, output_size=total)[:, None]
        sizes = torch.repeat_interleave(torch.diff(point_offsets), query_counts, output_size=total)[:, None]
        positions = _with_source_grad(source_points, positions, indices, sizes, row_base)
    return indices, distances, positions


def query_knn(
    bvh: BVHHandle | BatchedBVHHandle | RaggedBVHHandle,
    query_points: torch.Tensor,
    k: int,
    *,
    query_offsets: torch.Tensor | None = None,
    source_points: torch.Tensor | None = None,
    sort_queries: bool = True,
):
    """Query exact k-NN. Dispatches on handle type.

    - ``BVHHandle`` -> single-sample, returns shape ``(M, k)``
    - ``BatchedBVHHandle`` -> batched, returns shape ``(B, M, k)``
    - ``RaggedBVHHandle`` -> packed ragged; ``query_offsets`` required, returns packed ``(total_M, k)``

    Returns ``(indices, squared_distances)`` or, when ``source_points`` is provided,
    ``(indices, squared_distances, neighbor_positions)``.
    """
    if isinstance(bvh, RaggedBVHHandle):
        if query_offsets is None:
            raise ValueError("query_knn: query_offsets is required when querying a ragged BVH")
        return _query_knn_ragged(bvh, query_points, query_offsets, k, source_points=source_points)
    if query_offsets is not None:
        raise TypeError("query_knn: query_offsets requires a RaggedBVHHandle")
    if isinstance(bvh, BatchedBVHHandle):
        return _query_knn_batched(bvh, query_points, k, source_points=source_points, sort_queries=sort_queries)
    return _query_knn_single(bvh, query_points, k, source_points=source_points, sort_queries=sort_queries)
