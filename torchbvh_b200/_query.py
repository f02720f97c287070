"""Build and query orchestration behind ``build_bvh`` / ``query_knn`` / ``BVH``.

Contract kept from torchbvh (torchbvh/_query.py:29-405): the same dispatch on
input shape and handle kind, the same payload fields, result shapes, local
indices, exception types and messages, and the same reference-named ``_C``
functions on the single and fixed-size batched paths.

Organisation here: every call resolves to one of three cloud layouts —
``single`` (one (N, D) cloud), ``batched`` (B clouds of N points) or
``ragged`` (packed clouds with offsets). A layout is a row of rule tables
(which argument shapes it accepts and what it says when they are wrong) plus
one native path. Single clouds run the batched native path with B = 1.
Ragged input is one packed native build and one packed query over all clouds
(the reference builds and queries each sample in a Python loop and
concatenates); per-sample handles are views into the packed payload, made on
first access.
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
    _reject_unless,
    _validate_cuda_float32,
    _validate_offsets,
    _validate_ragged_points,
    _validate_supported_k,
)

_INT32_MAX = 2**31 - 1
_SINGLE, _BATCHED, _RAGGED = "single", "batched", "ragged"


def _validate_narrow_build_extent(prefix: str, points: torch.Tensor) -> None:
    # Point indices and sort values are 32-bit inside the native path.
    total = points.numel() // max(int(points.size(-1)), 1)
    _reject_unless(total <= _INT32_MAX, f"{prefix}: total point count must fit in signed int32")


# ---------------------------------------------------------------------------
# Rule tables. Each entry is (holds(tensor, payload), message); they run in order.
# ---------------------------------------------------------------------------

_BUILD_RULES = {
    _SINGLE: (
        (lambda p: p.dim() == 2, "build_bvh: points must have shape (N, D)"),
        (lambda p: p.size(1) in SUPPORTED_DIMS, "build_bvh: D must be 2 or 3"),
    ),
    _BATCHED: (
        (lambda p: p.dim() == 3, "build_bvh: batched points must have shape (B, N, D)"),
        (lambda p: p.size(2) in SUPPORTED_DIMS, "build_bvh: D must be 2 or 3"),
    ),
}

_QUERY_SHAPE_RULES = {
    _SINGLE: (
        (lambda q, d: q.dim() == 2, "query_knn: query_points must have shape (M, D)"),
        (lambda q, d: q.size(1) == d["dim"], "query_knn: query_points second dimension must match BVH dim"),
    ),
    _BATCHED: (
        (lambda q, d: q.dim() == 3, "query_knn: batched query_points must have shape (B, M, D)"),
        (lambda q, d: q.size(0) == d["batch_size"], "query_knn: query_points batch size must match BVH batch_size"),
        (lambda q, d: q.size(2) == d["dim"], "query_knn: query_points last dimension must match BVH dim"),
    ),
    _RAGGED: (
        (lambda q, d: q.dim() == 2, "query_knn: ragged query_points must have shape (total_M, D)"),
        (lambda q, d: q.size(1) == d["dim"], "query_knn: query_points second dimension must match BVH dim"),
    ),
}

# Source-point rules take the payload's size facts: (num_leaves or total_N, batch_size, dim).
_SOURCE_SHAPE_RULES = {
    _SINGLE: (
        (lambda s, n, b, d: s.dim() == 2, "source_points must have shape (N, D)"),
        (lambda s, n, b, d: s.size(0) == n, "source_points first dimension must match BVH num_leaves"),
        (lambda s, n, b, d: s.size(1) == d, "source_points second dimension must match BVH dim"),
    ),
    _BATCHED: (
        (lambda s, n, b, d: s.dim() == 3, "source_points must have shape (B, N, D)"),
        (lambda s, n, b, d: s.size(0) == b, "source_points batch size must match BVH batch_size"),
        (lambda s, n, b, d: s.size(1) == n, "source_points second dimension must match BVH num_leaves"),
        (lambda s, n, b, d: s.size(2) == d, "source_points last dimension must match BVH dim"),
    ),
    _RAGGED: (
        (lambda s, n, b, d: s.dim() == 2, "ragged source_points must have shape (total_N, D)"),
        (lambda s, n, b, d: s.size(0) == n, "source_points first dimension must match BVH total_N"),
        (lambda s, n, b, d: s.size(1) == d, "source_points second dimension must match BVH dim"),
    ),
}


def _check_source_points(layout: str, prefix: str, source: torch.Tensor, rows: int, batch: int | None, dim: int,
                         device: torch.device) -> torch.Tensor:
    for holds, text in _SOURCE_SHAPE_RULES[layout]:
        _reject_unless(holds(source, rows, batch, dim), f"{prefix}: {text}")
    _validate_cuda_float32(prefix, source, "source_points")
    _reject_unless(source.device == device, f"{prefix}: source_points must be on the same device as the BVH")
    return _as_contiguous(source)


def _validate_single_source_points(prefix: str, data: Mapping, source_points: torch.Tensor) -> None:
    _check_source_points(_SINGLE, prefix, source_points, data["num_leaves"], None, data["dim"],
                         data["sorted_indices"].device)


def _validate_batched_source_points(prefix: str, data: Mapping, source_points: torch.Tensor) -> None:
    _check_source_points(_BATCHED, prefix, source_points, data["num_leaves"], data["batch_size"], data["dim"],
                         data["sorted_indices"].device)


# ---------------------------------------------------------------------------
# Builders
# ---------------------------------------------------------------------------

def _checked_build_points(layout: str, points: torch.Tensor) -> torch.Tensor:
    for holds, text in _BUILD_RULES[layout]:
        _reject_unless(holds(points), text)
    _validate_cuda_float32("build_bvh", points, "points")
    points = _as_contiguous(points)
    _validate_narrow_build_extent("build_bvh", points)
    return points


def _build_bvh_single(points: torch.Tensor) -> BVHHandle:
    points = _checked_build_points(_SINGLE, points)
    payload = _C.build_bvh_batched_cooperative(points.unsqueeze(0))
    # One cloud is a batch of one: drop the batch dimension of the per-cloud fields.
    fields = {key: (value[0] if key in ("node_aabbs", "sorted_indices", "scene_min", "scene_max") else value)
              for key, value in payload.items() if key != "batch_size"}
    return BVHHandle(fields)


def _build_bvh_batched(points: torch.Tensor) -> BatchedBVHHandle:
    return BatchedBVHHandle(_C.build_bvh_batched_cooperative(_checked_build_points(_BATCHED, points)))


def _sample_payload(packed: Mapping, batch: int) -> dict:
    """Per-sample handle payload: views of the packed ragged build."""
    p0, p1 = packed["point_offsets"][batch], packed["point_offsets"][batch + 1]
    r0, r1 = packed["row_offsets"][batch], packed["row_offsets"][batch + 1]
    fields = _C.tree_scalars(p1 - p0)
    fields.update(
        node_aabbs=packed["node_aabbs"][r0:r1],
        sorted_indices=packed["sorted_indices"][p0:p1],
        scene_min=packed["scene_min"][batch],
        scene_max=packed["scene_max"][batch],
        dim=packed["dim"],
    )
    fields.update(_C.deferred_traversal_arrays(p1 - p0, packed["node_aabbs"].device))
    return fields


def _build_bvh_ragged(points: torch.Tensor, batch_offsets: torch.Tensor) -> RaggedBVHHandle:
    points = _as_contiguous(points)
    batch_offsets = _as_contiguous_int64(batch_offsets)
    offsets = _validate_ragged_points("build_bvh", points, batch_offsets)
    packed = dict(_C.build_bvh_ragged(points, batch_offsets, offsets))
    # The handle keeps its own copy of the offsets.
    packed["point_offsets_device"] = batch_offsets.clone()
    samples = [_LazyBVHHandle(lambda b=b: _sample_payload(packed, b)) for b in range(len(offsets) - 1)]
    meta = {
        "batch_offsets": packed["point_offsets_device"],
        "num_leaves_per_sample": torch.diff(batch_offsets),
        "batch_size": len(offsets) - 1,
        "dim": int(points.size(1)),
    }
    return RaggedBVHHandle(meta, samples, packed)


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
        _reject_unless(points.dim() == 2, "build_bvh: ragged mode requires 2-D points (total_N, D)")
        return _build_bvh_ragged(points, batch_offsets)
    builders = {2: _build_bvh_single, 3: _build_bvh_batched}
    _reject_unless(points.dim() in builders, "build_bvh: points must have shape (N, D) or (B, N, D)")
    return builders[points.dim()](points)


# ---------------------------------------------------------------------------
# Queries
# ---------------------------------------------------------------------------

def _checked_queries(layout: str, data: Mapping, query_points: torch.Tensor, device: torch.device) -> torch.Tensor:
    for holds, text in _QUERY_SHAPE_RULES[layout]:
        _reject_unless(holds(query_points, data), text)
    _validate_cuda_float32("query_knn", query_points, "query_points")
    _reject_unless(query_points.device == device, "query_knn: query_points must be on the same device as the BVH")
    return _as_contiguous(query_points)


def _checked_out(out, shape: tuple, device: torch.device, source: torch.Tensor | None):
    """``out=(indices, squared_distances)``: caller-owned result tensors of the
    call's result shape (int64 / float32, contiguous), on the BVH's device or in
    pinned host memory; they are complete once the current stream has passed the
    call."""
    if out is None:
        return None
    _reject_unless(source is None, "query_knn: out cannot be combined with source_points")
    _reject_unless(isinstance(out, (tuple, list)) and len(out) == 2,
                   "query_knn: out must be a pair (indices, squared_distances)")
    for t, dtype, name in zip(out, (torch.int64, torch.float32), ("indices", "squared_distances")):
        _reject_unless(isinstance(t, torch.Tensor) and t.dtype == dtype,
                       f"query_knn: out {name} must be a {dtype} tensor")
        _reject_unless(tuple(t.shape) == tuple(shape), f"query_knn: out {name} must have shape {tuple(shape)}")
        _reject_unless(t.is_contiguous(), f"query_knn: out {name} must be contiguous")
        _reject_unless(t.device == device or (t.device.type == "cpu" and t.is_pinned()),
                       "query_knn: out tensors must be on the BVH's device or in pinned host memory")
    return tuple(out)


def _run_fixed_size(data: Mapping, queries: torch.Tensor, k: int, source: torch.Tensor | None, sort_queries: bool,
                    squeeze: bool, out=None):
    """Single clouds (as B = 1) and fixed-size batches: Morton order of the
    queries against each cloud's scene box, then the traversal."""
    lift = (lambda t: t.unsqueeze(0)) if squeeze else (lambda t: t)
    queries_b = lift(queries)
    tree = (lift(data["node_aabbs"]), lift(data["sorted_indices"]))
    sizes = (data["num_leaves"], data["num_real_nodes"], data["dim"], k)
    order = None
    if sort_queries:
        order = _C.morton_sort_queries_narrow(queries_b, lift(data["scene_min"]), lift(data["scene_max"])).contiguous()
    if source is not None:
        idx, dist, pos = _C.query_knn_gather_positions(*tree, queries_b, order, lift(source.detach()), *sizes)
        n = int(data["num_leaves"])
        base = None if squeeze else (torch.arange(idx.size(0), device=idx.device, dtype=torch.int64) * n).view(-1, 1, 1)
        if squeeze:
            idx, dist, pos = idx[0], dist[0], pos[0]
        return idx, dist, _with_source_grad(source, pos, idx, n, base)
    kw = {"out": tuple(lift(t) for t in out)} if _on_device(out) else {}
    if sort_queries:
        idx, dist = _C.query_knn_batched_cached_bounds_ordered(*tree, queries_b, order, *sizes, **kw)
    else:
        idx, dist = _C.query_knn_batched_cached_bounds(*tree, queries_b, *sizes, **kw)
    if out is not None:
        return _deliver(out, idx, dist)
    return (idx[0], dist[0]) if squeeze else (idx, dist)


def _on_device(out) -> bool:
    return out is not None and out[0].is_cuda


def _deliver(out, idx: torch.Tensor, dist: torch.Tensor):
    """The result in the caller's ``out`` pair. Device tensors were written by the
    traversal itself. Pinned host tensors receive one asynchronous copy of each
    result tensor on the current stream: the kernel could store the rows into
    host memory directly (the C ABI allows it), but the rows land at scattered
    query rows, which PCIe serves far more slowly than one bulk copy (measured on
    B200, 6.4 GB of rows: 16.5 GB/s direct against 52 GB/s copied)."""
    if not out[0].is_cuda:
        out[0].copy_(idx.view(out[0].shape), non_blocking=True)
        out[1].copy_(dist.view(out[1].shape), non_blocking=True)
    return out


def _query_knn_single(bvh: BVHHandle, query_points: torch.Tensor, k: int, *,
                      source_points: torch.Tensor | None = None, sort_queries: bool = True, out=None):
    _validate_supported_k("query_knn", k)
    data = _bvh_data(bvh, "query_knn")
    device = data["sorted_indices"].device
    queries = _checked_queries(_SINGLE, data, query_points, device)
    if source_points is not None:
        source_points = _check_source_points(_SINGLE, "query_knn", source_points, data["num_leaves"], None,
                                             data["dim"], device)
    out = _checked_out(out, (queries.size(0), k), device, source_points)
    return _run_fixed_size(data, queries, k, source_points, sort_queries, squeeze=True, out=out)


def _query_knn_batched(bvh: BatchedBVHHandle, query_points: torch.Tensor, k: int, *,
                       source_points: torch.Tensor | None = None, sort_queries: bool = True, out=None):
    _validate_supported_k("query_knn", k)
    data = _batched_bvh_data(bvh, "query_knn")
    device = data["sorted_indices"].device
    queries = _checked_queries(_BATCHED, data, query_points, device)
    if source_points is not None:
        source_points = _check_source_points(_BATCHED, "query_knn", source_points, data["num_leaves"],
                                             data["batch_size"], data["dim"], device)
    out = _checked_out(out, (queries.size(0), queries.size(1), k), device, source_points)
    return _run_fixed_size(data, queries, k, source_points, sort_queries, squeeze=False, out=out)


def _query_knn_ragged(bvh: RaggedBVHHandle, query_points: torch.Tensor, query_offsets: torch.Tensor, k: int, *,
                      source_points: torch.Tensor | None = None, out=None):
    _validate_supported_k("query_knn", k)
    data, packed = _ragged_bvh_data(bvh, "query_knn")
    device = data["batch_offsets"].device
    queries = _checked_queries(_RAGGED, data, query_points, device)
    query_offsets = _as_contiguous_int64(query_offsets)
    q_offsets = _validate_offsets("query_knn", query_offsets, total_rows=int(queries.size(0)), device=queries.device)
    _reject_unless(len(q_offsets) - 1 == data["batch_size"],
                   "query_knn: query_offsets batch size must match BVH batch_size")
    p_offsets = packed["point_offsets"]
    _reject_unless(all(b - a >= k for a, b in zip(p_offsets, p_offsets[1:])),
                   "query_knn: each source sample must contain at least k points")
    if source_points is not None:
        source_points = _check_source_points(_RAGGED, "query_knn", source_points, p_offsets[-1], None, data["dim"],
                                             device)
    total = q_offsets[-1]
    out = _checked_out(out, (total, k), device, source_points)
    order = _C.morton_sort_queries_ragged(queries, query_offsets, total, packed["scene_min"], packed["scene_max"])
    if source_points is None:
        if out is None:
            return _C.query_knn_ragged(packed, queries, query_offsets, total, order, k)
        kw = {"out": out} if _on_device(out) else {}
        return _deliver(out, *_C.query_knn_ragged(packed, queries, query_offsets, total, order, k, **kw))
    idx, dist, pos = _C.query_knn_ragged(packed, queries, query_offsets, total, order, k,
                                         source_points=source_points.detach())
    if torch.is_grad_enabled() and source_points.requires_grad:
        # Each query row's cloud: its first source row and its point count.
        per_query = torch.diff(query_offsets)
        starts = packed["point_offsets_device"]
        row_base = torch.repeat_interleave(starts[:-1], per_query, output_size=total)[:, None]
        sizes = torch.repeat_interleave(torch.diff(starts), per_query, output_size=total)[:, None]
        pos = _with_source_grad(source_points, pos, idx, sizes, row_base)
    return idx, dist, pos


def query_knn(
    bvh: BVHHandle | BatchedBVHHandle | RaggedBVHHandle,
    query_points: torch.Tensor,
    k: int,
    *,
    query_offsets: torch.Tensor | None = None,
    source_points: torch.Tensor | None = None,
    sort_queries: bool = True,
    out=None,
):
    """Query exact k-NN. Dispatches on handle type.

    - ``BVHHandle`` -> single-sample, returns shape ``(M, k)``
    - ``BatchedBVHHandle`` -> batched, returns shape ``(B, M, k)``
    - ``RaggedBVHHandle`` -> packed ragged; ``query_offsets`` required, returns packed ``(total_M, k)``

    Returns ``(indices, squared_distances)`` or, when ``source_points`` is provided,
    ``(indices, squared_distances, neighbor_positions)``.

    ``out=(indices, squared_distances)`` (an addition to the reference's
    signature) writes the result into caller-owned tensors of the result shape
    and returns them: tensors on the BVH's device are written by the traversal
    itself (no result allocation); pinned host tensors receive an asynchronous
    copy on the current stream. Read them after the current stream has passed
    the call (``torch.cuda.current_stream().synchronize()`` or an event).
    """
    if isinstance(bvh, RaggedBVHHandle):
        _reject_unless(query_offsets is not None, "query_knn: query_offsets is required when querying a ragged BVH")
        return _query_knn_ragged(bvh, query_points, query_offsets, k, source_points=source_points, out=out)
    if query_offsets is not None:
        raise TypeError("query_knn: query_offsets requires a RaggedBVHHandle")
    run = _query_knn_batched if isinstance(bvh, BatchedBVHHandle) else _query_knn_single
    return run(bvh, query_points, k, source_points=source_points, sort_queries=sort_queries, out=out)


# ---------------------------------------------------------------------------
# Differentiable neighbour positions from the fused gather
# ---------------------------------------------------------------------------

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
