"""Displaced-query k-NN for multi-head point models (torchbvh/_multihead.py).

``query_displaced_knn`` is the caller of the batched k-NN path that
torchbvh/_multihead.py:38-82 defines: one BVH per sample over ``pos`` and the
per-point, per-head queries ``q`` flattened to ``(B, N*H, D)``, answered by the
Morton-ordered traversal with the neighbour positions gathered inside the same
kernel. ``gather_neighbor_values`` and ``interpolate_displaced``
(torchbvh/_multihead.py:85-190) are the matching-head gather and the
inverse-squared-distance interpolation built on it.
"""
from __future__ import annotations

import torch

from ._constants import EXACT_DISTANCE_EPSILON, SUPPORTED_DIMS
from ._handles import _temporary_bvh
from ._query import _build_bvh_batched, _query_knn_batched
from ._validation import _as_contiguous, _as_contiguous_int64, _validate_cuda_float32

__all__ = ["query_displaced_knn", "gather_neighbor_values", "interpolate_displaced"]


def _check_displaced(prefix: str, pos: torch.Tensor, q: torch.Tensor) -> None:
    """Shape, dtype and device checks of torchbvh/_multihead.py:17-35, same order and messages."""
    if pos.dim() != 3:
        raise ValueError(f"{prefix}: pos must have shape (B, N, D)")
    if q.dim() != 4:
        raise ValueError(f"{prefix}: q must have shape (B, N, H, D)")
    if pos.size(2) not in SUPPORTED_DIMS:
        raise ValueError(f"{prefix}: D must be 2 or 3")
    if q.size(0) != pos.size(0):
        raise ValueError(f"{prefix}: q batch size must match pos")
    if q.size(1) != pos.size(1):
        raise ValueError(f"{prefix}: q point dimension must match pos")
    if q.size(3) != pos.size(2):
        raise ValueError(f"{prefix}: q last dimension must match pos")
    if q.size(2) < 1:
        raise ValueError(f"{prefix}: q must contain at least one head")
    _validate_cuda_float32(prefix, pos, "pos")
    _validate_cuda_float32(prefix, q, "q")
    if pos.device != q.device:
        raise ValueError(f"{prefix}: pos and q must be on the same device")


def query_displaced_knn(pos: torch.Tensor, q: torch.Tensor, k: int = 8, *, return_positions: bool = True):
    """k-NN of every per-point, per-head displaced position ``q (B, N, H, D)``
    among the sample's points ``pos (B, N, D)``.

    Returns ``indices (B, N, H, k)`` int64 (local to the sample),
    ``squared_distances (B, N, H, k)`` float32 ascending and, unless
    ``return_positions`` is False, ``neighbor_positions (B, N, H, k, D)``. The
    BVH is built over ``pos.detach()`` and dropped on return; none of the
    outputs carries gradient (torchbvh/_multihead.py:38-82).
    """
    _check_displaced("query_displaced_knn", pos, q)
    batch, n, heads, dim = q.shape
    flat = _as_contiguous(q).reshape(batch, n * heads, dim)
    sources = _as_contiguous(pos).detach()
    with _temporary_bvh(_build_bvh_batched, sources) as bvh:
        if return_positions:
            idx, dist, positions = _query_knn_batched(bvh, flat, k, source_points=sources, sort_queries=True)
            return (idx.reshape(batch, n, heads, k), dist.reshape(batch, n, heads, k),
                    positions.reshape(batch, n, heads, k, dim))
        idx, dist = _query_knn_batched(bvh, flat, k, sort_queries=True)
        return idx.reshape(batch, n, heads, k), dist.reshape(batch, n, heads, k)


def gather_neighbor_values(values: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """``out[b, i, h, j] = values[b, indices[b, i, h, j], h]``: each head reads its
    own channel block only. ``values (B, N, H, Ch)`` float32, ``indices
    (B, N, H, k)`` int64 local source indices -> ``(B, N, H, k, Ch)``;
    differentiable in ``values`` (torchbvh/_multihead.py:85-120)."""
    prefix = "gather_neighbor_values"
    if values.dim() != 4:
        raise ValueError(f"{prefix}: values must have shape (B, N, H, Ch)")
    if indices.dim() != 4:
        raise ValueError(f"{prefix}: indices must have shape (B, N, H, k)")
    if values.size(0) != indices.size(0):
        raise ValueError(f"{prefix}: indices batch size must match values")
    if values.size(1) != indices.size(1):
        raise ValueError(f"{prefix}: indices point dimension must match values")
    if values.size(2) != indices.size(2):
        raise ValueError(f"{prefix}: indices head dimension must match values")
    if values.size(3) < 1:
        raise ValueError(f"{prefix}: values must have at least one channel")
    _validate_cuda_float32(prefix, values, "values")
    if indices.dtype != torch.int64:
        raise ValueError(f"{prefix}: indices must be int64")
    if values.device != indices.device:
        raise ValueError(f"{prefix}: values and indices must be on the same device")
    values = _as_contiguous(values)
    indices = _as_contiguous_int64(indices)
    if indices.numel() > 0:
        lo, hi = torch.aminmax(indices)
        if int(lo) < 0 or int(hi) >= values.size(1):
            raise ValueError(f"{prefix}: indices must be local source indices")
    batch, n, heads, channels = values.shape
    k = indices.size(-1)
    # Row of (b, source i, head h) in values viewed as (B*N*H, Ch).
    sample_base = (torch.arange(batch, device=values.device) * (n * heads)).view(batch, 1, 1, 1)
    head = torch.arange(heads, device=values.device).view(1, 1, heads, 1)
    rows = sample_base + indices * heads + head
    return values.reshape(batch * n * heads, channels).index_select(0, rows.reshape(-1)).reshape(
        batch, n, heads, k, channels)


def interpolate_displaced(pos: torch.Tensor, q: torch.Tensor, values: torch.Tensor, k: int = 8, *,
                          reduction: str = "weighted_mean") -> torch.Tensor:
    """Matching-head values interpolated at the displaced queries
    (torchbvh/_multihead.py:151-190): weights ``1 / (d2 + 1e-12)`` normalised
    over the k neighbours; a query with neighbours at ``d2 <= 1e-12`` takes the
    plain mean of those exact hits instead. ``values (B, N, H, Ch)`` ->
    ``(B, N, H, Ch)``, differentiable in ``values`` only."""
    if reduction != "weighted_mean":
        raise ValueError("interpolate_displaced: reduction must be 'weighted_mean'")
    prefix = "interpolate_displaced"
    _check_displaced(prefix, pos, q)
    if values.dim() != 4:
        raise ValueError(f"{prefix}: values must have shape (B, N, H, Ch)")
    if values.size(0) != pos.size(0) or values.size(1) != pos.size(1):
        raise ValueError(f"{prefix}: values first two dimensions must match pos")
    if values.size(2) != q.size(2):
        raise ValueError(f"{prefix}: values head dimension must match q")
    if values.size(3) < 1:
        raise ValueError(f"{prefix}: values must have at least one channel")
    _validate_cuda_float32(prefix, values, "values")
    if values.device != pos.device:
        raise ValueError(f"{prefix}: values must be on the same device as pos")

    indices, d2 = query_displaced_knn(pos, q, k, return_positions=False)
    neighbours = gather_neighbor_values(values, indices)  # (B, N, H, k, Ch)
    weights = torch.reciprocal(d2 + EXACT_DISTANCE_EPSILON)
    weights = weights / weights.sum(dim=-1, keepdim=True).clamp(min=EXACT_DISTANCE_EPSILON)
    out = torch.einsum("bnhkc,bnhk->bnhc", neighbours, weights)
    exact = d2 <= EXACT_DISTANCE_EPSILON
    if bool(exact.any()):
        hits = exact.to(values.dtype)
        mean = torch.einsum("bnhkc,bnhk->bnhc", neighbours, hits) / hits.sum(dim=-1, keepdim=True).clamp(min=1.0)
        out = torch.where(exact.any(dim=-1, keepdim=True), mean, out)
    return out
