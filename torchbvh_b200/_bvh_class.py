"""``BVH``: the object-style entry point (torchbvh/_bvh_class.py:14-105, k-NN part).

``BVH(points[, batch_offsets=...])`` builds at construction through
``build_bvh`` (same dispatch: (N, D) single, (B, N, D) batched, packed
(total_N, D) with offsets ragged), ``.knn(...)`` forwards to ``query_knn``,
and the object owns its handle: ``destroy()`` / ``with`` release it. The
handle's fields stay private (the class is not a mapping).
"""

from __future__ import annotations

import torch

from ._handles import destroy_bvh
from ._query import build_bvh, query_knn
from ._validation import _reject_unless


class BVH:
    """Unified BVH wrapper. Dispatches on points shape and batch_offsets.

    - ``BVH(points)`` where ``points`` is ``(N, D)`` -> single-sample BVH
    - ``BVH(points)`` where ``points`` is ``(B, N, D)`` -> fixed-size batched BVH
    - ``BVH(points, batch_offsets=offsets)`` where ``points`` is ``(total_N, D)``
      -> ragged packed BVH

    Owns handle lifetime. Supports the context-manager protocol.
    """

    def __init__(self, points: torch.Tensor, *, batch_offsets: torch.Tensor | None = None) -> None:
        # The class reports shape problems under its own name before building.
        if batch_offsets is not None:
            _reject_unless(points.dim() == 2, "BVH: ragged mode requires 2-D points (total_N, D)")
        else:
            _reject_unless(points.dim() in (2, 3), "BVH: points must have shape (N, D) or (B, N, D)")
        self._handle = build_bvh(points, batch_offsets=batch_offsets)
        self._points = points

    @property
    def destroyed(self) -> bool:
        return self._handle.destroyed

    def knn(self, query_points: torch.Tensor, k: int, *, query_offsets: torch.Tensor | None = None,
            source_points: torch.Tensor | None = None, sort_queries: bool = True, out=None):
        """Query k nearest neighbors (see ``query_knn``).

        For ragged BVHs ``query_offsets`` is required. For single/batched BVHs
        ``sort_queries`` controls Morton-sorted traversal (default True).
        ``out=(indices, squared_distances)``: caller-owned result tensors on the
        BVH's device (written by the traversal) or in pinned host memory (an
        asynchronous copy on the current stream).
        """
        return query_knn(self._handle, query_points, k, query_offsets=query_offsets, source_points=source_points,
                         sort_queries=sort_queries, out=out)

    def destroy(self) -> None:
        destroy_bvh(self._handle)

    def __enter__(self) -> "BVH":
        return self

    def __exit__(self, *exc) -> None:
        self.destroy()
