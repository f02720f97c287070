"""BVH handles: the Python objects ``build_bvh`` returns.

Contract kept from torchbvh (torchbvh/_handles.py:7-120): a handle is a
read-only ``Mapping`` over its payload, ``destroyed`` tells whether it was
released, ``destroy()`` is idempotent and drops the tensor references, any
later access raises ``RuntimeError`` with the handle kind's message, a ragged
handle destroys its per-sample handles with it, and helpers reject foreign
objects with ``TypeError``.

Design here: a payload field may be *deferred* — stored as a ``_Deferred``
thunk and computed on first read, then kept. Builds use that for the
traversal arrays (``left_child_mem`` / ``right_child_mem`` / ``mem_to_leaf``,
which depend only on the point count and which the k-NN path never reads) and
ragged builds for their per-sample handles, which are views into one packed
payload materialised only when a caller asks for them.
"""

from __future__ import annotations

from collections.abc import Callable, Iterator, Mapping
from contextlib import contextmanager

import torch


class _Deferred:
    """A payload field computed on first read."""

    __slots__ = ("make",)

    def __init__(self, make: Callable[[], object]):
        self.make = make


class _Handle(Mapping):
    kind_message = "BVH handle has been destroyed"
    marker: str | None = None

    def __init__(self, fields: Mapping):
        self._fields = dict(fields)
        if self.marker is not None:
            self._fields[self.marker] = True
        self._alive = True

    @property
    def destroyed(self) -> bool:
        return not self._alive

    def destroy(self) -> None:
        self._alive = False
        self._fields = {}

    def _live_fields(self) -> dict:
        if not self._alive:
            raise RuntimeError(self.kind_message)
        return self._fields

    def _require_live(self) -> dict:
        """The raw payload (deferred fields not computed): what the query paths read."""
        return self._live_fields()

    def __getitem__(self, key):
        fields = self._live_fields()
        value = fields[key]
        if isinstance(value, _Deferred):
            value = fields[key] = value.make()
        return value

    def __iter__(self) -> Iterator:
        return iter(list(self._live_fields()))

    def __len__(self) -> int:
        return len(self._live_fields())


class BVHHandle(_Handle):
    """One cloud's BVH payload."""


class _LazyBVHHandle(BVHHandle):
    """A per-sample handle of a ragged build: its whole payload comes from
    `factory` on first access."""

    def __init__(self, factory: Callable[[], Mapping]):
        super().__init__({})
        self._factory: Callable[[], Mapping] | None = factory

    def _live_fields(self) -> dict:
        fields = super()._live_fields()
        if self._factory is not None:
            fields.update(self._factory())
            self._factory = None
        return fields

    def destroy(self) -> None:
        self._factory = None
        super().destroy()


class BatchedBVHHandle(_Handle):
    """Fixed-size batch of BVHs (leading batch dimension on every tensor field)."""

    kind_message = "Batched BVH handle has been destroyed"
    marker = "_batched"


class RaggedBVHHandle(_Handle):
    """Ragged batch: metadata fields, per-sample handles (``_handles``) and the
    packed payload of the one native build behind them."""

    kind_message = "Ragged BVH handle has been destroyed"
    marker = "_ragged"

    def __init__(self, fields: Mapping, handles: list[BVHHandle], packed: Mapping | None = None):
        super().__init__(fields)
        self._handles = list(handles)
        self._packed = dict(packed or {})

    def destroy(self) -> None:
        if self._alive:
            for inner in self._handles:
                inner.destroy()
        self._handles = []
        self._packed = {}
        super().destroy()

    def _require_handles(self) -> list[BVHHandle]:
        self._live_fields()
        return self._handles

    def _require_packed(self) -> dict:
        self._live_fields()
        return self._packed


def _payload_of(bvh, expected: type, prefix: str, what: str) -> Mapping:
    """Live payload of `bvh` if it is a handle of the expected kind (the three
    kinds are unrelated classes, so a batched or ragged handle never passes
    for a single one)."""
    if isinstance(bvh, expected):
        return bvh._require_live()
    raise TypeError(f"{prefix}: bvh must be a {what} returned by build_bvh")


def _bvh_data(bvh, prefix: str = "query_knn") -> Mapping:
    return _payload_of(bvh, BVHHandle, prefix, "BVHHandle")


def _batched_bvh_data(bvh, prefix: str = "query_knn") -> Mapping:
    return _payload_of(bvh, BatchedBVHHandle, prefix, "BatchedBVHHandle")


def _ragged_bvh_data(bvh, prefix: str = "query_knn") -> tuple[Mapping, dict]:
    return _payload_of(bvh, RaggedBVHHandle, prefix, "RaggedBVHHandle"), bvh._require_packed()


@contextmanager
def _temporary_bvh(build_fn, points: torch.Tensor):
    """A handle from `build_fn(points)` that is destroyed when the block exits."""
    handle = build_fn(points)
    try:
        yield handle
    finally:
        destroy_bvh(handle)


def destroy_bvh(bvh: BVHHandle | BatchedBVHHandle | RaggedBVHHandle) -> None:
    """Destroy a Python BVH handle and release its tensor references."""
    if not isinstance(bvh, _Handle):
        raise TypeError("destroy_bvh: bvh must be a handle returned by build_bvh")
    bvh.destroy()
