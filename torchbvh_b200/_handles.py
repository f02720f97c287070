"""Python-owned BVH handles.

Same contract as torchbvh/_handles.py:7-120: Mapping access to the tensor
payload, a ``destroyed`` flag, idempotent ``destroy()``, ``RuntimeError`` on
use after destroy, cascade destroy for ragged handles, ``TypeError`` for
foreign objects.

Ragged handles additionally keep the packed device payload of one on-device
build (``_packed``); their per-sample ``BVHHandle`` views are materialised
lazily so that building 64 clouds does not cost 64 Python dictionaries of
tensor views unless a caller asks for them.
"""

from __future__ import annotations

from collections.abc import Callable, Iterator, Mapping
from contextlib import contextmanager

import torch


class _MappingBVHHandle(Mapping):
    """Shared mapping/liveness behaviour for Python-owned BVH handles."""

    _destroyed_message = "BVH handle has been destroyed"

    def __init__(self, data: Mapping, *, marker: str | None = None):
        self._data = dict(data)
        if marker is not None:
            self._data[marker] = True
        self._destroyed = False

    @property
    def destroyed(self) -> bool:
        return self._destroyed

    def destroy(self) -> None:
        self._destroyed = True
        self._data.clear()

    def _require_live(self) -> dict:
        if self._destroyed:
            raise RuntimeError(self._destroyed_message)
        return self._data

    def __getitem__(self, key):
        return self._require_live()[key]

    def __iter__(self) -> Iterator:
        return iter(self._require_live())

    def __len__(self) -> int:
        return len(self._require_live())


class BVHHandle(_MappingBVHHandle):
    """Lifecycle wrapper around one cloud's BVH payload."""


class _LazyBVHHandle(BVHHandle):
    """Per-sample handle of a ragged build whose payload is built on first use."""

    def __init__(self, factory: Callable[[], Mapping]):
        super().__init__({})
        self._factory: Callable[[], Mapping] | None = factory

    def _require_live(self) -> dict:
        data = super()._require_live()
        if self._factory is not None:
            data.update(self._factory())
            self._factory = None
        return data

    def destroy(self) -> None:
        self._factory = None
        super().destroy()


class BatchedBVHHandle(_MappingBVHHandle):
    """Lifecycle wrapper around a fixed-size batched BVH payload."""

    _destroyed_message = "Batched BVH handle has been destroyed"

    def __init__(self, data: Mapping):
        super().__init__(data, marker="_batched")


class RaggedBVHHandle(_MappingBVHHandle):
    """Lifecycle wrapper around packed ragged metadata, payload and sample handles."""

    _destroyed_message = "Ragged BVH handle has been destroyed"

    def __init__(self, data: Mapping, handles: list[BVHHandle], packed: Mapping | None = None):
        super().__init__(data, marker="_ragged")
        self._handles = list(handles)
        self._packed = dict(packed) if packed is not None else {}

    def destroy(self) -> None:
        if not self._destroyed:
            for handle in self._handles:
                handle.destroy()
        self._destroyed = True
        self._handles.clear()
        self._packed.clear()
        self._data.clear()

    def _require_handles(self) -> list[BVHHandle]:
        self._require_live()
        return self._handles

    def _require_packed(self) -> dict:
        self._require_live()
        return self._packed


def _bvh_data(bvh, prefix: str = "query_knn") -> Mapping:
    if isinstance(bvh, (BatchedBVHHandle, RaggedBVHHandle)):
        raise TypeError(f"{prefix}: bvh must be a BVHHandle returned by build_bvh")
    if isinstance(bvh, BVHHandle):
        return bvh._require_live()
    raise TypeError(f"{prefix}: bvh must be a BVHHandle returned by build_bvh")


def _batched_bvh_data(bvh, prefix: str = "query_knn") -> Mapping:
    if isinstance(bvh, BatchedBVHHandle):
        return bvh._require_live()
    raise TypeError(f"{prefix}: bvh must be a BatchedBVHHandle returned by build_bvh")


def _ragged_bvh_data(bvh, prefix: str = "query_knn") -> tuple[Mapping, dict]:
    if isinstance(bvh, RaggedBVHHandle):
        return bvh._require_live(), bvh._require_packed()
    raise TypeError(f"{prefix}: bvh must be a RaggedBVHHandle returned by build_bvh")


@contextmanager
def _temporary_bvh(build_fn, points: torch.Tensor):
    handle = build_fn(points)
    try:
        yield handle
    finally:
        destroy_bvh(handle)


def destroy_bvh(bvh: BVHHandle | BatchedBVHHandle | RaggedBVHHandle) -> None:
    """Destroy a Python BVH handle and release its tensor references."""
    if isinstance(bvh, (RaggedBVHHandle, BatchedBVHHandle, BVHHandle)):
        bvh.destroy()
        return
    raise TypeError("destroy_bvh: bvh must be a handle returned by build_bvh")
