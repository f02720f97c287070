"""Argument checks of the public calls.

The exception types and message texts are part of the drop-in contract:
``ValueError`` with the reference's wording (torchbvh/_validation.py:6-75),
e.g. ``"build_bvh: points must be a CUDA tensor"``. Checks run in the
reference's order, so an input with several problems reports the same one.

Everything is phrased as small predicates over one tensor plus the message
to raise, so each call site reads as the list of its rules.
"""

from __future__ import annotations

import torch

from ._constants import SUPPORTED_DIMS, SUPPORTED_K


def _reject_unless(ok: bool, message: str) -> None:
    if not ok:
        raise ValueError(message)


def _validate_supported_k(prefix: str, k: int) -> None:
    # The reference's text stays a prefix of the message; k = 32 is this package's addition.
    _reject_unless(k in SUPPORTED_K, f"{prefix}: k must be 4, 8, or 16 (or 32)")


def _as_contiguous(tensor: torch.Tensor) -> torch.Tensor:
    return tensor.contiguous()


def _as_contiguous_int64(tensor: torch.Tensor) -> torch.Tensor:
    # Only int64 offsets are made contiguous here; any other dtype is reported
    # by the offsets check with its own message.
    return tensor.contiguous() if tensor.dtype == torch.int64 else tensor


def _validate_cuda_float32(prefix: str, tensor: torch.Tensor, name: str) -> None:
    _reject_unless(tensor.is_cuda, f"{prefix}: {name} must be a CUDA tensor")
    _reject_unless(tensor.dtype == torch.float32, f"{prefix}: {name} must be float32")


def _validate_offset_values(prefix: str, values: list[int], total_rows: int) -> list[int]:
    """Host copy of an offsets vector: starts at 0, ends at the packed length, strictly increasing."""
    _reject_unless(values[0] == 0, f"{prefix}: offsets must start at 0")
    _reject_unless(values[-1] == total_rows, f"{prefix}: final offset must match the packed tensor length")
    _reject_unless(all(b > a for a, b in zip(values, values[1:])), f"{prefix}: offsets must be strictly increasing")
    return values


def _validate_offsets(prefix: str, offsets: torch.Tensor, *, total_rows: int, device: torch.device) -> list[int]:
    """Checks a (B + 1,) int64 CUDA offsets tensor and returns its host values."""
    rules = (
        (lambda: offsets.dim() == 1, "offsets must have shape (B + 1,)"),
        (lambda: offsets.numel() >= 2, "offsets must contain at least two entries"),
        (lambda: offsets.dtype == torch.int64, "offsets must be int64"),
        (lambda: offsets.is_cuda, "offsets must be a CUDA tensor"),
        (lambda: offsets.is_contiguous(), "offsets must be contiguous"),
        (lambda: offsets.device == device, "offsets must be on the same device as the packed tensor"),
    )
    for holds, text in rules:
        _reject_unless(holds(), f"{prefix}: {text}")
    return _validate_offset_values(prefix, [int(v) for v in offsets.detach().cpu().tolist()], total_rows)


def _validate_ragged_points(prefix: str, points: torch.Tensor, offsets: torch.Tensor) -> list[int]:
    """Packed (total_N, D) CUDA float32 points plus their offsets; returns the host offsets."""
    _reject_unless(points.dim() == 2, f"{prefix}: points must have shape (total_N, D)")
    _reject_unless(points.size(1) in SUPPORTED_DIMS, f"{prefix}: D must be 2 or 3")
    _validate_cuda_float32(prefix, points, "points")
    _reject_unless(points.is_contiguous(), f"{prefix}: points must be contiguous")
    return _validate_offsets(prefix, offsets, total_rows=int(points.size(0)), device=points.device)
