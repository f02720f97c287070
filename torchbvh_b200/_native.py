"""Native boundary: the C-ABI library and the ``_C`` function namespace.

``_C`` mirrors the reference's pybind module functions for this path
(torchbvh/csrc/bindings.cpp:137-157,192-199): same names, same argument
meaning, same ``RuntimeError`` on invalid native arguments (the reference's
TORCH_CHECK). Each function allocates its outputs and workspace with the
PyTorch caching allocator, passes the current CUDA stream, and calls one
``extern "C"`` entry point of ``libtorchbvh_b200.so`` (include/torchbvh_b200.h)
through ctypes. There is no fallback: if the library is missing, every call
raises.

Functions without a reference counterpart (``build_bvh_ragged``,
``morton_sort_queries_ragged``, ``query_knn_ragged``) carry the ragged batch
through the same entry points in one launch sequence instead of the
reference's per-sample Python loop (torchbvh/_query.py:68-85,299-366).
"""

from __future__ import annotations

import ctypes
import os
import threading
import types
from pathlib import Path

import torch

# The in-tree build; TORCHBVH_B200_LIBRARY may name another build of the same sources
# (e.g. one compiled with different tuning macros).
LIB_PATH = Path(os.environ.get("TORCHBVH_B200_LIBRARY") or Path(__file__).resolve().with_name("libtorchbvh_b200.so"))

TBVH_OK = 0
TBVH_ERR_BAD_ARG = 1
TBVH_ERR_UNSUPPORTED_K = 2
TBVH_ERR_CUDA = 3
TBVH_ERR_WORKSPACE = 4

# Device status bits (tbvh_device_status).
TBVH_DEVICE_LOOKBACK_TIMEOUT = 1
TBVH_DEVICE_STACK_OVERFLOW = 2
TBVH_DEVICE_TREE_COUNTER = 4
TBVH_DEVICE_BAD_INDEX = 8

_lib = None
_lib_lock = threading.Lock()

_i32 = ctypes.c_int
_i64 = ctypes.c_int64
_ptr = ctypes.c_void_p
_size = ctypes.c_size_t

_SIGNATURES = {
    "tbvh_last_error": (ctypes.c_char_p, []),
    "tbvh_abi_version": (_i32, []),
    "tbvh_device_status": (_i32, [_i32, ctypes.POINTER(ctypes.c_uint), _i32]),
    "tbvh_real_node_count": (_i64, [_i64]),
    "tbvh_build_workspace_size": (_size, [_i64, _i64, _ptr, _i32]),
    "tbvh_build": (
        _i32,
        [_i32, _ptr, _i64, _i64, _ptr, _ptr, _i32, _ptr, _ptr, _ptr, _ptr, _ptr, _ptr, _ptr, _i32, _ptr, _size, _ptr],
    ),
    "tbvh_traversal_arrays": (_i32, [_i32, _i64, _ptr, _ptr, _ptr, _ptr]),
    "tbvh_selftest_workspace_size": (_size, []),
    "tbvh_selftest_lookback_timeout": (_i32, [_i32, _ptr, _size, _ptr, ctypes.POINTER(ctypes.c_uint)]),
    "tbvh_sort_queries_workspace_size": (_size, [_i64, _i64, _i32]),
    "tbvh_sort_queries": (_i32, [_i32, _ptr, _i64, _i64, _ptr, _i64, _i32, _ptr, _ptr, _ptr, _ptr, _size, _ptr]),
    "tbvh_query_knn_workspace_size": (_size, [_i64, _i64]),
    "tbvh_scene_bounds_workspace_size": (_size, []),
    "tbvh_scene_bounds": (_i32, [_i32, _ptr, _i64, _i32, _ptr, _ptr, _ptr, _size, _ptr]),
    "tbvh_share_queries_workspace_size": (_size, [_i64, _i32]),
    "tbvh_share_queries": (
        _i32, [_i32, _ptr, _i64, _i32, _ptr, _ptr, _i32, _i32, _i64, _ptr, ctypes.POINTER(_i64), _ptr, _size, _ptr],
    ),
    "tbvh_peer_handle_bytes": (_size, []),
    "tbvh_peer_alloc": (_i32, [_i32, _size, ctypes.POINTER(_ptr), _ptr]),
    "tbvh_peer_free": (_i32, [_i32, _ptr]),
    "tbvh_peer_open": (_i32, [_i32, _ptr, ctypes.POINTER(_ptr)]),
    "tbvh_peer_close": (_i32, [_i32, _ptr]),
    "tbvh_query_knn_share": (
        _i32,
        [_i32, _ptr, _ptr, _i64, _ptr, _i64, _ptr, _i64, _i32, _i32, _i32, ctypes.POINTER(_ptr),
         ctypes.POINTER(_ptr), _ptr],
    ),
    "tbvh_query_knn_share_i32": (
        _i32,
        [_i32, _ptr, _ptr, _i64, _ptr, _i64, _ptr, _i64, _i32, _i32, _i32, ctypes.POINTER(_ptr),
         ctypes.POINTER(_ptr), _ptr],
    ),
    "tbvh_query_knn_share_multicast": (
        _i32, [_i32, _ptr, _ptr, _i64, _ptr, _i64, _ptr, _i64, _i32, _i32, _ptr, _ptr, _ptr],
    ),
    "tbvh_widen_indices": (_i32, [_i32, _ptr, _ptr, _i64, _ptr]),
    "tbvh_query_knn_gather": (
        _i32,
        [_i32, _ptr, _ptr, _i64, _i64, _ptr, _ptr, _ptr, _i64, _ptr, _i64, _ptr, _i32, _i32, _ptr, _ptr, _ptr, _ptr,
         _i32, _ptr, _size, _ptr],
    ),
    "tbvh_query_knn": (
        _i32,
        [_i32, _ptr, _ptr, _i64, _i64, _ptr, _ptr, _ptr, _i64, _ptr, _i64, _ptr, _i32, _i32, _ptr, _ptr, _ptr, _size,
         _ptr],
    ),
}

ABI_VERSION = 1


def load_library() -> ctypes.CDLL:
    """Loads ``libtorchbvh_b200.so`` once; raises if it is missing or stale."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"torchbvh_b200: native library {LIB_PATH.name} is not built; run "
                "`python -m torchbvh_b200._build_lib` (or __graft_entry__.build())"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        version = lib.tbvh_abi_version()
        if version != ABI_VERSION:
            raise RuntimeError(f"torchbvh_b200: native ABI {version} != expected {ABI_VERSION}; rebuild the library")
        _lib = lib
        return lib


def _check(rc: int) -> None:
    if rc != TBVH_OK:
        msg = load_library().tbvh_last_error().decode("utf-8", "replace")
        raise RuntimeError(msg or f"torchbvh_b200 native call failed with status {rc}")


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def real_node_count(n: int) -> int:
    n = int(n)
    if n <= 0:
        return 0
    leaf_level = (n - 1).bit_length()
    return 2 * n - 1 + ((1 << leaf_level) - n).bit_count()


def _tree_scalars(n: int) -> dict:
    leaf_level = (n - 1).bit_length()
    return {
        "num_leaves": n,
        "num_real_nodes": real_node_count(n),
        "leaf_level": leaf_level,
        "virtual_leaves": (1 << leaf_level) - n,
    }


def traversal_arrays(num_points: int, device: torch.device) -> dict:
    """left_child_mem / right_child_mem / mem_to_leaf int32 of one cloud of
    `num_points` points (bvh_build.cu:361-398 values), computed on `device`."""
    lib = load_library()
    rows = real_node_count(num_points)
    out = {key: torch.empty((rows,), dtype=torch.int32, device=device)
           for key in ("left_child_mem", "right_child_mem", "mem_to_leaf")}
    _check(lib.tbvh_traversal_arrays(device.index, int(num_points), out["left_child_mem"].data_ptr(),
                                     out["right_child_mem"].data_ptr(), out["mem_to_leaf"].data_ptr(),
                                     _stream(device)))
    return out


def deferred_traversal_arrays(num_points: int, device: torch.device) -> dict:
    """The three traversal-array payload fields as deferred entries: the k-NN
    path never reads them and they depend only on the point count, so they are
    computed (once, together) when a caller first reads one of them."""
    from ._handles import _Deferred

    made: dict = {}

    def field(key):
        def make():
            if not made:
                made.update(traversal_arrays(num_points, device))
            return made[key]
        return _Deferred(make)

    return {key: field(key) for key in ("left_child_mem", "right_child_mem", "mem_to_leaf")}


def device_status(device: int | torch.device | None = None, clear: bool = True) -> int:
    """Error bits raised by bounded device waits (0 when healthy). Synchronises."""
    lib = load_library()
    if device is None:
        device = torch.cuda.current_device()
    index = device.index if isinstance(device, torch.device) else int(device)
    out = ctypes.c_uint(0)
    torch.cuda.synchronize(index)
    _check(lib.tbvh_device_status(index, ctypes.byref(out), 1 if clear else 0))
    return int(out.value)


# ---------------------------------------------------------------------------
# Build
# ---------------------------------------------------------------------------

def build_bvh_batched_cooperative(points: torch.Tensor) -> dict:
    """(B, N, D) points -> BVH payload dict (bvh_build.cu:679-721, bindings.cpp:137-153)."""
    op = "build_bvh_batched_cooperative"
    if not (points.is_cuda and points.is_contiguous() and points.dtype == torch.float32):
        raise RuntimeError(f"{op}: points must be contiguous CUDA float32")
    if not (points.dim() == 3 and points.size(0) >= 1 and points.size(1) >= 1 and points.size(2) in (2, 3)):
        raise RuntimeError(f"{op}: points must have shape (B, N, 2|3)")
    batch, n, dim = (int(s) for s in points.shape)
    if batch * n > 2**31 - 1:
        raise RuntimeError(f"{op}: total point count must fit in signed int32")
    lib = load_library()
    device = points.device
    nr = real_node_count(n)
    node_aabbs = torch.empty((batch, nr, 2 * dim), dtype=torch.float32, device=device)
    sorted_indices = torch.empty((batch, n), dtype=torch.int64, device=device)
    scene_min = torch.empty((batch, dim), dtype=torch.float32, device=device)
    scene_max = torch.empty((batch, dim), dtype=torch.float32, device=device)
    ws_bytes = lib.tbvh_build_workspace_size(batch, n, None, dim)
    ws = _workspace(ws_bytes, device)
    _check(lib.tbvh_build(
        device.index, points.data_ptr(), batch, n, None, None, dim,
        node_aabbs.data_ptr(), sorted_indices.data_ptr(), scene_min.data_ptr(), scene_max.data_ptr(),
        None, None, None, 0,
        ws.data_ptr(), ws.numel(), _stream(device),
    ))
    out = {
        "node_aabbs": node_aabbs,
        "sorted_indices": sorted_indices,
        "scene_min": scene_min,
        "scene_max": scene_max,
        "batch_size": batch,
        "dim": dim,
        # One shared set for every cloud of the batch (they have the same size).
        **deferred_traversal_arrays(n, device),
    }
    out.update(_tree_scalars(n))
    return out


def build_bvh_ragged(points: torch.Tensor, batch_offsets: torch.Tensor, offsets: list[int]) -> dict:
    """Packed ragged build: one launch sequence for every cloud (no reference counterpart).

    ``offsets`` is the validated host copy of ``batch_offsets``. Returns packed
    tensors plus per-cloud row offsets into ``node_aabbs``.
    """
    op = "build_bvh_ragged"
    if not (points.is_cuda and points.is_contiguous() and points.dtype == torch.float32):
        raise RuntimeError(f"{op}: points must be contiguous CUDA float32")
    dim = int(points.size(1))
    clouds = len(offsets) - 1
    counts = [offsets[b + 1] - offsets[b] for b in range(clouds)]
    rows = [real_node_count(c) for c in counts]
    row_offsets = [0]
    for r in rows:
        row_offsets.append(row_offsets[-1] + r)
    lib = load_library()
    device = points.device
    node_aabbs = torch.empty((row_offsets[-1], 2 * dim), dtype=torch.float32, device=device)
    sorted_indices = torch.empty((offsets[-1],), dtype=torch.int64, device=device)
    scene_min = torch.empty((clouds, dim), dtype=torch.float32, device=device)
    scene_max = torch.empty((clouds, dim), dtype=torch.float32, device=device)
    host_offsets = (ctypes.c_int64 * len(offsets))(*offsets)
    ws_bytes = lib.tbvh_build_workspace_size(clouds, 0, ctypes.cast(host_offsets, _ptr), dim)
    ws = _workspace(ws_bytes, device)
    _check(lib.tbvh_build(
        device.index, points.data_ptr(), clouds, 0, batch_offsets.data_ptr(), ctypes.cast(host_offsets, _ptr), dim,
        node_aabbs.data_ptr(), sorted_indices.data_ptr(), scene_min.data_ptr(), scene_max.data_ptr(),
        None, None, None, 1,
        ws.data_ptr(), ws.numel(), _stream(device),
    ))
    return {
        "node_aabbs": node_aabbs,
        "sorted_indices": sorted_indices,
        "scene_min": scene_min,
        "scene_max": scene_max,
        "row_offsets": row_offsets,
        "point_offsets": list(offsets),
        "point_offsets_device": batch_offsets,
        "dim": dim,
    }


# ---------------------------------------------------------------------------
# Query ordering
# ---------------------------------------------------------------------------

def morton_sort_queries_narrow(queries: torch.Tensor, scene_min: torch.Tensor, scene_max: torch.Tensor) -> torch.Tensor:
    """(B, M, D) queries -> (B, M) int64 Morton permutation (morton_sort.cu:264-287)."""
    op = "morton_sort_queries_narrow"
    if not (queries.is_cuda and queries.is_contiguous() and queries.dtype == torch.float32):
        raise RuntimeError(f"{op}: queries must be contiguous CUDA float32")
    if not (scene_min.is_cuda and scene_max.is_cuda and scene_min.is_contiguous() and scene_max.is_contiguous()):
        raise RuntimeError(f"{op}: bounds must be contiguous CUDA tensors")
    if not (queries.dim() == 3 and queries.size(2) in (2, 3)):
        raise RuntimeError(f"{op}: queries must have shape (B, M, 2|3)")
    if not (scene_min.shape == scene_max.shape and scene_min.size(0) == queries.size(0)
            and scene_min.size(1) == queries.size(2)):
        raise RuntimeError(f"{op}: bounds shape mismatch")
    batch, m, dim = (int(s) for s in queries.shape)
    device = queries.device
    order = torch.empty((batch, m), dtype=torch.int64, device=device)
    if batch * m == 0:
        return order
    lib = load_library()
    ws = _workspace(lib.tbvh_sort_queries_workspace_size(batch, batch * m, dim), device)
    _check(lib.tbvh_sort_queries(
        device.index, queries.data_ptr(), batch, m, None, batch * m, dim,
        scene_min.data_ptr(), scene_max.data_ptr(), order.data_ptr(), ws.data_ptr(), ws.numel(), _stream(device),
    ))
    return order


def scene_bounds(points: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(scene_min, scene_max) of one (N, D) cloud on the current stream,
    bit-identical to the build's (tbvh_scene_bounds)."""
    if not (points.is_cuda and points.is_contiguous() and points.dtype == torch.float32 and points.dim() == 2):
        raise RuntimeError("scene_bounds: points must be contiguous CUDA float32 (N, D)")
    n, dim = int(points.size(0)), int(points.size(1))
    device = points.device
    lib = load_library()
    box = torch.empty((2, dim), dtype=torch.float32, device=device)
    ws = _workspace(lib.tbvh_scene_bounds_workspace_size(), device)
    _check(lib.tbvh_scene_bounds(device.index, points.data_ptr(), n, dim, box[0].data_ptr(), box[1].data_ptr(),
                                 ws.data_ptr(), ws.numel(), _stream(device)))
    return box[0], box[1]


def share_queries(queries: torch.Tensor, scene_min: torch.Tensor, scene_max: torch.Tensor, rank: int, world: int,
                  chunk: int) -> torch.Tensor:
    """This rank's share of the (M, D) queries of one cloud, as int64 query
    indices in Morton order (see tbvh_share_queries). Synchronises the stream."""
    if not (queries.is_cuda and queries.is_contiguous() and queries.dtype == torch.float32 and queries.dim() == 2):
        raise RuntimeError("share_queries: queries must be contiguous CUDA float32 (M, D)")
    m, dim = int(queries.size(0)), int(queries.size(1))
    device = queries.device
    lib = load_library()
    out = torch.empty((m,), dtype=torch.int64, device=device)
    ws = _workspace(lib.tbvh_share_queries_workspace_size(m, dim), device)
    count = ctypes.c_int64(0)
    _check(lib.tbvh_share_queries(device.index, queries.data_ptr(), m, dim, scene_min.contiguous().data_ptr(),
                                  scene_max.contiguous().data_ptr(), int(rank), int(world), int(chunk),
                                  out.data_ptr(), ctypes.byref(count), ws.data_ptr(), ws.numel(), _stream(device)))
    return out[: count.value]


def morton_sort_queries_ragged(queries: torch.Tensor, query_offsets: torch.Tensor, total: int,
                               scene_min: torch.Tensor, scene_max: torch.Tensor) -> torch.Tensor:
    """Packed ragged query permutation (local index per cloud, packed)."""
    clouds = int(query_offsets.numel()) - 1
    dim = int(queries.size(1))
    device = queries.device
    order = torch.empty((total,), dtype=torch.int64, device=device)
    lib = load_library()
    ws = _workspace(lib.tbvh_sort_queries_workspace_size(clouds, total, dim), device)
    _check(lib.tbvh_sort_queries(
        device.index, queries.data_ptr(), clouds, 0, query_offsets.data_ptr(), total, dim,
        scene_min.data_ptr(), scene_max.data_ptr(), order.data_ptr(), ws.data_ptr(), ws.numel(), _stream(device),
    ))
    return order


# ---------------------------------------------------------------------------
# k-NN
# ---------------------------------------------------------------------------

def _result_pair(op: str, out, shape: tuple, device: torch.device):
    """The (indices, distances) the kernel writes: new tensors on ``device``, or the
    caller's ``out`` pair (int64 / float32, contiguous, ``shape``), each on
    ``device`` or in pinned host memory, which the kernel fills across PCIe."""
    if out is None:
        return (torch.empty(shape, dtype=torch.int64, device=device),
                torch.empty(shape, dtype=torch.float32, device=device))
    if not (isinstance(out, (tuple, list)) and len(out) == 2):
        raise RuntimeError(f"{op}: out must be a pair (indices, distances)")
    for t, dtype in zip(out, (torch.int64, torch.float32)):
        if not (isinstance(t, torch.Tensor) and t.dtype == dtype and tuple(t.shape) == tuple(shape)
                and t.is_contiguous()):
            raise RuntimeError(f"{op}: out tensors must be contiguous int64 / float32 of shape {tuple(shape)}")
        if not (t.device == device or (t.device.type == "cpu" and t.is_pinned())):
            raise RuntimeError(f"{op}: out tensors must be on {device} or in pinned host memory")
    return out[0], out[1]


def _query_impl(op, node_aabbs, sorted_indices, query_points, query_order, num_leaves, num_real_nodes, dim, k,
                source_points=None, spatial=False, out=None):
    if dim not in (2, 3):
        raise RuntimeError(f"{op}: D must be 2 or 3")
    if not (query_points.is_cuda and query_points.is_contiguous() and query_points.dtype == torch.float32):
        raise RuntimeError(f"{op}: query_points must be contiguous CUDA float32")
    if not (query_points.dim() == 3 and query_points.size(2) == dim):
        raise RuntimeError(f"{op}: query_points must have shape (B, M, D)")
    if not (node_aabbs.is_cuda and node_aabbs.is_contiguous() and node_aabbs.dtype == torch.float32):
        raise RuntimeError(f"{op}: node_aabbs must be contiguous CUDA float32")
    if not (node_aabbs.dim() == 3 and node_aabbs.size(0) == query_points.size(0)
            and node_aabbs.size(1) == num_real_nodes and node_aabbs.size(2) == 2 * dim):
        raise RuntimeError(f"{op}: node_aabbs has incompatible shape")
    if not (sorted_indices.is_cuda and sorted_indices.is_contiguous() and sorted_indices.dtype == torch.int64):
        raise RuntimeError(f"{op}: sorted_indices must be contiguous CUDA int64")
    if not (sorted_indices.dim() == 2 and sorted_indices.size(0) == query_points.size(0)
            and sorted_indices.size(1) == num_leaves):
        raise RuntimeError(f"{op}: sorted_indices has incompatible shape")
    if query_order is not None:
        if not (query_order.is_cuda and query_order.is_contiguous() and query_order.dtype == torch.int64):
            raise RuntimeError(f"{op}: query_order must be contiguous CUDA int64")
        if not (query_order.dim() == 2 and query_order.size(0) == query_points.size(0)
                and query_order.size(1) == query_points.size(1)):
            raise RuntimeError(f"{op}: query_order must have shape (B, M)")
    if num_leaves < k:
        raise RuntimeError(f"{op}: num_leaves must be >= k")
    if num_real_nodes != real_node_count(num_leaves):
        raise RuntimeError(f"{op}: num_real_nodes does not match num_leaves")
    device = query_points.device
    tensors = [node_aabbs, sorted_indices] + ([query_order] if query_order is not None else [])
    if any(t.device != device for t in tensors):
        raise RuntimeError(f"{op}: all inputs must share a device")
    if k not in (4, 8, 16, 32):
        raise RuntimeError(f"{op}: k must be 4, 8, or 16 (or 32), got {k}")
    if source_points is not None:
        if not (source_points.is_cuda and source_points.is_contiguous() and source_points.dtype == torch.float32
                and source_points.shape == (query_points.size(0), num_leaves, dim)
                and source_points.device == device):
            raise RuntimeError(f"{op}: source_points must be contiguous CUDA float32 of shape (B, N, D)")
    batch, m = int(query_points.size(0)), int(query_points.size(1))
    indices, distances = _result_pair(op, out, (batch, m, k), device)
    positions = (torch.empty((batch, m, k, dim), dtype=torch.float32, device=device)
                 if source_points is not None else None)
    if batch * m == 0:
        return (indices, distances) if positions is None else (indices, distances, positions)
    lib = load_library()
    hooks = _knn_hooks
    if hooks:
        for h in hooks:
            h("start", device)
    _check(lib.tbvh_query_knn_gather(
        device.index, node_aabbs.data_ptr(), sorted_indices.data_ptr(), batch, int(num_leaves), None, None,
        query_points.data_ptr(), m, None, batch * m,
        query_order.data_ptr() if query_order is not None else None, dim, int(k),
        indices.data_ptr(), distances.data_ptr(),
        source_points.data_ptr() if source_points is not None else None,
        positions.data_ptr() if positions is not None else None, 1 if spatial else 0,
        None, 0, _stream(device),
    ))
    if hooks:
        for h in hooks:
            h("end", device)
    return (indices, distances) if positions is None else (indices, distances, positions)


def query_knn_batched_cached_bounds(node_aabbs, sorted_indices, query_points, num_leaves, num_real_nodes, dim, k,
                                    *, out=None):
    """Unordered exact k-NN (knn_query.cu:419-431). ``out``: optional (B, M, k)
    result pair to write into (see ``_result_pair``)."""
    return _query_impl("query_knn_batched_cached_bounds", node_aabbs, sorted_indices, query_points, None,
                       num_leaves, num_real_nodes, dim, k, out=out)


def query_knn_batched_cached_bounds_ordered(node_aabbs, sorted_indices, query_points, query_order,
                                            num_leaves, num_real_nodes, dim, k, *, out=None):
    """Morton-ordered exact k-NN (knn_query.cu:433-446); outputs in original query order."""
    return _query_impl("query_knn_batched_cached_bounds_ordered", node_aabbs, sorted_indices, query_points,
                       query_order, num_leaves, num_real_nodes, dim, k, out=out)


def query_knn_batched_cached_bounds_spatial(node_aabbs, sorted_indices, query_points, query_order,
                                            num_leaves, num_real_nodes, dim, k):
    """Morton-ordered exact k-NN with outputs left in the sorted order (knn_query.cu:448-461):
    row m of cloud b holds the neighbours of query ``query_order[b, m]``."""
    return _query_impl("query_knn_batched_cached_bounds_spatial", node_aabbs, sorted_indices, query_points,
                       query_order, num_leaves, num_real_nodes, dim, k, spatial=True)


def query_knn_gather_positions(node_aabbs, sorted_indices, query_points, query_order, source_points,
                               num_leaves, num_real_nodes, dim, k):
    """Exact k-NN that also returns ``source_points`` gathered at the neighbour indices,
    (B, M, k, D), from the same kernel (no reference counterpart: the reference gathers
    in a second pass, torchbvh/_query.py:174,203-215)."""
    op = ("query_knn_batched_cached_bounds_ordered" if query_order is not None
          else "query_knn_batched_cached_bounds")
    return _query_impl(op, node_aabbs, sorted_indices, query_points, query_order, num_leaves, num_real_nodes,
                       dim, k, source_points=source_points)


def query_knn_ragged(packed: dict, query_points: torch.Tensor, query_offsets: torch.Tensor, total_queries: int,
                     order: torch.Tensor | None, k: int, source_points: torch.Tensor | None = None, *, out=None):
    """Packed ragged exact k-NN over every cloud in one launch (no reference counterpart)."""
    dim = int(packed["dim"])
    device = query_points.device
    clouds = len(packed["point_offsets"]) - 1
    indices, distances = _result_pair("query_knn_ragged", out, (total_queries, k), device)
    positions = (torch.empty((total_queries, k, dim), dtype=torch.float32, device=device)
                 if source_points is not None else None)
    if total_queries == 0:
        return (indices, distances) if positions is None else (indices, distances, positions)
    lib = load_library()
    host_offsets = (ctypes.c_int64 * (clouds + 1))(*packed["point_offsets"])
    ws = _workspace(lib.tbvh_query_knn_workspace_size(clouds, 0), device)
    hooks = _knn_hooks
    if hooks:
        for h in hooks:
            h("start", device)
    _check(lib.tbvh_query_knn_gather(
        device.index, packed["node_aabbs"].data_ptr(), packed["sorted_indices"].data_ptr(), clouds, 0,
        packed["point_offsets_device"].data_ptr(), ctypes.cast(host_offsets, _ptr),
        query_points.data_ptr(), 0, query_offsets.data_ptr(), total_queries,
        order.data_ptr() if order is not None else None, dim, int(k),
        indices.data_ptr(), distances.data_ptr(),
        source_points.data_ptr() if source_points is not None else None,
        positions.data_ptr() if positions is not None else None, 0,
        ws.data_ptr(), ws.numel(), _stream(device),
    ))
    if hooks:
        for h in hooks:
            h("end", device)
    return (indices, distances) if positions is None else (indices, distances, positions)


# ---------------------------------------------------------------------------
# Peer-delivered results (one cloud sharded over the GPUs of a node)
# ---------------------------------------------------------------------------

def peer_alloc(device: int, nbytes: int) -> tuple[int, bytes]:
    """IPC-shareable device buffer: (pointer, handle bytes for the other processes)."""
    lib = load_library()
    handle = ctypes.create_string_buffer(int(lib.tbvh_peer_handle_bytes()))
    ptr = _ptr()
    _check(lib.tbvh_peer_alloc(int(device), int(nbytes), ctypes.byref(ptr), ctypes.cast(handle, _ptr)))
    return int(ptr.value), handle.raw


def peer_open(device: int, handle: bytes) -> int:
    """Maps another process's buffer (from peer_alloc) on `device`; returns its address there."""
    lib = load_library()
    buf = ctypes.create_string_buffer(handle, len(handle))
    ptr = _ptr()
    _check(lib.tbvh_peer_open(int(device), ctypes.cast(buf, _ptr), ctypes.byref(ptr)))
    return int(ptr.value)


def peer_close(device: int, ptr: int) -> None:
    _check(load_library().tbvh_peer_close(int(device), _ptr(ptr)))


def peer_free(device: int, ptr: int) -> None:
    _check(load_library().tbvh_peer_free(int(device), _ptr(ptr)))


class _DeviceView:
    """__cuda_array_interface__ of a raw device buffer, for a zero-copy tensor view."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


# Array-interface type strings of the dtypes a shared buffer can hold.
_TYPESTR = {torch.int64: "<i8", torch.int32: "<i4", torch.float32: "<f4"}


def device_tensor(ptr: int, shape: tuple, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """Tensor over memory this module owns (no copy; the owner must outlive it)."""
    typestr = _TYPESTR[dtype]
    with torch.cuda.device(device):
        return torch.as_tensor(_DeviceView(ptr, shape, typestr), device=device)


def widen_indices(src: torch.Tensor, dst: torch.Tensor) -> None:
    """dst (int64) = src (int32), same number of elements, on the current stream."""
    if not (src.is_cuda and dst.is_cuda and src.is_contiguous() and dst.is_contiguous()
            and src.dtype == torch.int32 and dst.dtype == torch.int64 and src.numel() == dst.numel()):
        raise RuntimeError("widen_indices: need contiguous CUDA int32 -> int64 tensors of equal size")
    _check(load_library().tbvh_widen_indices(src.device.index, src.data_ptr(), dst.data_ptr(), src.numel(),
                                             _stream(src.device)))


def query_knn_share(node_aabbs: torch.Tensor, sorted_indices: torch.Tensor, num_points: int,
                    queries: torch.Tensor, share: torch.Tensor, k: int,
                    dest_indices: list[int], dest_distances: list[int], index_bits: int = 64,
                    multicast: bool = False) -> None:
    """k-NN of the queries listed in `share` (int64 indices into `queries`), each result
    row written at the query's row of every destination buffer (tbvh_query_knn_share;
    index_bits = 32: int32 destination index buffers, tbvh_query_knn_share_i32;
    multicast: one pair of multicast addresses, tbvh_query_knn_share_multicast)."""
    op = "query_knn_share"
    if not (queries.is_cuda and queries.is_contiguous() and queries.dtype == torch.float32 and queries.dim() == 2):
        raise RuntimeError(f"{op}: queries must be contiguous CUDA float32 (M, D)")
    if not (share.is_cuda and share.is_contiguous() and share.dtype == torch.int64 and share.dim() == 1):
        raise RuntimeError(f"{op}: share must be contiguous CUDA int64 (count,)")
    if len(dest_indices) != len(dest_distances) or not dest_indices:
        raise RuntimeError(f"{op}: one distance buffer per index buffer")
    device = queries.device
    lib = load_library()
    n_dest = len(dest_indices)
    idx_arr = (_ptr * n_dest)(*[_ptr(p) for p in dest_indices])
    dist_arr = (_ptr * n_dest)(*[_ptr(p) for p in dest_distances])
    hooks = _knn_hooks
    if hooks:
        for h in hooks:
            h("start", device)
    if index_bits not in (32, 64):
        raise RuntimeError(f"{op}: index_bits must be 32 or 64")
    if multicast:
        if n_dest != 1 or index_bits != 32:
            raise RuntimeError(f"{op}: multicast takes one pair of addresses and int32 indices")
        _check(lib.tbvh_query_knn_share_multicast(
            device.index, node_aabbs.data_ptr(), sorted_indices.data_ptr(), int(num_points), queries.data_ptr(),
            int(queries.size(0)), share.data_ptr(), int(share.numel()), int(queries.size(1)), int(k),
            dest_indices[0], dest_distances[0], _stream(device),
        ))
    else:
        entry = lib.tbvh_query_knn_share_i32 if index_bits == 32 else lib.tbvh_query_knn_share
        _check(entry(
            device.index, node_aabbs.data_ptr(), sorted_indices.data_ptr(), int(num_points), queries.data_ptr(),
            int(queries.size(0)), share.data_ptr(), int(share.numel()), int(queries.size(1)), int(k), n_dest,
            idx_arr, dist_arr, _stream(device),
        ))
    if hooks:
        for h in hooks:
            h("end", device)


# Optional observers of the traversal launch (bench.py times the kernel with
# CUDA events on the launching stream through this list). Empty by default.
_knn_hooks: list = []

_C = types.SimpleNamespace(
    build_bvh_batched_cooperative=build_bvh_batched_cooperative,
    morton_sort_queries_narrow=morton_sort_queries_narrow,
    query_knn_batched_cached_bounds=query_knn_batched_cached_bounds,
    query_knn_batched_cached_bounds_ordered=query_knn_batched_cached_bounds_ordered,
    query_knn_batched_cached_bounds_spatial=query_knn_batched_cached_bounds_spatial,
    query_knn_gather_positions=query_knn_gather_positions,
    build_bvh_ragged=build_bvh_ragged,
    morton_sort_queries_ragged=morton_sort_queries_ragged,
    query_knn_ragged=query_knn_ragged,
    tree_scalars=_tree_scalars,
    deferred_traversal_arrays=deferred_traversal_arrays,
)
