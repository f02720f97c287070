"""numpy wrappers over the C oracle (oracle/tbvh_oracle.c) -- test infrastructure only.

Each function restates part of the reference algorithm; see tbvh_oracle.h for
the reference file:line each follows and the floating-point mode.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "libtbvh_oracle.so"
REF_LIB_PATH = ORACLE_DIR / "_ref" / "libtbvh_ref_headers.so"

_lock = threading.Lock()
_lib = None
_ref = None

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int


def reference_root() -> Path:
    """The reference checkout: TORCHBVH_REFERENCE_ROOT, else a directory named
    "reference" beside this repository (it need not exist)."""
    return Path(os.environ.get("TORCHBVH_REFERENCE_ROOT", str(ORACLE_DIR.parent.parent / "reference")))


def compile_libs(ref: bool = False) -> None:
    """Builds the oracle (and, when asked and the reference sources exist, the header shim)."""
    targets = ["all"] + (["ref", f"REF_ROOT={reference_root()}"] if ref else [])
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR), *targets], check=True)


def _stale(lib: Path, *sources: str) -> bool:
    if not lib.exists():
        return True
    return any((ORACLE_DIR / s).stat().st_mtime > lib.stat().st_mtime for s in sources)


def lib() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            if _stale(LIB_PATH, "tbvh_oracle.c", "tbvh_oracle.h"):
                compile_libs()
            l = ctypes.CDLL(str(LIB_PATH))
            l.tbo_real_node_count.restype = _i64
            l.tbo_real_node_count.argtypes = [_i64]
            l.tbo_leaf_level.restype = _i32
            l.tbo_leaf_level.argtypes = [_i64]
            l.tbo_build_and_query.argtypes = [_p, _p, _p, _p, _i64, _i32, _i32, _p, _p, _i32,
                                              ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
            for name, args in {
                "tbo_scene_bounds": [_p, _i64, _i32, _p, _p],
                "tbo_morton_codes": [_p, _i64, _i32, _p, _p, _p],
                "tbo_stable_argsort_u32": [_p, _i64, _p],
                "tbo_build_tree": [_p, _p, _i64, _i32, _p, _p, _p, _p],
                "tbo_build": [_p, _i64, _i32, _p, _p, _p, _p, _p, _p, _p],
                "tbo_knn_reference": [_p, _p, _i64, _i32, _p, _i64, _i32, _p, _p, _i32],
                "tbo_knn_bruteforce": [_p, _i64, _i32, _p, _i64, _i32, _p, _p, _i32],
                "tbo_pair_distances": [_p, _i64, _i32, _p, _i64, _i32, _p, _p],
            }.items():
                getattr(l, name).argtypes = args
                getattr(l, name).restype = None
            _lib = l
    return _lib


def ref_lib() -> ctypes.CDLL | None:
    """The reference's own Morton / implicit-tree headers compiled for the host, if available."""
    global _ref
    with _lock:
        if _ref is None:
            if not REF_LIB_PATH.exists():
                return None
            r = ctypes.CDLL(str(REF_LIB_PATH))
            r.tbr_morton_encode_3d.restype = ctypes.c_uint32
            r.tbr_morton_encode_3d.argtypes = [ctypes.c_float] * 3 + [_p, _p]
            r.tbr_morton_encode_2d.restype = ctypes.c_uint32
            r.tbr_morton_encode_2d.argtypes = [ctypes.c_float] * 2 + [_p, _p]
            for name in ("tbr_real_node_count", "tbr_leaf_level", "tbr_virtual_leaves"):
                getattr(r, name).restype = _i32
                getattr(r, name).argtypes = [_i32]
            for name in ("tbr_memory_index", "tbr_is_virtual"):
                getattr(r, name).restype = _i32
                getattr(r, name).argtypes = [_i32, _i32]
            _ref = r
    return _ref


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def default_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


def real_node_count(n: int) -> int:
    return int(lib().tbo_real_node_count(n))


def leaf_level(n: int) -> int:
    return int(lib().tbo_leaf_level(n))


def scene_bounds(points) -> tuple[np.ndarray, np.ndarray]:
    pts = _f32(points)
    n, d = pts.shape
    lo = np.empty(d, np.float32)
    hi = np.empty(d, np.float32)
    lib().tbo_scene_bounds(_ptr(pts), n, d, _ptr(lo), _ptr(hi))
    return lo, hi


def morton_codes(points, lo, hi) -> np.ndarray:
    pts = _f32(points)
    lo, hi = _f32(lo), _f32(hi)
    n, d = pts.shape
    codes = np.empty(n, np.uint32)
    lib().tbo_morton_codes(_ptr(pts), n, d, _ptr(lo), _ptr(hi), _ptr(codes))
    return codes


def stable_argsort(keys) -> np.ndarray:
    keys = np.ascontiguousarray(keys, dtype=np.uint32)
    perm = np.empty(keys.size, np.int64)
    lib().tbo_stable_argsort_u32(_ptr(keys), keys.size, _ptr(perm))
    return perm


def build_tree(points, sorted_indices) -> dict:
    pts = _f32(points)
    n, d = pts.shape
    sidx = np.ascontiguousarray(sorted_indices, dtype=np.int64)
    nr = real_node_count(n)
    nodes = np.empty((nr, 2 * d), np.float32)
    left = np.empty(nr, np.int32)
    right = np.empty(nr, np.int32)
    m2l = np.empty(nr, np.int32)
    lib().tbo_build_tree(_ptr(pts), _ptr(sidx), n, d, _ptr(nodes), _ptr(left), _ptr(right), _ptr(m2l))
    return {"node_aabbs": nodes, "left_child_mem": left, "right_child_mem": right, "mem_to_leaf": m2l}


def build(points) -> dict:
    """Whole reference build for one cloud (bounds, Morton codes, stable sort, tree)."""
    pts = _f32(points)
    n, d = pts.shape
    nr = real_node_count(n)
    out = {
        "node_aabbs": np.empty((nr, 2 * d), np.float32),
        "sorted_indices": np.empty(n, np.int64),
        "scene_min": np.empty(d, np.float32),
        "scene_max": np.empty(d, np.float32),
        "left_child_mem": np.empty(nr, np.int32),
        "right_child_mem": np.empty(nr, np.int32),
        "mem_to_leaf": np.empty(nr, np.int32),
    }
    lib().tbo_build(_ptr(pts), n, d, *(_ptr(out[k]) for k in (
        "node_aabbs", "sorted_indices", "scene_min", "scene_max", "left_child_mem", "right_child_mem",
        "mem_to_leaf")))
    leaf = leaf_level(n)
    out.update(num_leaves=n, num_real_nodes=nr, leaf_level=leaf, virtual_leaves=(1 << leaf) - n, dim=d)
    return out


def knn_reference(tree: dict, queries, k: int, threads: int = 1) -> tuple[np.ndarray, np.ndarray]:
    """The reference's DFS traversal over `tree` (node_aabbs + sorted_indices)."""
    q = _f32(queries)
    m, d = q.shape
    nodes = _f32(tree["node_aabbs"])
    sidx = np.ascontiguousarray(tree["sorted_indices"], dtype=np.int64)
    idx = np.empty((m, k), np.int64)
    dist = np.empty((m, k), np.float32)
    lib().tbo_knn_reference(_ptr(nodes), _ptr(sidx), sidx.size, d, _ptr(q), m, k, _ptr(idx), _ptr(dist), threads)
    return idx, dist


def knn_bruteforce(points, queries, k: int, threads: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """Exhaustive k-NN ordered by (distance, index) with the reference arithmetic."""
    pts = _f32(points)
    q = _f32(queries)
    n, d = pts.shape
    m = q.shape[0]
    idx = np.empty((m, k), np.int64)
    dist = np.empty((m, k), np.float32)
    lib().tbo_knn_bruteforce(_ptr(pts), n, d, _ptr(q), m, k, _ptr(idx), _ptr(dist),
                             threads if threads > 0 else default_threads())
    return idx, dist


def pair_distances(points, queries, idx) -> np.ndarray:
    """Squared distance of each (query row, returned index) pair with the reference arithmetic."""
    pts = _f32(points)
    q = _f32(queries)
    idx = np.ascontiguousarray(idx, dtype=np.int64)
    m, k = idx.shape
    out = np.empty((m, k), np.float32)
    lib().tbo_pair_distances(_ptr(pts), pts.shape[0], pts.shape[1], _ptr(q), m, k, _ptr(idx), _ptr(out))
    return out


def build_and_query(points, pt_offsets, queries, q_offsets, k: int, threads: int = 0):
    """Reference build + DFS query for packed clouds; returns (idx, dist, build_s, query_s)."""
    pts = _f32(points)
    q = _f32(queries)
    po = np.ascontiguousarray(pt_offsets, dtype=np.int64)
    qo = np.ascontiguousarray(q_offsets, dtype=np.int64)
    d = pts.shape[1]
    m = q.shape[0]
    idx = np.empty((m, k), np.int64)
    dist = np.empty((m, k), np.float32)
    tb = ctypes.c_double(0.0)
    tq = ctypes.c_double(0.0)
    lib().tbo_build_and_query(_ptr(pts), _ptr(po), _ptr(q), _ptr(qo), po.size - 1, d, k, _ptr(idx), _ptr(dist),
                              threads if threads > 0 else default_threads(), ctypes.byref(tb), ctypes.byref(tq))
    return idx, dist, tb.value, tq.value


def tie_equivalent(idx_a, dist_a, idx_b, dist_b) -> tuple[bool, str]:
    """Compares two k-NN results row by row, allowing differences only among exactly tied distances.

    Distances must be bitwise equal. Within each group of equal distances the
    index sets must match, except the last (k-th) group, which may be cut at a
    different member of the tie.
    """
    idx_a, idx_b = np.asarray(idx_a), np.asarray(idx_b)
    dist_a, dist_b = np.asarray(dist_a), np.asarray(dist_b)
    if idx_a.shape != idx_b.shape or dist_a.shape != dist_b.shape:
        return False, f"shape mismatch {idx_a.shape} vs {idx_b.shape}"
    k = idx_a.shape[-1]
    ia = idx_a.reshape(-1, k)
    ib = idx_b.reshape(-1, k)
    da = dist_a.reshape(-1, k)
    db = dist_b.reshape(-1, k)
    if not np.array_equal(da.view(np.uint32), db.view(np.uint32)):
        bad = np.nonzero((da.view(np.uint32) != db.view(np.uint32)).any(axis=1))[0]
        r = int(bad[0])
        return False, f"{bad.size} rows differ in distance bits; first row {r}: {da[r]} vs {db[r]}"
    same = (ia == ib).all(axis=1)
    for r in np.nonzero(~same)[0]:
        row_d = da[r]
        start = 0
        while start < k:
            end = start
            while end + 1 < k and row_d[end + 1] == row_d[start]:
                end += 1
            sa, sb = set(ia[r, start:end + 1].tolist()), set(ib[r, start:end + 1].tolist())
            if end + 1 < k and sa != sb:
                return False, f"row {r}: tie group {start}..{end} differs: {sorted(sa)} vs {sorted(sb)}"
            start = end + 1
    return True, ""
