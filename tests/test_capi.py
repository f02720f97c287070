"""C-ABI checks that need no GPU: the library loads, exports every entry point
declared in include/torchbvh_b200.h, sizes workspaces, and rejects bad
arguments before touching CUDA."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from torchbvh_b200 import _native

HEADER = Path(__file__).resolve().parents[1] / "include" / "torchbvh_b200.h"


def _declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(tbvh_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared_functions()
    for required in ("tbvh_build", "tbvh_sort_queries", "tbvh_query_knn", "tbvh_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol(native_lib):
    missing = [name for name in _declared_functions() if not hasattr(native_lib, name)]
    assert not missing, missing


def test_abi_version(native_lib):
    assert native_lib.tbvh_abi_version() == _native.ABI_VERSION


@pytest.mark.parametrize("n", [1, 2, 3, 5, 10_000, 65_536, 262_144, 16_777_216])
def test_real_node_count_matches_python(native_lib, n):
    assert native_lib.tbvh_real_node_count(n) == _native.real_node_count(n)


def test_workspace_sizes_are_positive(native_lib):
    assert native_lib.tbvh_build_workspace_size(16, 65_536, None, 3) > 16 * 65_536 * 16
    offs = (ctypes.c_int64 * 4)(0, 5, 1029, 3000)
    assert native_lib.tbvh_build_workspace_size(3, 0, ctypes.cast(offs, ctypes.c_void_p), 3) > 0
    assert native_lib.tbvh_sort_queries_workspace_size(8, 8 * 262_144, 2) > 0
    assert native_lib.tbvh_query_knn_workspace_size(64, 0) >= 64 * 8


def test_build_rejects_bad_dim_without_cuda(native_lib):
    rc = native_lib.tbvh_build(-1, 1, 1, 16, None, None, 4, 1, 1, 1, 1, None, None, None, 0, 1, 1 << 20, None)
    assert rc == _native.TBVH_ERR_BAD_ARG
    assert b"D must be 2 or 3" in native_lib.tbvh_last_error()


def test_build_rejects_small_workspace(native_lib):
    rc = native_lib.tbvh_build(-1, 1, 1, 16, None, None, 3, 1, 1, 1, 1, None, None, None, 0, 1, 16, None)
    assert rc == _native.TBVH_ERR_WORKSPACE


def test_build_rejects_ragged_without_offsets(native_lib):
    rc = native_lib.tbvh_build(-1, 1, 2, 0, None, None, 3, 1, 1, 1, 1, None, None, None, 0, 1, 1 << 20, None)
    assert rc == _native.TBVH_ERR_BAD_ARG


def test_build_rejects_non_increasing_offsets(native_lib):
    offs = (ctypes.c_int64 * 3)(0, 5, 5)
    rc = native_lib.tbvh_build(-1, 1, 2, 0, 1, ctypes.cast(offs, ctypes.c_void_p), 3, 1, 1, 1, 1, None, None,
                               None, 0, 1, 1 << 20, None)
    assert rc == _native.TBVH_ERR_BAD_ARG
    assert b"strictly increasing" in native_lib.tbvh_last_error()


def test_build_rejects_partial_traversal_arrays(native_lib):
    rc = native_lib.tbvh_build(-1, 1, 1, 16, None, None, 3, 1, 1, 1, 1, 1, None, None, 0, 1, 1 << 20, None)
    assert rc == _native.TBVH_ERR_BAD_ARG


def test_build_rejects_int32_overflow(native_lib):
    rc = native_lib.tbvh_build(-1, 1, 2, 2**30 + 1, None, None, 3, 1, 1, 1, 1, None, None, None, 0, 1, 1, None)
    assert rc == _native.TBVH_ERR_BAD_ARG
    assert b"int32" in native_lib.tbvh_last_error()


@pytest.mark.parametrize("k", [1, 5, 12, 64])
def test_query_rejects_unsupported_k(native_lib, k):
    rc = native_lib.tbvh_query_knn(-1, 1, 1, 1, 64, None, None, 1, 8, None, 8, None, 3, k, 1, 1, None, 0, None)
    assert rc == _native.TBVH_ERR_UNSUPPORTED_K
    assert b"k must be 4, 8, or 16" in native_lib.tbvh_last_error()


def test_query_rejects_too_few_points(native_lib):
    rc = native_lib.tbvh_query_knn(-1, 1, 1, 1, 8, None, None, 1, 8, None, 8, None, 3, 16, 1, 1, None, 0, None)
    assert rc == _native.TBVH_ERR_BAD_ARG
    assert b"num_leaves must be >= k" in native_lib.tbvh_last_error()


def test_query_rejects_ragged_cloud_smaller_than_k(native_lib):
    offs = (ctypes.c_int64 * 3)(0, 3, 40)
    rc = native_lib.tbvh_query_knn(-1, 1, 1, 2, 0, 1, ctypes.cast(offs, ctypes.c_void_p), 1, 0, 1, 8, None, 3, 4,
                                   1, 1, 1, 4096, None)
    assert rc == _native.TBVH_ERR_BAD_ARG


def test_query_rejects_mismatched_query_count(native_lib):
    rc = native_lib.tbvh_query_knn(-1, 1, 1, 2, 64, None, None, 1, 8, None, 15, None, 3, 4, 1, 1, None, 0, None)
    assert rc == _native.TBVH_ERR_BAD_ARG


def test_sort_queries_rejects_bad_dim(native_lib):
    rc = native_lib.tbvh_sort_queries(-1, 1, 1, 8, None, 8, 5, 1, 1, 1, 1, 1 << 20, None)
    assert rc == _native.TBVH_ERR_BAD_ARG


def test_empty_query_batch_is_a_no_op(native_lib):
    rc = native_lib.tbvh_query_knn(-1, 1, 1, 1, 64, None, None, 1, 0, 1, 0, None, 3, 4, 1, 1, None, 0, None)
    assert rc == _native.TBVH_OK


def test_gather_rejects_source_without_positions(native_lib):
    rc = native_lib.tbvh_query_knn_gather(-1, 1, 1, 1, 64, None, None, 1, 8, None, 8, None, 3, 4, 1, 1,
                                          1, None, 0, None, 0, None)
    assert rc == _native.TBVH_ERR_BAD_ARG
    assert b"both" in native_lib.tbvh_last_error()


def test_gather_rejects_spatial_without_order(native_lib):
    rc = native_lib.tbvh_query_knn_gather(-1, 1, 1, 1, 64, None, None, 1, 8, None, 8, None, 3, 4, 1, 1,
                                          None, None, 1, None, 0, None)
    assert rc == _native.TBVH_ERR_BAD_ARG
    assert b"spatial" in native_lib.tbvh_last_error()


def test_gather_checks_the_same_arguments_as_query(native_lib):
    rc = native_lib.tbvh_query_knn_gather(-1, 1, 1, 1, 64, None, None, 1, 8, None, 8, None, 3, 12, 1, 1,
                                          1, 1, 0, None, 0, None)
    assert rc == _native.TBVH_ERR_UNSUPPORTED_K


def test_peer_handle_is_a_cuda_ipc_handle(native_lib):
    assert native_lib.tbvh_peer_handle_bytes() == 64


def _share(native_lib, **kw):
    args = dict(device=-1, nodes=1, sorted=1, n=64, queries=1, m=16, order=1, count=16, dim=3, k=4,
                ndest=1, didx=None, ddist=None)
    args.update(kw)
    ptrs = (ctypes.c_void_p * 8)(*([1] * 8))
    didx = args["didx"] if args["didx"] is not None else ptrs
    ddist = args["ddist"] if args["ddist"] is not None else ptrs
    return native_lib.tbvh_query_knn_share(args["device"], args["nodes"], args["sorted"], args["n"], args["queries"],
                                           args["m"], args["order"], args["count"], args["dim"], args["k"],
                                           args["ndest"], didx, ddist, None)


@pytest.mark.parametrize("kw,code", [
    ({"dim": 4}, "BAD_ARG"), ({"k": 12}, "UNSUPPORTED_K"), ({"n": 2}, "BAD_ARG"),
    ({"count": 17}, "BAD_ARG"), ({"count": -1}, "BAD_ARG"), ({"ndest": 0}, "BAD_ARG"), ({"ndest": 9}, "BAD_ARG"),
])
def test_share_rejects_bad_arguments(native_lib, kw, code):
    assert _share(native_lib, **kw) == getattr(_native, "TBVH_ERR_" + code)


def test_share_rejects_null_destination(native_lib):
    ptrs = (ctypes.c_void_p * 8)(1, None, 1, 1, 1, 1, 1, 1)
    assert _share(native_lib, ndest=2, didx=ptrs) == _native.TBVH_ERR_BAD_ARG
    assert b"destination" in native_lib.tbvh_last_error()


def test_empty_share_is_a_no_op(native_lib):
    assert _share(native_lib, count=0) == _native.TBVH_OK


def test_multicast_share_checks_its_addresses_before_any_cuda_call(native_lib):
    """tbvh_query_knn_share_multicast takes one pair of 16-byte aligned multicast
    addresses; misaligned or NULL ones are refused with no CUDA call (no GPU here)."""
    call = native_lib.tbvh_query_knn_share_multicast
    args = dict(device=-1, nodes=16, sorted=16, n=64, queries=16, m=16, order=16, count=0, dim=3, k=8)

    def run(idx, dist, count=0):
        a = dict(args, count=count)
        return call(a["device"], a["nodes"], a["sorted"], a["n"], a["queries"], a["m"], a["order"], a["count"],
                    a["dim"], a["k"], idx, dist, None)

    assert run(4096 + 4, 8192) == _native.TBVH_ERR_BAD_ARG
    assert b"16-byte aligned" in native_lib.tbvh_last_error()
    assert run(4096, 8192 + 8) == _native.TBVH_ERR_BAD_ARG
    assert run(None, 8192) == _native.TBVH_ERR_BAD_ARG
    assert run(4096, 8192) == _native.TBVH_OK  # an empty share launches nothing
