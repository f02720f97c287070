"""Full-output parity with the reference on the five benchmark configurations.

Every result row, tree and query permutation of c1–c5 at full size is compared
with digests of the reference's own CUDA outputs on the same seeded inputs
(``tests/golden/reference_configs.npz``, made by ``tests/golden/make_golden.py``
from the unmodified reference; c4's k = 32 from the reference's traversal
kernel instantiated at K = 32):

* per cloud: ``sorted_indices`` and ``node_aabbs`` bit-identical (SHA-256 of
  the bytes), the query Morton permutation identical;
* per 65,536-row block: canonical rows (each row's (distance bits, index)
  pairs in ascending order) identical, i.e. bit-identical distances and the
  same neighbour sets, in any order among exact ties;
* rows whose k-th distance ties with a (k+1)-th candidate: ``tie_equivalent``
  against the reference's stored rows (the tie may be cut at another member).

Reference behaviour matched: index-exact k-NN (torchbvh tests/test_knn.py:126-157),
batched ≡ per-cloud (tests/test_batched_knn.py:59-71), ragged ≡ per-cloud loop
(tests/test_ragged_knn.py:14-88).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import torchbvh_b200 as torchbvh
from tests.golden import digests
from torchbvh_b200 import _native, workloads

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_configs.npz"


@pytest.fixture(scope="module")
def golden():
    if not GOLDEN.exists():
        pytest.fail(f"{GOLDEN.name} missing: run tests/golden/make_golden.py on a GPU box")
    return np.load(GOLDEN)


def _per_cloud_inputs(w, pts, q):
    if w.points.dim() == 3:
        return [(b, pts[b], q[b]) for b in range(pts.shape[0])]
    if w.batch_offsets is not None:
        o, qo = w.batch_offsets.tolist(), w.query_offsets.tolist()
        return [(b, pts[o[b]:o[b + 1]], q[qo[b]:qo[b + 1]].contiguous()) for b in range(len(o) - 1)]
    return [(0, pts, q)]


def _cloud_handle(bvh, w, b):
    """(sorted_indices, node_aabbs, scene_min, scene_max) of cloud b."""
    if w.batch_offsets is not None:
        h = bvh._handles[b]
        return h["sorted_indices"], h["node_aabbs"], h["scene_min"], h["scene_max"]
    if w.points.dim() == 3:
        return bvh["sorted_indices"][b], bvh["node_aabbs"][b], bvh["scene_min"][b], bvh["scene_max"][b]
    return bvh["sorted_indices"], bvh["node_aabbs"], bvh["scene_min"], bvh["scene_max"]


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c5", "c4"])
def test_config_matches_reference(golden, oracle, name):
    dev = torch.device("cuda", 0)
    w = workloads.make(name)
    k = w.k
    pts, q = w.points.to(dev), w.queries.to(dev)
    bo = w.batch_offsets.to(dev) if w.batch_offsets is not None else None
    qo = w.query_offsets.to(dev) if w.query_offsets is not None else None
    bvh = torchbvh.build_bvh(pts, batch_offsets=bo)
    idx, dist = (torchbvh.query_knn(bvh, q, k, query_offsets=qo) if bo is not None
                 else torchbvh.query_knn(bvh, q, k))
    torch.cuda.synchronize()
    assert torchbvh.device_status() == 0

    # Trees and query permutations, cloud by cloud.
    sorted_sha = golden[f"{name}/tree_sorted_sha"]
    nodes_sha = golden[f"{name}/tree_nodes_sha"]
    order_sha = golden[f"{name}/order_sha"]
    clouds = _per_cloud_inputs(w, pts, q)
    assert len(clouds) == len(sorted_sha)
    packed_order = None
    if bo is not None:
        packed = bvh._require_packed()
        packed_order = _native.morton_sort_queries_ragged(q, qo, w.num_queries, packed["scene_min"],
                                                          packed["scene_max"])
    qo_h = w.query_offsets.tolist() if qo is not None else None
    for b, _, q_b in clouds:
        s_b, n_b, lo_b, hi_b = _cloud_handle(bvh, w, b)
        assert digests.tensor_digest(s_b) == sorted_sha[b], f"{name}: sorted_indices of cloud {b} differ"
        assert digests.tensor_digest(n_b) == nodes_sha[b], f"{name}: node_aabbs of cloud {b} differ"
        order = _native.morton_sort_queries_narrow(q_b.unsqueeze(0).contiguous(), lo_b.unsqueeze(0).contiguous(),
                                                   hi_b.unsqueeze(0).contiguous())[0]
        assert digests.tensor_digest(order) == order_sha[b], f"{name}: query permutation of cloud {b} differs"
        if packed_order is not None:
            assert digests.tensor_digest(packed_order[qo_h[b]:qo_h[b + 1]]) == order_sha[b], \
                f"{name}: packed ragged query permutation of cloud {b} differs"

    # Every result row.
    rows = int(golden[f"{name}/rows"])
    flat_idx, flat_dist = idx.reshape(-1, k), dist.reshape(-1, k)
    assert flat_idx.shape[0] == rows
    ties = golden[f"{name}/tie_rows"]
    keys = digests.canonical_keys(flat_idx, flat_dist)
    got = digests.block_digests(keys, ties)
    want = golden[f"{name}/block_sha"]
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, (f"{name}: {bad.size} of {want.size} blocks of {digests.BLOCK_ROWS} rows differ from the "
                           f"reference; first block {int(bad[0])} (rows {int(bad[0]) * digests.BLOCK_ROWS}...)")
    if ties.size:
        sel = torch.as_tensor(ties, device=dev)
        ok, msg = oracle.tie_equivalent(flat_idx.index_select(0, sel).cpu().numpy(),
                                        flat_dist.index_select(0, sel).cpu().numpy(),
                                        golden[f"{name}/tie_idx"], golden[f"{name}/tie_dist"])
        assert ok, f"{name}: boundary-tie rows: {msg}"
