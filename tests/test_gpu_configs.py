"""The five benchmark configurations at full size on the GPU.

Per configuration: size-independent properties over every output row (on the
GPU), a seeded sample of queries against the exhaustive oracle (bit-identical
distances, canonical indices), a larger sample against the oracle's
restatement of the reference traversal over the GPU-built tree
(tie-equivalent), and the tree itself against the oracle rebuilt from the
GPU's Morton order (exact).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import torchbvh_b200 as torchbvh
from torchbvh_b200 import workloads

pytestmark = pytest.mark.gpu

SAMPLE_BRUTE = {"c1": 10_000, "c2": 256, "c3": 256, "c4": 384, "c5": 64}
SAMPLE_TREE = {"c1": 0, "c2": 4096, "c3": 4096, "c4": 65_536, "c5": 512}


def _clouds(w, dev):
    pts, q = w.points.to(dev), w.queries.to(dev)
    if w.batch_offsets is not None:
        return pts, q, w.batch_offsets.to(dev), w.query_offsets.to(dev)
    return pts, q, None, None


def _check_rows(idx: torch.Tensor, dist: torch.Tensor, n_per_row: torch.Tensor) -> None:
    assert torch.all(dist[:, 1:] >= dist[:, :-1])
    assert torch.all(idx >= 0)
    assert torch.all(idx < n_per_row[:, None])
    srt = idx.sort(dim=1).values
    assert torch.all(srt[:, 1:] != srt[:, :-1]), "duplicate neighbour in a row"


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c5", "c4"])
def test_config_full_size(oracle, name):
    dev = torch.device("cuda", 0)
    w = workloads.make(name)
    pts, q, bo, qo = _clouds(w, dev)
    k = w.k
    bvh = torchbvh.build_bvh(pts, batch_offsets=bo)
    if bo is not None:
        idx, dist = torchbvh.query_knn(bvh, q, k, query_offsets=qo)
    else:
        idx, dist = torchbvh.query_knn(bvh, q, k)
    torch.cuda.synchronize()
    assert torchbvh.device_status() == 0
    d = w.dim
    flat_idx = idx.reshape(-1, k)
    flat_dist = dist.reshape(-1, k)
    sizes = w.cloud_sizes()
    if bo is not None:
        qcounts = torch.diff(w.query_offsets).tolist()
        n_row = torch.repeat_interleave(torch.tensor(sizes, device=dev), torch.tensor(qcounts, device=dev))
        q_cloud = torch.repeat_interleave(torch.arange(len(sizes), device=dev), torch.tensor(qcounts, device=dev))
    else:
        per = w.num_queries // len(sizes)
        n_row = torch.full((w.num_queries,), sizes[0], device=dev)
        q_cloud = torch.arange(len(sizes), device=dev).repeat_interleave(per)
    _check_rows(flat_idx, flat_dist, n_row)

    # Cloud-local point arrays on the host.
    host_pts = w.points.numpy()
    host_q = w.queries.reshape(-1, d).numpy()
    if w.points.dim() == 3:
        cloud_pts = [host_pts[b] for b in range(host_pts.shape[0])]
    elif bo is not None:
        o = w.batch_offsets.tolist()
        cloud_pts = [host_pts[o[b]:o[b + 1]] for b in range(len(sizes))]
    else:
        cloud_pts = [host_pts]

    rng = np.random.default_rng(99)
    rows = rng.choice(w.num_queries, size=min(SAMPLE_BRUTE[name], w.num_queries), replace=False)
    rows.sort()
    rows_t = torch.from_numpy(rows).to(dev)
    gi = flat_idx.index_select(0, rows_t).cpu().numpy()
    gd = flat_dist.index_select(0, rows_t).cpu().numpy()
    clouds_of = q_cloud.index_select(0, rows_t).cpu().numpy()
    for b in np.unique(clouds_of):
        sel = clouds_of == b
        bi, bd = oracle.knn_bruteforce(cloud_pts[b], host_q[rows[sel]], k)
        np.testing.assert_array_equal(gd[sel].view(np.uint32), bd.view(np.uint32))
        np.testing.assert_array_equal(gi[sel], bi)

    if SAMPLE_TREE[name]:
        # Restated reference traversal over the GPU-built tree of one cloud.
        b = int(clouds_of[0]) if w.points.dim() == 3 or bo is not None else 0
        if w.points.dim() == 3:
            nodes = bvh["node_aabbs"][b].cpu().numpy()
            sidx = bvh["sorted_indices"][b].cpu().numpy()
            qrows = np.arange(b * (w.num_queries // len(sizes)), (b + 1) * (w.num_queries // len(sizes)))
        elif bo is not None:
            handle = bvh._handles[b]
            nodes = handle["node_aabbs"].cpu().numpy()
            sidx = handle["sorted_indices"].cpu().numpy()
            qo_h = w.query_offsets.tolist()
            qrows = np.arange(qo_h[b], qo_h[b + 1])
        else:
            nodes = bvh["node_aabbs"].cpu().numpy()
            sidx = bvh["sorted_indices"].cpu().numpy()
            qrows = np.arange(w.num_queries)
        tree_np = {"node_aabbs": nodes, "sorted_indices": sidx}
        rebuilt = oracle.build_tree(cloud_pts[b], sidx)
        np.testing.assert_array_equal(nodes, rebuilt["node_aabbs"])
        pick = np.sort(rng.choice(qrows, size=min(SAMPLE_TREE[name], qrows.size), replace=False))
        ri, rd = oracle.knn_reference(tree_np, host_q[pick], k, threads=oracle.default_threads())
        pick_t = torch.from_numpy(pick).to(dev)
        ok, msg = oracle.tie_equivalent(flat_idx.index_select(0, pick_t).cpu().numpy(),
                                        flat_dist.index_select(0, pick_t).cpu().numpy(), ri, rd)
        assert ok, msg
