"""Batched and ragged k-NN on the GPU (ports tests/test_batched_knn.py and
tests/test_ragged_knn.py of the reference): per-sample results equal the
single-cloud path exactly, match the oracle, and indices stay local."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import torchbvh_b200 as torchbvh

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().cpu().numpy()


def _offsets(lengths):
    return torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int64, device="cuda")


@pytest.mark.parametrize("d", [2, 3])
@pytest.mark.parametrize("n", [16, 17, 31, 2000])
@pytest.mark.parametrize("k", [4, 8, 16])
def test_batched_matches_single_loop_and_oracle(oracle, d, n, k):
    rng = np.random.default_rng(13100 + d * 100 + n * 10 + k)
    pts = rng.random((3, n, d), dtype=np.float32)
    q = rng.random((3, 9 if n < 100 else 333, d), dtype=np.float32)
    pts_t, q_t = torch.from_numpy(pts).cuda(), torch.from_numpy(q).cuda()
    bvh = torchbvh.build_bvh(pts_t)
    idx, dist, pos = torchbvh.query_knn(bvh, q_t, k, source_points=pts_t)
    assert idx.shape == (3, q.shape[1], k) and dist.shape == idx.shape and pos.shape == (*idx.shape, d)
    for b in range(3):
        single = torchbvh.build_bvh(pts_t[b].contiguous())
        si, sd = torchbvh.query_knn(single, q_t[b].contiguous(), k)
        assert torch.equal(idx[b], si) and torch.equal(dist[b], sd)
        bi, bd = oracle.knn_bruteforce(pts[b], q[b], k)
        np.testing.assert_array_equal(_np(idx[b]), bi)
        np.testing.assert_array_equal(_np(dist[b]).view(np.uint32), bd.view(np.uint32))
        assert torch.equal(pos[b], pts_t[b][idx[b]])
    assert torchbvh.device_status() == 0


@pytest.mark.parametrize("k", [4, 8])
def test_batched_pathological_fixed_size_clouds(oracle, k):
    base17 = np.linspace(-1, 1, 17, dtype=np.float32)
    pts = np.stack([
        np.zeros((17, 2), np.float32),
        np.stack([base17, -2 * base17], 1),
        np.stack([base17 ** 2, np.full_like(base17, 3.0)], 1),
    ]).astype(np.float32)
    q = (pts[:, :7] + np.array([0.03, -0.02], np.float32)).astype(np.float32)
    bvh = torchbvh.build_bvh(torch.from_numpy(pts).cuda())
    idx, dist = torchbvh.query_knn(bvh, torch.from_numpy(q).cuda(), k)
    for b in range(3):
        bi, bd = oracle.knn_bruteforce(pts[b], q[b], k)
        np.testing.assert_array_equal(_np(idx[b]), bi)
        np.testing.assert_array_equal(_np(dist[b]).view(np.uint32), bd.view(np.uint32))


def test_batched_indices_are_local_not_flattened():
    g = torch.Generator().manual_seed(13200)
    pts = torch.rand((4, 20, 2), generator=g)
    pts[1:] += torch.tensor([10.0, -7.0])
    pts = pts.cuda()
    bvh = torchbvh.build_bvh(pts)
    idx, dist = torchbvh.query_knn(bvh, pts[:, :5].contiguous(), 4)
    assert int(idx.max()) < 20 and int(idx.min()) >= 0
    assert torch.all(dist[:, :, 0] == 0.0)


@pytest.mark.parametrize("d", [2, 3])
@pytest.mark.parametrize("k", [4, 8, 16, 32])
def test_ragged_matches_single_loop(oracle, d, k):
    rng = np.random.default_rng(14100 + d * 10 + k)
    counts = [k, k + 3, k + 9, 1500, k + 40, 70_001]
    qcounts = [3, 6, 4, 700, 33, 2049]
    pts = np.concatenate([rng.random((c, d), dtype=np.float32) + np.float32(20 * b) for b, c in enumerate(counts)])
    q = np.concatenate([rng.random((c, d), dtype=np.float32) + np.float32(20 * b) for b, c in enumerate(qcounts)])
    pts_t, q_t = torch.from_numpy(pts).cuda(), torch.from_numpy(q).cuda()
    bo, qo = _offsets(counts), _offsets(qcounts)
    bvh = torchbvh.build_bvh(pts_t, batch_offsets=bo)
    idx, dist, pos = torchbvh.query_knn(bvh, q_t, k, query_offsets=qo, source_points=pts_t)
    assert idx.shape == (sum(qcounts), k)
    start = 0
    for b, (c, qc) in enumerate(zip(counts, qcounts)):
        p0 = int(bo[b])
        sp = pts_t[p0:p0 + c].contiguous()
        sq = q_t[start:start + qc].contiguous()
        single = torchbvh.build_bvh(sp)
        si, sd, spos = torchbvh.query_knn(single, sq, k, source_points=sp)
        assert torch.equal(idx[start:start + qc], si), b
        assert torch.equal(dist[start:start + qc], sd), b
        assert torch.equal(pos[start:start + qc], spos), b
        if c * qc <= 20_000_000:
            bi, bd = oracle.knn_bruteforce(pts[p0:p0 + c], q[start:start + qc], k)
            np.testing.assert_array_equal(_np(si), bi)
            np.testing.assert_array_equal(_np(sd).view(np.uint32), bd.view(np.uint32))
        start += qc
    assert torchbvh.device_status() == 0


def test_ragged_queries_straddling_warps_and_clouds(oracle):
    # Query counts that are not multiples of 32 put several clouds in one warp.
    rng = np.random.default_rng(4)
    counts = [40, 50, 33, 64, 100]
    qcounts = [1, 5, 31, 2, 77]
    pts = np.concatenate([rng.random((c, 3), dtype=np.float32) * np.float32(b + 1) for b, c in enumerate(counts)])
    q = np.concatenate([rng.random((c, 3), dtype=np.float32) * np.float32(b + 1) for b, c in enumerate(qcounts)])
    bvh = torchbvh.build_bvh(torch.from_numpy(pts).cuda(), batch_offsets=_offsets(counts))
    idx, dist = torchbvh.query_knn(bvh, torch.from_numpy(q).cuda(), 4, query_offsets=_offsets(qcounts))
    pstart = qstart = 0
    for c, qc in zip(counts, qcounts):
        bi, bd = oracle.knn_bruteforce(pts[pstart:pstart + c], q[qstart:qstart + qc], 4)
        np.testing.assert_array_equal(_np(idx[qstart:qstart + qc]), bi)
        np.testing.assert_array_equal(_np(dist[qstart:qstart + qc]).view(np.uint32), bd.view(np.uint32))
        pstart += c
        qstart += qc


@pytest.mark.parametrize("d", [2, 3])
@pytest.mark.parametrize("k", [4, 8, 16])
def test_ragged_true_ties_are_local_members(oracle, d, k):
    dirs = np.concatenate([np.eye(d), -np.eye(d)]).astype(np.float32)
    counts = [k + 3, k + 7, k + 11]
    shifts = [np.full(d, -40.0, np.float32), np.full(d, 40.0, np.float32), np.linspace(-25, 25, d).astype(np.float32)]
    dup = np.zeros(d, np.float32)
    dup[0] = 1.0
    alt = np.zeros(d, np.float32)
    alt[-1] = -1.0
    samples = [
        np.broadcast_to(dup, (counts[0], d)) + shifts[0],
        np.tile(dirs, ((counts[1] + len(dirs) - 1) // len(dirs), 1))[: counts[1]] + shifts[1],
        np.broadcast_to(alt, (counts[2], d)) + shifts[2],
    ]
    pts = np.concatenate(samples).astype(np.float32)
    qcounts = [2, 3, 1]
    q = np.concatenate([np.broadcast_to(s, (c, d)) for s, c in zip(shifts, qcounts)]).astype(np.float32)
    bvh = torchbvh.build_bvh(torch.from_numpy(pts).cuda(), batch_offsets=_offsets(counts))
    idx, dist = torchbvh.query_knn(bvh, torch.from_numpy(q).cuda(), k, query_offsets=_offsets(qcounts))
    assert torch.all(dist == 1.0)
    pstart = qstart = 0
    for s, c, qc in zip(samples, counts, qcounts):
        bi, bd = oracle.knn_bruteforce(pts[pstart:pstart + c], q[qstart:qstart + qc], k)
        np.testing.assert_array_equal(_np(idx[qstart:qstart + qc]), bi)
        pstart += c
        qstart += qc


def test_ragged_neighbor_positions_gradients_flow_to_source_points_only():
    g = torch.Generator().manual_seed(51030)
    counts, qcounts = [8, 10, 12], [3, 4, 5]
    pts = torch.cat([torch.randn((c, 3), generator=g) + 20.0 * b for b, c in enumerate(counts)]).cuda()
    pts.requires_grad_()
    q = torch.cat([pts.detach()[sum(counts[:b]):sum(counts[:b]) + qc] + 0.025 for b, qc in enumerate(qcounts)])
    q.requires_grad_()
    bvh = torchbvh.build_bvh(pts, batch_offsets=_offsets(counts))
    idx, dist, pos = torchbvh.query_knn(bvh, q, 4, query_offsets=_offsets(qcounts), source_points=pts)
    assert not idx.requires_grad and not dist.requires_grad and pos.requires_grad
    pos.square().sum().backward()
    assert pts.grad is not None and torch.count_nonzero(pts.grad) > 0
    assert q.grad is None
