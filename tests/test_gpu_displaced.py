"""Displaced-query k-NN and matching-head interpolation on the GPU.

Behavioural ports of the reference's tests/test_displaced_query.py cases:
flattened-query equivalence, per-sample BVH with flattened queries only,
matching-head gather, the weighted-mean and exact-hit interpolation rules and
the gradient boundary (values only).
"""
from __future__ import annotations

import pytest
import torch

import torchbvh_b200 as torchbvh
import torchbvh_b200._multihead as multihead_module

pytestmark = pytest.mark.gpu


def _inputs(batch=2, n=24, heads=3, dim=3, channels=4, seed=0):
    g = torch.Generator().manual_seed(9000 + seed + batch * 100 + n * 10 + heads + dim)
    pos = torch.rand((batch, n, dim), generator=g)
    pos = pos + 8.0 * torch.arange(batch, dtype=torch.float32).view(batch, 1, 1)
    q = pos[:, :, None, :] + 0.015 * torch.randn((batch, n, heads, dim), generator=g)
    values = torch.randn((batch, n, heads, channels), generator=g)
    return pos.cuda().contiguous(), q.cuda().contiguous(), values.cuda().contiguous()


def _hard_geometry(dim):
    """Two samples of 32 points: four coincident points at the origin, a tiny
    cluster (1e-5), a far cluster (1e4), a stretched line (1e-3 x 1e3); heads 0
    sit exactly on the points (exact hits), heads 1-2 are displaced."""
    n = 32
    t = torch.linspace(-1.0, 1.0, n - 4)
    cols = [t, 0.5 * t] + ([torch.zeros_like(t)] if dim == 3 else [])
    rows = torch.stack(cols, dim=-1)
    rows[0:6] = 0.0
    rows[0:6, 0] = 1.0e-5 * t[:6]
    rows[6:14, 0] = 1.0e4 + 17.0 * t[6:14]
    rows[6:14, 1] = -2.0e4 + 3.0 * t[6:14]
    rows[14:22, 0] = 1.0e-3 * t[14:22]
    rows[14:22, 1] = 1.0e3 * t[14:22]
    base = torch.zeros((n, dim))
    base[4:] = rows
    pos = base.unsqueeze(0) + 7.5e4 * torch.arange(2, dtype=torch.float32).view(2, 1, 1)
    q = pos[:, :, None, :].repeat(1, 1, 3, 1)
    q[:, :, 1, :] += 0.013
    q[:, :, 2, 0] += torch.linspace(-0.02, 0.02, n)
    values = torch.arange(2 * n * 3 * 5, dtype=torch.float32).reshape(2, n, 3, 5)
    return pos.cuda().contiguous(), q.cuda().contiguous(), values.cuda().contiguous()


def _weighted_mean_oracle(values, indices, d2):
    """Per-element restatement of torchbvh/_multihead.py:123-190 in float64."""
    b, n, h, k = indices.shape
    vals = values.double().cpu()
    idx = indices.cpu()
    dd = d2.double().cpu()
    out = torch.empty((b, n, h, values.size(-1)), dtype=torch.float64)
    for bi in range(b):
        for i in range(n):
            for hi in range(h):
                d = dd[bi, i, hi]
                neigh = vals[bi, idx[bi, i, hi], hi]
                exact = d <= 1.0e-12
                if bool(exact.any()):
                    out[bi, i, hi] = neigh[exact].mean(dim=0)
                else:
                    w = 1.0 / (d + 1.0e-12)
                    w = w / w.sum()
                    out[bi, i, hi] = (neigh * w[:, None]).sum(dim=0)
    return out.float().cuda()


def test_displaced_returns_local_sorted_results_and_positions():
    pos, q, _ = _inputs(batch=3, n=28, heads=2, dim=2)
    idx, d2, npos = torchbvh.query_displaced_knn(pos, q, 4)
    assert idx.shape == (3, 28, 2, 4) and d2.shape == (3, 28, 2, 4) and npos.shape == (3, 28, 2, 4, 2)
    assert idx.dtype == torch.int64 and d2.dtype == torch.float32
    assert int(idx.min()) >= 0 and int(idx.max()) < 28
    assert torch.all(d2[..., :-1] <= d2[..., 1:])
    for b in range(3):
        assert torch.equal(npos[b], pos[b, idx[b]])
    torch.testing.assert_close(d2, (npos - q[:, :, :, None, :]).square().sum(-1), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("k", [4, 8, 16, 32])
def test_displaced_equals_flattened_batched_query(k):
    pos, q, _ = _inputs(batch=2, n=40, heads=4, dim=3, seed=k)
    b, n, h, d = q.shape
    bvh = torchbvh.build_bvh(pos)
    fi, fd, fp = torchbvh.query_knn(bvh, q.reshape(b, n * h, d), k, source_points=pos)
    idx, d2, npos = torchbvh.query_displaced_knn(pos, q, k)
    assert torch.equal(idx, fi.reshape(b, n, h, k))
    assert torch.equal(d2, fd.reshape(b, n, h, k))
    assert torch.equal(npos, fp.reshape(b, n, h, k, d))


def test_displaced_builds_per_sample_and_flattens_queries_only(monkeypatch):
    pos, q, _ = _inputs(batch=2, n=10, heads=3, dim=3)
    calls = []

    def fake_build(points):
        calls.append(("build", tuple(points.shape), points.requires_grad))
        return torchbvh.BatchedBVHHandle({})

    def fake_query(bvh, query_points, k, *, source_points=None, sort_queries=True):
        calls.append(("query", tuple(query_points.shape), k,
                      None if source_points is None else tuple(source_points.shape), sort_queries))
        b, m, d = query_points.shape
        idx = torch.zeros((b, m, k), dtype=torch.int64, device=query_points.device)
        dist = torch.zeros((b, m, k), device=query_points.device)
        if source_points is None:
            return idx, dist
        return idx, dist, torch.zeros((b, m, k, d), device=query_points.device)

    monkeypatch.setattr(multihead_module, "_build_bvh_batched", fake_build)
    monkeypatch.setattr(multihead_module, "_query_knn_batched", fake_query)
    idx, d2, npos = torchbvh.query_displaced_knn(pos.requires_grad_(), q.requires_grad_(), 4)
    assert idx.shape == (2, 10, 3, 4) and npos.shape == (2, 10, 3, 4, 3)
    assert calls == [("build", (2, 10, 3), False), ("query", (2, 30, 3), 4, (2, 10, 3), True)]


def test_displaced_can_skip_positions():
    pos, q, _ = _inputs(batch=2, n=20, heads=2, dim=2)
    result = torchbvh.query_displaced_knn(pos, q, 4, return_positions=False)
    assert len(result) == 2 and result[0].shape == (2, 20, 2, 4)


def test_displaced_rejects_unsupported_k():
    pos, q, _ = _inputs(batch=2, n=16, heads=2, dim=2)
    with pytest.raises(ValueError, match="k must be 4, 8, or 16"):
        torchbvh.query_displaced_knn(pos, q, 5)


@pytest.mark.parametrize("bad", ["pos_rank", "q_rank", "batch", "points", "dtype"])
def test_displaced_shape_validation_on_gpu(bad):
    pos, q, _ = _inputs()
    if bad == "pos_rank":
        pos, match = pos[0], "pos.*shape"
    elif bad == "q_rank":
        q, match = q.reshape(q.size(0), -1, q.size(3)), "q.*shape"
    elif bad == "batch":
        pos, match = pos[:1], "batch size"
    elif bad == "points":
        q, match = q[:, :3], "point dimension"
    else:
        q, match = q.double(), "float32"
    with pytest.raises(ValueError, match=match):
        torchbvh.query_displaced_knn(pos, q, 4)


def test_gather_neighbor_values_reads_matching_head_only():
    g = torch.Generator().manual_seed(5)
    values = torch.arange(2 * 6 * 3 * 4, dtype=torch.float32).reshape(2, 6, 3, 4).cuda()
    indices = torch.randint(0, 6, (2, 6, 3, 2), generator=g).cuda()
    out = torchbvh.gather_neighbor_values(values, indices)
    assert out.shape == (2, 6, 3, 2, 4)
    for b in range(2):
        for i in range(6):
            for h in range(3):
                assert torch.equal(out[b, i, h], values[b, indices[b, i, h], h])


def test_gather_neighbor_values_rejects_foreign_indices():
    values = torch.zeros((1, 4, 2, 3), device="cuda")
    with pytest.raises(ValueError, match="local source indices"):
        torchbvh.gather_neighbor_values(values, torch.full((1, 4, 2, 2), 4, dtype=torch.int64, device="cuda"))
    with pytest.raises(ValueError, match="values must be float32"):
        torchbvh.gather_neighbor_values(values.double(), torch.zeros((1, 4, 2, 2), dtype=torch.int64, device="cuda"))


def test_gather_neighbor_values_gradients_reach_values():
    values = torch.randn((2, 6, 3, 4), device="cuda", requires_grad=True)
    indices = torch.randint(0, 6, (2, 6, 3, 2), device="cuda")
    torchbvh.gather_neighbor_values(values, indices).square().sum().backward()
    assert values.grad is not None and torch.count_nonzero(values.grad) > 0


def test_interpolate_weighted_mean_matches_oracle():
    pos, q, values = _inputs(batch=2, n=24, heads=2, dim=3, channels=3)
    out = torchbvh.interpolate_displaced(pos, q, values, 4)
    idx, d2 = torchbvh.query_displaced_knn(pos, q, 4, return_positions=False)
    assert not bool((d2 <= 1e-12).any())
    assert out.shape == (2, 24, 2, 3)
    torch.testing.assert_close(out, _weighted_mean_oracle(values, idx, d2), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize(("dim", "k"), [(2, 4), (3, 8), (3, 16)])
def test_hard_geometry_matches_flattened_query(dim, k):
    pos, q, values = _hard_geometry(dim)
    b, n, h, _ = q.shape
    fi, fd, fp = torchbvh.query_knn(torchbvh.build_bvh(pos), q.reshape(b, n * h, dim), k, source_points=pos)
    idx, d2, npos = torchbvh.query_displaced_knn(pos, q, k)
    assert torch.all(d2[..., :-1] <= d2[..., 1:])
    assert torch.equal(idx, fi.reshape(b, n, h, k))
    assert torch.equal(d2, fd.reshape(b, n, h, k))
    assert torch.equal(npos, fp.reshape(b, n, h, k, dim))


def test_interpolate_exact_hits_average_and_gradient_boundary():
    pos, q, values = _hard_geometry(2)
    pos = pos.requires_grad_(True)
    q = q.requires_grad_(True)
    values = values.requires_grad_(True)
    out = torchbvh.interpolate_displaced(pos, q, values, 4)
    idx, d2 = torchbvh.query_displaced_knn(pos, q, 4, return_positions=False)
    exact = d2 <= 1e-12
    assert bool(exact[:, 0, 0].all())
    torch.testing.assert_close(out, _weighted_mean_oracle(values.detach(), idx, d2), rtol=1e-5, atol=1e-5)
    out.square().sum().backward()
    assert values.grad is not None and torch.count_nonzero(values.grad) > 0
    assert pos.grad is None and q.grad is None


def test_displaced_outputs_are_detached():
    pos, q, _ = _inputs(batch=2, n=20, heads=2, dim=3)
    pos.requires_grad_(True)
    q.requires_grad_(True)
    idx, d2, npos = torchbvh.query_displaced_knn(pos, q, 4)
    assert not (idx.requires_grad or d2.requires_grad or npos.requires_grad)
