"""Host logic of the multi-GPU layer on CPU: world_size-2 gloo process groups,
the CPU oracle standing in for the CUDA k-NN. Checks sharding, partition,
gather order and that a failing rank surfaces as an error on its peer
instead of a hang."""

from __future__ import annotations

import os
import socket
import tempfile
import traceback
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from torchbvh_b200 import distributed as tdist


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def oracle_knn(points, queries, k, *, batch_offsets=None, query_offsets=None):
    from oracle import pyoracle

    p, q = points.numpy(), queries.numpy()
    if p.ndim == 3:
        res = [pyoracle.knn_bruteforce(p[b], q[b], k, threads=1) for b in range(p.shape[0])]
        return (torch.from_numpy(np.stack([r[0] for r in res])), torch.from_numpy(np.stack([r[1] for r in res])))
    if batch_offsets is not None:
        bo, qo = batch_offsets.tolist(), query_offsets.tolist()
        res = [pyoracle.knn_bruteforce(p[bo[c]:bo[c + 1]], q[qo[c]:qo[c + 1]], k, threads=1)
               for c in range(len(bo) - 1)]
        return torch.from_numpy(np.concatenate([r[0] for r in res])), torch.from_numpy(np.concatenate([r[1] for r in res]))
    i, d = pyoracle.knn_bruteforce(p, q, k, threads=1)
    return torch.from_numpy(i), torch.from_numpy(d)


def oracle_order(points, queries):
    """Morton order of the queries against the points' bounding box (the CPU oracle's codes)."""
    from oracle import pyoracle

    lo = points.min(0).values.numpy()
    hi = points.max(0).values.numpy()
    codes = pyoracle.morton_codes(queries.numpy(), lo, hi)
    return torch.from_numpy(pyoracle.stable_argsort(codes).astype(np.int64))


def _data():
    g = torch.Generator().manual_seed(5)
    single_p = torch.rand((700, 3), generator=g)
    single_q = torch.rand((333, 3), generator=g)
    batched_p = torch.rand((5, 200, 2), generator=g)
    batched_q = torch.rand((5, 41, 2), generator=g)
    sizes = [50, 300, 17, 120, 64, 33, 200]
    qsizes = [5, 30, 1, 12, 9, 4, 20]
    bo = np.concatenate([[0], np.cumsum(sizes)]).tolist()
    qo = np.concatenate([[0], np.cumsum(qsizes)]).tolist()
    ragged_p = torch.rand((bo[-1], 3), generator=g)
    ragged_q = torch.rand((qo[-1], 3), generator=g)
    return single_p, single_q, batched_p, batched_q, ragged_p, bo, ragged_q, qo


def _worker(rank, world, port, outdir, mode):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
        sp, sq, bp, bq, rp, bo, rq, qo = _data()
        out = {}
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected host-side failure on rank 1")
        out["single_all"] = tdist.knn_sharded_single_cloud(sp if rank == 0 else None, sq, 8, num_points=700, dim=3,
                                                           split="contiguous", knn_fn=oracle_knn)
        out["single_root"] = tdist.knn_sharded_single_cloud(sp if rank == 0 else None, sq, 4, num_points=700, dim=3,
                                                            gather="root", split="contiguous", knn_fn=oracle_knn)
        out["morton_all"] = tdist.knn_sharded_single_cloud(sp if rank == 0 else None, sq, 8, num_points=700, dim=3,
                                                           order_fn=oracle_order, knn_fn=oracle_knn)
        out["morton_root"] = tdist.knn_sharded_single_cloud(sp if rank == 0 else None, sq, 4, num_points=700, dim=3,
                                                            gather="root", order_fn=oracle_order, knn_fn=oracle_knn)
        out["morton_none"] = tdist.knn_sharded_single_cloud(sp if rank == 0 else None, sq, 4, num_points=700, dim=3,
                                                            gather="none", order_fn=oracle_order, knn_fn=oracle_knn)
        out["batched"] = tdist.knn_sharded_batched(bp, bq, 4, knn_fn=oracle_knn)
        # An even split: every rank's block has the same length (gathered in place).
        out["batched_even"] = tdist.knn_sharded_batched(bp[:4].contiguous(), bq[:4].contiguous(), 4,
                                                        knn_fn=oracle_knn)
        out["ragged"] = tdist.knn_sharded_ragged(rp, bo, rq, qo, 4, knn_fn=oracle_knn)
        torch.save(out, Path(outdir) / f"rank{rank}.pt")
        dist.destroy_process_group()
    except Exception:
        (Path(outdir) / f"rank{rank}.err").write_text(traceback.format_exc())


def _run(world, mode):
    outdir = tempfile.mkdtemp()
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, outdir, mode)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    return Path(outdir)


def test_shard_range_covers_everything():
    for total in (0, 1, 7, 64, 1001):
        for world in (1, 2, 3, 8):
            spans = [tdist.shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(e - s for s, e in spans) - min(e - s for s, e in spans) <= 1


def test_partition_is_balanced_and_complete():
    sizes = [1024, 1_048_576, 5000, 700_000, 3000, 3000, 250_000, 90_000]
    parts = tdist.partition_clouds(sizes, 3)
    assert sorted(c for p in parts for c in p) == list(range(len(sizes)))
    loads = [sum(sizes[c] for c in p) for p in parts]
    assert max(loads) == 1_048_576  # the largest cloud alone bounds the makespan
    assert tdist.partition_clouds(sizes, 3) == parts  # deterministic


@pytest.mark.timeout(300)
def test_sharded_paths_match_single_process():
    outdir = _run(2, "ok")
    errs = list(outdir.glob("*.err"))
    assert not errs, errs[0].read_text()
    r0, r1 = torch.load(outdir / "rank0.pt"), torch.load(outdir / "rank1.pt")
    sp, sq, bp, bq, rp, bo, rq, qo = _data()
    ei, ed = oracle_knn(sp, sq, 8)
    for r in (r0, r1):
        assert torch.equal(r["single_all"][0], ei) and torch.equal(r["single_all"][1], ed)
    ei4, ed4 = oracle_knn(sp, sq, 4)
    assert torch.equal(r0["single_root"][0], ei4) and torch.equal(r0["single_root"][1], ed4)
    assert r1["single_root"] == (None, None)
    # Morton split: same results in the original query order; the shares are
    # consecutive ranges of the Morton order and cover every query once.
    for r in (r0, r1):
        assert torch.equal(r["morton_all"][0], ei) and torch.equal(r["morton_all"][1], ed)
    assert torch.equal(r0["morton_root"][0], ei4) and torch.equal(r0["morton_root"][1], ed4)
    assert r1["morton_root"] == (None, None)
    order = oracle_order(sp, sq)
    owned = torch.cat([r0["morton_none"][2], r1["morton_none"][2]])
    assert torch.equal(owned, order)
    for r in (r0, r1):
        i, d, rows = r["morton_none"]
        assert torch.equal(i, ei4[rows]) and torch.equal(d, ed4[rows])
    bi, bd = oracle_knn(bp, bq, 4)
    ri, rd = oracle_knn(rp, rq, 4, batch_offsets=torch.tensor(bo), query_offsets=torch.tensor(qo))
    for r in (r0, r1):
        assert torch.equal(r["batched"][0], bi) and torch.equal(r["batched"][1], bd)
        assert torch.equal(r["batched_even"][0], bi[:4]) and torch.equal(r["batched_even"][1], bd[:4])
        assert torch.equal(r["ragged"][0], ri) and torch.equal(r["ragged"][1], rd)


@pytest.mark.timeout(300)
def test_failing_rank_is_reported_not_hung():
    outdir = _run(2, "fail")
    err1 = (outdir / "rank1.err").read_text()
    assert "injected host-side failure" in err1
    # Rank 0 must leave its first collective with an error (peer gone), not wait forever.
    assert (outdir / "rank0.err").exists()
    assert not (outdir / "rank0.pt").exists()
