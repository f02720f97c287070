"""The multi-GPU layer on real GPUs: NCCL process groups of 1 and 2 ranks (one
per GPU) running the sharded k-NN forms with the CUDA path, compared with the
single-GPU result. The 1-rank group runs on any GPU box (it still goes through
the IPC-shared result buffers and both index widths); the 2-rank group is
skipped on machines with fewer than 2 GPUs. NVLS is switched off and each group
has a short timeout."""

from __future__ import annotations

import os
import socket
import tempfile
import traceback
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(21)
    big_p = torch.rand((200_000, 3), generator=g)
    big_q = torch.rand((70_001, 3), generator=g)
    bp = torch.rand((5, 20_000, 2), generator=g)
    bq = torch.rand((5, 3_001, 2), generator=g)
    sizes = [5000, 40_000, 1024, 77_777, 3000]
    qsizes = [100, 2000, 10, 5000, 333]
    bo = [0]
    qo = [0]
    for a, b in zip(sizes, qsizes):
        bo.append(bo[-1] + a)
        qo.append(qo[-1] + b)
    rp = torch.rand((bo[-1], 3), generator=g)
    rq = torch.rand((qo[-1], 3), generator=g)
    return big_p, big_q, bp, bq, rp, bo, rq, qo


def _peer_query_sets(big_q):
    """A different query set per reuse of the same PeerResults buffers, so stale or
    racing rows from the previous call cannot pass as correct."""
    g = torch.Generator().manual_seed(22)
    return [big_q, big_q.flip(0).contiguous(), torch.rand(big_q.shape, generator=g)]


_PEER_FORMS = ((32, "peer"), (64, "peer"), (32, "multicast"))


def _worker(rank, world, port, outdir):
    import datetime

    import torch.distributed as dist

    from torchbvh_b200 import distributed as tdist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        big_p, big_q, bp, bq, rp, bo, rq, qo = _inputs()
        out = {}
        i, d = tdist.knn_sharded_single_cloud(big_p.to(dev) if rank == 0 else None, big_q.to(dev), 32,
                                              num_points=big_p.shape[0], dim=3, device=dev)
        out["single"] = (i.cpu(), d.cpu())
        i, d = tdist.knn_sharded_single_cloud(big_p.to(dev) if rank == 0 else None, big_q.to(dev), 32,
                                              num_points=big_p.shape[0], dim=3, device=dev, split="contiguous")
        out["single_contiguous"] = (i.cpu(), d.cpu())
        i, d, rows = tdist.knn_sharded_single_cloud(big_p.to(dev) if rank == 0 else None, big_q.to(dev), 32,
                                                    num_points=big_p.shape[0], dim=3, device=dev, gather="none")
        out["single_none"] = (i.cpu(), d.cpu(), rows.cpu())
        # Fused all-gather: each rank's traversal writes its rows into every
        # rank's buffers over NVLink (int32 or int64 indices on the wire); the
        # same buffers serve consecutive calls.
        # The multicast transport needs two or more GPUs whose switch supports it.
        for bits, transport in _PEER_FORMS:
            if transport == "multicast" and world == 1:
                continue
            try:
                peer = tdist.PeerResults(big_q.shape[0], 32, device=dev, index_bits=bits, transport=transport)
            except RuntimeError as exc:
                if "not available" not in str(exc):
                    raise
                out[f"transport{bits}{transport}"] = "unavailable"  # every rank sees the same answer
                continue
            out[f"transport{bits}{transport}"] = peer.transport_used
            for rep, (split, qset) in enumerate(zip(("morton", "morton", "contiguous"), _peer_query_sets(big_q))):
                i, d = tdist.knn_sharded_single_cloud(big_p.to(dev) if rank == 0 else None, qset.to(dev), 32,
                                                      num_points=big_p.shape[0], dim=3, device=dev, split=split,
                                                      out=peer)
                out[f"peer{bits}{transport}_{rep}"] = (i.cpu().clone(), d.cpu().clone())
            peer.close()
        i, d = tdist.knn_sharded_batched(bp.to(dev), bq.to(dev), 8)
        out["batched"] = (i.cpu(), d.cpu())
        i, d = tdist.knn_sharded_batched(bp[:4].to(dev), bq[:4].to(dev), 8)  # equal blocks on 1, 2 and 4 ranks
        out["batched_even"] = (i.cpu(), d.cpu())
        i, d = tdist.knn_sharded_ragged(rp.to(dev), bo, rq.to(dev), qo, 16)
        out["ragged"] = (i.cpu(), d.cpu())
        torch.cuda.synchronize(dev)
        torch.save(out, Path(outdir) / f"rank{rank}.pt")
        dist.destroy_process_group()
    except Exception:
        (Path(outdir) / f"rank{rank}.err").write_text(traceback.format_exc())


@pytest.mark.parametrize("world", [1, pytest.param(2, marks=pytest.mark.skipif(
    torch.cuda.device_count() < 2, reason="needs 2 GPUs"))])
@pytest.mark.timeout(600)
def test_sharded_knn_matches_one_gpu(world):
    import torchbvh_b200 as torchbvh

    outdir = tempfile.mkdtemp()
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, outdir)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    hung = [p for p in procs if p.is_alive()]
    for p in hung:
        p.kill()
    assert not hung, "a rank hung"
    errs = list(Path(outdir).glob("*.err"))
    assert not errs, errs[0].read_text()
    big_p, big_q, bp, bq, rp, bo, rq, qo = _inputs()
    dev = torch.device("cuda", 0)
    with torchbvh.BVH(big_p.to(dev)) as bvh:
        si, sd = bvh.knn(big_q.to(dev), 32)
        peer_want = [tuple(t.cpu() for t in bvh.knn(qset.to(dev), 32)) for qset in _peer_query_sets(big_q)]
    with torchbvh.BVH(bp.to(dev)) as bvh:
        bi, bd = bvh.knn(bq.to(dev), 8)
    bot = torch.tensor(bo, device=dev)
    qot = torch.tensor(qo, device=dev)
    with torchbvh.BVH(rp.to(dev), batch_offsets=bot) as bvh:
        ri, rd = bvh.knn(rq.to(dev), 16, query_offsets=qot)
    for r in range(world):
        got = torch.load(Path(outdir) / f"rank{r}.pt")
        assert torch.equal(got["single"][0], si.cpu()) and torch.equal(got["single"][1], sd.cpu())
        assert torch.equal(got["single_contiguous"][0], si.cpu())
        assert torch.equal(got["single_contiguous"][1], sd.cpu())
        i, d, rows = got["single_none"]
        assert torch.equal(i, si.cpu()[rows]) and torch.equal(d, sd.cpu()[rows])
        for bits, transport in _PEER_FORMS:
            used = got.get(f"transport{bits}{transport}")
            if used in (None, "unavailable"):  # multicast on one GPU, or a switch without it
                continue
            assert used == transport
            for rep in range(3):
                wi, wd = peer_want[rep]
                gi, gd = got[f"peer{bits}{transport}_{rep}"]
                assert torch.equal(gi, wi) and torch.equal(gd, wd), (bits, transport, rep)
        assert torch.equal(got["batched"][0], bi.cpu()) and torch.equal(got["batched"][1], bd.cpu())
        assert torch.equal(got["batched_even"][0], bi[:4].cpu()) and torch.equal(got["batched_even"][1], bd[:4].cpu())
        assert torch.equal(got["ragged"][0], ri.cpu()) and torch.equal(got["ragged"][1], rd.cpu())
    shares = [torch.load(Path(outdir) / f"rank{r}.pt")["single_none"][2] for r in range(world)]
    owned = torch.cat(shares)
    assert torch.equal(torch.sort(owned).values, torch.arange(big_q.shape[0]))
