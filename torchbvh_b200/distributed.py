"""Multi-GPU k-NN over ``torch.distributed`` (one process per GPU).

The reference is single-GPU; this module adds the sharded forms of its three
input shapes:

* ``knn_sharded_single_cloud``: one large cloud. Rank ``src`` holds the
  points; they are broadcast (NCCL over NVLink), every rank builds the same
  BVH, takes its share of the queries, queries it, and the result slices are
  all-gathered (or gathered to ``src``, or left where they were computed).
  The share is a contiguous range of the queries' Morton order
  (``split="morton"``, the default) or of their given order
  (``split="contiguous"``): Morton ranges keep each warp's 32 queries
  spatially close and each rank's walk to one region of the tree, where a
  slice of randomly ordered queries spreads every warp over the whole cloud.
* ``knn_sharded_batched``: fixed-size batches, clouds split contiguously over
  ranks, results all-gathered in cloud order.
* ``knn_sharded_ragged``: ragged batches, clouds assigned by a size-balanced
  greedy partition (largest first onto the least-loaded rank), results
  returned in the original packed order.

The collectives are the only data exchange. ``knn_fn`` defaults to this
package's CUDA path; tests pass a CPU function to exercise the host logic over
the gloo backend. All ranks call every collective in the same order.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
import torch.distributed as dist

KnnFn = Callable[..., tuple[torch.Tensor, torch.Tensor]]


def default_knn(points: torch.Tensor, queries: torch.Tensor, k: int, *, batch_offsets=None,
                query_offsets=None) -> tuple[torch.Tensor, torch.Tensor]:
    """One build + query through the public API (the CUDA path)."""
    from ._bvh_class import BVH

    with BVH(points, batch_offsets=batch_offsets) as bvh:
        if batch_offsets is not None:
            return bvh.knn(queries, k, query_offsets=query_offsets)
        return bvh.knn(queries, k)


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, end) slice of `total` items owned by `rank` (sizes differ by at most one)."""
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def partition_clouds(sizes: list[int], world: int) -> list[list[int]]:
    """Greedy longest-processing-time partition: clouds by size (desc, then index), each
    onto the currently least-loaded rank (lowest rank on ties). Returns cloud ids per
    rank, each list in ascending cloud order."""
    load = [0] * world
    parts: list[list[int]] = [[] for _ in range(world)]
    for c in sorted(range(len(sizes)), key=lambda i: (-sizes[i], i)):
        r = min(range(world), key=lambda j: (load[j], j))
        parts[r].append(c)
        load[r] += sizes[c]
    return [sorted(p) for p in parts]


def _world(group) -> tuple[int, int]:
    return dist.get_world_size(group), dist.get_rank(group)


def _all_gather_rows(local: torch.Tensor, counts: list[int], group) -> torch.Tensor:
    """Every rank's row block, concatenated in rank order. Equal blocks are
    gathered straight into the result (one collective, no copies); blocks of
    different lengths are padded to the longest and compacted afterwards."""
    world, _ = _world(group)
    width = tuple(local.shape[1:])
    longest = max(counts)
    gathered = torch.empty((longest * world, *width), dtype=local.dtype, device=local.device)
    if all(c == longest for c in counts):
        dist.all_gather_into_tensor(gathered, local.contiguous(), group=group)
        return gathered
    padded = torch.zeros((longest, *width), dtype=local.dtype, device=local.device)
    padded[: local.shape[0]] = local
    dist.all_gather_into_tensor(gathered, padded, group=group)
    return torch.cat([gathered[r * longest: r * longest + c] for r, c in enumerate(counts)])


SPLITS = ("morton", "interleaved", "contiguous")

# Optional observers of the phases of one sharded single-cloud call, each
# called as hook(phase, device) on the host as the phase's work is enqueued
# (bench.py records CUDA events there). Empty by default.
_phase_hooks: list = []


def _phase(name: str, device) -> None:
    for hook in _phase_hooks:
        hook(name, device)


_RUNS_PER_RANK = 32  # ownership runs per rank of the interleaved split


def _split_chunk(m: int, world: int, split: str) -> int:
    """Queries per ownership run: one run per rank ("morton"), or 32 runs per rank
    dealt round-robin over the Morton order ("interleaved")."""
    if split == "morton":
        return -(-m // world)
    return max(1, -(-m // (world * _RUNS_PER_RANK)))


def _owned_by_order(order: torch.Tensor, m: int, world: int, rank: int, split: str) -> torch.Tensor:
    """This rank's queries from a full traversal order (CPU paths and tests): the
    positions of `order` whose run (position // chunk) the rank owns."""
    chunk = _split_chunk(m, world, split)
    runs = torch.arange(m, device=order.device) // chunk
    return order[runs % world == rank]


def _owned_queries_cuda(handle, queries: torch.Tensor, rank: int, world: int, split: str) -> torch.Tensor:
    """This rank's query indices in traversal order on the CUDA path. Morton
    splits select and sort only the rank's own share (tbvh_share_queries);
    every rank derives the same split, so the shares partition the queries."""
    from ._native import share_queries

    m = queries.shape[0]
    if split == "contiguous":
        q0, q1 = shard_range(m, world, rank)
        return torch.arange(q0, q1, dtype=torch.int64, device=queries.device)
    return share_queries(queries, handle["scene_min"], handle["scene_max"], rank, world,
                         _split_chunk(m, world, split))


_SIDE_STREAMS: dict = {}


def _side_stream(device: torch.device) -> torch.cuda.Stream:
    """One extra stream per device for work that runs beside the build."""
    key = torch.device(device).index
    if key not in _SIDE_STREAMS:
        _SIDE_STREAMS[key] = torch.cuda.Stream(device=device)
    return _SIDE_STREAMS[key]


def _build_and_share(points: torch.Tensor, queries: torch.Tensor, rank: int, world: int, split: str):
    """The BVH of `points` (built on the current stream) and this rank's share of
    the queries, selected at the same time on a side stream: the share needs only
    the scene box, which tbvh_scene_bounds gives bit-identical to the build's, so
    the selection overlaps the build's sort and tree kernels. The current stream
    waits for the share before anything after this call. Returns (bvh, share)."""
    from ._bvh_class import BVH
    from ._native import scene_bounds, share_queries

    main = torch.cuda.current_stream(points.device)
    ready = torch.cuda.Event()
    ready.record(main)
    bvh = BVH(points)
    _phase("build", queries.device)
    m = queries.shape[0]
    if split == "contiguous":
        q0, q1 = shard_range(m, world, rank)
        return bvh, torch.arange(q0, q1, dtype=torch.int64, device=queries.device)
    side = _side_stream(points.device)
    side.wait_event(ready)
    with torch.cuda.stream(side):
        lo, hi = scene_bounds(points)
        share = share_queries(queries, lo, hi, rank, world, _split_chunk(m, world, split))
    main.wait_stream(side)
    share.record_stream(main)
    return bvh, share


class PeerResults:
    """(M, k) result buffers on every rank of `group`, each mapped on every other
    rank through CUDA IPC, for ``knn_sharded_single_cloud(..., gather="all", out=...)``.

    With it, the all-gather is fused into the traversal: each rank writes every
    result row of its share into all ranks' buffers (NVLink stores) as the rows
    are produced, instead of an NCCL all-gather after the traversal.
    ``indices`` / ``distances`` are this rank's (M, k) buffers; a call
    overwrites them. Each call begins with a collective on every rank's current
    stream before any rank writes, so reads of the previous results enqueued on
    the current stream (or finished on the host) are safe on every rank; reads
    on other streams must be ordered before the next call by the caller.
    Create once, reuse across calls, ``close()`` on every rank together (a
    collective).

    ``index_bits=32`` (default): indices cross NVLink as int32 (8 instead of 12
    bytes per neighbour; point counts are below 2^31) into a shared int32
    buffer, and each rank widens its copy into the int64 ``indices`` tensor
    after the rows have arrived. ``index_bits=64`` writes int64 directly.

    ``transport``: "peer" (default) maps every rank's buffers on every other
    rank (CUDA IPC) and the traversal stores each row once per rank;
    "multicast" binds every rank's buffer to one NVLink multicast object
    (PyTorch symmetric memory) and the traversal stores each row once, through
    the multicast address, for the switch to deliver to all ranks (int32
    indices only; a RuntimeError on every rank if some rank lacks multicast
    support). On 8 B200 the multicast stores made c4's traversal slower
    (9.0-10.0 ms against 7.3-8.1 ms with peer stores), so peer is the default.
    ``transport_used`` says which one is in use.
    """

    def __init__(self, num_queries: int, k: int, *, group=None, device: torch.device | None = None,
                 index_bits: int = 32, transport: str = "peer"):
        from . import _native

        if index_bits not in (32, 64):
            raise ValueError("PeerResults: index_bits must be 32 or 64")
        if transport not in ("multicast", "peer"):
            raise ValueError("PeerResults: transport must be 'multicast' or 'peer'")
        if transport == "multicast" and index_bits != 32:
            raise ValueError("PeerResults: the multicast transport carries int32 indices (index_bits=32)")
        self.group = group
        self.world, self.rank = _world(group)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.num_queries, self.k = int(num_queries), int(k)
        self.index_bits = index_bits
        self.closed = False
        self._flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._opened: list[int] = []
        self._own: list = []
        self._symm = None
        shape = (self.num_queries, self.k)
        if transport == "multicast":
            if not self._open_multicast(shape):
                raise RuntimeError("PeerResults: NVLink multicast is not available on every rank")
            self.transport_used = "multicast"
            return
        self.transport_used = "peer"
        dev = self.device.index
        rows = max(self.num_queries, 1) * self.k
        self._own = [_native.peer_alloc(dev, rows * index_bits // 8), _native.peer_alloc(dev, rows * 4)]
        handles = [None] * self.world
        dist.all_gather_object(handles, (self._own[0][1], self._own[1][1]), group=group)
        self._opened: list[int] = []
        self.dest_indices: list[int] = []
        self.dest_distances: list[int] = []
        for r in range(self.world):
            if r == self.rank:
                pi, pd = self._own[0][0], self._own[1][0]
            else:
                pi = _native.peer_open(dev, handles[r][0])
                pd = _native.peer_open(dev, handles[r][1])
                self._opened += [pi, pd]
            self.dest_indices.append(pi)
            self.dest_distances.append(pd)
        shape = (self.num_queries, self.k)
        if index_bits == 64:
            self.indices = _native.device_tensor(self._own[0][0], shape, torch.int64, self.device)
            self._wire_indices = None
        else:
            self._wire_indices = _native.device_tensor(self._own[0][0], shape, torch.int32, self.device)
            self.indices = torch.empty(shape, dtype=torch.int64, device=self.device)
        self.distances = _native.device_tensor(self._own[1][0], shape, torch.float32, self.device)

    def _open_multicast(self, shape: tuple) -> bool:
        """One symmetric-memory buffer per rank (int32 indices, then float32
        distances), all bound to one multicast object. A collective; every rank
        reaches the same answer."""
        from torch.distributed import _symmetric_memory as symm_mem
        from torch._C._distributed_c10d import _SymmetricMemory

        ok = self.world > 1
        if ok:
            try:
                ok = bool(_SymmetricMemory.has_multicast_support(symm_mem.DeviceType.CUDA, self.device.index))
            except Exception:
                ok = False
        if not self._all_ranks(ok):
            return False
        rows = max(self.num_queries, 1) * self.k
        try:
            buf = symm_mem.empty(2 * rows, dtype=torch.int32, device=self.device)
            handle = symm_mem.rendezvous(buf, self.group if self.group is not None else dist.group.WORLD)
            mc = int(handle.multicast_ptr)
        except Exception:  # e.g. no symmetric-memory backend: every rank falls back together
            buf = handle = None
            mc = 0
        if not self._all_ranks(mc != 0):
            del handle, buf
            return False
        # The multicast address of this tensor: same offset as in the local buffer.
        at = mc + (buf.data_ptr() - int(handle.buffer_ptrs[handle.rank]))
        self._symm = (buf, handle)
        self.dest_indices = [at]
        self.dest_distances = [at + rows * 4]
        self._wire_indices = buf[:rows].view(-1)[: shape[0] * shape[1]].view(shape)
        self.distances = buf[rows:].view(torch.float32)[: shape[0] * shape[1]].view(shape)
        self.indices = torch.empty(shape, dtype=torch.int64, device=self.device)
        return True

    def _all_ranks(self, ok: bool) -> bool:
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=self.device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.group)
        return bool(flag.item())

    def delivered(self) -> None:
        """Collective on the current stream after the writing launches: once it
        completes on a rank, every peer's rows have arrived in its buffers."""
        dist.all_reduce(self._flag, group=self.group)

    def _widen(self) -> None:
        """int32 wire indices -> this rank's int64 ``indices`` (after delivered())."""
        if self._wire_indices is not None:
            from . import _native

            _native.widen_indices(self._wire_indices, self.indices)

    def close(self) -> None:
        from . import _native

        if self.closed:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._opened:
            _native.peer_close(self.device.index, p)
        self.indices = self.distances = self._wire_indices = None
        self._symm = None  # every rank releases its multicast binding after the barrier above
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p, _ in self._own:
            _native.peer_free(self.device.index, p)
        self.closed = True

    def __enter__(self) -> "PeerResults":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


def _share_to_peers(points: torch.Tensor, queries: torch.Tensor, k: int, rank: int, world: int, split: str,
                    out: PeerResults):
    """One BVH build; this rank's share of the queries; results delivered to
    every rank's `out`."""
    from ._native import query_knn_share

    bvh, share = _build_and_share(points, queries, rank, world, split)
    with bvh:
        h = bvh._handle
        # No rank may store into a peer's buffers while that peer still reads the
        # previous call's rows: a collective on every rank's current stream, after
        # its earlier reads and before any traversal, orders them.
        out.delivered()
        _phase("share", queries.device)
        query_knn_share(h["node_aabbs"], h["sorted_indices"], points.shape[0], queries, share, k,
                        out.dest_indices, out.dest_distances, index_bits=out.index_bits,
                        multicast=out.transport_used == "multicast")
    _phase("traversal", queries.device)
    out.delivered()
    out._widen()
    _phase("delivered", queries.device)
    return out.indices, out.distances


def knn_sharded_single_cloud(points: torch.Tensor | None, queries: torch.Tensor, k: int, *,
                             num_points: int, dim: int, src: int = 0, group=None, gather: str = "all",
                             split: str = "morton", order_fn: Callable | None = None,
                             knn_fn: KnnFn = default_knn, device: torch.device | None = None,
                             out: "PeerResults | None" = None):
    """Exact k-NN of one cloud with the queries split over ranks.

    `points` is read on rank `src` only (other ranks may pass None); every rank
    passes the full `queries` tensor. `split` ("morton", "interleaved",
    "contiguous") decides which queries each rank serves:

    * "morton": one contiguous range of the queries' Morton order (codes
      against the shared BVH's scene box), of nearly equal size per rank;
    * "interleaved": runs of the Morton order (32 per rank) dealt to the ranks
      in turn, so that every rank gets queries from every region of the cloud
      and the per-rank cost evens out;
    * "contiguous": a contiguous slice of the given query order.

    On the CUDA path each rank selects and sorts only its own share. With
    `order_fn(points, queries)` (a full traversal order) or a custom
    `knn_fn`, the Morton splits are taken from `order_fn`'s order (default:
    this package's Morton sort).

    `gather`: "all" returns the full (M, k) results in the original query order
    on every rank, "root" only on `src` (None elsewhere), "none" returns this
    rank's rows and which queries they belong to (the (start, end) range for
    "contiguous", else the int64 query indices).

    `out` (a PeerResults, gather="all" with the CUDA path only): the traversal
    itself delivers every row to every rank; the returned tensors are views of
    `out`, valid until the next call with it.
    """
    if split not in SPLITS:
        raise ValueError("knn_sharded_single_cloud: split must be 'morton', 'interleaved' or 'contiguous'")
    world, rank = _world(group)
    dev = device or queries.device
    buf = points if rank == src else torch.empty((num_points, dim), dtype=torch.float32, device=dev)
    buf = buf.contiguous()
    _phase("start", dev)
    dist.broadcast(buf, src=src, group=group)
    _phase("broadcast", dev)
    m = queries.shape[0]
    q0, q1 = shard_range(m, world, rank)
    queries = queries.contiguous()
    if out is not None:
        if gather != "all" or knn_fn is not default_knn or order_fn is not None:
            raise ValueError("knn_sharded_single_cloud: out= needs gather='all' and the CUDA path")
        if out.num_queries != m or out.k != k:
            raise ValueError("knn_sharded_single_cloud: out= was made for another query count or k")
        return _share_to_peers(buf, queries, k, rank, world, split, out)
    if split == "contiguous":
        idx, dist_sq = knn_fn(buf, queries[q0:q1].contiguous(), k)
        owned = torch.arange(q0, q1, dtype=torch.int64, device=queries.device)
    elif order_fn is None and knn_fn is default_knn:
        bvh, owned = _build_and_share(buf, queries, rank, world, split)
        with bvh:
            idx, dist_sq = bvh.knn(queries.index_select(0, owned), k, sort_queries=False)
    else:
        order = order_fn(buf, queries) if order_fn is not None else _full_morton_order(buf, queries)
        owned = _owned_by_order(order, m, world, rank, split)
        idx, dist_sq = knn_fn(buf, queries.index_select(0, owned).contiguous(), k)
    if gather == "none":
        return idx, dist_sq, ((q0, q1) if split == "contiguous" else owned)
    counts = _share_sizes(owned.numel(), group, owned.device)
    if gather == "root":
        idx_all = _gather_to(idx, counts, src, group)
        dist_all = _gather_to(dist_sq, counts, src, group)
        owners = _gather_to(owned.unsqueeze(1), counts, src, group)
        if rank != src:
            return None, None
        return _to_query_order(idx_all, owners[:, 0]), _to_query_order(dist_all, owners[:, 0])
    idx_all = _all_gather_rows(idx, counts, group)
    dist_all = _all_gather_rows(dist_sq, counts, group)
    owners = _all_gather_rows(owned.unsqueeze(1), counts, group)[:, 0]
    return _to_query_order(idx_all, owners), _to_query_order(dist_all, owners)


def _full_morton_order(points: torch.Tensor, queries: torch.Tensor) -> torch.Tensor:
    """All queries in Morton order against the points' BVH (CUDA)."""
    from ._bvh_class import BVH
    from ._native import _C

    with BVH(points) as bvh:
        h = bvh._handle
        return _C.morton_sort_queries_narrow(queries.unsqueeze(0), h["scene_min"].unsqueeze(0),
                                             h["scene_max"].unsqueeze(0))[0]


def _share_sizes(n: int, group, device: torch.device) -> list[int]:
    """Every rank's share size (one small all-gather)."""
    world, _ = _world(group)
    mine = torch.tensor([n], dtype=torch.int64, device=device)
    sizes = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(sizes, mine, group=group)
    return [int(s.item()) for s in sizes]


def _to_query_order(rows: torch.Tensor, owners: torch.Tensor) -> torch.Tensor:
    """Rows gathered rank by rank -> rows in query order (row p belongs to query owners[p])."""
    out = torch.empty_like(rows)
    out.index_copy_(0, owners.to(rows.device), rows)
    return out


def _gather_to(local: torch.Tensor, counts: list[int], dst: int, group) -> torch.Tensor | None:
    world, rank = _world(group)
    longest = max(counts)
    padded = torch.zeros((longest, *local.shape[1:]), dtype=local.dtype, device=local.device)
    padded[: local.shape[0]] = local
    bufs = [torch.empty_like(padded) for _ in range(world)] if rank == dst else None
    dist.gather(padded, bufs, dst=dst, group=group)
    if rank != dst:
        return None
    return torch.cat([b[:c] for b, c in zip(bufs, counts)])


def knn_sharded_batched(points: torch.Tensor, queries: torch.Tensor, k: int, *, group=None,
                        knn_fn: KnnFn = default_knn) -> tuple[torch.Tensor, torch.Tensor]:
    """(B, N, D) clouds split contiguously over ranks; returns full (B, M, k) on every rank."""
    world, rank = _world(group)
    b = points.shape[0]
    c0, c1 = shard_range(b, world, rank)
    m = queries.shape[1]
    _phase("start", queries.device)
    if c1 > c0:
        idx, dist_sq = knn_fn(points[c0:c1].contiguous(), queries[c0:c1].contiguous(), k)
    else:
        idx = torch.empty((0, m, k), dtype=torch.int64, device=queries.device)
        dist_sq = torch.empty((0, m, k), dtype=torch.float32, device=queries.device)
    _phase("compute", queries.device)
    counts = [shard_range(b, world, r)[1] - shard_range(b, world, r)[0] for r in range(world)]
    gathered = _all_gather_rows(idx, counts, group), _all_gather_rows(dist_sq, counts, group)
    _phase("gathered", queries.device)
    return gathered


def knn_sharded_ragged(points: torch.Tensor, batch_offsets: list[int], queries: torch.Tensor,
                       query_offsets: list[int], k: int, *, group=None,
                       knn_fn: KnnFn = default_knn) -> tuple[torch.Tensor, torch.Tensor]:
    """Ragged clouds (host offsets) partitioned by size; returns packed (total_M, k) on every rank."""
    world, rank = _world(group)
    nb = len(batch_offsets) - 1
    sizes = [batch_offsets[c + 1] - batch_offsets[c] for c in range(nb)]
    parts = partition_clouds(sizes, world)
    _phase("start", queries.device)
    mine = parts[rank]
    dev = queries.device
    if mine:
        p_local = torch.cat([points[batch_offsets[c]:batch_offsets[c + 1]] for c in mine])
        q_local = torch.cat([queries[query_offsets[c]:query_offsets[c + 1]] for c in mine])
        lo = [0]
        qlo = [0]
        for c in mine:
            lo.append(lo[-1] + sizes[c])
            qlo.append(qlo[-1] + query_offsets[c + 1] - query_offsets[c])
        idx, dist_sq = knn_fn(p_local, q_local, k,
                              batch_offsets=torch.tensor(lo, dtype=torch.int64, device=dev),
                              query_offsets=torch.tensor(qlo, dtype=torch.int64, device=dev))
    else:
        idx = torch.empty((0, k), dtype=torch.int64, device=dev)
        dist_sq = torch.empty((0, k), dtype=torch.float32, device=dev)
    qcount = [sum(query_offsets[c + 1] - query_offsets[c] for c in parts[r]) for r in range(world)]
    _phase("compute", dev)
    all_idx = _all_gather_rows(idx, qcount, group)
    all_dist = _all_gather_rows(dist_sq, qcount, group)
    # Back to the original packed order: gathered row p (clouds rank by rank, each
    # rank's clouds ascending) is packed query row owner[p], computed on the device.
    clouds = [c for r in range(world) for c in parts[r]]
    lens = torch.tensor([query_offsets[c + 1] - query_offsets[c] for c in clouds], dtype=torch.int64)
    gathered_start = torch.cumsum(lens, 0) - lens
    shift = torch.tensor([query_offsets[c] for c in clouds], dtype=torch.int64) - gathered_start
    total = int(lens.sum())
    owner = torch.repeat_interleave(shift.to(dev), lens.to(dev), output_size=total) + \
        torch.arange(total, dtype=torch.int64, device=dev)
    result = _to_query_order(all_idx, owner), _to_query_order(all_dist, owner)
    _phase("gathered", dev)
    return result
