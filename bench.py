"""Benchmark of the B200 BVH k-NN path (build + query), one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c1..c5]
                    [--impl b200|reference|reference_cuda]

A step is one ``BVH(points)`` build plus one ``.knn(queries, k)`` query over one
batch of the seeded synthetic workload (torchbvh_b200.workloads), through the
public API. Default workload: c4, the largest configuration and the only one
that is strong-scaled (one sphere-shell cloud of 16,777,216 3-D points, as many
queries, k = 32). Metric: k-NN queries/sec (build + query).

* ``value``: device-resident inputs, CUDA events around each step on the
  current stream, L2 flushed (256 MiB write) between steps outside the events,
  summed over K steps, max over ranks. On one GPU: build + query. On N > 1
  GPUs, c4 is one cloud sharded over the ranks (strong scaling): rank 0's
  points broadcast, the BVH built on every rank, the queries split by Morton
  range, and every result row delivered to every rank (the traversal writes
  each row into all ranks' buffers over NVLink), i.e. results all-gathered;
  ``results_in_place`` times the same step with the rows left on the rank
  that computed them, ``nccl_all_gather`` with an NCCL all-gather after the
  traversal instead. c2 / c3 / c5 on N GPUs are sharded by cloud (strong
  scaling: each rank builds and queries its clouds, results all-gathered by
  NCCL); ``--replicas`` runs N independent replicas instead (weak scaling);
  c1 always runs replicas.
* ``e2e``: the same public API with the inputs in pinned host memory: per step
  H2D copy of points and queries, build, query with ``out=`` pinned host
  tensors (D2H copy of indices and distances), all inside the events.
* ``roofline``: the traversal kernel (dominant), algorithmic query bytes per
  launch over its event-timed duration, against MEASURED_PEAKS.json hbm_gbs.
* ``cpu_baseline``: the CPU port of the reference algorithm (oracle/, C,
  all host threads) on a bounded sample of the same workload, rank 0 only.
* ``cpu_bruteforce``: ``torch.cdist`` + ``topk`` on all host threads over a
  bounded sample, extrapolated (rank 0, one GPU only).
* ``--impl reference``: that CPU port as the reference arm (the reference's k-NN
  has no CPU implementation of its own). ``--impl reference_cuda``: the
  reference's CUDA path from baseline/_ref, if installed.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "k-NN queries/sec (build+query)"
UNIT = "queries/s"
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="c4", choices=["c1", "c2", "c3", "c4", "c5"])
    ap.add_argument("--impl", default="b200", choices=["b200", "reference", "reference_cuda"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--replicas", action="store_true",
                    help="c2 / c3 / c5 on N > 1 GPUs: N independent replicas of the whole workload "
                         "(weak scaling) instead of the clouds sharded over the ranks")
    ap.add_argument("--c4-points", type=int, default=16_777_216,
                    help="points (= queries) of workload c4; smaller values make ncu-sized cases")
    ap.add_argument("--c4-index-bits", type=int, default=32, choices=[32, 64],
                    help="c4 on N > 1 GPUs: width of the indices the traversal sends over NVLink")
    ap.add_argument("--c4-transport", default="peer", choices=["peer", "multicast"],
                    help="c4 on N > 1 GPUs: rows to every rank by one NVLink store per peer (default) or "
                         "one multicast store per row")
    ap.add_argument("--c4-split", default="morton", choices=["morton", "interleaved", "contiguous"],
                    help="c4 on N > 1 GPUs: share of the queries per rank (one range of their Morton order, "
                         "runs of it dealt to the ranks in turn, or a range of their given order)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------

def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# clocks (NVML, read-only sampling during the timed region)
# ---------------------------------------------------------------------------

_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
    0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


class ClockSampler:
    def __init__(self, device_index: int, period_s: float = 0.01):
        self.samples: list[tuple[int, int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._period = period_s
        try:
            import pynvml

            pynvml.nvmlInit()
            uuid = torch.cuda.get_device_properties(device_index).uuid
            handle = None
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                u = pynvml.nvmlDeviceGetUUID(h)
                u = u.decode() if isinstance(u, bytes) else u
                if u.replace("GPU-", "") == str(uuid).replace("GPU-", ""):
                    handle = h
                    break
            if handle is None:
                handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self._nvml = pynvml
            self._handle = handle
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # no NVML: report the absence instead of guessing
            self._nvml = None
            self.error = str(exc)

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                util = nv.nvmlDeviceGetUtilizationRates(self._handle).gpu
                self.samples.append((mhz, reasons, util))
            except Exception:
                pass
            time.sleep(self._period)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict:
        if self._nvml is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "note": f"NVML unavailable: {getattr(self, 'error', '')}"}
        loaded = [s for s in self.samples if not (s[1] & 0x1)] or self.samples
        reasons = set()
        for _, r, _ in loaded:
            for bit, name in _REASONS.items():
                if r & bit and bit != 0x1:
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(s[0] for s in loaded) if loaded else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(reasons),
            "samples": len(loaded),
        }


# ---------------------------------------------------------------------------
# workload helpers
# ---------------------------------------------------------------------------

def load_workload(name: str, args=None):
    from torchbvh_b200 import workloads

    if name == "c4" and args is not None and args.c4_points != 16_777_216:
        return workloads.make("c4", n=args.c4_points, m=args.c4_points)
    return workloads.make(name)


def workload_config(w, world: int) -> dict:
    cfg = {
        "workload": w.name,
        "clouds": w.num_clouds,
        "points": w.num_points,
        "queries": w.num_queries,
        "dim": w.dim,
        "k": w.k,
        "l2": "flushed between steps (256 MiB write outside the timed events)",
        "parallelism": f"dp{world} (every rank runs the full workload on its own GPU)" if world > 1 else "single GPU",
    }
    if w.batch_offsets is not None:
        sizes = w.cloud_sizes()
        cfg["cloud_size_min"] = min(sizes)
        cfg["cloud_size_max"] = max(sizes)
    return cfg


def algorithmic_bytes(w) -> tuple[int, int]:
    from torchbvh_b200 import workloads

    sizes = w.cloud_sizes()
    if w.query_offsets is not None:
        qsizes = torch.diff(w.query_offsets).tolist()
    else:
        qsizes = [w.num_queries // len(sizes)] * len(sizes)
    return workloads.algorithmic_bytes(sizes, qsizes, w.dim, w.k)


def measured_peak_hbm() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def profiled_traffic(workload: str):
    p = ROOT / "profiles" / "knn_traffic.json"
    if not p.exists():
        return None, None
    try:
        data = json.loads(p.read_text())
        entry = data.get(workload)
        if entry is None:
            return None, None
        return float(entry["bytes_per_launch"]), entry.get("source")
    except Exception:
        return None, None


# ---------------------------------------------------------------------------
# the B200 arm
# ---------------------------------------------------------------------------

def run_b200(args, world, rank, local):
    import torchbvh_b200 as torchbvh
    from torchbvh_b200 import _native

    device = torch.device("cuda", local)
    w = load_workload(args.workload, args)
    points = w.points.to(device)
    queries = w.queries.to(device)
    offsets = w.batch_offsets.to(device) if w.batch_offsets is not None else None
    qoffsets = w.query_offsets.to(device) if w.query_offsets is not None else None
    k = w.k

    def step(p, q, o, qo, result=None):
        bvh = torchbvh.BVH(p, batch_offsets=o)
        out = bvh.knn(q, k, query_offsets=qo, out=result) if o is not None else bvh.knn(q, k, out=result)
        return bvh, out

    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    # traversal-kernel timing through the native hook (events on the launching stream)
    knn_events: list = []

    def hook(phase, dev):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(dev))
        knn_events.append((phase, ev))

    # Warm-up holds references the way the timed loop does (the previous step's
    # BVH and results stay alive while the next step runs), so the caching
    # allocator has grown to its steady state before timing starts; otherwise
    # the second timed step pays for new device segments.
    bvh = out = None
    for _ in range(args.warmup):
        bvh, out = step(points, queries, offsets, qoffsets)
    torch.cuda.synchronize(device)
    assert torchbvh.device_status(device) == 0

    # ---- timed region (device-resident inputs) ----
    build_ms = []
    step_ms = []
    launches0 = _native.load_library().tbvh_kernel_launch_count()
    barrier(world)
    torch.cuda.synchronize(device)
    _native._knn_hooks.append(hook)
    sampler = ClockSampler(local)
    with sampler:
        for _ in range(args.steps):
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e2 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            bvh = torchbvh.BVH(points, batch_offsets=offsets)
            e1.record(stream)
            out = bvh.knn(queries, k, query_offsets=qoffsets) if offsets is not None else bvh.knn(queries, k)
            e2.record(stream)
            build_ms.append((e0, e1))
            step_ms.append((e0, e2))
        torch.cuda.synchronize(device)
    _native._knn_hooks.remove(hook)
    barrier(world)
    torch.cuda.synchronize(device)
    launches = _native.load_library().tbvh_kernel_launch_count() - launches0
    status = torchbvh.device_status(device)

    total_ms = sum(a.elapsed_time(b) for a, b in step_ms)
    build_total_ms = sum(a.elapsed_time(b) for a, b in build_ms)
    starts = [e for ph, e in knn_events if ph == "start"]
    ends = [e for ph, e in knn_events if ph == "end"]
    knn_ms = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    total_ms_max = max_over_ranks(total_ms, world)
    queries_total = w.num_queries * args.steps * world
    value = queries_total / (total_ms_max / 1e3)

    # ---- e2e: pinned host inputs, copies inside the timed region ----
    e2e = None
    if not args.no_e2e:
        hp = w.points.pin_memory()
        hq = w.queries.pin_memory()
        ho = w.batch_offsets.pin_memory() if w.batch_offsets is not None else None
        hqo = w.query_offsets.pin_memory() if w.query_offsets is not None else None
        qshape = (*w.queries.shape[:-1], k)
        out_idx = torch.empty(qshape, dtype=torch.int64).pin_memory()
        out_dist = torch.empty(qshape, dtype=torch.float32).pin_memory()
        e2e_steps = max(3, min(args.steps, 20))

        def e2e_step():
            p = hp.to(device, non_blocking=True)
            q = hq.to(device, non_blocking=True)
            o = ho.to(device, non_blocking=True) if ho is not None else None
            qo = hqo.to(device, non_blocking=True) if hqo is not None else None
            # out= pinned host tensors: the result is copied into them on the
            # current stream (one bulk D2H copy per tensor).
            step(p, q, o, qo, (out_idx, out_dist))

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize(device)
        barrier(world)
        ev = []
        for _ in range(e2e_steps):
            flush.zero_()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            e2e_step()
            b.record(stream)
            ev.append((a, b))
        torch.cuda.synchronize(device)
        e2e_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev), world)
        h2d = hp.numel() * 4 + hq.numel() * 4 + (ho.numel() * 8 if ho is not None else 0) + \
            (hqo.numel() * 8 if hqo is not None else 0)
        d2h = out_idx.numel() * 8 + out_dist.numel() * 4
        e2e = {"value": w.num_queries * e2e_steps * world / (e2e_ms / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": e2e_ms / e2e_steps,
               "api": "torchbvh_b200.BVH(points).knn(queries, k, out=(pinned host indices, distances))"}

    # ---- roofline of the traversal kernel ----
    build_bytes, query_bytes = algorithmic_bytes(w)
    peak, peak_kind = measured_peak_hbm()
    knn_avg_ms = sum(knn_ms) / len(knn_ms) if knn_ms else float("nan")
    achieved = query_bytes / (knn_avg_ms / 1e3) / 1e9 if knn_ms else None
    traffic, traffic_src = profiled_traffic(args.workload)
    roofline = {
        "kernel": "k_knn (warp-packet BVH traversal)",
        "bound": "hbm",
        "achieved": achieved,
        "peak": peak,
        "unit": "GB/s",
        "frac": achieved / peak if achieved else None,
        "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback 6.65 TB/s",
        "traffic": traffic,
        "traffic_source": traffic_src,
        "algorithmic_bytes_per_launch": query_bytes,
        "avg_launch_ms": knn_avg_ms,
        "launches": len(knn_ms),
    }

    cpu = cpu_bf = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w, args)
        cpu_bf = cpu_bruteforce_throughput(w)

    result = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": total_ms_max / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded CPU generator, torchbvh_b200.workloads)",
        "config": workload_config(w, world),
        "build_ms": build_total_ms / args.steps,
        "build_ms_per_1m_points": build_total_ms / args.steps / (w.num_points / 1e6),
        "query_ms": (total_ms - build_total_ms) / args.steps,
        "knn_kernel_ms": knn_avg_ms,
        "build_algorithmic_bytes": build_bytes,
        "roofline": roofline,
        "cpu_baseline": cpu,
        "cpu_bruteforce": cpu_bf,
        "e2e": e2e,
        "gpu_launches": launches,
        "gpu_launches_per_step": launches / args.steps,
        "device_status": status,
        "clocks": sampler.summary(),
        "gpu": torch.cuda.get_device_name(device),
    }
    return result


def run_b200_clouds_sharded(args, world, rank, local):
    """c2 / c3 / c5 on N > 1 GPUs, sharded by cloud (strong scaling).

    Every rank holds the whole batch; one step is
    ``distributed.knn_sharded_batched`` (fixed-size clouds split into contiguous
    ranges) or ``knn_sharded_ragged`` (ragged clouds by a longest-first
    partition): each rank builds and queries its clouds, then the results are
    all-gathered (NCCL) into the original order on every rank.
    """
    from torchbvh_b200 import _native
    from torchbvh_b200 import distributed as tdist
    import torchbvh_b200 as torchbvh

    device = torch.device("cuda", local)
    w = load_workload(args.workload, args)
    k = w.k
    points = w.points.to(device)
    queries = w.queries.to(device)
    if w.batch_offsets is not None:
        bo = [int(v) for v in w.batch_offsets.tolist()]
        qo = [int(v) for v in w.query_offsets.tolist()]

        def step():
            return tdist.knn_sharded_ragged(points, bo, queries, qo, k)
        form = "knn_sharded_ragged: clouds by a longest-first partition of their sizes"
    else:
        def step():
            return tdist.knn_sharded_batched(points, queries, k)
        form = "knn_sharded_batched: contiguous cloud ranges"
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    phase_events: list = []

    def phase_hook(name, dev):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(dev))
        phase_events.append((name, ev))

    out = None
    for _ in range(args.warmup):
        out = step()
    torch.cuda.synchronize(device)
    barrier(world)
    launches0 = _native.load_library().tbvh_kernel_launch_count()
    ev = []
    sampler = ClockSampler(local)
    tdist._phase_hooks.append(phase_hook)
    with sampler:
        for _ in range(args.steps):
            flush.zero_()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            out = step()
            b.record(stream)
            ev.append((a, b))
        torch.cuda.synchronize(device)
    tdist._phase_hooks.remove(phase_hook)
    del out
    launches = _native.load_library().tbvh_kernel_launch_count() - launches0
    total_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev), world)
    # Per-rank phases: own clouds' build + query, then the all-gather (and reorder).
    import torch.distributed as dist

    names = ["start", "compute", "gathered"]
    steps_ev = [phase_events[i:i + 3] for i in range(0, len(phase_events), 3)]
    phases = {f"{b}_ms": sum(st[i][1].elapsed_time(st[i + 1][1]) for st in steps_ev) / len(steps_ev)
              for i, b in enumerate(names[1:])}
    per_rank = [None] * world
    dist.all_gather_object(per_rank, {"step_ms": sum(a.elapsed_time(b) for a, b in ev) / args.steps, **phases})
    cfg = workload_config(w, world)
    cfg["parallelism"] = (f"{form} over {world} GPUs, every result row all-gathered (NCCL) into the "
                          f"original order on every rank")
    return {
        "metric": METRIC,
        "value": w.num_queries * args.steps / (total_ms / 1e3),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded CPU generator, torchbvh_b200.workloads)",
        "config": cfg,
        "per_rank_ms": per_rank,
        "roofline": None,
        "cpu_baseline": None,
        "e2e": None,
        "gpu_launches": launches,
        "gpu_launches_per_step": launches / args.steps,
        "device_status": torchbvh.device_status(device),
        "clocks": sampler.summary(),
        "gpu": torch.cuda.get_device_name(device),
    }


def run_b200_single_cloud_sharded(args, world, rank, local):
    """c4 on N > 1 GPUs, the sharded single-cloud form (strong scaling).

    One step: rank 0's points are broadcast (NCCL), every rank builds the same
    BVH, sorts all queries by Morton code against it, takes its range of that
    order and queries it; the results stay on the rank that computed them
    (`value`). `all_gather` times the same step followed by the all-gather of
    every result row into the original query order on every rank.
    """
    import torchbvh_b200 as torchbvh
    from torchbvh_b200 import _native
    from torchbvh_b200 import distributed as tdist

    device = torch.device("cuda", local)
    w = load_workload("c4", args)
    n, m, dim, k = w.num_points, w.num_queries, w.dim, w.k
    points = w.points.to(device) if rank == 0 else None
    queries = w.queries.to(device)

    def step(p, q, gather, out=None):
        return tdist.knn_sharded_single_cloud(p, q, k, num_points=n, dim=dim, gather=gather,
                                              split=args.c4_split, device=device, out=out)

    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    knn_events: list = []

    def hook(phase, dev):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(dev))
        knn_events.append((phase, ev))

    def timed(gather, steps, warmup, inputs, peer=None):
        out = None
        for _ in range(warmup):
            out = step(*inputs(), gather, peer)
        torch.cuda.synchronize(device)
        barrier(world)
        launches0 = _native.load_library().tbvh_kernel_launch_count()
        ev = []
        for _ in range(steps):
            flush.zero_()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            out = step(*inputs(), gather, peer)
            b.record(stream)
            ev.append((a, b))
        torch.cuda.synchronize(device)
        del out
        launches = _native.load_library().tbvh_kernel_launch_count() - launches0
        return sum(a.elapsed_time(b) for a, b in ev), launches

    resident = lambda: (points, queries)  # noqa: E731
    # value: results all-gathered, the traversal delivering every row to every
    # rank's buffer over NVLink (PeerResults, reused across steps).
    gather_steps = max(3, min(args.steps, 10))
    # Phase markers of the sharded call (events on the current stream), to
    # split a rank's step into broadcast / build / share / traversal / delivery.
    phase_events: list = []

    def phase_hook(name, dev):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(dev))
        phase_events.append((name, ev))

    with tdist.PeerResults(m, k, device=device, index_bits=args.c4_index_bits,
                           transport=args.c4_transport) as peer:
        transport_used = peer.transport_used
        _native._knn_hooks.append(hook)
        tdist._phase_hooks.append(phase_hook)
        sampler = ClockSampler(local)
        with sampler:
            total_ms, launches = timed("all", args.steps, args.warmup, resident, peer)
        tdist._phase_hooks.remove(phase_hook)
        _native._knn_hooks.remove(hook)
        total_ms_max = max_over_ranks(total_ms, world)
        starts = [e for ph, e in knn_events if ph == "start"][-args.steps:]
        ends = [e for ph, e in knn_events if ph == "end"][-args.steps:]
        knn_local_ms = sum(a.elapsed_time(b) for a, b in zip(starts, ends)) / len(starts)
        knn_avg_ms = max_over_ranks(knn_local_ms, world)
        import torch.distributed as dist

        order = ["start", "broadcast", "build", "share", "traversal", "delivered"]
        steps_ev = [phase_events[i:i + len(order)] for i in range(0, len(phase_events), len(order))][-args.steps:]
        phases = {}
        for a_name, b_name in zip(order, order[1:]):
            ia, ib = order.index(a_name), order.index(b_name)
            phases[b_name + "_ms"] = sum(s[ia][1].elapsed_time(s[ib][1]) for s in steps_ev) / len(steps_ev)
        per_rank = [None] * world
        dist.all_gather_object(per_rank, {"knn_ms": knn_local_ms, "step_ms": total_ms / args.steps, **phases})
    inplace_ms = max_over_ranks(timed("none", gather_steps, 3, resident)[0], world)
    nccl_gather_ms = max_over_ranks(timed("all", gather_steps, 3, resident)[0], world)
    status = torchbvh.device_status(device)

    e2e = None
    if not args.no_e2e:
        hp = w.points.pin_memory() if rank == 0 else None
        hq = w.queries.pin_memory()
        # The rank's share size depends on the split; it is the same every step.
        share_rows = int(step(points, queries, "none")[2].numel()) if args.c4_split != "contiguous" else \
            tdist.shard_range(m, world, rank)[1] - tdist.shard_range(m, world, rank)[0]
        host_idx = torch.empty((share_rows, k), dtype=torch.int64).pin_memory()
        host_dist = torch.empty((share_rows, k), dtype=torch.float32).pin_memory()

        def e2e_inputs():
            p = hp.to(device, non_blocking=True) if rank == 0 else None
            return p, hq.to(device, non_blocking=True)

        def e2e_step_ms(steps):
            ev = []
            for i in range(steps + 2):
                flush.zero_()
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record(stream)
                idx, dist_sq, _ = step(*e2e_inputs(), "none")
                host_idx.copy_(idx, non_blocking=True)
                host_dist.copy_(dist_sq, non_blocking=True)
                b.record(stream)
                if i >= 2:
                    ev.append((a, b))
            torch.cuda.synchronize(device)
            return sum(a.elapsed_time(b) for a, b in ev)

        e2e_steps = max(3, min(args.steps, 10))
        e2e_ms = max_over_ranks(e2e_step_ms(e2e_steps), world)
        e2e = {"value": m * e2e_steps / (e2e_ms / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": (n * dim * 4 if rank == 0 else 0) + m * dim * 4,
               "d2h_bytes_per_step": share_rows * k * 12,
               "ms_per_step": e2e_ms / e2e_steps,
               "api": "torchbvh_b200.distributed.knn_sharded_single_cloud(..., gather='none') from pinned host "
                      "buffers (byte counts of rank 0)"}

    from torchbvh_b200 import workloads

    share = -(-m // world)
    _, query_bytes = workloads.algorithmic_bytes([n], [share], dim, k)
    peak, peak_kind = measured_peak_hbm()
    achieved = query_bytes / (knn_avg_ms / 1e3) / 1e9
    return {
        "metric": METRIC,
        "value": m * args.steps / (total_ms_max / 1e3),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": total_ms_max / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded CPU generator, torchbvh_b200.workloads)",
        "config": {**workload_config(w, world),
                   "parallelism": (f"points broadcast from rank 0 (NCCL), BVH built on each of {world} GPUs, "
                                   f"queries split by {'Morton-order' if args.c4_split == 'morton' else 'index'} "
                                   f"range, every result row delivered to every rank by the traversal "
                                   f"({'one NVLink multicast store per row' if transport_used == 'multicast' else 'NVLink stores to every peer'}, "
                                   f"int{args.c4_index_bits} indices on the wire): results all-gathered"),
                   "transport": transport_used, "index_bits": args.c4_index_bits},
        "results_in_place": {"value": m * gather_steps / (inplace_ms / 1e3), "unit": UNIT,
                             "ms_per_step": inplace_ms / gather_steps,
                             "note": "same step with each result row left on the rank that computed it"},
        "nccl_all_gather": {"value": m * gather_steps / (nccl_gather_ms / 1e3), "unit": UNIT,
                            "ms_per_step": nccl_gather_ms / gather_steps,
                            "note": "rows left in place by the traversal, then an NCCL all-gather into query order"},
        "knn_kernel_ms": knn_avg_ms,
        "per_rank_ms": per_rank,
        "roofline": {"kernel": "k_knn (warp-packet BVH traversal), one rank's share", "bound": "hbm",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)", "traffic": None,
                     "algorithmic_bytes_per_launch": query_bytes, "avg_launch_ms": knn_avg_ms},
        "cpu_baseline": None,
        "e2e": e2e,
        "gpu_launches": launches,
        "gpu_launches_per_step": launches / args.steps,
        "device_status": status,
        "clocks": sampler.summary(),
        "gpu": torch.cuda.get_device_name(device),
    }


# ---------------------------------------------------------------------------
# CPU port (oracle) timing: cpu_baseline and the reference arm
# ---------------------------------------------------------------------------

def _cpu_sample(w):
    """Per-cloud point and query arrays of a workload (CPU tensors)."""
    sizes = w.cloud_sizes()
    if w.points.dim() == 3:
        pts = [w.points[b] for b in range(w.points.shape[0])]
        qs = [w.queries[b] for b in range(w.queries.shape[0])]
    elif w.batch_offsets is not None:
        o = w.batch_offsets.tolist()
        qo = w.query_offsets.tolist()
        pts = [w.points[o[b]:o[b + 1]] for b in range(len(sizes))]
        qs = [w.queries[qo[b]:qo[b + 1]] for b in range(len(sizes))]
    else:
        pts, qs = [w.points], [w.queries]
    return sizes, pts, qs


class CpuPortSample:
    """The C port of the reference algorithm (oracle/, build + DFS traversal) over a
    bounded sample of a workload, on the host cores.

    Construction builds the first clouds in full, one thread each (the port's
    build is serial), until about `build_budget_s` is spent; clouds are
    independent, so a whole workload builds `min(threads, clouds)` clouds at a
    time. Each `step(budget_s)` traverses fresh queries of those clouds (a
    rolling window over each cloud's queries) on `threads` threads for about
    `budget_s` seconds. A traversal costs the same per query whichever queries of
    a cloud are drawn, so the measured rate scales to the whole workload:
    estimated seconds = build s/point x points / min(threads, clouds)
    + traversal s/query x queries.
    """

    def __init__(self, w, build_budget_s: float = 4.0):
        import numpy as np

        from oracle import pyoracle

        self._np, self._oracle = np, pyoracle
        self.w = w
        self.threads = pyoracle.default_threads()
        sizes, pts, qs = _cpu_sample(w)
        self.total_clouds = len(sizes)
        self.trees, self.queries = [], []
        build_s = 0.0
        self.built_points = 0
        for b in range(len(sizes)):
            p = np.ascontiguousarray(pts[b].numpy())
            t0 = time.perf_counter()
            tree = pyoracle.build(p)
            build_s += time.perf_counter() - t0
            self.built_points += p.shape[0]
            self.trees.append({"node_aabbs": tree["node_aabbs"], "sorted_indices": tree["sorted_indices"]})
            self.queries.append(np.ascontiguousarray(qs[b].numpy()))
            if build_s > build_budget_s:
                break
        self.build_s = build_s
        self.build_s_per_point = build_s / self.built_points
        self._cursor = [0] * len(self.trees)
        self.chunk = 2048

    def step(self, budget_s: float) -> tuple[float, int]:
        """Traverses fresh queries for about `budget_s` s; returns (seconds, queries)."""
        done = 0
        t0 = time.perf_counter()
        while True:
            for c, (tree, q) in enumerate(zip(self.trees, self.queries)):
                s = self._cursor[c] % q.shape[0]
                e = min(s + self.chunk, q.shape[0])
                self._oracle.knn_reference(tree, q[s:e], self.w.k, threads=self.threads)
                self._cursor[c] = e
                done += e - s
            if time.perf_counter() - t0 >= budget_s:
                break
        return time.perf_counter() - t0, done

    def estimate(self, seconds: float, queries: int) -> float:
        build_parallel = min(self.threads, self.total_clouds)
        est = (self.build_s_per_point * self.w.num_points / build_parallel
               + seconds / queries * self.w.num_queries)
        return self.w.num_queries / est

    def describe(self, seconds: float, queries: int) -> str:
        return (f"{len(self.trees)} of {self.total_clouds} clouds built in full ({self.built_points} points, "
                f"{self.build_s:.2f} s on 1 thread), then {queries} of their queries traversed in {seconds:.2f} s on "
                f"{self.threads} threads; extrapolated to the whole workload (build s/point x points / "
                f"min(threads, clouds) + traversal s/query x queries); C restatement of the reference build + DFS "
                f"traversal (oracle/tbvh_oracle.c)")


def cpu_baseline(w, args, budget_s: float = 12.0) -> dict:
    """`cpu_baseline` of the JSON line: the CPU port on a bounded sample (rank 0, one GPU)."""
    sampler = CpuPortSample(w, build_budget_s=budget_s / 3)
    seconds, queries = sampler.step(max(1.0, budget_s - sampler.build_s))
    return {
        "value": sampler.estimate(seconds, queries),
        "unit": UNIT,
        "cores": sampler.threads,
        "kind": "port",
        "extrapolated": True,
        "sample": sampler.describe(seconds, queries),
        "build_s_per_mpoints": sampler.build_s_per_point * 1e6,
        "query_us_per_query": seconds / queries * 1e6,
    }


def cpu_bruteforce_throughput(w, budget_s: float = 8.0, chunk_bytes: int = 1 << 28) -> dict:
    """CPU brute force the north star asks to report beside the GPU numbers:
    ``torch.cdist(q, p).topk(k, largest=False)`` (default compute mode) plus the
    square, on all host threads, over a bounded sample: queries of the first
    clouds, in chunks whose distance matrix stays near `chunk_bytes`, until
    about `budget_s` seconds are spent. Brute force costs the same per query
    within a cloud, so per-cloud query rates extrapolate to the whole workload.
    """
    threads = os.cpu_count() or 1
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        sizes, pts, qs = _cpu_sample(w)
        qcounts = ([int(q.shape[0]) for q in qs])
        est_s = 0.0
        sampled = 0
        spent = 0.0
        clouds_used = 0
        per_query_s = []
        for b in range(len(sizes)):
            p = pts[b].contiguous()
            q_all = qs[b]
            rows = max(1, min(int(q_all.shape[0]), chunk_bytes // max(1, 4 * int(p.shape[0]))))
            done = 0
            t_cloud = 0.0
            while done < q_all.shape[0] and (t_cloud < budget_s / 4 or done == 0):
                q = q_all[done:done + rows].contiguous()
                t0 = time.perf_counter()
                d, i = torch.cdist(q, p).topk(w.k, dim=1, largest=False)
                d = d.square()
                t_cloud += time.perf_counter() - t0
                done += q.shape[0]
            per_query_s.append(t_cloud / done)
            sampled += done
            spent += t_cloud
            clouds_used += 1
            if spent > budget_s:
                break
        # Clouds not sampled cost like the sampled one closest in size (cost ~ N per query).
        for b in range(len(sizes)):
            j = min(range(len(per_query_s)), key=lambda c: abs(sizes[c] - sizes[b]))
            est_s += per_query_s[j] * (sizes[b] / sizes[j]) * qcounts[b]
        return {
            "value": w.num_queries / est_s,
            "unit": UNIT,
            "cores": threads,
            "kind": "torch.cdist + topk brute force",
            "sample": (f"{sampled} queries of {clouds_used} of {len(sizes)} clouds, chunks of up to "
                       f"{chunk_bytes >> 20} MiB of distances; per-query time scaled by cloud size to the "
                       f"whole workload"),
        }
    finally:
        torch.set_num_threads(prev)


def run_reference(args, world, rank):
    """The reference arm: the CPU port of the reference algorithm (the reference's
    k-NN path is CUDA-only), rank 0 only. Every step traverses a fresh bounded
    query sample; the clouds are built once, before the first warm-up step."""
    if rank != 0:
        return None
    w = load_workload(args.workload, args)
    t_build0 = time.perf_counter()
    sampler = CpuPortSample(w)
    build_wall = time.perf_counter() - t_build0
    per_step_budget = max(0.5, 60.0 / max(1, args.steps + args.warmup))
    vals, secs, counts = [], [], []
    for i in range(args.warmup + args.steps):
        seconds, queries = sampler.step(per_step_budget)
        if i >= args.warmup:
            vals.append(sampler.estimate(seconds, queries))
            secs.append(seconds)
            counts.append(queries)
    value = statistics.median(vals)
    cpu = {"value": value, "unit": UNIT, "cores": sampler.threads, "kind": "port", "extrapolated": True,
           "sample": sampler.describe(sum(secs), sum(counts))}
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": statistics.median(secs) * 1e3,
        "extrapolated": True,
        "queries_per_step": statistics.median(counts),
        "measured_s": {"build_once": build_wall, "timed_steps": sum(secs)},
        "estimated_ms_per_workload": w.num_queries / value * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded CPU generator, torchbvh_b200.workloads)",
        "config": workload_config(w, 1),
        "cpu_baseline": cpu,
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("the reference's k-NN path is CUDA-only; this arm times the C restatement of its algorithm "
                 "(oracle/) on the host cores. A step traverses a bounded sample of fresh queries "
                 "(ms_per_step is that measured time); value extrapolates to the whole workload"),
    }


def run_reference_cuda(args, world, rank, local):
    """The reference's own CUDA path (baseline/_ref), timed exactly like the B200 arm's value.

    k = 32 (c4) is not offered by the reference's dispatch; there a step is the
    reference's build and query sort plus its own traversal kernel instantiated
    at K = 32 (oracle/ref_knn_harness.cu), labelled as such.
    """
    ref_dir = ROOT / "baseline" / "_ref"
    if rank != 0:
        return None
    if not (ref_dir / "torchbvh").exists():
        return {"impl": "reference_cuda", "unavailable": "baseline/_ref not installed"}
    sys.path.insert(0, str(ref_dir))
    # The reference compiles its extension on first use; one built beside the install
    # (baseline/_ref/torch_ext) is reused instead of rebuilding on the GPU box.
    os.environ.setdefault("TORCH_EXTENSIONS_DIR", str(ref_dir / "torch_ext"))
    try:
        import torchbvh as ref  # noqa: F401
    except Exception as exc:
        return {"impl": "reference_cuda", "unavailable": f"import failed: {exc}"}
    w = load_workload(args.workload, args)
    device = torch.device("cuda", local)
    points, queries = w.points.to(device), w.queries.to(device)
    offsets = w.batch_offsets.to(device) if w.batch_offsets is not None else None
    qoffsets = w.query_offsets.to(device) if w.query_offsets is not None else None
    path = "reference public API: torchbvh.BVH(points).knn(queries, k)"
    if w.k in ref.SUPPORTED_K:
        def step():
            bvh = ref.BVH(points, batch_offsets=offsets)
            return bvh.knn(queries, w.k, query_offsets=qoffsets) if offsets is not None else bvh.knn(queries, w.k)
    else:
        if offsets is not None or points.dim() != 2:
            return {"impl": "reference_cuda", "unavailable": f"k={w.k} not supported by the reference"}
        from oracle import ref_harness

        harness = ref_harness.load()
        path = (f"reference algorithm, K={w.k} instantiation (not a shipped reference path): reference "
                f"build_bvh + morton_sort_queries_narrow + its traversal kernel template at K={w.k}")

        def step():
            h = ref.build_bvh(points)
            order = ref._C.morton_sort_queries_narrow(queries.unsqueeze(0), h["scene_min"].unsqueeze(0),
                                                      h["scene_max"].unsqueeze(0))
            return harness.knn_ordered_any_k(h["node_aabbs"].unsqueeze(0), h["sorted_indices"].unsqueeze(0),
                                             queries.unsqueeze(0), order.contiguous(), int(h["num_leaves"]),
                                             int(h["num_real_nodes"]), int(h["dim"]), w.k)

    out = None
    for _ in range(args.warmup):
        out = step()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    torch.cuda.synchronize(device)
    ev = []
    sampler = ClockSampler(local)
    with sampler:
        for _ in range(args.steps):
            flush.zero_()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            out = step()
            b.record(stream)
            ev.append((a, b))
        torch.cuda.synchronize(device)
    del out
    total_ms = sum(a.elapsed_time(b) for a, b in ev)
    value = w.num_queries * args.steps / (total_ms / 1e3)
    return {"impl": "reference_cuda", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "config": workload_config(w, 1), "dtype": "f32", "path": path,
            "reference_version": getattr(ref, "__version__", None), "clocks": sampler.summary(),
            "gpu": torch.cuda.get_device_name(device),
            "data": "synthetic (seeded CPU generator, torchbvh_b200.workloads)"}


def main():
    args = parse_args()
    # stdout carries the one result line only: whatever else writes to it
    # (NCCL's version banner at process-group start, for one) goes to stderr.
    sys.stdout.flush()
    result_fd = os.dup(1)
    os.dup2(2, 1)
    if args.warmup < 3 and args.impl == "b200":
        print("note: fewer than 3 warm-up steps; this run is not a reportable measurement", file=sys.stderr)
    world, rank, local = dist_setup(args) if args.impl != "reference" else (
        int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0)
    try:
        if args.impl == "reference":
            result = run_reference(args, world, rank)
        elif args.impl == "reference_cuda":
            result = run_reference_cuda(args, world, rank, local)
        elif args.workload == "c4" and world > 1:
            result = run_b200_single_cloud_sharded(args, world, rank, local)
        elif args.workload in ("c2", "c3", "c5") and world > 1 and not args.replicas:
            result = run_b200_clouds_sharded(args, world, rank, local)
        else:
            result = run_b200(args, world, rank, local)
        if rank == 0 and result is not None:
            os.write(result_fd, (json.dumps(result) + "\n").encode())
    finally:
        if world > 1 and args.impl != "reference":
            import torch.distributed as dist

            if dist.is_initialized():
                dist.destroy_process_group()


if __name__ == "__main__":
    main()
