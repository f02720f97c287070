"""Benchmark of the B200 BVH k-NN path (build + query), one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c1..c5]
                    [--impl b200|reference|reference_cuda]

A step is one ``BVH(points)`` build plus one ``.knn(queries, k)`` query over one
batch of the seeded synthetic workload (torchbvh_b200.workloads), through the
public API. Default workload: c2 (16 Gaussian-mixture clouds x 65,536 3-D
points, k = 16). Metric: k-NN queries/sec (build + query).

* ``value``: device-resident inputs, CUDA events around each step on the
  current stream, L2 flushed (256 MiB write) between steps outside the events,
  summed over K steps, max over ranks. Under torchrun every rank runs the
  workload on its own GPU with no data exchange (weak scaling), except c4:
  one cloud, its points broadcast from rank 0, queries split by Morton range,
  results left on the computing rank (strong scaling), with an ``all_gather``
  figure where the traversal delivers every row to every GPU over NVLink.
* ``e2e``: the same public API with the inputs in pinned host memory: per step
  H2D copy of points and queries, build, query, D2H copy of indices and
  distances, all inside the events.
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
    ap.add_argument("--workload", default="c2", choices=["c1", "c2", "c3", "c4", "c5"])
    ap.add_argument("--impl", default="b200", choices=["b200", "reference", "reference_cuda"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--c4-points", type=int, default=16_777_216,
                    help="points (= queries) of workload c4; smaller values make ncu-sized cases")
    ap.add_argument("--c4-split", default="morton", choices=["morton", "contiguous"],
                    help="c4 on N > 1 GPUs: share of the queries per rank (a range of their Morton order, "
                         "or of their given order)")
    ap.add_argument("--cpu-sample-queries", type=int, default=0,
                    help="queries per sampled cloud for the CPU baseline (0 = automatic)")
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

    def step(p, q, o, qo):
        bvh = torchbvh.BVH(p, batch_offsets=o)
        out = bvh.knn(q, k, query_offsets=qo) if o is not None else bvh.knn(q, k)
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
            _, (idx, dist) = step(p, q, o, qo)
            out_idx.copy_(idx, non_blocking=True)
            out_dist.copy_(dist, non_blocking=True)

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
               "ms_per_step": e2e_ms / e2e_steps, "api": "torchbvh_b200.BVH(points).knn(queries, k)"}

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
    _native._knn_hooks.append(hook)
    sampler = ClockSampler(local)
    with sampler:
        total_ms, launches = timed("none", args.steps, args.warmup, resident)
    _native._knn_hooks.remove(hook)
    total_ms_max = max_over_ranks(total_ms, world)
    starts = [e for ph, e in knn_events if ph == "start"][-args.steps:]
    ends = [e for ph, e in knn_events if ph == "end"][-args.steps:]
    knn_local_ms = sum(a.elapsed_time(b) for a, b in zip(starts, ends)) / len(starts)
    knn_avg_ms = max_over_ranks(knn_local_ms, world)
    import torch.distributed as dist

    per_rank = [None] * world
    dist.all_gather_object(per_rank, {"knn_ms": knn_local_ms, "step_ms": total_ms / args.steps})

    gather_steps = max(3, min(args.steps, 10))
    nccl_gather_ms = max_over_ranks(timed("all", gather_steps, 3, resident)[0], world)
    with tdist.PeerResults(m, k, device=device) as peer:
        gather_ms = max_over_ranks(timed("all", gather_steps, 3, resident, peer)[0], world)
    status = torchbvh.device_status(device)

    e2e = None
    if not args.no_e2e:
        hp = w.points.pin_memory() if rank == 0 else None
        hq = w.queries.pin_memory()
        q0, q1 = tdist.shard_range(m, world, rank)
        host_idx = torch.empty((q1 - q0, k), dtype=torch.int64).pin_memory()
        host_dist = torch.empty((q1 - q0, k), dtype=torch.float32).pin_memory()

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
               "d2h_bytes_per_step": (q1 - q0) * k * 12,
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
                                   f"range, results left on the computing rank")},
        "all_gather": {"value": m * gather_steps / (gather_ms / 1e3), "unit": UNIT,
                       "ms_per_step": gather_ms / gather_steps,
                       "note": ("same step with every (M, k) result row delivered to every rank in query order: "
                                "the traversal writes each row into all ranks' buffers over NVLink as it "
                                "finishes (tbvh_query_knn_share)"),
                       "nccl_all_gather_ms_per_step": nccl_gather_ms / gather_steps},
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

def _cpu_sample(w, sample_queries: int):
    """Bounded sample: the first clouds (whole), a prefix of their queries."""
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


def cpu_port_throughput(w, args, budget_s: float = 12.0) -> dict:
    """Times the C port of the reference algorithm on host cores; extrapolates q/s.

    Per sampled cloud: full build timed, then a prefix of its queries (the
    per-query cost is independent of how many are run). Clouds are sampled
    until about `budget_s` seconds of CPU work are spent.
    """
    import numpy as np

    from oracle import pyoracle

    threads = pyoracle.default_threads()
    sizes, pts, qs = _cpu_sample(w, 0)
    m_total = w.num_queries
    per_cloud_q = args.cpu_sample_queries or (8192 if w.num_points <= 20_000_000 else 65536)
    build_s = query_s = 0.0
    built_points = sampled_queries = 0
    clouds_used = 0
    t_start = time.perf_counter()
    order = sorted(range(len(sizes)), key=lambda b: b)  # deterministic: first clouds first
    for b in order:
        p = np.ascontiguousarray(pts[b].numpy())
        q = np.ascontiguousarray(qs[b][:per_cloud_q].numpy())
        po = np.array([0, p.shape[0]], np.int64)
        qo = np.array([0, q.shape[0]], np.int64)
        _, _, tb, tq = pyoracle.build_and_query(p, po, q, qo, w.k, threads)
        build_s += tb
        query_s += tq
        built_points += p.shape[0]
        sampled_queries += q.shape[0]
        clouds_used += 1
        if time.perf_counter() - t_start > budget_s:
            break
    build_per_point = build_s / built_points
    query_per_query = query_s / sampled_queries
    est_s = build_per_point * w.num_points + query_per_query * m_total
    return {
        "value": m_total / est_s,
        "unit": UNIT,
        "cores": threads,
        "kind": "port",
        "sample": (f"{clouds_used} of {len(sizes)} clouds built in full ({built_points} points), "
                   f"{sampled_queries} queries traversed (first {per_cloud_q} per cloud); build time scaled by "
                   f"points and query time by queries to the whole workload; C restatement of the reference "
                   f"build + DFS traversal (oracle/tbvh_oracle.c), {threads} threads"),
        "build_s_per_mpoints": build_per_point * 1e6,
        "query_us_per_query": query_per_query * 1e6,
    }


def cpu_baseline(w, args) -> dict:
    return cpu_port_throughput(w, args)


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
        sizes, pts, qs = _cpu_sample(w, 0)
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
    if rank != 0:
        return None
    w = load_workload(args.workload, args)
    vals = []
    per_step_budget = max(2.0, 60.0 / max(1, args.steps + args.warmup))
    cpu = None
    for i in range(args.warmup + args.steps):
        cpu = cpu_port_throughput(w, args, budget_s=per_step_budget)
        if i >= args.warmup:
            vals.append(cpu["value"])
    value = statistics.median(vals)
    cpu["value"] = value
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": w.num_queries / value * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded CPU generator, torchbvh_b200.workloads)",
        "config": workload_config(w, 1),
        "cpu_baseline": cpu,
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("the reference's k-NN path is CUDA-only; this arm times the C restatement of its algorithm "
                 "(oracle/) on the host cores"),
    }


def run_reference_cuda(args, world, rank, local):
    """The reference's own CUDA path (baseline/_ref), timed exactly like the B200 arm's value."""
    ref_dir = ROOT / "baseline" / "_ref"
    if rank != 0:
        return None
    if not (ref_dir / "torchbvh").exists():
        return {"impl": "reference_cuda", "unavailable": "baseline/_ref not installed"}
    sys.path.insert(0, str(ref_dir))
    try:
        import torchbvh as ref  # noqa: F401
    except Exception as exc:
        return {"impl": "reference_cuda", "unavailable": f"import failed: {exc}"}
    w = load_workload(args.workload, args)
    if w.k not in ref.SUPPORTED_K:
        return {"impl": "reference_cuda", "unavailable": f"k={w.k} not supported by the reference"}
    device = torch.device("cuda", local)
    points, queries = w.points.to(device), w.queries.to(device)
    offsets = w.batch_offsets.to(device) if w.batch_offsets is not None else None
    qoffsets = w.query_offsets.to(device) if w.query_offsets is not None else None

    def step():
        bvh = ref.BVH(points, batch_offsets=offsets)
        return bvh.knn(queries, w.k, query_offsets=qoffsets) if offsets is not None else bvh.knn(queries, w.k)

    for _ in range(args.warmup):
        step()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    torch.cuda.synchronize(device)
    ev = []
    for _ in range(args.steps):
        flush.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        step()
        b.record(stream)
        ev.append((a, b))
    torch.cuda.synchronize(device)
    total_ms = sum(a.elapsed_time(b) for a, b in ev)
    value = w.num_queries * args.steps / (total_ms / 1e3)
    return {"impl": "reference_cuda", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "config": workload_config(w, 1), "dtype": "f32",
            "data": "synthetic (seeded CPU generator, torchbvh_b200.workloads)"}


def main():
    args = parse_args()
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
        else:
            result = run_b200(args, world, rank, local)
        if rank == 0 and result is not None:
            print(json.dumps(result), flush=True)
    finally:
        if world > 1 and args.impl != "reference":
            import torch.distributed as dist

            if dist.is_initialized():
                dist.destroy_process_group()


if __name__ == "__main__":
    main()
