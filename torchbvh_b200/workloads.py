"""Seeded synthetic workloads for the five benchmark configurations.

Inputs are generated on the CPU with ``torch.Generator().manual_seed(seed)``
and only then copied to a device, so they are identical for any GPU count.
No public dataset is involved; distributions and sizes follow the benchmark
configurations of this project (single uniform cloud; 16 Gaussian-mixture
clouds; 8 uniform 2-D clouds; one 16.7 M-point sphere shell with background;
64 log-uniform ragged anisotropic clouds).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass
class Workload:
    name: str
    points: torch.Tensor              # (N, D), (B, N, D) or packed (total, D); CPU float32
    queries: torch.Tensor             # same layout as points
    k: int
    batch_offsets: torch.Tensor | None = None   # ragged only, int64 (B + 1,)
    query_offsets: torch.Tensor | None = None

    @property
    def dim(self) -> int:
        return int(self.points.shape[-1])

    @property
    def num_queries(self) -> int:
        return int(self.queries.numel() // self.dim)

    @property
    def num_points(self) -> int:
        return int(self.points.numel() // self.dim)

    @property
    def num_clouds(self) -> int:
        if self.batch_offsets is not None:
            return int(self.batch_offsets.numel() - 1)
        return int(self.points.shape[0]) if self.points.dim() == 3 else 1

    def cloud_sizes(self) -> list[int]:
        if self.batch_offsets is not None:
            return torch.diff(self.batch_offsets).tolist()
        if self.points.dim() == 3:
            return [int(self.points.shape[1])] * int(self.points.shape[0])
        return [int(self.points.shape[0])]


def _gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def c1_single_uniform(n: int = 10_000, m: int = 10_000, seed: int = 1001) -> Workload:
    g = _gen(seed)
    pts = torch.rand((n, 3), generator=g)
    q = torch.rand((m, 3), generator=g)
    return Workload("c1_single3d_uniform_10k_k4", pts, q, 4)


def c2_batched_gaussian(batch: int = 16, n: int = 65_536, seed: int = 1002) -> Workload:
    g = _gen(seed)
    pts = torch.empty((batch, n, 3))
    for b in range(batch):
        centers = torch.rand((32, 3), generator=g)
        comp = torch.randint(0, 32, (n,), generator=g)
        pts[b] = centers[comp] + 0.02 * torch.randn((n, 3), generator=g)
    q = pts + 0.01 * torch.randn(pts.shape, generator=g)
    return Workload("c2_batched3d_gaussian_16x65536_k16", pts, q, 16)


def c3_batched_uniform_2d(batch: int = 8, n: int = 262_144, seed: int = 1003) -> Workload:
    g = _gen(seed)
    pts = torch.rand((batch, n, 2), generator=g)
    q = torch.rand((batch, n, 2), generator=g)
    return Workload("c3_batched2d_uniform_8x262144_k8", pts, q, 8)


def _sphere_shell(n: int, seed: int) -> torch.Tensor:
    g = _gen(seed)
    n_shell = (9 * n) // 10
    u = torch.randn((n_shell, 3), generator=g)
    u = u / u.norm(dim=1, keepdim=True)
    shell = u * (1.0 + 1.0e-3 * torch.randn((n_shell, 1), generator=g))
    background = 3.0 * torch.rand((n - n_shell, 3), generator=g) - 1.5
    both = torch.cat([shell, background])
    return both[torch.randperm(n, generator=g)].contiguous()


def c4_sphere_shell(n: int = 16_777_216, m: int | None = None, seed: int = 1004, query_seed: int = 2004) -> Workload:
    pts = _sphere_shell(n, seed)
    q = _sphere_shell(m if m is not None else n, query_seed)
    return Workload(f"c4_single3d_sphere_{n}_k32", pts, q, 32)


def c5_ragged_anisotropic(clouds: int = 64, lo: int = 1024, hi: int = 1_048_576, seed: int = 1005) -> Workload:
    g = _gen(seed)
    u = torch.rand((clouds,), generator=g, dtype=torch.float64)
    sizes = torch.floor(torch.exp(math.log(lo) + u * (math.log(hi) - math.log(lo)))).to(torch.int64)
    offsets = torch.zeros(clouds + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(sizes, 0)
    total = int(offsets[-1])
    pts = torch.rand((total, 3), generator=g) * torch.tensor([1.0, 0.1, 0.01])
    return Workload("c5_ragged3d_anisotropic_64_k16", pts, pts.clone(), 16, offsets, offsets.clone())


CONFIGS = {
    "c1": c1_single_uniform,
    "c2": c2_batched_gaussian,
    "c3": c3_batched_uniform_2d,
    "c4": c4_sphere_shell,
    "c5": c5_ragged_anisotropic,
}


def make(name: str, **kwargs) -> Workload:
    return CONFIGS[name](**kwargs)


def algorithmic_bytes(sizes: list[int], queries_per_cloud: list[int], dim: int, k: int) -> tuple[int, int]:
    """(build, query) algorithmic HBM bytes of one step.

    Per cloud: build = 4*D*N (read points) + 8*N (write int64 sorted_indices)
    + 8*D*nr (write node AABBs); query = 4*D*M (read queries) + 12*K*M (write
    int64 indices + float32 distances) + 8*D*nr + 8*N (read the tree once).
    """
    from ._native import real_node_count

    build = query = 0
    for n, m in zip(sizes, queries_per_cloud):
        nr = real_node_count(n)
        build += 4 * dim * n + 8 * n + 8 * dim * nr
        query += 4 * dim * m + 12 * k * m + 8 * dim * nr + 8 * n
    return build, query
