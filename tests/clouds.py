"""Deterministic point clouds shared by the CPU and GPU tests.

The shapes follow the reference's own test inputs (tests/test_bvh_build.py:133-340,
tests/test_knn.py:160-324), regenerated here with numpy.
"""

from __future__ import annotations

import numpy as np


def _f(a):
    return np.asarray(a, dtype=np.float32)


def boundary_cloud(n: int, d: int) -> np.ndarray:
    base = np.arange(n, dtype=np.float32)
    cols = [((base * (a + 3)) % 11) + base * np.float32(0.125 + 0.25 * a) for a in range(d)]
    return _f(np.stack(cols, axis=1))


def linspace(a, b, n):
    return np.linspace(a, b, n, dtype=np.float32)


def pathological_clouds() -> list[tuple[str, np.ndarray]]:
    return [
        ("single_2d", _f([[4.0, -2.0]])),
        ("single_3d", _f([[-1.0, 3.0, 5.0]])),
        ("pair_2d", _f([[0.0, 0.0], [10.0, -2.0]])),
        ("pair_3d", _f([[0.0, 0.0, 0.0], [10.0, -2.0, 0.5]])),
        ("line_2d", np.stack([linspace(-3, 3, 9), linspace(6, -6, 9)], axis=1)),
        ("line_3d", np.stack([linspace(-2, 2, 11), linspace(4, -4, 11), linspace(1, 9, 11)], axis=1)),
        ("plane_3d", _f([[-2, -1, 7], [-1, 2, 7], [0, -3, 7], [1, 4, 7], [2, -5, 7], [3, 6, 7]])),
        ("duplicates_3d", np.full((9, 3), 2.5, np.float32)),
        ("wide_2d", _f([[0, 0], [1e6, 1e-3], [2e6, -1e-3], [3e6, 2e-3], [4e6, -2e-3]])),
        ("wide_3d", _f([[0, 0, 0], [1e-3, 1e6, 2], [-1e-3, 2e6, -2], [2e-3, 3e6, 4], [-2e-3, 4e6, -4]])),
        ("tiny_2d", _f([[1e-7, -2e-7], [1.5e-7, -2.5e-7], [2e-7, -1.5e-7], [2.5e-7, -3e-7], [3e-7, -1e-7]])),
        ("mixed_3d", _f([[1, 1e-6, -1e3], [2, 1.5e-6, -5e2], [3, 2e-6, 0], [4, 2.5e-6, 5e2], [5, 3e-6, 1e3],
                         [6, 3.5e-6, 1.5e3], [7, 4e-6, 2e3]])),
        ("mixed_2d", _f([[1e-4, -1e8], [2e-4, -5e7], [3e-4, 0], [4e-4, 5e7], [5e-4, 1e8]])),
        ("flat_3d", _f([[-1e6, 1e-5, 2], [-5e5, 2e-5, 2], [0, 3e-5, 2], [5e5, 4e-5, 2], [1e6, 5e-5, 2],
                        [1.5e6, 6e-5, 2]])),
        ("degenerate_2d", _f([[7, -3], [7, -3], [7, -3]])),
        ("explicit_2d", _f([[0, 0], [1, 0], [0.25, 0.75], [0.25, 0.75], [2, -1]])),
        ("explicit_3d", _f([[1, 2, 0], [1, 2, 0], [3, 2, -1], [0, 2, 4], [5, 2, 4], [2, 2, 4]])),
    ]


def single_child_cloud(n: int) -> np.ndarray:
    a = np.arange(n, dtype=np.float32)
    return _f(np.stack([a, np.remainder(a, 3), -a], axis=1))


BUILD_CASES = (
    pathological_clouds()
    + [(f"boundary_n{n}_d{d}", boundary_cloud(n, d)) for d in (2, 3)
       for n in (1, 2, 3, 4, 7, 8, 9, 15, 16, 17, 31, 32, 33, 63, 64, 65)]
    + [(f"single_child_n{n}", single_child_cloud(n)) for n in (3, 5, 6, 9, 10, 17, 18)]
)


def directions(d: int) -> np.ndarray:
    eye = np.eye(d, dtype=np.float32)
    return _f(np.stack([v for axis in eye for v in (axis, -axis)]))


def symmetric_tie_cloud(d: int) -> tuple[np.ndarray, np.ndarray, float]:
    """Unit directions repeated 4x plus a shell at radius 3; queries at the origin
    (tests/test_knn.py:292-324). Every k <= 4 * 2d neighbour is tied at distance 1."""
    dirs = directions(d)
    pts = np.concatenate([np.repeat(dirs, 4, axis=0), 3.0 * dirs]).astype(np.float32)
    q = np.zeros((2, d), np.float32)
    return pts, q, 1.0


def knn_pathological_cases() -> list[tuple[str, np.ndarray, int]]:
    """(points, k) pairs of tests/test_knn.py:160-258."""
    rng = np.random.default_rng(77)
    return [
        ("line_2d", np.stack([linspace(-3, 3, 17), linspace(6, -6, 17)], axis=1), 4),
        ("line_3d", np.stack([linspace(-2, 2, 19), linspace(4, -4, 19), linspace(1, 9, 19)], axis=1), 8),
        ("zigzag_3d", _f([[i - 2.0, (i + 1.0) * (-1) ** (i + 1), 7.0] for i in range(12)]), 4),
        ("duplicates_3d", np.full((18, 3), 2.5, np.float32), 16),
        ("wide_2d", _f([[i * 1e6, ((i + 1) // 2) * 1e-3 * (-1) ** (i + 1)] for i in range(9)]), 8),
        ("wide_3d", _f([[((i + 1) // 2) * 1e-3 * (-1) ** (i + 1), i * 1e6, ((i + 1) // 2) * 2.0 * (-1) ** (i + 1)]
                        for i in range(9)]), 8),
        ("outlier_2d", np.concatenate([rng.random((20, 2), dtype=np.float32), _f([[1000.0, -1000.0]])]), 4),
    ]
