"""bench.py helpers that run without a GPU: the CPU baselines on small seeded
workloads and the workload description of the JSON line."""
from __future__ import annotations

import importlib.util
from pathlib import Path

import pytest

from torchbvh_b200 import workloads

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_bruteforce_baseline_reports_a_rate(bench):
    w = workloads.make("c1", n=2000, m=500)
    out = bench.cpu_bruteforce_throughput(w, budget_s=0.5)
    assert out["value"] > 0 and out["cores"] >= 1
    assert out["kind"].startswith("torch.cdist")
    assert "queries of 1 of 1 clouds" in out["sample"]


def test_bruteforce_baseline_covers_ragged_clouds(bench):
    w = workloads.make("c5", clouds=4, lo=1024, hi=4096)
    out = bench.cpu_bruteforce_throughput(w, budget_s=0.2)
    assert out["value"] > 0
    assert "of 4 clouds" in out["sample"]


def test_workload_config_names_the_workload(bench):
    w = workloads.make("c1", n=2000, m=500)
    cfg = bench.workload_config(w, 1)
    assert cfg["workload"].startswith("c1") and cfg["k"] == 4 and cfg["parallelism"] == "single GPU"
    assert "dp8" in bench.workload_config(w, 8)["parallelism"]


def test_bruteforce_baseline_covers_batched_clouds(bench):
    w = workloads.make("c2", batch=3, n=2048)
    out = bench.cpu_bruteforce_throughput(w, budget_s=0.2)
    assert out["value"] > 0 and "of 3 clouds" in out["sample"]
