"""Generates the golden fixtures from the reference torchbvh 0.3.4 CUDA path.

Two files, both from seeded inputs:

* ``reference_cuda.npz`` — small and edge cases stored in full: the
  reference's tree (every handle field), its k-NN results through the sorted
  and the unsorted query paths, and its own query Morton permutation
  (``_C.morton_sort_queries_narrow``, torchbvh/csrc/morton_sort.cu:212-287),
  plus the full c1 workload.
* ``reference_configs.npz`` — the five benchmark configurations at full size,
  as digests (``tests/golden/digests.py``): per cloud the SHA-256 of the
  reference's ``sorted_indices``, ``node_aabbs`` and query permutation; per
  65,536-row block the SHA-256 of the canonical result rows; and, stored
  verbatim, every row whose k-th distance is tied with a (k+1)-th candidate.
  c1, c2, c3 and c5 run the reference's public API (c5 is its per-cloud
  ragged loop). c4 has k = 32, which the reference's dispatch does not offer:
  it runs the reference's own traversal kernel instantiated at K = 32
  (``oracle/ref_knn_harness.cu``) over the reference's build and query
  order. The (k+1)-th neighbour comes from the same harness at K = 9, 17, 33
  (from the stock path at k = 8 for c1).

The reference is the unmodified package installed into baseline/_ref
(``pip install --no-deps --target baseline/_ref``), its extension built by its
own loader into baseline/_ref/torch_ext; the harness is built by
``python oracle/ref_harness.py <reference root>``. Needs a CUDA GPU:

    TORCH_CUDA_ARCH_LIST=10.0 TORCH_EXTENSIONS_DIR=baseline/_ref/torch_ext \\
        python tests/golden/make_golden.py [--cases OUT.npz] [--configs OUT.npz]

Inputs are generated with numpy / torch CPU generators from fixed seeds; the
small cases store them, the configurations regenerate them from
torchbvh_b200.workloads.
"""

from __future__ import annotations

import argparse
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "baseline" / "_ref"))

import torchbvh as ref  # noqa: E402  (the reference package from baseline/_ref)

from tests import clouds  # noqa: E402
from tests.golden import digests  # noqa: E402
from torchbvh_b200 import workloads  # noqa: E402

CONFIGS = ("c1", "c2", "c3", "c5", "c4")


def cases():
    rng = np.random.default_rng(424242)
    out = []
    for d, n, m, k in [(3, 20000, 3000, 16), (2, 20000, 3000, 8), (3, 4097, 500, 4), (2, 1000, 500, 16),
                       (3, 33, 50, 8), (2, 5, 10, 4), (3, 1025, 300, 4)]:
        pts = rng.random((n, d), dtype=np.float32)
        q = rng.random((m, d), dtype=np.float32)
        out.append((f"rand_d{d}_n{n}_k{k}", "single", pts, q, k, True))
    g = torch.Generator().manual_seed(77)
    centers = torch.rand((32, 3), generator=g)
    comp = torch.randint(0, 32, (16384,), generator=g)
    gm = (centers[comp] + 0.02 * torch.randn((16384, 3), generator=g)).numpy()
    gq = (torch.from_numpy(gm[:2048]) + 0.01 * torch.randn((2048, 3), generator=g)).numpy()
    out.append(("gaussian_mixture_16384_k16", "single", gm, gq, 16, True))
    for name, pts, k in clouds.knn_pathological_cases():
        q = pts[: min(7, pts.shape[0])] + np.float32(0.125)
        out.append((f"patho_{name}", "single", pts, q, k, True))
    for d in (2, 3):
        pts, q, _ = clouds.symmetric_tie_cloud(d)
        out.append((f"ties_d{d}", "single", pts, q, 8, True))
        out.append((f"duplicates_d{d}", "single", np.full((20, d), 3.5, np.float32), np.full((3, d), 3.5, np.float32),
                    16, True))
    for name, pts in clouds.BUILD_CASES:
        out.append((f"build_{name}", "single", pts, pts[:1], 4, pts.shape[0] >= 4))
    bpts = rng.random((3, 3000, 3), dtype=np.float32)
    bpts[1] *= 50.0
    bq = rng.random((3, 200, 3), dtype=np.float32)
    out.append(("batched_3x3000_k8", "batched", bpts, bq, 8, True))
    return out


def _order(h, q: torch.Tensor) -> torch.Tensor:
    """The reference's query Morton permutation for a single-cloud handle, (M,) int64."""
    return ref._C.morton_sort_queries_narrow(q.unsqueeze(0), h["scene_min"].unsqueeze(0),
                                             h["scene_max"].unsqueeze(0))[0]


def run_single(pts, q, k, do_query):
    p = torch.from_numpy(np.ascontiguousarray(pts)).cuda()
    h = ref.build_bvh(p)
    res = {key: h[key].cpu().numpy() for key in ("node_aabbs", "sorted_indices", "scene_min", "scene_max",
                                                   "left_child_mem", "right_child_mem", "mem_to_leaf")}
    qt = torch.from_numpy(np.ascontiguousarray(q)).cuda()
    if p.dim() == 3:
        res["query_order"] = ref._C.morton_sort_queries_narrow(qt, h["scene_min"], h["scene_max"]).cpu().numpy()
    else:
        res["query_order"] = _order(h, qt).cpu().numpy()
    if do_query:
        i, d = ref.query_knn(h, qt, k)
        iu, du = ref.query_knn(h, qt, k, sort_queries=False)
        res.update(indices=i.cpu().numpy(), distances=d.cpu().numpy(), indices_unsorted=iu.cpu().numpy(),
                   distances_unsorted=du.cpu().numpy())
    return res


def make_cases(out_path: str) -> None:
    arrays = {}
    names = []
    for name, mode, pts, q, k, do_query in cases():
        res = run_single(pts, q, k, do_query)  # batched input goes through the reference's batched path too
        names.append(name)
        arrays[f"{name}/points"] = pts
        arrays[f"{name}/queries"] = q
        arrays[f"{name}/k"] = np.array(k)
        arrays[f"{name}/mode"] = np.array(mode)
        for key, val in res.items():
            arrays[f"{name}/{key}"] = val
    w = workloads.c1_single_uniform()
    res = run_single(w.points.numpy(), w.queries.numpy(), w.k, True)
    names.append("c1")
    arrays["c1/k"] = np.array(w.k)
    arrays["c1/mode"] = np.array("workload_c1")
    for key, val in res.items():
        arrays[f"c1/{key}"] = val
    arrays["_cases"] = np.array(names)
    arrays["_meta"] = _meta()
    np.savez_compressed(out_path, **arrays)
    print(f"wrote {len(names)} cases to {out_path}", flush=True)


def _meta() -> np.ndarray:
    return np.array([f"torchbvh {ref.__version__}", torch.__version__, torch.version.cuda,
                     torch.cuda.get_device_name(0)])


# ---------------------------------------------------------------------------
# Full configurations
# ---------------------------------------------------------------------------

def _knn_one_cloud(h, q: torch.Tensor, order: torch.Tensor, k: int, harness):
    """Reference results of one cloud: the stock API where k is offered, else the
    K-instantiated reference kernel over the same build and query order."""
    if k in ref.SUPPORTED_K:
        return ref.query_knn(h, q, k)
    i, d = harness.knn_ordered_any_k(h["node_aabbs"].unsqueeze(0), h["sorted_indices"].unsqueeze(0),
                                     q.unsqueeze(0), order.unsqueeze(0).contiguous(), int(h["num_leaves"]),
                                     int(h["num_real_nodes"]), int(h["dim"]), k)
    return i[0], d[0]


def _kth_plus_one(h, q: torch.Tensor, order: torch.Tensor, k: int, harness) -> torch.Tensor:
    """Distances of the k + 1 (or more) nearest neighbours of each query, (M, >= k + 1)."""
    if k == 4:
        return ref.query_knn(h, q, 8)[1]
    i, d = harness.knn_ordered_any_k(h["node_aabbs"].unsqueeze(0), h["sorted_indices"].unsqueeze(0),
                                     q.unsqueeze(0), order.unsqueeze(0).contiguous(), int(h["num_leaves"]),
                                     int(h["num_real_nodes"]), int(h["dim"]), k + 1)
    del i
    return d[0]


def reference_config(name: str, harness) -> dict:
    w = workloads.make(name)
    dev = torch.device("cuda", 0)
    k = w.k
    pts = w.points.to(dev)
    q = w.queries.to(dev)
    tree_sorted, tree_nodes, order_sha = [], [], []
    idx_parts, dist_parts, far_parts = [], [], []
    t0 = time.perf_counter()
    if w.points.dim() == 3:
        clouds_in = [(pts[b], q[b]) for b in range(pts.shape[0])]
    elif w.batch_offsets is not None:
        o = w.batch_offsets.tolist()
        qo = w.query_offsets.tolist()
        clouds_in = [(pts[o[b]:o[b + 1]].contiguous(), q[qo[b]:qo[b + 1]].contiguous()) for b in range(len(o) - 1)]
    else:
        clouds_in = [(pts, q)]
    if w.points.dim() == 3:
        # The batched reference path: one batched build, one batched query.
        h = ref.build_bvh(pts)
        order = ref._C.morton_sort_queries_narrow(q, h["scene_min"], h["scene_max"])
        for b in range(pts.shape[0]):
            tree_sorted.append(digests.tensor_digest(h["sorted_indices"][b]))
            tree_nodes.append(digests.tensor_digest(h["node_aabbs"][b]))
            order_sha.append(digests.tensor_digest(order[b]))
        i, d = ref.query_knn(h, q, k)
        idx_parts.append(i.reshape(-1, k))
        dist_parts.append(d.reshape(-1, k))
        for b in range(pts.shape[0]):
            hb = ref.build_bvh(pts[b].contiguous())
            far_parts.append(_kth_plus_one(hb, q[b].contiguous(), _order(hb, q[b].contiguous()), k, harness))
            del hb
    else:
        for p_b, q_b in clouds_in:
            h = ref.build_bvh(p_b)
            order = _order(h, q_b)
            tree_sorted.append(digests.tensor_digest(h["sorted_indices"]))
            tree_nodes.append(digests.tensor_digest(h["node_aabbs"]))
            order_sha.append(digests.tensor_digest(order))
            i, d = _knn_one_cloud(h, q_b, order, k, harness)
            idx_parts.append(i)
            dist_parts.append(d)
            far_parts.append(_kth_plus_one(h, q_b, order, k, harness))
            del h
    idx = torch.cat(idx_parts)
    dist = torch.cat(dist_parts)
    far = torch.cat([f[:, :k + 1] for f in far_parts])
    ties = digests.boundary_tie_rows(far, k)
    keys = digests.canonical_keys(idx, dist)
    blocks = digests.block_digests(keys, ties)
    tsel = torch.as_tensor(ties, dtype=torch.int64, device=dev)
    out = {
        "k": np.array(k),
        "rows": np.array(idx.shape[0]),
        "block_sha": blocks,
        "tie_rows": ties,
        "tie_idx": idx.index_select(0, tsel).cpu().numpy(),
        "tie_dist": dist.index_select(0, tsel).cpu().numpy(),
        "tree_sorted_sha": np.array(tree_sorted),
        "tree_nodes_sha": np.array(tree_nodes),
        "order_sha": np.array(order_sha),
        "source": np.array("reference K=32 kernel instantiation (oracle/ref_knn_harness.cu)" if k == 32
                           else "reference public API"),
    }
    print(f"{name}: {idx.shape[0]} rows, {len(blocks)} blocks, {ties.size} boundary-tie rows, "
          f"{time.perf_counter() - t0:.1f} s", flush=True)
    return out


def make_configs(out_path: str, names=CONFIGS) -> None:
    from oracle import ref_harness

    harness = ref_harness.load()
    arrays = {}
    for name in names:
        for key, val in reference_config(name, harness).items():
            arrays[f"{name}/{key}"] = val
        torch.cuda.empty_cache()
    arrays["_configs"] = np.array(list(names))
    arrays["_meta"] = _meta()
    np.savez_compressed(out_path, **arrays)
    print(f"wrote {len(names)} configurations to {out_path}", flush=True)


def main() -> None:
    here = Path(__file__).resolve().parent
    ap = argparse.ArgumentParser()
    ap.add_argument("--cases", default=str(here / "reference_cuda.npz"))
    ap.add_argument("--configs", default=str(here / "reference_configs.npz"))
    ap.add_argument("--only", choices=["cases", "configs"], default=None)
    args = ap.parse_args()
    if args.only != "configs":
        make_cases(args.cases)
    if args.only != "cases":
        make_configs(args.configs)


if __name__ == "__main__":
    main()
