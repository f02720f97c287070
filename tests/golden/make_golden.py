"""Generates tests/golden/reference_cuda.npz: outputs of the reference torchbvh
0.3.4 CUDA path on seeded inputs, used to pin the CPU oracle and the B200 path.

The reference is the unmodified package installed into baseline/_ref (pip
install --no-deps --target baseline/_ref), its extension compiled with its own
loader into baseline/_ref/torch_ext. Needs a CUDA GPU:

    TORCH_CUDA_ARCH_LIST=10.0 TORCH_EXTENSIONS_DIR=baseline/_ref/torch_ext \
        python tests/golden/make_golden.py tests/golden/reference_cuda.npz

Inputs are generated with numpy / torch CPU generators from fixed seeds and
stored next to the outputs (except the c1 workload, regenerated from
torchbvh_b200.workloads.c1_single_uniform()).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "baseline" / "_ref"))

import torchbvh as ref  # noqa: E402  (the reference package from baseline/_ref)

from tests import clouds  # noqa: E402
from torchbvh_b200 import workloads  # noqa: E402


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


def run_single(pts, q, k, do_query):
    p = torch.from_numpy(np.ascontiguousarray(pts)).cuda()
    h = ref.build_bvh(p)
    res = {key: h[key].cpu().numpy() for key in ("node_aabbs", "sorted_indices", "scene_min", "scene_max",
                                                   "left_child_mem", "right_child_mem", "mem_to_leaf")}
    if do_query:
        qt = torch.from_numpy(np.ascontiguousarray(q)).cuda()
        i, d = ref.query_knn(h, qt, k)
        iu, du = ref.query_knn(h, qt, k, sort_queries=False)
        res.update(indices=i.cpu().numpy(), distances=d.cpu().numpy(), indices_unsorted=iu.cpu().numpy(),
                   distances_unsorted=du.cpu().numpy())
    return res


def main(out_path: str) -> None:
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
    arrays["_meta"] = np.array([f"torchbvh {ref.__version__}", torch.__version__, torch.version.cuda,
                                torch.cuda.get_device_name(0)])
    np.savez_compressed(out_path, **arrays)
    print(f"wrote {len(names)} cases to {out_path}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(Path(__file__).with_name("reference_cuda.npz")))
