"""torchbvh_b200: B200-native exact BVH k-NN, a drop-in for torchbvh's k-NN path.

``import torchbvh_b200 as torchbvh`` exposes the same k-NN surface as
torchbvh 0.3.4 (torchbvh/__init__.py:1-54): ``BVH``, ``build_bvh``,
``query_knn``, ``destroy_bvh``, the handle classes, the displaced-query
helpers of torchbvh/_multihead.py and the
``SUPPORTED_K`` / ``SUPPORTED_DIMS`` constants (k = 32 added). Every kernel
behind it is hand-written CUDA for sm_100a in ``libtorchbvh_b200.so``; there
is no CPU fallback.
"""

from ._bvh_class import BVH
from ._constants import SUPPORTED_DIMS, SUPPORTED_K
from ._handles import BVHHandle, BatchedBVHHandle, RaggedBVHHandle, destroy_bvh
from ._multihead import gather_neighbor_values, interpolate_displaced, query_displaced_knn
from ._native import device_status
from ._query import build_bvh, query_knn
from ._version import __version__

__all__ = [
    "BVH",
    "BVHHandle",
    "BatchedBVHHandle",
    "RaggedBVHHandle",
    "build_bvh",
    "destroy_bvh",
    "query_knn",
    "query_displaced_knn",
    "gather_neighbor_values",
    "interpolate_displaced",
    "device_status",
    "SUPPORTED_K",
    "SUPPORTED_DIMS",
]
