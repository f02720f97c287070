"""Public constants (torchbvh/_constants.py:1-2), with k = 32 added."""

SUPPORTED_K = (4, 8, 16, 32)
SUPPORTED_DIMS = (2, 3)
