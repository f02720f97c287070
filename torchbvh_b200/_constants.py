"""Public constants (torchbvh/_constants.py:1-2), with k = 32 added."""

SUPPORTED_K = (4, 8, 16, 32)
SUPPORTED_DIMS = (2, 3)

# Squared distance at or below which a neighbour counts as an exact hit in
# interpolate_displaced, and the inverse-distance weight regulariser
# (torchbvh/_constants.py:3).
EXACT_DISTANCE_EPSILON = 1.0e-12
