"""CPU oracle for the BVH k-NN path -- test infrastructure only.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU baseline and
reference arm as the checker; the product path (torchbvh_b200) never uses it.
"""
