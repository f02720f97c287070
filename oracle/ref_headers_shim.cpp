// Exposes the reference's own header-only Morton and implicit-tree functions
// (torchbvh/csrc/morton.cuh, torchbvh/csrc/implicit_tree.cuh, both written to
// compile as host C++) through a C ABI, so tests can pin the oracle's
// restatement against the reference code itself. Built by oracle/Makefile
// from the reference sources in place; the result stays in oracle/_ref/.
#include <cstdint>

#include "implicit_tree.cuh"
#include "morton.cuh"

extern "C" {

uint32_t tbr_morton_encode_3d(float x, float y, float z, const float* lo, const float* hi) {
  return implicit_bvh::morton::morton_encode_3d(x, y, z, make_float3(lo[0], lo[1], lo[2]),
                                                make_float3(hi[0], hi[1], hi[2]));
}

uint32_t tbr_morton_encode_2d(float x, float y, const float* lo, const float* hi) {
  return implicit_bvh::morton::morton_encode_2d(x, y, make_float2(lo[0], lo[1]), make_float2(hi[0], hi[1]));
}

int tbr_real_node_count(int t) { return implicit_bvh::tree::real_node_count(t); }
int tbr_leaf_level(int t) { return implicit_bvh::tree::leaf_level(t); }
int tbr_virtual_leaves(int t) { return implicit_bvh::tree::virtual_leaves(t); }
int tbr_memory_index(int t, int implicit_idx) { return implicit_bvh::tree::memory_index(t, implicit_idx); }
int tbr_is_virtual(int t, int implicit_idx) { return implicit_bvh::tree::is_virtual(t, implicit_idx) ? 1 : 0; }

}  // extern "C"
