/*
 * CPU oracle for the BVH k-NN path -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference algorithm (torchbvh 0.3.4) used as
 * the checker by tests/, by __graft_entry__.smoke() and by bench.py's CPU
 * baseline / reference arm. The product path never calls it.
 *
 * Floating point follows the reference's CUDA build (--use_fast_math):
 * float32 throughout, flush-to-zero + denormals-are-zero set in MXCSR for the
 * duration of every call, fused multiply-add exactly where nvcc contracts
 * `dist += delta * delta`. One documented difference: the Morton
 * normalisation divides with IEEE division here, whereas fast-math CUDA
 * division may differ in the last bits, so a point lying within a few ulp of
 * a quantisation boundary can get a neighbouring Morton cell. Tree invariants
 * and k-NN results do not depend on that; bit-equal sorted_indices against
 * the reference are pinned by the golden vectors in tests/golden/.
 */
#ifndef TBVH_ORACLE_H_
#define TBVH_ORACLE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Scene AABB: per axis min/max seeded with +/-1e30 (bvh_build.cu:453-494). */
void tbo_scene_bounds(const float* pts, int64_t n, int d, float* lo, float* hi);

/* Morton codes against lo/hi (morton.cuh:19-68). */
void tbo_morton_codes(const float* pts, int64_t n, int d, const float* lo, const float* hi, uint32_t* codes);

/* Stable argsort of uint32 keys (ties keep ascending index), as the stable
 * segmented radix sort of bvh_build.cu:551-600. */
void tbo_stable_argsort_u32(const uint32_t* keys, int64_t n, int64_t* perm);

/* Implicit tree sizes (implicit_tree.cuh:56-66). */
int64_t tbo_real_node_count(int64_t n);
int tbo_leaf_level(int64_t n);

/* Node AABBs in memory order plus traversal arrays (bvh_build.cu:241-398). */
void tbo_build_tree(const float* pts, const int64_t* sorted, int64_t n, int d, float* node_aabbs,
                    int32_t* left, int32_t* right, int32_t* mem_to_leaf);

/* Whole single-cloud build: bounds -> codes -> stable sort -> tree. */
void tbo_build(const float* pts, int64_t n, int d, float* node_aabbs, int64_t* sorted, float* scene_min,
               float* scene_max, int32_t* left, int32_t* right, int32_t* mem_to_leaf);

/* The reference's depth-first branch-and-bound k-NN (knn_query.cu:20-154):
 * closer child first (left on equal bounds), deferred sibling with its bound,
 * prune when bound > k-th, insert when distance < k-th. Results ascending,
 * ties in the reference's discovery order. `threads` <= 0 uses one thread. */
void tbo_knn_reference(const float* node_aabbs, const int64_t* sorted, int64_t n, int d, const float* queries,
                       int64_t m, int k, int64_t* out_idx, float* out_dist, int threads);

/* Exhaustive k-NN with the same distance arithmetic, ordered by
 * (distance, source index): the canonical answer the B200 kernel returns. */
void tbo_knn_bruteforce(const float* pts, int64_t n, int d, const float* queries, int64_t m, int k,
                        int64_t* out_idx, float* out_dist, int threads);

/* Squared distances of given (query, source index) pairs with the reference
 * arithmetic; negative indices give FLT_MAX. out[m*k] for idx[m*k]. */
void tbo_pair_distances(const float* pts, int64_t n, int d, const float* queries, int64_t m, int k,
                        const int64_t* idx, float* out);

/* Build + reference k-NN for `clouds` independent clouds laid out
 * back-to-back (points/queries/outputs packed by offsets), multi-threaded
 * across queries: the CPU baseline of bench.py. */
void tbo_build_and_query(const float* pts, const int64_t* pt_offsets, const float* queries, const int64_t* q_offsets,
                         int64_t clouds, int d, int k, int64_t* out_idx, float* out_dist, int threads,
                         double* build_seconds, double* query_seconds);

#ifdef __cplusplus
}
#endif

#endif
