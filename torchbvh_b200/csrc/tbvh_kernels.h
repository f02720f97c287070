// Host-visible launch interface between the C-ABI layer (tbvh_capi.cu) and the
// kernel translation units (tbvh_build.cu, tbvh_knn.cu). No torch types.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "tbvh_common.cuh"

namespace tbvh {

// ---- radix sort (stable LSD, 8-bit digits, decoupled look-back) -----------
constexpr int kSortThreads = 256;
// Keys per thread of a sort tile. Measured on B200 (build ms, c1 / c3 / c5 / c4):
// 8: 0.071 / 0.288 / 1.123 / 1.606; 12: 0.075 / 0.294 / 1.127 / 1.560;
// 16: 0.087 / 0.317 / 1.146 / 1.560 (80 registers in every form).
#ifndef TBVH_SORT_IPT
#define TBVH_SORT_IPT 12
#endif
constexpr int kSortIpt = TBVH_SORT_IPT;  // keys per thread in one sort tile
constexpr int kSortTile = kSortThreads * kSortIpt;  // elements per tile
constexpr int kRadix = 256;
constexpr int kMaxSortPasses = 8;

// The sort key of element e is the composite (cloud(e) << code_bits) | code(e);
// pass p orders by composite bits [8p, 8p + 8). Values are packed element
// indices, so the cloud of an element is recovered from its value.
struct SortPlan {
  int code_bits = 0;   // 30 (3-D) or 32 (2-D)
  int cloud_bits = 0;  // ceil(log2(num_clouds))
  int passes = 0;
  int64_t n = 0;       // elements
  int64_t tiles = 0;
};

SortPlan make_sort_plan(int64_t n, int num_clouds, int dim);

struct SortScratch {
  uint32_t* keys[2];
  uint32_t* vals[2];
  uint32_t* hist;         // passes x 256
  uint32_t* tile_ctr;     // passes
  uint64_t* lookback[2];  // 2 x (tiles x 256), ping-pong between passes
};

size_t sort_scratch_bytes(const SortPlan& plan);
void carve_sort_scratch(const SortPlan& plan, char*& cursor, SortScratch& s);

// ---- build -----------------------------------------------------------------
constexpr int kTreeThreads = 256;
constexpr int kTreeSubLevels = 10;  // one build block owns 2^10 leaves
constexpr int kTreeHopLevels = 8;   // upper levels are merged 8 levels per hop

// Host-side per-cloud facts (the device table mirrors this for ragged input).
CloudTree cloud_tree_facts(int64_t n);
int64_t cloud_tree_blocks(const CloudTree& t);
int64_t cloud_tree_counters(const CloudTree& t);

struct BuildLaunch {
  // inputs
  const float* points;
  CloudMap clouds;
  int dim;
  // outputs
  float* node_aabbs;
  int64_t* sorted_indices;
  float* scene_min;
  float* scene_max;
  int32_t* left_child;   // nullable
  int32_t* right_child;  // nullable
  int32_t* mem_to_leaf;  // nullable
  bool arrays_per_cloud;
  // plan
  SortPlan sort;
  int64_t tree_blocks;
  int64_t tree_counters;
  CloudTree uniform;        // valid when clouds.uniform_n > 0
  int64_t uniform_rows;     // nr of one uniform cloud
  // scratch
  SortScratch ss;
  uint32_t* bounds_enc;     // num_clouds x 2D
  CloudTree* table;         // ragged only
  uint32_t* tree_counter;   // tree_counters entries
};

cudaError_t launch_build(const BuildLaunch& b, cudaStream_t stream);

// Bounded-wait self-test: one sort pass whose tile 0 is never claimed, so the
// look-back wait of tile 1 gives up after spin_limit polls and raises
// kDevErrLookbackTimeout. Scratch of selftest_scratch_bytes().
size_t selftest_scratch_bytes();
cudaError_t launch_lookback_selftest(void* scratch, int spin_limit, cudaStream_t stream);

// left_child_mem / right_child_mem / mem_to_leaf of one cloud of n points.
cudaError_t launch_traversal_arrays(int64_t n, int32_t* left, int32_t* right, int32_t* m2l, cudaStream_t stream);

struct QuerySortLaunch {
  const float* queries;
  CloudMap clouds;
  int dim;
  const float* scene_min;
  const float* scene_max;
  int64_t* order_out;
  SortPlan sort;
  SortScratch ss;
};

cudaError_t launch_query_sort(const QuerySortLaunch& q, cudaStream_t stream);

// Scene box of one cloud (the build's bounds step alone); enc: 2·D words of scratch.
cudaError_t launch_scene_bounds(const float* points, int64_t n, int D, uint32_t* enc, float* smin, float* smax,
                                cudaStream_t stream);

// One rank's share of the queries of one cloud, in Morton order (see
// k_share_cells in tbvh_build.cu). Synchronous: the share size comes back to
// the host (*count_out) before the share is sorted.
struct ShareLaunch {
  const float* queries;
  int64_t num_queries;
  int dim;
  const float* scene_min;
  const float* scene_max;
  int rank;
  int world;
  int64_t chunk;        // queries per ownership run (M / world: contiguous Morton ranges)
  int64_t* share_out;   // capacity num_queries
  void* workspace;      // share_scratch_bytes(num_queries, dim)
};
size_t share_scratch_bytes(int64_t m, int dim);
cudaError_t launch_share_queries(const ShareLaunch& q, int64_t* count_out, cudaStream_t stream);

// ---- k-NN traversal ----------------------------------------------------------
constexpr int kMaxDest = 8;  // result destinations of one k-NN launch (GPUs of one node)
struct KnnLaunch {
  const float* node_aabbs;
  const int64_t* sorted_indices;
  const float* queries;
  const int64_t* order;  // nullable: identity order
  int64_t* out_idx;
  float* out_dist;
  CloudMap points;
  CloudMap queries_map;
  const CloudTree* table;  // ragged only (written by launch_knn's init kernel)
  CloudTree* table_scratch;
  CloudTree uniform;
  int64_t uniform_rows;
  int64_t total_queries;
  int dim;
  int k;
  const float* source_points = nullptr;  // fused neighbour-position gather (nullable)
  float* out_positions = nullptr;
  bool spatial = false;                  // output rows in sorted order
  // Result rows delivered to every destination (row = query index), instead of
  // out_idx/out_dist, when num_dest > 0. Destinations may be peer-mapped
  // buffers of other GPUs (NVLink stores).
  int num_dest = 0;
  bool dest_idx32 = false;  // dest_idx buffers hold int32 indices (the caller widens them)
  // dest_idx[0] / dest_dist[0] are multicast addresses (num_dest == 1, int32
  // indices): one multimem store per 16 bytes reaches every GPU of the group.
  bool dest_multimem = false;
  int64_t* dest_idx[kMaxDest] = {};
  float* dest_dist[kMaxDest] = {};
};

cudaError_t launch_knn(const KnnLaunch& q, cudaStream_t stream);

// Sets the calling thread's tbvh_last_error() text and returns `code`.
int record_error(int code, const char* message);

// Host-side count of kernel launches issued by this library (all devices).
void count_launches(int n);
uint64_t launches_so_far();

// Device status word (error bits from bounded waits / guards), per device.
cudaError_t read_device_status(unsigned* out, bool clear);
unsigned* device_status_ptr();

}  // namespace tbvh
