// C-ABI entry points (include/torchbvh_b200.h): argument validation, plans,
// workspace carving and launch orchestration. No allocation happens here;
// callers provide outputs and workspace.
#include <climits>
#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/torchbvh_b200.h"
#include "tbvh_kernels.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(TBVH_ERR_CUDA, "%s: CUDA error %s (%s)", where, cudaGetErrorName(e), cudaGetErrorString(e));
}

int set_device(int device, const char* op) {
  if (device < 0) return TBVH_OK;
  int cur = -1;
  cudaError_t e = cudaGetDevice(&cur);
  if (e == cudaSuccess && cur == device) return TBVH_OK;
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, op);
  return TBVH_OK;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Whether the traversal on the current device may store to `p`: memory of that
// device, managed memory, or page-locked host memory mapped at the same address
// (unified addressing), which the kernel then fills across PCIe. Pageable host
// memory and other devices' memory are refused here, before a launch could fault.
bool kernel_writable(const void* p) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  switch (at.type) {
    case cudaMemoryTypeDevice: return at.device == dev;
    case cudaMemoryTypeManaged: return true;
    case cudaMemoryTypeHost: return at.devicePointer == p;
    default: return false;
  }
}

// Cloud description shared by build and query.
struct Clouds {
  int64_t num = 0;
  int64_t uniform_n = 0;        // > 0: fixed-size
  const int64_t* off_host = nullptr;
  int64_t total = 0;
  int64_t min_n = 0;
};

int describe(const char* op, int64_t num, int64_t uniform_n, const int64_t* off_host, Clouds& c,
             bool need_host_offsets) {
  c = Clouds{};
  if (num < 1 || num > INT_MAX) return fail(TBVH_ERR_BAD_ARG, "%s: number of clouds must be in [1, 2^31)", op);
  c.num = num;
  c.uniform_n = uniform_n;
  c.off_host = off_host;
  if (uniform_n > 0) {
    if (uniform_n > INT_MAX || num * uniform_n > INT_MAX)
      return fail(TBVH_ERR_BAD_ARG, "%s: total point count must fit in signed int32", op);
    c.total = num * uniform_n;
    c.min_n = uniform_n;
    return TBVH_OK;
  }
  if (off_host == nullptr) {
    if (need_host_offsets) return fail(TBVH_ERR_BAD_ARG, "%s: ragged input needs host offsets", op);
    return TBVH_OK;
  }
  if (off_host[0] != 0) return fail(TBVH_ERR_BAD_ARG, "%s: offsets must start at 0", op);
  int64_t mn = INT64_MAX;
  for (int64_t b = 0; b < num; ++b) {
    const int64_t sz = off_host[b + 1] - off_host[b];
    if (sz <= 0) return fail(TBVH_ERR_BAD_ARG, "%s: offsets must be strictly increasing", op);
    if (sz < mn) mn = sz;
  }
  c.total = off_host[num];
  c.min_n = mn;
  if (c.total > INT_MAX) return fail(TBVH_ERR_BAD_ARG, "%s: total point count must fit in signed int32", op);
  return TBVH_OK;
}

tbvh::CloudMap device_map(const Clouds& c, const int64_t* off_dev) {
  tbvh::CloudMap m;
  m.offsets = off_dev;
  m.uniform_n = c.uniform_n;
  m.num_clouds = int(c.num);
  return m;
}

// ---- build plan --------------------------------------------------------------
struct BuildPlan {
  tbvh::SortPlan sort;
  int64_t rows = 0;
  int64_t tree_blocks = 0;
  int64_t tree_counters = 0;
  tbvh::CloudTree uni{};
  int64_t uni_rows = 0;
  size_t sort_bytes = 0, bounds_bytes = 0, table_bytes = 0, counter_bytes = 0;
  size_t total_bytes() const { return sort_bytes + bounds_bytes + table_bytes + counter_bytes; }
};

void plan_build(const Clouds& c, int dim, BuildPlan& p) {
  p.sort = tbvh::make_sort_plan(c.total, int(c.num), dim);
  if (c.uniform_n > 0) {
    p.uni = tbvh::cloud_tree_facts(c.uniform_n);
    p.uni_rows = tbvh::real_node_count(c.uniform_n);
    p.rows = p.uni_rows * c.num;
    p.tree_blocks = tbvh::cloud_tree_blocks(p.uni) * c.num;
    p.tree_counters = tbvh::cloud_tree_counters(p.uni) * c.num;
  } else {
    for (int64_t b = 0; b < c.num; ++b) {
      const int64_t n = c.off_host[b + 1] - c.off_host[b];
      const tbvh::CloudTree t = tbvh::cloud_tree_facts(n);
      p.rows += tbvh::real_node_count(n);
      p.tree_blocks += tbvh::cloud_tree_blocks(t);
      p.tree_counters += tbvh::cloud_tree_counters(t);
    }
  }
  p.sort_bytes = tbvh::sort_scratch_bytes(p.sort);
  p.bounds_bytes = align_up(size_t(c.num) * 2 * dim * 4, 256);
  p.table_bytes = c.uniform_n > 0 ? 0 : align_up(size_t(c.num) * sizeof(tbvh::CloudTree), 256);
  p.counter_bytes = align_up(size_t(p.tree_counters > 0 ? p.tree_counters : 1) * 4, 256);
}

}  // namespace

int tbvh::record_error(int code, const char* message) {
  g_last_error = message;
  return code;
}

extern "C" {

const char* tbvh_last_error(void) { return g_last_error.c_str(); }

int tbvh_abi_version(void) { return 1; }

uint64_t tbvh_kernel_launch_count(void) { return tbvh::launches_so_far(); }

int tbvh_device_status(int device, unsigned* out_bits, int clear) {
  if (out_bits == nullptr) return fail(TBVH_ERR_BAD_ARG, "tbvh_device_status: out_bits is NULL");
  int rc = set_device(device, "tbvh_device_status");
  if (rc) return rc;
  cudaError_t e = tbvh::read_device_status(out_bits, clear != 0);
  if (e != cudaSuccess) return cuda_fail(e, "tbvh_device_status");
  return TBVH_OK;
}

size_t tbvh_selftest_workspace_size(void) { return tbvh::selftest_scratch_bytes(); }

int tbvh_selftest_lookback_timeout(int device, void* workspace, size_t workspace_bytes, void* stream,
                                   unsigned* out_bits) {
  const char* op = "tbvh_selftest_lookback_timeout";
  g_last_error.clear();
  if (out_bits == nullptr) return fail(TBVH_ERR_BAD_ARG, "%s: out_bits is NULL", op);
  if (workspace == nullptr || workspace_bytes < tbvh::selftest_scratch_bytes())
    return fail(TBVH_ERR_WORKSPACE, "%s: workspace of %zu bytes is smaller than the required %zu", op,
                workspace_bytes, tbvh::selftest_scratch_bytes());
  int rc = set_device(device, op);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = tbvh::read_device_status(out_bits, true);  // start from a clear word
  if (e == cudaSuccess) e = tbvh::launch_lookback_selftest(workspace, 1 << 12, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = tbvh::read_device_status(out_bits, true);
  if (e != cudaSuccess) return cuda_fail(e, op);
  return TBVH_OK;
}

int64_t tbvh_real_node_count(int64_t num_points) {
  return num_points > 0 ? tbvh::real_node_count(num_points) : 0;
}

size_t tbvh_build_workspace_size(int64_t num_clouds, int64_t points_per_cloud, const int64_t* offsets_host,
                                 int dim) {
  Clouds c;
  if (describe("tbvh_build_workspace_size", num_clouds, points_per_cloud, offsets_host, c, true)) return 0;
  if (dim != 2 && dim != 3) return 0;
  BuildPlan p;
  plan_build(c, dim, p);
  return p.total_bytes();
}

int tbvh_build(int device, const float* points, int64_t num_clouds, int64_t points_per_cloud,
               const int64_t* offsets_dev, const int64_t* offsets_host, int dim,
               float* node_aabbs, int64_t* sorted_indices, float* scene_min, float* scene_max,
               int32_t* left_child_mem, int32_t* right_child_mem, int32_t* mem_to_leaf,
               int traversal_arrays_per_cloud,
               void* workspace, size_t workspace_bytes, void* stream) {
  const char* op = "build_bvh";
  g_last_error.clear();
  if (dim != 2 && dim != 3) return fail(TBVH_ERR_BAD_ARG, "%s: D must be 2 or 3", op);
  Clouds c;
  int rc = describe(op, num_clouds, points_per_cloud, offsets_host, c, true);
  if (rc) return rc;
  if (points_per_cloud <= 0 && offsets_dev == nullptr)
    return fail(TBVH_ERR_BAD_ARG, "%s: ragged input needs device offsets", op);
  if (!points || !node_aabbs || !sorted_indices || !scene_min || !scene_max)
    return fail(TBVH_ERR_BAD_ARG, "%s: NULL input/output pointer", op);
  const int arrays = (left_child_mem != nullptr) + (right_child_mem != nullptr) + (mem_to_leaf != nullptr);
  if (arrays != 0 && arrays != 3)
    return fail(TBVH_ERR_BAD_ARG, "%s: traversal arrays must be all present or all NULL", op);
  BuildPlan p;
  plan_build(c, dim, p);
  if (workspace == nullptr || workspace_bytes < p.total_bytes())
    return fail(TBVH_ERR_WORKSPACE, "%s: workspace of %zu bytes is smaller than the required %zu", op,
                workspace_bytes, p.total_bytes());
  rc = set_device(device, op);
  if (rc) return rc;

  tbvh::BuildLaunch b{};
  b.points = points;
  b.clouds = device_map(c, offsets_dev);
  b.dim = dim;
  b.node_aabbs = node_aabbs;
  b.sorted_indices = sorted_indices;
  b.scene_min = scene_min;
  b.scene_max = scene_max;
  b.left_child = left_child_mem;
  b.right_child = right_child_mem;
  b.mem_to_leaf = mem_to_leaf;
  b.arrays_per_cloud = traversal_arrays_per_cloud != 0;
  b.sort = p.sort;
  b.tree_blocks = p.tree_blocks;
  b.tree_counters = p.tree_counters;
  b.uniform = p.uni;
  b.uniform_rows = p.uni_rows;
  char* cur = static_cast<char*>(workspace);
  tbvh::carve_sort_scratch(p.sort, cur, b.ss);
  b.bounds_enc = reinterpret_cast<uint32_t*>(cur);
  cur += p.bounds_bytes;
  b.table = p.table_bytes ? reinterpret_cast<tbvh::CloudTree*>(cur) : nullptr;
  cur += p.table_bytes;
  b.tree_counter = reinterpret_cast<uint32_t*>(cur);
  cudaError_t e = tbvh::launch_build(b, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, op);
  return TBVH_OK;
}

int tbvh_traversal_arrays(int device, int64_t num_points, int32_t* left_child_mem, int32_t* right_child_mem,
                          int32_t* mem_to_leaf, void* stream) {
  const char* op = "build_traversal_arrays";
  g_last_error.clear();
  if (num_points < 1 || num_points > INT_MAX)
    return fail(TBVH_ERR_BAD_ARG, "%s: point count must be in [1, 2^31)", op);
  if (!left_child_mem || !right_child_mem || !mem_to_leaf)
    return fail(TBVH_ERR_BAD_ARG, "%s: NULL output pointer", op);
  int rc = set_device(device, op);
  if (rc) return rc;
  cudaError_t e = tbvh::launch_traversal_arrays(num_points, left_child_mem, right_child_mem, mem_to_leaf,
                                                static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, op);
  return TBVH_OK;
}

size_t tbvh_sort_queries_workspace_size(int64_t num_clouds, int64_t total_queries, int dim) {
  if (num_clouds < 1 || total_queries < 0 || (dim != 2 && dim != 3)) return 0;
  const tbvh::SortPlan p = tbvh::make_sort_plan(total_queries, int(num_clouds), dim);
  return tbvh::sort_scratch_bytes(p);
}

int tbvh_sort_queries(int device, const float* queries, int64_t num_clouds, int64_t queries_per_cloud,
                      const int64_t* query_offsets_dev, int64_t total_queries, int dim,
                      const float* scene_min, const float* scene_max, int64_t* order_out,
                      void* workspace, size_t workspace_bytes, void* stream) {
  const char* op = "morton_sort_queries_narrow";
  g_last_error.clear();
  if (dim != 2 && dim != 3) return fail(TBVH_ERR_BAD_ARG, "%s: D must be 2 or 3", op);
  if (num_clouds < 1 || num_clouds > INT_MAX) return fail(TBVH_ERR_BAD_ARG, "%s: bad number of clouds", op);
  if (total_queries < 0 || total_queries > INT_MAX)
    return fail(TBVH_ERR_BAD_ARG, "%s: total query count must fit in signed int32", op);
  if (queries_per_cloud <= 0 && query_offsets_dev == nullptr)
    return fail(TBVH_ERR_BAD_ARG, "%s: ragged queries need device offsets", op);
  if (queries_per_cloud > 0 && queries_per_cloud * num_clouds != total_queries)
    return fail(TBVH_ERR_BAD_ARG, "%s: queries_per_cloud * num_clouds != total_queries", op);
  if (total_queries == 0) return TBVH_OK;
  if (!queries || !scene_min || !scene_max || !order_out)
    return fail(TBVH_ERR_BAD_ARG, "%s: NULL input/output pointer", op);
  const tbvh::SortPlan p = tbvh::make_sort_plan(total_queries, int(num_clouds), dim);
  const size_t need = tbvh::sort_scratch_bytes(p);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(TBVH_ERR_WORKSPACE, "%s: workspace of %zu bytes is smaller than the required %zu", op,
                workspace_bytes, need);
  int rc = set_device(device, op);
  if (rc) return rc;
  tbvh::QuerySortLaunch q{};
  q.queries = queries;
  q.clouds.offsets = query_offsets_dev;
  q.clouds.uniform_n = queries_per_cloud > 0 ? queries_per_cloud : 0;
  q.clouds.num_clouds = int(num_clouds);
  q.dim = dim;
  q.scene_min = scene_min;
  q.scene_max = scene_max;
  q.order_out = order_out;
  q.sort = p;
  char* cur = static_cast<char*>(workspace);
  tbvh::carve_sort_scratch(p, cur, q.ss);
  cudaError_t e = tbvh::launch_query_sort(q, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, op);
  return TBVH_OK;
}

size_t tbvh_scene_bounds_workspace_size(void) { return 256; }

int tbvh_scene_bounds(int device, const float* points, int64_t num_points, int dim, float* scene_min,
                      float* scene_max, void* workspace, size_t workspace_bytes, void* stream) {
  const char* op = "scene_bounds";
  g_last_error.clear();
  if (dim != 2 && dim != 3) return fail(TBVH_ERR_BAD_ARG, "%s: D must be 2 or 3", op);
  if (num_points < 1 || num_points > INT_MAX)
    return fail(TBVH_ERR_BAD_ARG, "%s: point count must be in [1, 2^31)", op);
  if (!points || !scene_min || !scene_max) return fail(TBVH_ERR_BAD_ARG, "%s: NULL pointer", op);
  if (workspace == nullptr || workspace_bytes < tbvh_scene_bounds_workspace_size())
    return fail(TBVH_ERR_WORKSPACE, "%s: workspace of %zu bytes is smaller than the required %zu", op,
                workspace_bytes, tbvh_scene_bounds_workspace_size());
  int rc = set_device(device, op);
  if (rc) return rc;
  const cudaError_t e = tbvh::launch_scene_bounds(points, num_points, dim, static_cast<uint32_t*>(workspace),
                                                  scene_min, scene_max, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, op);
  return TBVH_OK;
}

size_t tbvh_share_queries_workspace_size(int64_t num_queries, int dim) {
  if (num_queries < 1 || num_queries > INT_MAX || (dim != 2 && dim != 3)) return 0;
  return tbvh::share_scratch_bytes(num_queries, dim);
}

int tbvh_share_queries(int device, const float* queries, int64_t num_queries, int dim, const float* scene_min,
                       const float* scene_max, int rank, int world, int64_t chunk, int64_t* share_out,
                       int64_t* share_count, void* workspace, size_t workspace_bytes, void* stream) {
  const char* op = "share_queries";
  g_last_error.clear();
  if (dim != 2 && dim != 3) return fail(TBVH_ERR_BAD_ARG, "%s: D must be 2 or 3", op);
  if (num_queries < 1 || num_queries > INT_MAX)
    return fail(TBVH_ERR_BAD_ARG, "%s: query count must be in [1, 2^31)", op);
  if (world < 1 || world > 256 || rank < 0 || rank >= world)
    return fail(TBVH_ERR_BAD_ARG, "%s: need 0 <= rank < world <= 256", op);
  if (chunk < 1) return fail(TBVH_ERR_BAD_ARG, "%s: chunk must be >= 1", op);
  if (!queries || !scene_min || !scene_max || !share_out || !share_count)
    return fail(TBVH_ERR_BAD_ARG, "%s: NULL pointer", op);
  const size_t need = tbvh::share_scratch_bytes(num_queries, dim);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(TBVH_ERR_WORKSPACE, "%s: workspace of %zu bytes is smaller than the required %zu", op,
                workspace_bytes, need);
  int rc = set_device(device, op);
  if (rc) return rc;
  tbvh::ShareLaunch q{};
  q.queries = queries;
  q.num_queries = num_queries;
  q.dim = dim;
  q.scene_min = scene_min;
  q.scene_max = scene_max;
  q.rank = rank;
  q.world = world;
  q.chunk = chunk;
  q.share_out = share_out;
  q.workspace = workspace;
  cudaError_t e = tbvh::launch_share_queries(q, share_count, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, op);
  return TBVH_OK;
}

size_t tbvh_query_knn_workspace_size(int64_t num_clouds, int64_t points_per_cloud) {
  if (num_clouds < 1) return 0;
  if (points_per_cloud > 0) return 256;
  return align_up(size_t(num_clouds) * sizeof(tbvh::CloudTree), 256);
}

int tbvh_query_knn_gather(int device, const float* node_aabbs, const int64_t* sorted_indices,
                          int64_t num_clouds, int64_t points_per_cloud,
                          const int64_t* point_offsets_dev, const int64_t* point_offsets_host,
                          const float* queries, int64_t queries_per_cloud, const int64_t* query_offsets_dev,
                          int64_t total_queries, const int64_t* order, int dim, int k,
                          int64_t* out_indices, float* out_distances,
                          const float* source_points, float* out_positions, int spatial_output,
                          void* workspace, size_t workspace_bytes, void* stream) {
  const char* op = spatial_output ? "query_knn_batched_cached_bounds_spatial"
                   : order        ? "query_knn_batched_cached_bounds_ordered"
                                  : "query_knn_batched_cached_bounds";
  if ((source_points == nullptr) != (out_positions == nullptr))
    return fail(TBVH_ERR_BAD_ARG, "%s: source_points and out_positions must both be given or both be NULL", op);
  if (spatial_output && order == nullptr)
    return fail(TBVH_ERR_BAD_ARG, "%s: spatial output needs a query order", op);
  g_last_error.clear();
  if (dim != 2 && dim != 3) return fail(TBVH_ERR_BAD_ARG, "%s: D must be 2 or 3", op);
  if (k != 4 && k != 8 && k != 16 && k != 32)
    return fail(TBVH_ERR_UNSUPPORTED_K, "%s: k must be 4, 8, or 16 (or 32), got %d", op, k);
  Clouds c;
  int rc = describe(op, num_clouds, points_per_cloud, point_offsets_host, c, false);
  if (rc) return rc;
  if (points_per_cloud <= 0 && point_offsets_dev == nullptr)
    return fail(TBVH_ERR_BAD_ARG, "%s: ragged input needs device point offsets", op);
  if (c.min_n > 0 && c.min_n < k) return fail(TBVH_ERR_BAD_ARG, "%s: num_leaves must be >= k", op);
  if (total_queries < 0 || total_queries > INT_MAX)
    return fail(TBVH_ERR_BAD_ARG, "%s: total query count must fit in signed int32", op);
  if (queries_per_cloud <= 0 && query_offsets_dev == nullptr)
    return fail(TBVH_ERR_BAD_ARG, "%s: ragged queries need device offsets", op);
  if (queries_per_cloud > 0 && queries_per_cloud * num_clouds != total_queries)
    return fail(TBVH_ERR_BAD_ARG, "%s: queries_per_cloud * num_clouds != total_queries", op);
  if (total_queries == 0) return TBVH_OK;
  if (!node_aabbs || !sorted_indices || !queries || !out_indices || !out_distances)
    return fail(TBVH_ERR_BAD_ARG, "%s: NULL input/output pointer", op);
  const size_t need = tbvh_query_knn_workspace_size(num_clouds, points_per_cloud);
  if (points_per_cloud <= 0 && (workspace == nullptr || workspace_bytes < need))
    return fail(TBVH_ERR_WORKSPACE, "%s: workspace of %zu bytes is smaller than the required %zu", op,
                workspace_bytes, need);
  rc = set_device(device, op);
  if (rc) return rc;
  if (!kernel_writable(out_indices) || !kernel_writable(out_distances) ||
      (out_positions && !kernel_writable(out_positions)))
    return fail(TBVH_ERR_BAD_ARG, "%s: outputs must be memory of this device or page-locked host memory", op);
  tbvh::KnnLaunch q{};
  q.node_aabbs = node_aabbs;
  q.sorted_indices = sorted_indices;
  q.queries = queries;
  q.order = order;
  q.out_idx = out_indices;
  q.out_dist = out_distances;
  q.points = device_map(c, point_offsets_dev);
  q.queries_map.offsets = query_offsets_dev;
  q.queries_map.uniform_n = queries_per_cloud > 0 ? queries_per_cloud : 0;
  q.queries_map.num_clouds = int(num_clouds);
  if (points_per_cloud > 0) {
    q.uniform = tbvh::cloud_tree_facts(points_per_cloud);
    q.uniform_rows = tbvh::real_node_count(points_per_cloud);
  }
  q.table_scratch = points_per_cloud > 0 ? nullptr : static_cast<tbvh::CloudTree*>(workspace);
  q.total_queries = total_queries;
  q.dim = dim;
  q.k = k;
  q.source_points = source_points;
  q.out_positions = out_positions;
  q.spatial = spatial_output != 0;
  cudaError_t e = tbvh::launch_knn(q, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, op);
  return TBVH_OK;
}

int tbvh_query_knn(int device, const float* node_aabbs, const int64_t* sorted_indices,
                   int64_t num_clouds, int64_t points_per_cloud,
                   const int64_t* point_offsets_dev, const int64_t* point_offsets_host,
                   const float* queries, int64_t queries_per_cloud, const int64_t* query_offsets_dev,
                   int64_t total_queries, const int64_t* order, int dim, int k,
                   int64_t* out_indices, float* out_distances,
                   void* workspace, size_t workspace_bytes, void* stream) {
  return tbvh_query_knn_gather(device, node_aabbs, sorted_indices, num_clouds, points_per_cloud,
                               point_offsets_dev, point_offsets_host, queries, queries_per_cloud,
                               query_offsets_dev, total_queries, order, dim, k, out_indices, out_distances,
                               nullptr, nullptr, 0, workspace, workspace_bytes, stream);
}

}  // extern "C"
