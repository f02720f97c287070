/*
 * torchbvh_b200 C ABI: the drop-in boundary of the B200 BVH k-NN path.
 *
 * Plain pointers and sizes only. Every device pointer must live on `device`;
 * every call enqueues work on `stream` (a cudaStream_t passed as void*) and
 * returns without synchronising. Outputs and workspace are caller-allocated
 * (the Python layer uses the PyTorch caching allocator). Return value 0 is
 * success; otherwise one of TBVH_ERR_* with a message in tbvh_last_error().
 *
 * Each entry point names the reference interface it replaces (paths inside
 * the torchbvh 0.3.4 project).
 */
#ifndef TORCHBVH_B200_H_
#define TORCHBVH_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  TBVH_OK = 0,
  TBVH_ERR_BAD_ARG = 1,        /* shape / pointer / size validation (reference: TORCH_CHECK) */
  TBVH_ERR_UNSUPPORTED_K = 2,  /* k not in {4, 8, 16, 32} */
  TBVH_ERR_CUDA = 3,           /* CUDA launch or runtime error */
  TBVH_ERR_WORKSPACE = 4       /* workspace smaller than the *_workspace_size() answer */
};

/* Device status bits, reported by tbvh_device_status(). */
enum {
  TBVH_DEVICE_LOOKBACK_TIMEOUT = 1, /* a radix-sort look-back wait hit its bound */
  TBVH_DEVICE_STACK_OVERFLOW = 2,   /* traversal stack guard tripped */
  TBVH_DEVICE_TREE_COUNTER = 4,     /* tree-build arrival counter out of range */
  TBVH_DEVICE_BAD_INDEX = 8         /* an index read from device memory was out of range (clamped) */
};

/* Message of the last failing call on this thread ("" if none). */
const char* tbvh_last_error(void);

/* ABI version of this library (bumped on any signature change). */
int tbvh_abi_version(void);

/* Reads (and optionally clears) the error bits kernels raised on `device`
 * instead of hanging. Synchronous. No reference counterpart (the reference
 * waits without bounds inside CUB). */
int tbvh_device_status(int device, unsigned* out_bits, int clear);

/* Self-test of the bounded device waits. No reference counterpart (the
 * reference's sort waits inside CUB without a bound). Runs one radix-sort
 * pass of this library over an internal key pattern in `workspace` whose
 * tile 0 is never claimed, so tile 1's look-back wait must give up after a
 * short bound (4,096 polls): the kernel records TBVH_DEVICE_LOOKBACK_TIMEOUT
 * and returns, and the device stays usable. Synchronous on `stream`: clears
 * the status word first, then stores the bits the pass raised in *out_bits
 * (and clears them). workspace: tbvh_selftest_workspace_size() bytes. */
size_t tbvh_selftest_workspace_size(void);
int tbvh_selftest_lookback_timeout(int device, void* workspace, size_t workspace_bytes, void* stream,
                                   unsigned* out_bits);

/* Number of kernels this library has launched in this process (all devices).
 * Host-side counter; lets callers attribute launches to this library. */
uint64_t tbvh_kernel_launch_count(void);

/* Real node count 2N - 1 + popcount(2^ceil(log2 N) - N) of one cloud
 * (torchbvh/csrc/implicit_tree.cuh:61-64). */
int64_t tbvh_real_node_count(int64_t num_points);

/* ---------------------------------------------------------------------------
 * BVH build. Replaces build_bvh_batched_cooperative_cuda
 * (torchbvh/csrc/bvh_build.cu:679-721, bound as build_bvh_batched_cooperative
 * in torchbvh/csrc/bindings.cpp:155-157,192) and, for ragged input, the
 * per-sample Python loop of _build_bvh_ragged (torchbvh/_query.py:68-85).
 *
 * Clouds: fixed size when points_per_cloud > 0 (points is (B, N, D)), else
 * ragged with offsets (B + 1 int64, both a device copy and a host copy).
 * Outputs, packed by cloud:
 *   node_aabbs      float32 [sum_b nr_b, 2*dim]  rows [lo.., hi..], implicit memory order
 *   sorted_indices  int64   [sum_b N_b]          local (in-cloud) point index per sorted leaf
 *   scene_min/max   float32 [B, dim]
 *   left_child_mem / right_child_mem / mem_to_leaf  int32, nullable (all three or none);
 *                   one shared set of nr entries when traversal_arrays_per_cloud == 0
 *                   (fixed-size batches), else packed per cloud.
 */
size_t tbvh_build_workspace_size(int64_t num_clouds, int64_t points_per_cloud,
                                 const int64_t* offsets_host, int dim);
int tbvh_build(int device, const float* points, int64_t num_clouds, int64_t points_per_cloud,
               const int64_t* offsets_dev, const int64_t* offsets_host, int dim,
               float* node_aabbs, int64_t* sorted_indices, float* scene_min, float* scene_max,
               int32_t* left_child_mem, int32_t* right_child_mem, int32_t* mem_to_leaf,
               int traversal_arrays_per_cloud,
               void* workspace, size_t workspace_bytes, void* stream);

/* Traversal arrays of one cloud of num_points points: left_child_mem,
 * right_child_mem, mem_to_leaf int32 [tbvh_real_node_count(num_points)], the
 * values build_traversal_arrays_kernel writes (torchbvh/csrc/bvh_build.cu:
 * 361-398). They depend on num_points only, so a caller may pass NULL for
 * them to tbvh_build and compute them here when they are first read. */
int tbvh_traversal_arrays(int device, int64_t num_points, int32_t* left_child_mem, int32_t* right_child_mem,
                          int32_t* mem_to_leaf, void* stream);

/* ---------------------------------------------------------------------------
 * Morton permutation of query points. Replaces morton_sort_queries_narrow_cuda
 * (torchbvh/csrc/morton_sort.cu:264-287, bound as morton_sort_queries_narrow in
 * torchbvh/csrc/bindings.cpp:195). order_out[p] is the local query index of
 * the p-th query of its cloud in (Morton code, index) order, codes taken
 * against that cloud's scene_min/scene_max.
 */
size_t tbvh_sort_queries_workspace_size(int64_t num_clouds, int64_t total_queries, int dim);
int tbvh_sort_queries(int device, const float* queries, int64_t num_clouds, int64_t queries_per_cloud,
                      const int64_t* query_offsets_dev, int64_t total_queries, int dim,
                      const float* scene_min, const float* scene_max, int64_t* order_out,
                      void* workspace, size_t workspace_bytes, void* stream);

/* Query Morton permutation that allocates nothing. No counterpart in the
 * reference. Same arguments and result as tbvh_sort_queries, minus the
 * workspace: for callers that cannot allocate device memory, such as a plugin
 * or FFI binding that only receives the buffers it reads and writes, or a
 * service that reserves its device memory at start-up and must not call
 * cudaMalloc later (allocation can stall the device or fail under pressure).
 * Its scratch is a fixed array inside the library, held in the memory of
 * every GPU that loads the library until the process exits; one call sorts
 * at most 262,144 queries (larger calls return TBVH_ERR_BAD_ARG). The first
 * call on a device looks up that array's device address once and keeps it for
 * the life of the process, so make it before any stream capture; a device
 * reset (cudaDeviceReset) is not supported afterwards. A negative `device`
 * means the current device, as for tbvh_sort_queries. Every call reuses the same array: the call
 * clears what must start at zero, but calls that overlap on the GPU (other
 * streams, unordered host threads) race on it; keep them on one stream. */
int tbvh_sort_queries_noalloc(int device, const float* queries, int64_t num_clouds, int64_t queries_per_cloud,
                              const int64_t* query_offsets_dev, int64_t total_queries, int dim,
                              const float* scene_min, const float* scene_max, int64_t* order_out, void* stream);

/* ---------------------------------------------------------------------------
 * Exact k-NN. Replaces query_knn_batched_cached_bounds_cuda and
 * query_knn_batched_cached_bounds_ordered_cuda (torchbvh/csrc/knn_query.cu:
 * 419-446, bound in torchbvh/csrc/bindings.cpp:197-198) and, for ragged
 * input, the per-sample loop of _query_knn_ragged (torchbvh/_query.py:299-366).
 * order may be NULL (identity order, the unordered reference kernel).
 * Outputs: out_indices int64 [total_queries, k] (local source indices),
 * out_distances float32 [total_queries, k], ascending, at the query's row.
 * k in {4, 8, 16, 32}; every cloud must hold at least k points.
 * The outputs (and out_positions below) may be memory of `device` or
 * page-locked host memory (cudaHostAlloc / cudaHostRegister, mapped at the
 * same address): the kernel then stores the finished rows across PCIe as it
 * goes, and they are readable on the host once the stream has passed the
 * call. Rows land at scattered query rows, which PCIe serves slowly (16.5 GB/s
 * measured for 6.4 GB of rows on B200, against 52 GB/s for one bulk copy of a
 * device result), so for large outputs a device result plus one copy is
 * faster. Any other output pointer (pageable host memory, another device's
 * memory) returns TBVH_ERR_BAD_ARG before a launch.
 */
size_t tbvh_query_knn_workspace_size(int64_t num_clouds, int64_t points_per_cloud);
int tbvh_query_knn(int device, const float* node_aabbs, const int64_t* sorted_indices,
                   int64_t num_clouds, int64_t points_per_cloud,
                   const int64_t* point_offsets_dev, const int64_t* point_offsets_host,
                   const float* queries, int64_t queries_per_cloud, const int64_t* query_offsets_dev,
                   int64_t total_queries, const int64_t* order, int dim, int k,
                   int64_t* out_indices, float* out_distances,
                   void* workspace, size_t workspace_bytes, void* stream);

/* tbvh_query_knn plus two options of the same traversal:
 *  - source_points / out_positions (both or neither): also writes
 *    out_positions[row, j, :] = source_points[cloud start + out_indices[row, j], :]
 *    (float32 [total_queries, k, dim]) in the same kernel; replaces the
 *    separate source_points[indices] / torch.gather of _query_knn_single /
 *    _query_knn_batched (torchbvh/_query.py:174,203-215). An empty slot
 *    (index -1, fewer than k reachable points) reads the cloud's last point.
 *  - spatial_output = 1 (requires order): row = sorted (Morton) position
 *    instead of the query's own row; replaces
 *    query_knn_batched_cached_bounds_spatial_cuda (torchbvh/csrc/knn_query.cu:
 *    448-461, bound in torchbvh/csrc/bindings.cpp:199). */
int tbvh_query_knn_gather(int device, const float* node_aabbs, const int64_t* sorted_indices,
                          int64_t num_clouds, int64_t points_per_cloud,
                          const int64_t* point_offsets_dev, const int64_t* point_offsets_host,
                          const float* queries, int64_t queries_per_cloud, const int64_t* query_offsets_dev,
                          int64_t total_queries, const int64_t* order, int dim, int k,
                          int64_t* out_indices, float* out_distances,
                          const float* source_points, float* out_positions, int spatial_output,
                          void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * One cloud sharded over the GPUs of a node, results delivered to every GPU.
 * No counterpart in the reference, which is single-GPU; this is the exchange
 * step of the broadcast + split + all-gather form of one large cloud.
 *
 * Buffers that other GPUs write into are shared with CUDA IPC:
 * tbvh_peer_alloc allocates `bytes` (rounded up to whole 2 MiB, so that the
 * buffer is an allocation of its own, which it then verifies with the
 * driver's cuMemGetAddressRange and refuses to share otherwise) on `device`
 * (cudaMalloc) and fills
 * out_handle (tbvh_peer_handle_bytes() bytes) for the other processes;
 * tbvh_peer_open maps such a handle on `device` (point-to-point mapping, no
 * multicast); tbvh_peer_close / tbvh_peer_free undo them. Synchronous.
 */
size_t tbvh_peer_handle_bytes(void);
int tbvh_peer_alloc(int device, size_t bytes, void** out_ptr, void* out_handle);
int tbvh_peer_free(int device, void* ptr);
int tbvh_peer_open(int device, const void* handle, void** out_ptr);
int tbvh_peer_close(int device, void* ptr);

/* Scene box of one cloud of num_points points: scene_min / scene_max (dim
 * floats each, device). The scene-AABB reduction of the build alone
 * (torchbvh/csrc/bvh_build.cu:453-494, the reduction tbvh_build runs first),
 * bit-identical to the scene_min / scene_max tbvh_build returns for the same
 * points. Lets a caller start work that needs only the box (the Morton share
 * of a sharded cloud's queries) on another stream while the build runs.
 * Workspace: tbvh_scene_bounds_workspace_size() bytes of device scratch. */
size_t tbvh_scene_bounds_workspace_size(void);
int tbvh_scene_bounds(int device, const float* points, int64_t num_points, int dim, float* scene_min,
                      float* scene_max, void* workspace, size_t workspace_bytes, void* stream);

/* This rank's share of the num_queries queries of one cloud, in Morton order
 * (codes against scene_min/scene_max, the BVH's scene box). No counterpart in
 * the reference. The code range is cut at cells of its top 15 bits; walking
 * the cells in code order, runs of about `chunk` queries go to ranks 0, 1, ..,
 * world-1, 0, 1, .. (chunk = ceil(num_queries / world) gives each rank one
 * contiguous Morton range; smaller chunks interleave the ranks over the
 * cloud). Every rank computes the same split from the same inputs, so the
 * shares of all ranks partition the queries with no exchange. Writes the
 * share's query indices (int64, ascending Morton code) to share_out (capacity
 * num_queries) and their number to *share_count (host). Synchronous on
 * `stream` (the count is read back before the share is sorted). */
size_t tbvh_share_queries_workspace_size(int64_t num_queries, int dim);
int tbvh_share_queries(int device, const float* queries, int64_t num_queries, int dim, const float* scene_min,
                       const float* scene_max, int rank, int world, int64_t chunk, int64_t* share_out,
                       int64_t* share_count, void* workspace, size_t workspace_bytes, void* stream);

/* Exact k-NN of this rank's share of the queries of one cloud (the BVH of
 * num_points points built by tbvh_build), with every result row written into
 * each of the num_dest (<= 8) destination buffers at the query's own row:
 * dest_indices[d] int64 [num_queries, k], dest_distances[d] float32
 * [num_queries, k], local or peer-mapped. `order` lists the share_count query
 * indices (into `queries`, [num_queries, dim]) this rank serves, normally a
 * contiguous range of their Morton order. Rows of other ranks' shares are not
 * touched. Remote rows are NVLink stores made as the traversal finishes each
 * query; the kernel ends with a system-scope fence, so a collective enqueued
 * after it on every rank (a barrier) orders all deliveries before any rank
 * reads its buffer. Callers must also order each rank's reads of the previous
 * results before the next call's writes (a collective at the start of the
 * step does). */
int tbvh_query_knn_share(int device, const float* node_aabbs, const int64_t* sorted_indices, int64_t num_points,
                         const float* queries, int64_t num_queries, const int64_t* order, int64_t share_count,
                         int dim, int k, int num_dest, int64_t* const* dest_indices,
                         float* const* dest_distances, void* stream);

/* tbvh_query_knn_share with int32 destination index buffers ([num_queries, k]):
 * 8 instead of 12 bytes per neighbour cross NVLink; every rank then widens its
 * own buffer with tbvh_widen_indices (local HBM traffic). No reference
 * counterpart. Point counts are below 2^31, so int32 holds every index (and -1). */
int tbvh_query_knn_share_i32(int device, const float* node_aabbs, const int64_t* sorted_indices, int64_t num_points,
                             const float* queries, int64_t num_queries, const int64_t* order, int64_t share_count,
                             int dim, int k, int num_dest, int32_t* const* dest_indices,
                             float* const* dest_distances, void* stream);

/* tbvh_query_knn_share_i32 with one pair of multicast destinations: mc_indices
 * (int32 [num_queries, k]) and mc_distances (float32 [num_queries, k]) are
 * addresses in a CUDA multicast object (cuMulticastCreate / cuMulticastBindMem,
 * mapped on this device; e.g. the multicast_ptr of a PyTorch symmetric-memory
 * buffer) with every rank's buffer bound to it. Each finished row is written
 * with 16-byte multimem.st stores: it leaves this GPU once and the NVLink
 * switch delivers it to every bound buffer, the local one included, instead of
 * one NVLink store per peer. Addresses must be 16-byte aligned and must be
 * multicast addresses (a plain device pointer is not valid for these stores).
 * Ordering as for tbvh_query_knn_share (system-scope fence at the end of the
 * kernel; a collective after it on every rank before reads). No reference
 * counterpart. */
int tbvh_query_knn_share_multicast(int device, const float* node_aabbs, const int64_t* sorted_indices,
                                   int64_t num_points, const float* queries, int64_t num_queries,
                                   const int64_t* order, int64_t share_count, int dim, int k,
                                   int32_t* mc_indices, float* mc_distances, void* stream);

/* dst[i] = src[i] (int32 -> int64) for i < count, on `stream`. No reference counterpart. */
int tbvh_widen_indices(int device, const int32_t* src, int64_t* dst, int64_t count, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TORCHBVH_B200_H_ */
