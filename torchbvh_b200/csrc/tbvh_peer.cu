// Peer-delivered k-NN results for one cloud sharded over the GPUs of a node.
//
// The reference is single-GPU and gathers nothing. Its sharded counterpart
// here (torchbvh_b200.distributed.knn_sharded_single_cloud) gives every rank a
// share of the queries; with an all-gathered result every rank needs every
// row. Instead of a collective after the traversal, tbvh_query_knn_share has
// the traversal write each finished row straight into every rank's (M, k)
// output at the query's own row: local rows to HBM, remote rows as NVLink
// stores into buffers mapped with CUDA IPC. The exchange then overlaps the
// rest of the traversal. No kernel waits on another GPU; ordering across ranks
// comes from the caller's collectives (see the header).
//
// The buffers are plain cudaMalloc allocations shared through
// cudaIpcGetMemHandle / cudaIpcOpenMemHandle: point-to-point mappings only,
// nothing is bound to an NVLink multicast object.
#include <climits>
#include <cstdio>

#include "../../include/torchbvh_b200.h"
#include "tbvh_kernels.h"

namespace {

int peer_fail(int code, const char* op, const char* what) {
  char buf[384];
  snprintf(buf, sizeof(buf), "%s: %s", op, what);
  return tbvh::record_error(code, buf);
}

int peer_cuda_fail(cudaError_t e, const char* op) {
  char buf[384];
  snprintf(buf, sizeof(buf), "%s: CUDA error %s (%s)", op, cudaGetErrorName(e), cudaGetErrorString(e));
  return tbvh::record_error(TBVH_ERR_CUDA, buf);
}

int peer_set_device(int device, const char* op) {
  int cur = -1;
  if (cudaGetDevice(&cur) == cudaSuccess && cur == device) return TBVH_OK;
  const cudaError_t e = cudaSetDevice(device);
  return e == cudaSuccess ? TBVH_OK : peer_cuda_fail(e, op);
}

// The driver's cuMemGetAddressRange (base and size of the allocation that
// contains a device pointer), fetched through the runtime so that the library
// needs no link-time dependency on libcuda. Signature of the driver API:
// CUresult cuMemGetAddressRange(CUdeviceptr* base, size_t* size, CUdeviceptr ptr).
using AddressRangeFn = int (*)(unsigned long long*, size_t*, unsigned long long);

AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult status;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &status) != cudaSuccess ||
        status != cudaDriverEntryPointSuccess)
      return AddressRangeFn(nullptr);
    return reinterpret_cast<AddressRangeFn>(p);
  }();
  return fn;
}

}  // namespace

extern "C" {

size_t tbvh_peer_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int tbvh_peer_alloc(int device, size_t bytes, void** out_ptr, void* out_handle) {
  const char* op = "tbvh_peer_alloc";
  tbvh::record_error(TBVH_OK, "");
  if (!out_ptr || !out_handle || bytes == 0) return peer_fail(TBVH_ERR_BAD_ARG, op, "bad arguments");
  int rc = peer_set_device(device, op);
  if (rc) return rc;
  // Whole 2 MiB units: a small request may be placed inside a larger block
  // that the driver shares between allocations, and an IPC handle maps the
  // block from its start, so another process would not see this pointer.
  constexpr size_t kUnit = size_t(2) << 20;
  bytes = (bytes + kUnit - 1) / kUnit * kUnit;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return peer_cuda_fail(e, op);
  // Refuse to share a buffer that does not start its own allocation: the other
  // ranks would map the allocation's start, not this pointer.
  const AddressRangeFn range = address_range_fn();
  if (range == nullptr) {
    cudaFree(p);
    return peer_fail(TBVH_ERR_CUDA, op, "cannot query allocation ranges (cuMemGetAddressRange unavailable)");
  }
  unsigned long long base = 0;
  size_t extent = 0;
  if (range(&base, &extent, reinterpret_cast<unsigned long long>(p)) != 0 ||
      base != reinterpret_cast<unsigned long long>(p) || extent < bytes) {
    cudaFree(p);
    return peer_fail(TBVH_ERR_CUDA, op, "the buffer is not the base of its own allocation; refusing to share it");
  }
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return peer_cuda_fail(e, op);
  }
  *out_ptr = p;
  *static_cast<cudaIpcMemHandle_t*>(out_handle) = h;
  return TBVH_OK;
}

int tbvh_peer_free(int device, void* ptr) {
  const char* op = "tbvh_peer_free";
  int rc = peer_set_device(device, op);
  if (rc) return rc;
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? TBVH_OK : peer_cuda_fail(e, op);
}

int tbvh_peer_open(int device, const void* handle, void** out_ptr) {
  const char* op = "tbvh_peer_open";
  tbvh::record_error(TBVH_OK, "");
  if (!handle || !out_ptr) return peer_fail(TBVH_ERR_BAD_ARG, op, "bad arguments");
  int rc = peer_set_device(device, op);
  if (rc) return rc;
  void* p = nullptr;
  const cudaError_t e =
      cudaIpcOpenMemHandle(&p, *static_cast<const cudaIpcMemHandle_t*>(handle), cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return peer_cuda_fail(e, op);
  *out_ptr = p;
  return TBVH_OK;
}

int tbvh_peer_close(int device, void* ptr) {
  const char* op = "tbvh_peer_close";
  int rc = peer_set_device(device, op);
  if (rc) return rc;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? TBVH_OK : peer_cuda_fail(e, op);
}

}  // extern "C"

namespace {

// tbvh_query_knn_share and tbvh_query_knn_share_i32: the destination index
// buffers hold int64 or int32 values.
int share_impl(const char* op, int device, const float* node_aabbs, const int64_t* sorted_indices,
               int64_t num_points, const float* queries, int64_t num_queries, const int64_t* order,
               int64_t share_count, int dim, int k, int num_dest, void* const* dest_indices,
               float* const* dest_distances, bool idx32, void* stream, bool multimem = false) {
  tbvh::record_error(TBVH_OK, "");
  if (dim != 2 && dim != 3) return peer_fail(TBVH_ERR_BAD_ARG, op, "D must be 2 or 3");
  if (k != 4 && k != 8 && k != 16 && k != 32)
    return peer_fail(TBVH_ERR_UNSUPPORTED_K, op, "k must be 4, 8, or 16 (or 32)");
  if (num_points < 1 || num_points > INT_MAX)
    return peer_fail(TBVH_ERR_BAD_ARG, op, "point count must be in [1, 2^31)");
  if (num_points < k) return peer_fail(TBVH_ERR_BAD_ARG, op, "num_leaves must be >= k");
  if (num_queries < 0 || num_queries > INT_MAX)
    return peer_fail(TBVH_ERR_BAD_ARG, op, "query count must fit in signed int32");
  if (share_count < 0 || share_count > num_queries)
    return peer_fail(TBVH_ERR_BAD_ARG, op, "share_count must be in [0, num_queries]");
  if (num_dest < 1 || num_dest > tbvh::kMaxDest)
    return peer_fail(TBVH_ERR_BAD_ARG, op, "num_dest must be in [1, 8]");
  if (!dest_indices || !dest_distances) return peer_fail(TBVH_ERR_BAD_ARG, op, "NULL destination list");
  for (int i = 0; i < num_dest; ++i)
    if (!dest_indices[i] || !dest_distances[i]) return peer_fail(TBVH_ERR_BAD_ARG, op, "NULL destination buffer");
  if (multimem && (num_dest != 1 || !idx32 || reinterpret_cast<uintptr_t>(dest_indices[0]) % 16 != 0 ||
                   reinterpret_cast<uintptr_t>(dest_distances[0]) % 16 != 0))
    return peer_fail(TBVH_ERR_BAD_ARG, op, "multicast destinations: one pair of 16-byte aligned addresses");
  if (share_count == 0) return TBVH_OK;
  if (!node_aabbs || !sorted_indices || !queries || !order)
    return peer_fail(TBVH_ERR_BAD_ARG, op, "NULL input pointer");
  int rc = peer_set_device(device, op);
  if (rc) return rc;
  tbvh::KnnLaunch q{};
  q.node_aabbs = node_aabbs;
  q.sorted_indices = sorted_indices;
  q.queries = queries;
  q.order = order;
  q.points.offsets = nullptr;
  q.points.uniform_n = num_points;
  q.points.num_clouds = 1;
  // One cloud of num_queries queries, of which this launch serves the
  // share_count positions listed in `order`.
  q.queries_map.offsets = nullptr;
  q.queries_map.uniform_n = num_queries;
  q.queries_map.num_clouds = 1;
  q.uniform = tbvh::cloud_tree_facts(num_points);
  q.uniform_rows = tbvh::real_node_count(num_points);
  q.total_queries = share_count;
  q.dim = dim;
  q.k = k;
  q.num_dest = num_dest;
  q.dest_idx32 = idx32;
  q.dest_multimem = multimem;
  for (int i = 0; i < num_dest; ++i) {
    q.dest_idx[i] = static_cast<int64_t*>(dest_indices[i]);
    q.dest_dist[i] = dest_distances[i];
  }
  const cudaError_t e = tbvh::launch_knn(q, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TBVH_OK : peer_cuda_fail(e, op);
}

// int32 -> int64, four values per thread when both ends are 16-byte aligned.
__global__ void __launch_bounds__(256) k_widen_i32(const int32_t* __restrict__ src, int64_t* __restrict__ dst,
                                                   int64_t count) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const int64_t quads = count / 4;
  const bool aligned = (reinterpret_cast<uintptr_t>(src) % 16 == 0) && (reinterpret_cast<uintptr_t>(dst) % 16 == 0);
  int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (aligned) {
    for (int64_t g = i; g < quads; g += stride) {
      const int4 v = reinterpret_cast<const int4*>(src)[g];
      reinterpret_cast<longlong2*>(dst)[2 * g] = make_longlong2(v.x, v.y);
      reinterpret_cast<longlong2*>(dst)[2 * g + 1] = make_longlong2(v.z, v.w);
    }
    for (int64_t j = quads * 4 + i; j < count; j += stride) dst[j] = src[j];
  } else {
    for (int64_t j = i; j < count; j += stride) dst[j] = src[j];
  }
}

}  // namespace

extern "C" {

int tbvh_query_knn_share(int device, const float* node_aabbs, const int64_t* sorted_indices, int64_t num_points,
                         const float* queries, int64_t num_queries, const int64_t* order, int64_t share_count,
                         int dim, int k, int num_dest, int64_t* const* dest_indices,
                         float* const* dest_distances, void* stream) {
  return share_impl("query_knn_share", device, node_aabbs, sorted_indices, num_points, queries, num_queries, order,
                    share_count, dim, k, num_dest, reinterpret_cast<void* const*>(dest_indices), dest_distances,
                    false, stream);
}

int tbvh_query_knn_share_i32(int device, const float* node_aabbs, const int64_t* sorted_indices, int64_t num_points,
                             const float* queries, int64_t num_queries, const int64_t* order, int64_t share_count,
                             int dim, int k, int num_dest, int32_t* const* dest_indices,
                             float* const* dest_distances, void* stream) {
  return share_impl("query_knn_share_i32", device, node_aabbs, sorted_indices, num_points, queries, num_queries,
                    order, share_count, dim, k, num_dest, reinterpret_cast<void* const*>(dest_indices),
                    dest_distances, true, stream);
}

int tbvh_query_knn_share_multicast(int device, const float* node_aabbs, const int64_t* sorted_indices,
                                   int64_t num_points, const float* queries, int64_t num_queries,
                                   const int64_t* order, int64_t share_count, int dim, int k,
                                   int32_t* mc_indices, float* mc_distances, void* stream) {
  void* idx[1] = {mc_indices};
  float* dst[1] = {mc_distances};
  return share_impl("query_knn_share_multicast", device, node_aabbs, sorted_indices, num_points, queries,
                    num_queries, order, share_count, dim, k, 1, idx, dst, true, stream, /*multimem=*/true);
}

int tbvh_widen_indices(int device, const int32_t* src, int64_t* dst, int64_t count, void* stream) {
  const char* op = "widen_indices";
  tbvh::record_error(TBVH_OK, "");
  if (count < 0 || (count > 0 && (!src || !dst))) return peer_fail(TBVH_ERR_BAD_ARG, op, "bad arguments");
  if (count == 0) return TBVH_OK;
  int rc = peer_set_device(device, op);
  if (rc) return rc;
  int64_t blocks = (count / 4 + 255) / 256;
  if (blocks < 1) blocks = 1;
  if (blocks > 148 * 16) blocks = 148 * 16;
  k_widen_i32<<<unsigned(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(src, dst, count);
  tbvh::count_launches(1);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TBVH_OK : peer_cuda_fail(e, op);
}

}  // extern "C"
