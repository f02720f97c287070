// tbvh_sort_queries_noalloc: the query Morton sort with library-owned scratch.
//
// Who needs it: callers that hold only the device pointers they were given
// and have no way to allocate more -- a plugin host or FFI binding that was
// handed input/output buffers but no CUDA allocator, or a service that
// reserves all of its device memory at start-up and may not call cudaMalloc
// afterwards (cudaMalloc can synchronise the device and can fail under memory
// pressure). tbvh_sort_queries needs a caller-provided workspace; this variant
// takes its scratch from a fixed array compiled into the library instead.
//
// The array lives in device memory of every GPU that loads this library and
// stays there until the process exits. Its size caps one call at
// kNoAllocMaxQueries queries; larger calls are rejected with an error.
//
// One-time set-up per device: the first call on a device (with that device
// current) resolves the array's device address with cudaGetSymbolAddress and
// caches it for the life of the process. Make that first call before any
// stream capture. A device reset (cudaDeviceReset) invalidates the cached
// address and is not supported while this library is loaded.
//
// All calls share the one array and it keeps whatever the last call left in
// it. The launch sequence clears what must start at zero (digit histograms,
// tile counters, look-back flags) at the start of every call. Calls whose
// work overlaps on the GPU (different streams, or different host threads
// without ordering) race on the array and corrupt each other's results:
// serialise them on one stream.
#include <climits>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/torchbvh_b200.h"
#include "tbvh_kernels.h"

namespace {

constexpr int64_t kNoAllocMaxQueries = int64_t(1) << 18;  // 262,144 queries per call

constexpr size_t round256(size_t v) { return (v + 255) / 256 * 256; }

// Scratch of one sort over kNoAllocMaxQueries elements (sort_scratch_bytes()
// layout: 4 key/value buffers, histograms, tile counters, two look-back areas).
constexpr size_t kNoAllocScratchBytes =
    4 * round256(size_t(kNoAllocMaxQueries) * 4) + round256(size_t(tbvh::kMaxSortPasses) * tbvh::kRadix * 4) +
    round256(size_t(tbvh::kMaxSortPasses) * 4) +
    2 * round256(size_t((kNoAllocMaxQueries + tbvh::kSortTile - 1) / tbvh::kSortTile) * tbvh::kRadix * 8);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mutex;

// Messages go to the library's per-thread error text (tbvh_last_error()).
int noalloc_fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return tbvh::record_error(code, buf);
}

// Device address of the static scratch on the current device (set up once).
int scratch_address(int device, void** out) {
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_addr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      return noalloc_fail(TBVH_ERR_CUDA, "tbvh_sort_queries_noalloc: cudaGetSymbolAddress failed: %s",
                          cudaGetErrorString(e));
    }
    g_scratch_addr[device] = p;
  }
  *out = g_scratch_addr[device];
  return TBVH_OK;
}

}  // namespace

extern "C" {

int tbvh_sort_queries_noalloc(int device, const float* queries, int64_t num_clouds, int64_t queries_per_cloud,
                              const int64_t* query_offsets_dev, int64_t total_queries, int dim,
                              const float* scene_min, const float* scene_max, int64_t* order_out, void* stream) {
  const char* op = "tbvh_sort_queries_noalloc";
  tbvh::record_error(TBVH_OK, "");
  if (dim != 2 && dim != 3) return noalloc_fail(TBVH_ERR_BAD_ARG, "%s: D must be 2 or 3", op);
  if (num_clouds < 1 || num_clouds > INT_MAX)
    return noalloc_fail(TBVH_ERR_BAD_ARG, "%s: bad number of clouds", op);
  if (total_queries < 0) return noalloc_fail(TBVH_ERR_BAD_ARG, "%s: negative query count", op);
  if (total_queries > kNoAllocMaxQueries)
    return noalloc_fail(TBVH_ERR_BAD_ARG,
                        "%s: %lld queries exceed the static scratch capacity of %lld queries per call; "
                        "use tbvh_sort_queries with a caller-provided workspace",
                        op, (long long)total_queries, (long long)kNoAllocMaxQueries);
  if (queries_per_cloud <= 0 && query_offsets_dev == nullptr)
    return noalloc_fail(TBVH_ERR_BAD_ARG, "%s: ragged queries need device offsets", op);
  if (queries_per_cloud > 0 && queries_per_cloud * num_clouds != total_queries)
    return noalloc_fail(TBVH_ERR_BAD_ARG, "%s: queries_per_cloud * num_clouds != total_queries", op);
  int cur = -1;
  cudaError_t e = cudaGetDevice(&cur);
  if (device < 0) {  // as in tbvh_sort_queries: a negative ordinal means the current device
    if (e != cudaSuccess) return noalloc_fail(TBVH_ERR_CUDA, "%s: cudaGetDevice: %s", op, cudaGetErrorString(e));
    device = cur;
  }
  if (device >= kMaxDevices) return noalloc_fail(TBVH_ERR_BAD_ARG, "%s: bad device ordinal", op);
  if (total_queries == 0) return TBVH_OK;
  if (!queries || !scene_min || !scene_max || !order_out)
    return noalloc_fail(TBVH_ERR_BAD_ARG, "%s: NULL input/output pointer", op);
  const tbvh::SortPlan plan = tbvh::make_sort_plan(total_queries, int(num_clouds), dim);
  if (tbvh::sort_scratch_bytes(plan) > kNoAllocScratchBytes)
    return noalloc_fail(TBVH_ERR_BAD_ARG, "%s: scratch plan exceeds the static array", op);

  if (e != cudaSuccess || cur != device) {
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return noalloc_fail(TBVH_ERR_CUDA, "%s: cudaSetDevice: %s", op, cudaGetErrorString(e));
  }
  void* scratch = nullptr;
  const int rc = scratch_address(device, &scratch);
  if (rc != TBVH_OK) return rc;

  tbvh::QuerySortLaunch q{};
  q.queries = queries;
  q.clouds.offsets = query_offsets_dev;
  q.clouds.uniform_n = queries_per_cloud > 0 ? queries_per_cloud : 0;
  q.clouds.num_clouds = int(num_clouds);
  q.dim = dim;
  q.scene_min = scene_min;
  q.scene_max = scene_max;
  q.order_out = order_out;
  q.sort = plan;
  char* cursor = static_cast<char*>(scratch);
  tbvh::carve_sort_scratch(plan, cursor, q.ss);
  e = tbvh::launch_query_sort(q, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return noalloc_fail(TBVH_ERR_CUDA, "%s: %s", op, cudaGetErrorString(e));
  return TBVH_OK;
}

}  // extern "C"
