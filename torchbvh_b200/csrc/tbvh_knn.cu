// Exact k-NN traversal for the B200 path.
//
// Replaces query_knn_batched_cached_bounds_kernel and its launchers
// (torchbvh/csrc/knn_query.cu:20-181,329-446). Same inputs (node_aabbs in the
// reference's memory order, int64 sorted_indices, optional Morton query
// order), same outputs (int64 local indices and float32 squared distances,
// ascending, written at the query's original row).
//
// Design (B200-first rather than one independent thread per query):
//  * One warp serves 32 consecutive queries of the (Morton-)sorted order, so
//    its queries are spatial neighbours. The warp walks the implicit tree as a
//    packet: a node is entered when any lane's lower bound admits it, child
//    order is a lane majority vote, and the deferred-sibling stack keeps the
//    node id once per warp (plus, optionally, one bound per lane) in shared
//    memory. Node box loads are warp-uniform (one transaction each).
//  * The tree is cut 5 levels above the leaves: a node there covers <= 32
//    consecutive sorted leaves ("bucket"), which the warp stages into shared
//    memory with one coalesced load (coordinates + original index) and then
//    scans with broadcast reads, every lane testing every point.
//  * Each lane keeps its top-k as packed (distance bits, original index) keys,
//    seeded from the sorted leaves around the query's own Morton rank before
//    the traversal starts. For k <= 8 the keys are an ascending list in
//    registers; for k >= 16 they are a per-lane max-heap in shared memory
//    (one insertion is a sift-down of log2(k) levels instead of k selects,
//    and the k keys leave the register file), heap-sorted in place at the end.
//    Pruning keeps the reference's rule (skip a node only if its lower bound
//    is strictly greater than the k-th distance), so the result is the exact k
//    smallest (distance, index) pairs: identical to the reference except for
//    the order among exactly tied distances, which the reference leaves
//    unspecified (docs/algorithms.md, k-NN Query).
//  * Queries of several clouds may share a warp (ragged batches); the warp
//    serves each cloud in turn with the other lanes disabled.
#include "tbvh_kernels.h"

namespace tbvh {
namespace {

// Tuning knobs (compile-time; the defaults are the measured best on B200).
// One warp per block: a block's resources are released as soon as its warp
// ends, so a slow warp never holds idle warps' slots (c4: 46.9 ms against
// 52.7 ms with four-warp blocks).
#ifndef TBVH_KNN_THREADS
#define TBVH_KNN_THREADS 32
#endif
constexpr int kKnnThreads = TBVH_KNN_THREADS;
constexpr int kKnnWarps = kKnnThreads / 32;
#ifndef TBVH_KNN_BUCKET_LEVELS
#define TBVH_KNN_BUCKET_LEVELS 5
#endif
constexpr int kBucketLevels = TBVH_KNN_BUCKET_LEVELS;  // bucket = 2^levels leaves (<= 32)
constexpr int kBucketSize = 1 << kBucketLevels;
static_assert(kBucketSize <= 32, "a bucket is staged by one warp");
// Deferred nodes: at most 3 per two-level step (one per level for a binary
// step) down to the bucket level, which is <= 26 for N < 2^31.
constexpr int kStackDepth = 44;
// Smallest k kept as a shared-memory heap (smaller k: register list).
#ifndef TBVH_KNN_HEAP_MIN_K
#define TBVH_KNN_HEAP_MIN_K 16
#endif
// 1: the stack keeps each lane's bound of a deferred node; 0: the bound is
// recomputed from the node box when the node is popped. Recomputing costs a
// warp-uniform box load per pop but frees 5.5 KB of shared memory per warp,
// which on B200 buys more resident warps (c4: 53 ms against 69 ms).
#ifndef TBVH_KNN_STACK_BOUNDS
#define TBVH_KNN_STACK_BOUNDS 0
#endif
// 1: above the last level before the buckets, a step tests the four
// grandchildren of the node (four consecutive rows of node_aabbs) and skips
// the children's level: half the steps and stack traffic, four independent
// box loads per step. 0: binary steps.
#ifndef TBVH_KNN_WIDE
#define TBVH_KNN_WIDE 1
#endif
constexpr bool kWideSteps = TBVH_KNN_WIDE != 0;
constexpr bool kStackBounds = TBVH_KNN_STACK_BOUNDS != 0;
// Seeding window: this many times k sorted leaves around the query's rank.
#ifndef TBVH_KNN_SEED_WINDOW
#define TBVH_KNN_SEED_WINDOW 2
#endif
constexpr int kSeedWindow = TBVH_KNN_SEED_WINDOW;
static_assert(kSeedWindow >= 1, "the window must hold at least k leaves");
#ifndef TBVH_KNN_SEED_ALIGN
#define TBVH_KNN_SEED_ALIGN 0
#endif
constexpr bool kSeedAlign = TBVH_KNN_SEED_ALIGN != 0;
// 1: the warp seeds every lane from the union of the lanes' windows (at most
// kUnionCap leaves, staged through shared memory); 0: each lane its own window.
// Measured on B200 (traversal ms, union / own window): c4 47.6 / 46.8, c2 1.96 /
// 1.88, c3 1.31 / 1.07, c5 42.4 / 43.8: the richer seed does not repay its
// extra insertions except on the ragged anisotropic clouds.
#ifndef TBVH_KNN_UNION_SEED
#define TBVH_KNN_UNION_SEED 0
#endif
constexpr bool kUnionSeed = TBVH_KNN_UNION_SEED != 0;
#ifndef TBVH_KNN_UNION_CAP
#define TBVH_KNN_UNION_CAP 256
#endif
constexpr int64_t kUnionCap = TBVH_KNN_UNION_CAP;
static_assert(TBVH_KNN_UNION_CAP >= 32, "the union holds at least k <= 32 leaves");
// Developer option: -DTBVH_KNN_PROFILE=1 sums, over warps, the clock cycles
// of each traversal phase and counts of its events into g_knn_profile
// (slots: 0 rank search, 1 seeding window, 2 node steps, 3 bucket load + marks,
// 4 insertion rounds, 5 stack pops, 6 heap sort + row writes; 7 bucket marks
// and 11 insertions of one lane per warp; 8 node steps, 9 buckets, 10
// insertion rounds, 12 pops, 13 warp passes, 14 active lanes). Off by default;
// timings taken with it on are not reported.
#ifndef TBVH_KNN_PROFILE
#define TBVH_KNN_PROFILE 0
#endif
// Levels of the tree, from the root, that a warp copies into shared memory
// (coalesced, once per cloud it serves) and reads node boxes of from there
// instead of through L1. 0: off (every box comes through L1).
#ifndef TBVH_KNN_TOP_LEVELS
#define TBVH_KNN_TOP_LEVELS 0
#endif
constexpr int kTopLevels = TBVH_KNN_TOP_LEVELS;
static_assert(kTopLevels >= 0 && kTopLevels <= 10, "staged top levels: 0..10");
constexpr int kTopRows = kTopLevels > 0 ? (1 << kTopLevels) - 1 : 1;
#if TBVH_KNN_PROFILE
__device__ unsigned long long g_knn_profile[16];
#define KNN_PF_LAP(slot)                  \
  do {                                    \
    const long long now_ = clock64();     \
    pf_[slot] += now_ - pf_t_;            \
    pf_t_ = now_;                         \
  } while (0)
#define KNN_PF_CNT(slot, n) (pf_[slot] += (n))
#else
#define KNN_PF_LAP(slot) ((void)0)
#define KNN_PF_CNT(slot, n) ((void)0)
#endif

template <int K>
__host__ __device__ constexpr bool heap_topk() { return K >= TBVH_KNN_HEAP_MIN_K; }

struct KnnArgs {
  const float* node_aabbs;
  const int64_t* sorted;
  const float* queries;
  const int64_t* order;
  int64_t* out_idx;
  float* out_dist;
  CloudMap pts;
  CloudMap qry;
  const CloudTree* table;
  CloudTree uni;
  int64_t uni_rows;
  int64_t total_q;
  const float* src_points;  // nullable: fused neighbour-position gather source
  float* out_pos;           // nullable: (rows, K, D) neighbour positions
  int spatial;              // 1: write row = sorted (Morton) position, else the query's own row
  int num_dest;             // > 0: rows go to dest_* (row = query index) instead of out_*
  int dest_idx32;           // 1: dest_idx buffers hold int32 indices
  int dest_multimem;        // 1: dest_idx[0] / dest_dist[0] are multicast addresses (int32 indices)
  int64_t* dest_idx[kMaxDest];
  float* dest_dist[kMaxDest];
  unsigned* status;
};

using u64 = unsigned long long;

template <int K>
struct KnnSmem {
  float4 bucket[kKnnWarps][32];
  uint32_t stack_node[kKnnWarps][kStackDepth];
  float stack_dist[kStackBounds ? kKnnWarps : 1][kStackBounds ? kStackDepth : 1][32];
  u64 heap[heap_topk<K>() ? kKnnWarps : 1][heap_topk<K>() ? K : 1][32];  // [warp][slot][lane]
  float top[kTopLevels > 0 ? kKnnWarps : 1][kTopRows * 6];                 // staged top-level node rows
};

// A top-k slot is one 64-bit key: distance bits above, source index below.
// Squared distances are >= +0, so unsigned key order is (distance, index)
// order. The empty slot (FLT_MAX, -1) is the largest key any accepted
// candidate can be compared with: candidates need distance < FLT_MAX, as for
// the reference's insertion into an empty list.
__device__ __forceinline__ u64 pack_key(float d, int32_t idx) {
  return (u64(__float_as_uint(d)) << 32) | u64(uint32_t(idx));
}
__device__ __forceinline__ float key_dist(u64 k) { return __uint_as_float(uint32_t(k >> 32)); }
__device__ __forceinline__ int32_t key_idx(u64 k) { return int32_t(uint32_t(k)); }
constexpr u64 kEmptyKey = (u64(0x7f7fffffu) << 32) | u64(0xffffffffu);

// ---------------------------------------------------------------------------
// Top-k containers. Both hold the K smallest keys offered so far; `kth` is the
// largest of them (the acceptance threshold: a candidate enters only if its
// key is strictly smaller).
// ---------------------------------------------------------------------------

// k <= 8: ascending list in registers. An insertion decides every slot from
// two independent comparisons (no serial chain).
template <int K, bool kHeap>
struct TopK {
  u64 key[K];
  u64 kth;

  __device__ __forceinline__ void init(u64* /*warp_heap*/, unsigned /*lane*/) {
#pragma unroll
    for (int i = 0; i < K; ++i) key[i] = kEmptyKey;
    kth = kEmptyKey;
  }
  // Fills the list from K keys given one at a time (any order), then sorts.
  __device__ __forceinline__ void seed_slot(int i, u64 v) {
#pragma unroll
    for (int s = 0; s < K; ++s)
      if (s == i) key[s] = v;
  }
  __device__ __forceinline__ void seed_done() {
    sort();
    kth = key[K - 1];
  }
  __device__ __forceinline__ void insert(u64 nk) {  // requires nk < kth
    bool before[K];
#pragma unroll
    for (int s = 0; s < K; ++s) before[s] = nk < key[s];
#pragma unroll
    for (int s = K - 1; s > 0; --s) key[s] = before[s] ? (before[s - 1] ? key[s - 1] : nk) : key[s];
    key[0] = before[0] ? nk : key[0];
    kth = key[K - 1];
  }
  __device__ __forceinline__ void finish() {}
  __device__ __forceinline__ u64 at(int i) const { return key[i]; }

  // In-register bitonic sort, ascending.
  __device__ __forceinline__ void sort() {
#pragma unroll
    for (int size = 2; size <= K; size <<= 1) {
#pragma unroll
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
        for (int i = 0; i < K; ++i) {
          const int j = i ^ stride;
          if (j > i) {
            const bool ascending = (i & size) == 0;
            const u64 a = key[i], b = key[j];
            const bool swap = ascending ? b < a : a < b;
            key[i] = swap ? b : a;
            key[j] = swap ? a : b;
          }
        }
      }
    }
  }
};

// Shared-memory word of slot s of lane l in a warp's heap area: row s, column
// l, so lanes reach distinct banks whatever slots they touch (the sift-downs).
// TBVH_KNN_SWIZZLE=1 uses column l XOR s instead, which makes the cooperative
// row reads (lane s reads slot s of one lane) conflict-free but lets lanes
// sifting different slots collide: c4 traversal 51.7 ms against 46.2 ms on
// B200, so the plain layout is the default and the row reads take the
// conflicts (one read per slot per row, once per query).
#ifndef TBVH_KNN_SWIZZLE
#define TBVH_KNN_SWIZZLE 0
#endif
// Cooperative row writes for heap top-k and the unrolled sift from the root
// are on by default. c4 traversal on B200: both 46.2 ms, sift only 46.6 ms,
// neither 46.9 ms (the writes matter more when rows go to peer GPUs).
#ifndef TBVH_KNN_COOP_WRITE
#define TBVH_KNN_COOP_WRITE 1
#endif
#ifndef TBVH_KNN_UNROLLED_SIFT
#define TBVH_KNN_UNROLLED_SIFT 1
#endif
// Children per heap node: 2 (binary) or 4 (a sift of a 32-slot heap is then 3
// dependent levels of four independent loads instead of 5 levels of two).
#ifndef TBVH_KNN_HEAP_ARITY
#define TBVH_KNN_HEAP_ARITY 2
#endif
constexpr int kArity = TBVH_KNN_HEAP_ARITY;
static_assert(kArity == 2 || kArity == 4, "heap arity 2 or 4");
__device__ __forceinline__ int heap_word(int s, unsigned l) {
  return TBVH_KNN_SWIZZLE ? s * 32 + int(l ^ unsigned(s & 31)) : s * 32 + int(l);
}

// k >= 16: max-heap per lane in shared memory (the warp's area, swizzled by
// heap_word), heap-sorted in place at the end.
template <int K>
struct TopK<K, true> {
  u64* hw;  // the warp's heap area
  unsigned ln;
  u64 kth;  // the root

  struct Slots {
    u64* hw;
    unsigned ln;
    __device__ __forceinline__ u64& operator[](int s) const { return hw[heap_word(s, ln)]; }
  };
  Slots h;

  __device__ __forceinline__ void init(u64* warp_heap, unsigned lane) {
    hw = warp_heap;
    ln = lane;
    h = Slots{warp_heap, lane};
    kth = kEmptyKey;
  }
  // Moves x down from slot i of a heap of n slots.
  __device__ __forceinline__ void sift_down(int i, u64 x, int n) {
#pragma unroll 1
    for (;;) {
      int c = kArity * i + 1;
      if (c >= n) break;
      u64 a = h[c];
#pragma unroll
      for (int d = 1; d < kArity; ++d) {
        if (c + d < n) {
          const u64 b = h[c + d];
          if (b > a) {
            a = b;
            c = kArity * i + 1 + d;
          }
        }
      }
      if (a <= x) break;
      h[i] = a;
      i = c;
    }
    h[i] = x;
  }
  __device__ __forceinline__ void seed_slot(int i, u64 v) { h[i] = v; }
  __device__ __forceinline__ void seed_done() {  // bottom-up heapify
#pragma unroll 1
    for (int i = (K - 2) / kArity; i >= 0; --i) sift_down(i, h[i], K);
    kth = h[0];
  }
  __device__ __forceinline__ void insert(u64 nk) {  // requires nk < kth: replaces the root
    if (!TBVH_KNN_UNROLLED_SIFT) {
      sift_down(0, nk, K);
      kth = h[0];
      return;
    }
    // The sift from the root unrolled over the heap's levels, the children of
    // a level loaded together.
    // The new root is known without reading it back: the larger child of
    // the root if the sift moved past level 0, else nk.
    constexpr int kLevels = kArity == 2 ? (K >= 32 ? 5 : K >= 16 ? 4 : K >= 8 ? 3 : 2)
                                        : (K >= 32 ? 3 : K >= 16 ? 2 : 2);
    int i = 0;
    bool moving = true;
    u64 root = nk;
#pragma unroll
    for (int lvl = 0; lvl < kLevels; ++lvl) {
      const int c = kArity * i + 1;
      if (moving && c < K) {
        u64 a = h[c];
        int pick = 0;
#pragma unroll
        for (int d = 1; d < kArity; ++d) {
          // A missing child reads as key 0, which never wins (keys are >= 0
          // and a move needs a child strictly above nk).
          const u64 b = c + d < K ? h[c + d] : 0ull;
          if (b > a) {
            a = b;
            pick = d;
          }
        }
        if (a > nk) {
          h[i] = a;
          if (lvl == 0) root = a;
          i = c + pick;
        } else {
          moving = false;
        }
      } else {
        moving = false;
      }
    }
    h[i] = nk;
    kth = root;
  }
  // In-place heap sort: slots end ascending.
  __device__ __forceinline__ void finish() {
#pragma unroll 1
    for (int end = K - 1; end > 0; --end) {
      const u64 top = h[0];
      const u64 last = h[end];
      h[end] = top;
      sift_down(0, last, end);
    }
  }
  __device__ __forceinline__ u64 at(int i) const { return h[i]; }
};

template <int D>
__device__ __forceinline__ void load_box(const float* rows, int64_t row, float* lo, float* hi) {
  const float* r = rows + row * (2 * D);
  if constexpr (D == 3) {
    const float2 a = __ldg(reinterpret_cast<const float2*>(r));
    const float2 b = __ldg(reinterpret_cast<const float2*>(r) + 1);
    const float2 c = __ldg(reinterpret_cast<const float2*>(r) + 2);
    lo[0] = a.x; lo[1] = a.y; lo[2] = b.x;
    hi[0] = b.y; hi[1] = c.x; hi[2] = c.y;
  } else {
    const float4 a = __ldg(reinterpret_cast<const float4*>(r));
    lo[0] = a.x; lo[1] = a.y;
    hi[0] = a.z; hi[1] = a.w;
  }
}

template <int D>
__device__ __forceinline__ void load_leaf(const float* rows, int64_t row, float* p) {
  const float* r = rows + row * (2 * D);
  const float2 xy = __ldg(reinterpret_cast<const float2*>(r));
  p[0] = xy.x;
  p[1] = xy.y;
  if constexpr (D == 3) p[2] = __ldg(r + 2);
}

// Writes the K ascending keys as one result row, four slots at a time.
template <int K, bool kHeap>
__device__ __forceinline__ void write_row(const TopK<K, kHeap>& top, int64_t* oi, float* od) {
#pragma unroll
  for (int i = 0; i < K; i += 4) {
    const u64 k0 = top.at(i), k1 = top.at(i + 1), k2 = top.at(i + 2), k3 = top.at(i + 3);
    reinterpret_cast<longlong2*>(oi)[i / 2] = make_longlong2(key_idx(k0), key_idx(k1));
    reinterpret_cast<longlong2*>(oi)[i / 2 + 1] = make_longlong2(key_idx(k2), key_idx(k3));
    reinterpret_cast<float4*>(od)[i / 4] = make_float4(key_dist(k0), key_dist(k1), key_dist(k2), key_dist(k3));
  }
}

// Result rows of a warp whose heaps are sorted, written cooperatively: for each
// lane j of `mask` (32 / K lanes per pass), lane s of the warp writes slot s of
// j's row, so one row is a single contiguous 8·K-byte index store and a 4·K-byte
// distance store (instead of 16-byte pieces of 32 scattered rows per warp
// instruction). Row `row_of_lane` of lane j; every destination buffer when
// kToDest (peer memory included), else out_idx / out_dist.
template <int K, bool kToDest>
__device__ __forceinline__ void write_rows_coop(const KnnArgs& a, const u64* hw, unsigned mask, int64_t row_of_lane,
                                                unsigned lane) {
  constexpr int kPerPass = 32 / K;
  const int sub = int(lane) / K;
  const int slot = int(lane) % K;
  while (mask) {
    int j = -1;
#pragma unroll
    for (int r = 0; r < kPerPass; ++r) {
      const int next = mask ? __ffs(mask) - 1 : -1;
      if (r == sub) j = next;
      if (mask) mask &= mask - 1u;
    }
    const int64_t row = __shfl_sync(kFullMask, row_of_lane, j < 0 ? 0 : j);
    if (j >= 0) {
      const u64 key = hw[heap_word(slot, unsigned(j))];
      const int64_t at = row * K + slot;
      if constexpr (kToDest) {
#pragma unroll 1
        for (int dst = 0; dst < a.num_dest; ++dst) {
          if (a.dest_idx32) {
            reinterpret_cast<int32_t*>(a.dest_idx[dst])[at] = key_idx(key);
          } else {
            a.dest_idx[dst][at] = key_idx(key);
          }
          a.dest_dist[dst][at] = key_dist(key);
        }
      } else {
        a.out_idx[at] = key_idx(key);
        a.out_dist[at] = key_dist(key);
      }
    }
  }
}

// One 16-byte store through a multicast address: the NVLink switch delivers it
// to the same offset of the buffer bound on every GPU of the multicast group
// (local GPU included). A row sent this way leaves the GPU once, whatever the
// number of GPUs.
__device__ __forceinline__ void multimem_store4(void* addr, float a, float b, float c, float d) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};"
               :: "l"(addr), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

// Result rows of a warp whose heaps are sorted, to multicast destinations
// (int32 indices): lane l writes slots 4·(l mod K/4) .. +3 of one row, one
// 16-byte store per array, so a warp instruction carries 128 / K rows.
template <int K>
__device__ __forceinline__ void write_rows_multimem(const KnnArgs& a, const u64* hw, unsigned mask,
                                                    int64_t row_of_lane, unsigned lane) {
  constexpr int kLanesPerRow = K / 4;
  constexpr int kRowsPerPass = 32 / kLanesPerRow;
  const int sub = int(lane) / kLanesPerRow;
  const int s0 = (int(lane) % kLanesPerRow) * 4;
  int32_t* idx = reinterpret_cast<int32_t*>(a.dest_idx[0]);
  float* dst = a.dest_dist[0];
  while (mask) {
    int j = -1;
#pragma unroll
    for (int r = 0; r < kRowsPerPass; ++r) {
      const int next = mask ? __ffs(mask) - 1 : -1;
      if (r == sub) j = next;
      if (mask) mask &= mask - 1u;
    }
    const int64_t row = __shfl_sync(kFullMask, row_of_lane, j < 0 ? 0 : j);
    if (j >= 0) {
      const u64 k0 = hw[heap_word(s0, unsigned(j))], k1 = hw[heap_word(s0 + 1, unsigned(j))];
      const u64 k2 = hw[heap_word(s0 + 2, unsigned(j))], k3 = hw[heap_word(s0 + 3, unsigned(j))];
      const int64_t at = row * K + s0;
      multimem_store4(idx + at, __int_as_float(key_idx(k0)), __int_as_float(key_idx(k1)),
                      __int_as_float(key_idx(k2)), __int_as_float(key_idx(k3)));
      multimem_store4(dst + at, key_dist(k0), key_dist(k1), key_dist(k2), key_dist(k3));
    }
  }
}

template <int D, int K, bool kToDest>
__device__ __forceinline__ void search_cloud(const KnnArgs& a, KnnSmem<K>& s, int cloud, bool mine, int64_t pos,
                                             unsigned lane, unsigned warp) {
  constexpr bool kHeap = heap_topk<K>();
  // Cloud facts.
  CloudTree t;
  if (a.table) {
    t = a.table[cloud];
  } else {
    t = a.uni;
    t.row_off = int64_t(cloud) * a.uni_rows;
  }
  const int64_t n = t.n;
  const int L = t.leaf_level;
  const int Lb = L > kBucketLevels ? L - kBucketLevels : 0;
  const int bucket_span = L - Lb;
  const int64_t pt_off = a.pts.start(cloud);
  const int64_t q_off = a.qry.start(cloud);
  const float* rows = a.node_aabbs + t.row_off * (2 * D);
  const int64_t* sorted = a.sorted + pt_off;
#if TBVH_KNN_PROFILE
  unsigned long long pf_[16] = {};
  long long pf_t_ = clock64();
  const int pf_leader = __ffs(__ballot_sync(kFullMask, mine)) - 1;
#endif

  // Lane l holds cnt(l) and rowoff(l) of level l (l <= L <= 31).
  const int64_t my_cnt = int(lane) <= L ? level_count(n, L, int(lane)) : 0;
  int64_t incl = my_cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t y = __shfl_up_sync(kFullMask, incl, o);
    if (lane >= unsigned(o)) incl += y;
  }
  const int64_t my_rowoff = incl - my_cnt;
  const int64_t leaf_row0 = __shfl_sync(kFullMask, my_rowoff, L);

  // The root box is the scene AABB the Morton codes were taken against.
  float root_lo[D], root_hi[D];
  load_box<D>(rows, 0, root_lo, root_hi);

  // Top levels staged in shared memory (rows [0, top_rows): whole levels).
  int64_t top_rows = 0;
  if constexpr (kTopLevels > 0) {
    top_rows = kTopLevels <= L ? __shfl_sync(kFullMask, my_rowoff, kTopLevels) : leaf_row0 + n;
    if (top_rows > kTopRows) top_rows = kTopRows;  // whole levels never exceed it; kept for safety
    for (int i = int(lane); i < int(top_rows) * 2 * D; i += 32) s.top[warp][i] = __ldg(rows + i);
    __syncwarp();
  }
  // Box of node row `row` (warp-uniform).
  auto node_box = [&](int64_t row, float* lo, float* hi) {
    if (kTopLevels > 0 && row < top_rows) {
      const float* r = &s.top[kTopLevels > 0 ? warp : 0][int(row) * 2 * D];
#pragma unroll
      for (int c = 0; c < D; ++c) {
        lo[c] = r[c];
        hi[c] = r[D + c];
      }
    } else {
      load_box<D>(rows, row, lo, hi);
    }
  };

  // Query.
  float q[D];
  int64_t gq = 0;
#pragma unroll
  for (int c = 0; c < D; ++c) q[c] = 0.0f;
  if (mine) {
    int64_t local = a.order ? a.order[pos] : pos - q_off;
    if (local < 0 || local >= a.qry.size(cloud)) {  // a foreign or corrupted order; keep the read in bounds
      atomicOr(a.status, kDevErrBadIndex);
      local = 0;
    }
    gq = q_off + local;
#pragma unroll
    for (int c = 0; c < D; ++c) q[c] = a.queries[gq * D + c];
  }

  TopK<K, kHeap> top;
  top.init(kHeap ? &s.heap[kHeap ? warp : 0][0][0] : nullptr, lane);
  float kth = mine ? kFar : -1.0f;  // disabled lanes admit nothing
  // Offers a candidate key whose distance is already known to be < FLT_MAX.
  auto offer = [&](u64 nk) {
    if (nk < top.kth) {
      top.insert(nk);
      kth = key_dist(top.kth);
    }
  };

  // Stages sorted leaves [start, start + count) (count <= 32) into the warp's
  // shared buffer with one coalesced load: coordinates and original index.
  auto stage_leaves = [&](int64_t start, int count) {
    if (int(lane) < count) {
      float p[D];
      load_leaf<D>(rows, leaf_row0 + start + lane, p);
      const int32_t src = int32_t(sorted[start + lane]);
      s.bucket[warp][lane] = make_float4(p[0], p[1], D == 3 ? p[2] : 0.0f, __int_as_float(src));
    }
    __syncwarp();
  };
  // Offers the staged points [from, count) to every lane: pass 1 marks those
  // within the lane's current k-th distance (less the `skip` bits), pass 2
  // inserts the marked points, one per lane per round.
  auto mark_and_insert = [&](int from, int count, uint32_t skip) {
    uint32_t cand = 0;
    if (from == 0 && count == 32) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float4 p = s.bucket[warp][i];
        if (point_dist2<D>(q, p.x, p.y, p.z) <= kth) cand |= 1u << i;
      }
    } else {
      for (int i = from; i < count; ++i) {
        const float4 p = s.bucket[warp][i];
        if (point_dist2<D>(q, p.x, p.y, p.z) <= kth) cand |= 1u << i;
      }
    }
    cand &= ~skip;
    __syncwarp();
    KNN_PF_LAP(3);
    KNN_PF_CNT(7, __popc(cand));
    while (__any_sync(kFullMask, cand != 0u)) {
      KNN_PF_CNT(10, 1);
      if (cand) {
        // Marks were taken against the k-th distance at the start of the
        // pass; insertions since may have lowered it. A lane first skips, in
        // a cheap per-lane loop, marks that no longer beat its k-th key, so a
        // round (one insertion) is only spent on one that does.
        u64 nk;
        bool take;
        do {
          const int i = __ffs(cand) - 1;
          cand &= cand - 1u;
          const float4 p = s.bucket[warp][i];
          const float d = point_dist2<D>(q, p.x, p.y, p.z);
          nk = pack_key(d, __float_as_int(p.w));
          take = d < kFar && nk < top.kth;
        } while (!take && cand);
        if (take) {
          KNN_PF_CNT(11, 1);
          top.insert(nk);
          kth = key_dist(top.kth);
        }
      }
    }
    __syncwarp();
    KNN_PF_LAP(4);
  };

  // ---- Seeding. Each lane locates its query's Morton rank among the sorted
  // leaves (binary search, leaf codes recomputed against the root box). Near
  // neighbours sit close to the query in Morton order, so scoring the leaves
  // around that rank makes the k-th distance tight before the exact traversal
  // starts; the traversal then skips the seeded leaves. The seed only affects
  // speed: every seeded point is fully evaluated.
  int64_t rank = 0;
  if (mine) {
    const uint32_t qcode = morton_code<D>(q, root_lo, root_hi);
    int64_t lo = 0, hi = n;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      float p[D];
      load_leaf<D>(rows, leaf_row0 + mid, p);
      if (morton_code<D>(p, root_lo, root_hi) < qcode) lo = mid + 1; else hi = mid;
    }
    rank = lo;
  }
  KNN_PF_LAP(0);
  int64_t w0, w1;  // seeded leaves [w0, w1): the lane's own (per-lane window) or the warp's (union)
  if constexpr (kUnionSeed) {
    // The union of the lanes' windows: [min rank - K, max rank + K), at least
    // K leaves, at most kUnionCap. Every lane scores every leaf of it, so a
    // lane whose own window is poor (a Morton-cell boundary) borrows its
    // neighbours' candidates. Staged 32 leaves at a time with coalesced loads;
    // the first K fill every lane's list.
    int64_t rmin = mine ? rank : n, rmax = mine ? rank : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const int64_t a = __shfl_xor_sync(kFullMask, rmin, o);
      const int64_t b = __shfl_xor_sync(kFullMask, rmax, o);
      rmin = a < rmin ? a : rmin;
      rmax = b > rmax ? b : rmax;
    }
    w0 = rmin - K < 0 ? 0 : rmin - K;
    w1 = rmax + K > n ? n : rmax + K;
    if (w1 - w0 < K) {  // n >= K: widen to K leaves inside [0, n)
      w1 = w0 + K > n ? n : w0 + K;
      w0 = w1 - K;
    }
    if (w1 - w0 > kUnionCap) w1 = w0 + kUnionCap;
    for (int64_t s0 = w0; s0 < w1; s0 += 32) {
      const int cnt = int(w1 - s0 < 32 ? w1 - s0 : 32);
      stage_leaves(s0, cnt);
      int from = 0;
      if (s0 == w0) {
        if (mine) {
          for (int i = 0; i < K; ++i) {
            const float4 p = s.bucket[warp][i];
            const float d = point_dist2<D>(q, p.x, p.y, p.z);
            top.seed_slot(i, d < kFar ? pack_key(d, __float_as_int(p.w)) : kEmptyKey);
          }
          top.seed_done();
          kth = key_dist(top.kth);
        } else {
          top.kth = 0ull;  // accepts nothing
        }
        from = K;
      }
      mark_and_insert(from, cnt, 0u);
    }
  } else {
    // Each lane's own window of kSeedWindow * K leaves around its rank.
    const int64_t win = n < int64_t(kSeedWindow * K) ? n : int64_t(kSeedWindow * K);
    w0 = 0;
    if (mine) {
      // Centred on the rank, or (TBVH_KNN_SEED_ALIGN) the aligned block of
      // `win` leaves that holds it, which is one subtree of the implicit tree.
      w0 = kSeedAlign ? rank / win * win : rank - win / 2;
      if (w0 > n - win) w0 = n - win;
      if (w0 < 0) w0 = 0;
    }
    w1 = mine ? w0 + win : 0;
    // The first K window points fill the list (only distances < FLT_MAX enter,
    // as with insertions into an empty list), then the rest are offered.
    if (mine) {
#pragma unroll
      for (int i = 0; i < K; ++i) {
        float p[D];
        load_leaf<D>(rows, leaf_row0 + w0 + i, p);
        const float d = point_dist2<D>(q, p[0], p[1], D == 3 ? p[2] : 0.0f);
        top.seed_slot(i, d < kFar ? pack_key(d, int32_t(sorted[w0 + i])) : kEmptyKey);
      }
      top.seed_done();
      kth = key_dist(top.kth);
    } else {
      top.kth = 0ull;  // accepts nothing
    }
    for (int64_t i = K; i < win; ++i) {
      if (mine) {
        float p[D];
        load_leaf<D>(rows, leaf_row0 + w0 + i, p);
        const float d = point_dist2<D>(q, p[0], p[1], D == 3 ? p[2] : 0.0f);
        if (d < kFar) offer(pack_key(d, int32_t(sorted[w0 + i])));
      }
    }
  }
  __syncwarp();
  KNN_PF_LAP(1);

  // ---- Exact packet traversal from the root.
  int level = 0;
  int64_t node = 0;
  float nd = box_dist2<D>(q, root_lo, root_hi);
  int sp = 0;
  if (__any_sync(kFullMask, nd <= kth)) {
    for (;;) {
      if (level == Lb) {
        // Bucket: sorted leaves [node << span, +32) clipped to n.
        const int64_t start = node << bucket_span;
        const int64_t rem = n - start;
        const int count = int(rem < (int64_t(1) << bucket_span) ? rem : (int64_t(1) << bucket_span));
        stage_leaves(start, count);
        // Points of the seeded range were scored already.
        uint32_t skip = 0;
        const int64_t slo = w0 - start;
        const int64_t shi = w1 - start;
        if (shi > 0 && slo < count) {
          const int b0 = slo > 0 ? int(slo) : 0;
          const int b1 = shi < count ? int(shi) : count;
          const uint32_t upto = b1 >= 32 ? 0xffffffffu : ((1u << b1) - 1u);
          skip = upto & ~((1u << b0) - 1u);
        }
        KNN_PF_CNT(9, 1);
        mark_and_insert(0, count, skip);
      } else if (kWideSteps && level + 2 <= Lb) {
        // Two levels at once: the node's four grandchildren are four consecutive
        // rows of the next-but-one level (the first is always real). A
        // grandchild box lies inside its parent's, so skipping the parents'
        // level never admits a node the binary walk would have pruned.
        const int gl = level + 2;
        const int64_t g0 = node * 4;
        const int64_t gleft = __shfl_sync(kFullMask, my_cnt, gl) - g0;
        const int64_t grow = __shfl_sync(kFullMask, my_rowoff, gl) + g0;
        float dg[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          dg[g] = INFINITY;
          if (g < gleft) {
            float lo[D], hi[D];
            node_box(grow + g, lo, hi);
            dg[g] = box_dist2<D>(q, lo, hi);
          }
        }
        // Warp-uniform order: the admitted grandchildren by how many lanes find
        // each one their nearest admitted box (ties: lower index first).
        int best = -1;
        float best_d = INFINITY;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          if (dg[g] <= kth && dg[g] < best_d) {
            best_d = dg[g];
            best = g;
          }
        }
        int key[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const bool admitted = __any_sync(kFullMask, dg[g] <= kth);
          const int votes = __popc(__ballot_sync(kFullMask, best == g));
          key[g] = admitted ? (votes << 2) | (3 - g) : -1;
        }
        auto swap_desc = [](int& x, int& y) {
          const int hi = x > y ? x : y;
          y = x > y ? y : x;
          x = hi;
        };
        swap_desc(key[0], key[1]);
        swap_desc(key[2], key[3]);
        swap_desc(key[0], key[2]);
        swap_desc(key[1], key[3]);
        swap_desc(key[1], key[2]);
        // Defer the others, least preferred deepest.
#pragma unroll
        for (int r = 3; r >= 1; --r) {
          if (key[r] >= 0) {
            const int g = 3 - (key[r] & 3);
            if (sp < kStackDepth) {
              if constexpr (kStackBounds) {
                s.stack_dist[warp][sp][lane] = g == 0 ? dg[0] : g == 1 ? dg[1] : g == 2 ? dg[2] : dg[3];
              }
              if (lane == 0) s.stack_node[warp][sp] = uint32_t(g0 + g) | (uint32_t(gl) << 27);
              ++sp;
            } else if (lane == 0) {
              atomicOr(a.status, kDevErrStackOverflow);
            }
          }
        }
        KNN_PF_CNT(8, 1);
        if (key[0] >= 0) {
          const int g = 3 - (key[0] & 3);
          level = gl;
          node = g0 + g;
          nd = g == 0 ? dg[0] : g == 1 ? dg[1] : g == 2 ? dg[2] : dg[3];
          KNN_PF_LAP(2);
          continue;
        }
        KNN_PF_LAP(2);
      } else {
        const int cl = level + 1;
        const int64_t c0 = node * 2;
        const int64_t ccnt = __shfl_sync(kFullMask, my_cnt, cl);
        const int64_t crow = __shfl_sync(kFullMask, my_rowoff, cl) + c0;
        const bool right_real = c0 + 1 < ccnt;
        float lo[D], hi[D];
        node_box(crow, lo, hi);
        const float d0 = box_dist2<D>(q, lo, hi);
        float d1 = INFINITY;
        if (right_real) {
          node_box(crow + 1, lo, hi);
          d1 = box_dist2<D>(q, lo, hi);
        }
        const bool n0 = d0 <= kth;
        const bool n1 = d1 <= kth;
        const bool want = n0 || n1;
        const bool pref_left = n0 && (!n1 || d0 <= d1);
        const int votes_left = __popc(__ballot_sync(kFullMask, want && pref_left));
        const int votes_all = __popc(__ballot_sync(kFullMask, want));
        const bool left_first = 2 * votes_left >= votes_all;
        const float near_d = left_first ? d0 : d1;
        const float far_d = left_first ? d1 : d0;
        const int64_t near_j = left_first ? c0 : c0 + 1;
        const int64_t far_j = left_first ? c0 + 1 : c0;
        if (__any_sync(kFullMask, far_d <= kth)) {
          if (sp < kStackDepth) {
            if constexpr (kStackBounds) s.stack_dist[warp][sp][lane] = far_d;
            if (lane == 0) s.stack_node[warp][sp] = uint32_t(far_j) | (uint32_t(cl) << 27);
            ++sp;
          } else if (lane == 0) {
            atomicOr(a.status, kDevErrStackOverflow);
          }
        }
        KNN_PF_CNT(8, 1);
        if (__any_sync(kFullMask, near_d <= kth)) {
          level = cl;
          node = near_j;
          nd = near_d;
          KNN_PF_LAP(2);
          continue;
        }
        KNN_PF_LAP(2);
      }
      // Pop the next deferred node that some lane still needs (against the
      // lane's current k-th distance).
      bool found = false;
      while (sp > 0) {
        --sp;
        KNN_PF_CNT(12, 1);
        __syncwarp();
        const uint32_t e = s.stack_node[warp][sp];
        const int el = int(e >> 27);
        const int64_t ej = int64_t(e & 0x07ffffffu);
        float d;
        if constexpr (kStackBounds) {
          d = s.stack_dist[warp][sp][lane];
        } else {
          float lo[D], hi[D];
          node_box(__shfl_sync(kFullMask, my_rowoff, el) + ej, lo, hi);
          d = box_dist2<D>(q, lo, hi);
        }
        if (__any_sync(kFullMask, d <= kth)) {
          level = el;
          node = ej;
          nd = d;
          found = true;
          break;
        }
      }
      KNN_PF_LAP(5);
      if (!found) break;
    }
  }
  (void)nd;

#if TBVH_KNN_PROFILE
  KNN_PF_CNT(13, 1);
  KNN_PF_CNT(14, __popc(__ballot_sync(kFullMask, mine)));
  if (mine) top.finish();
  KNN_PF_LAP(6);
  if (int(lane) == pf_leader) {
    for (int i = 0; i < 16; ++i) atomicAdd(&g_knn_profile[i], pf_[i]);
  }
#else
  if (mine) top.finish();
#endif
  if constexpr (kHeap && TBVH_KNN_COOP_WRITE) {
    // Rows leave through the cooperative writer; result rows (and, over
    // NVLink, the peers' copies) are then whole-row stores.
    __syncwarp();
    const int64_t row = kToDest ? gq : (a.spatial ? pos : gq);
    if (kToDest && a.dest_multimem) {
      write_rows_multimem<K>(a, top.hw, __ballot_sync(kFullMask, mine), row, lane);
    } else {
      write_rows_coop<K, kToDest>(a, top.hw, __ballot_sync(kFullMask, mine), row, lane);
    }
    if constexpr (!kToDest) {
      if (mine && a.out_pos) {
        // Fused source_points[indices] gather (see below for the rule on -1).
        const float* src = a.src_points + pt_off * D;
        float* op = a.out_pos + row * K * D;
#pragma unroll 4
        for (int i = 0; i < K; ++i) {
          int64_t idx = key_idx(top.at(i));
          if (idx < 0) idx = n - 1;
#pragma unroll
          for (int c = 0; c < D; ++c) op[i * D + c] = __ldg(src + idx * D + c);
        }
      }
    }
    return;
  }
  if (!mine) return;
  if constexpr (kToDest) {
    // Result row delivered to every destination buffer at the query's row.
    // Destinations on other GPUs are written over NVLink as the results come
    // out of the traversal, so the exchange overlaps the remaining compute.
    // Four slots at a time, each chunk to every destination, so only four keys
    // are live in registers.
#pragma unroll
    for (int i = 0; i < K; i += 4) {
      const u64 k0 = top.at(i), k1 = top.at(i + 1), k2 = top.at(i + 2), k3 = top.at(i + 3);
      const longlong2 i01 = make_longlong2(key_idx(k0), key_idx(k1));
      const longlong2 i23 = make_longlong2(key_idx(k2), key_idx(k3));
      const float4 d4 = make_float4(key_dist(k0), key_dist(k1), key_dist(k2), key_dist(k3));
      if (a.dest_multimem) {
        multimem_store4(reinterpret_cast<int32_t*>(a.dest_idx[0]) + gq * K + i, __int_as_float(key_idx(k0)),
                        __int_as_float(key_idx(k1)), __int_as_float(key_idx(k2)), __int_as_float(key_idx(k3)));
        multimem_store4(a.dest_dist[0] + gq * K + i, d4.x, d4.y, d4.z, d4.w);
        continue;
      }
#pragma unroll 1
      for (int dst = 0; dst < a.num_dest; ++dst) {
        if (a.dest_idx32) {
          *reinterpret_cast<int4*>(reinterpret_cast<int32_t*>(a.dest_idx[dst]) + gq * K + i) =
              make_int4(key_idx(k0), key_idx(k1), key_idx(k2), key_idx(k3));
        } else {
          longlong2* oi = reinterpret_cast<longlong2*>(a.dest_idx[dst] + gq * K + i);
          oi[0] = i01;
          oi[1] = i23;
        }
        *reinterpret_cast<float4*>(a.dest_dist[dst] + gq * K + i) = d4;
      }
    }
  } else {
    // Output row: the query's own row, or its position in the sorted order
    // (the reference's spatial variant, knn_query.cu:448-461).
    const int64_t row = a.spatial ? pos : gq;
    write_row<K, kHeap>(top, a.out_idx + row * K, a.out_dist + row * K);
    if (a.out_pos) {
      // Fused source_points[indices] gather. An empty slot (index -1) reads the
      // cloud's last point, as PyTorch's negative indexing would.
      const float* src = a.src_points + pt_off * D;
      float* op = a.out_pos + row * K * D;
      // Register lists need constant slot indices (full unroll); heap slots are
      // shared-memory reads, so four at a time keep few loads in flight.
      constexpr int kGatherUnroll = kHeap ? 4 : K;
#pragma unroll kGatherUnroll
      for (int i = 0; i < K; ++i) {
        int64_t idx = key_idx(top.at(i));
        if (idx < 0) idx = n - 1;
#pragma unroll
        for (int c = 0; c < D; ++c) op[i * D + c] = __ldg(src + idx * D + c);
      }
    }
  }
}

template <int D, int K, bool kToDest>
__global__ void __launch_bounds__(kKnnThreads) k_knn(KnnArgs a) {
  extern __shared__ __align__(16) unsigned char knn_smem_raw[];
  KnnSmem<K>& s = *reinterpret_cast<KnnSmem<K>*>(knn_smem_raw);
  const unsigned lane = threadIdx.x & 31u;
  const unsigned warp = threadIdx.x >> 5;
  const int64_t pos = (int64_t(blockIdx.x) * kKnnWarps + warp) * 32 + lane;
  const bool valid = pos < a.total_q;
  const int cloud = valid ? a.qry.find(pos) : -1;
  unsigned pending = __ballot_sync(kFullMask, valid);
  while (pending) {
    const int leader = __ffs(pending) - 1;
    const int cur = __shfl_sync(kFullMask, cloud, leader);
    const bool mine = valid && cloud == cur;
    pending &= ~__ballot_sync(kFullMask, mine);
    search_cloud<D, K, kToDest>(a, s, cur, mine, pos, lane, warp);
    __syncwarp();
  }
  // Peer stores must be visible system-wide before the kernel counts as done:
  // the caller's next collective tells the other GPUs that their rows arrived.
  if constexpr (kToDest) __threadfence_system();
}

// Per-cloud table for ragged queries (n, leaf level, first node row).
__global__ void __launch_bounds__(256) k_knn_table(CloudMap pts, CloudTree* table) {
  __shared__ int64_t s_warp[8];
  int64_t carry = 0;
  for (int base = 0; base < pts.num_clouds; base += 256) {
    const int b = base + int(threadIdx.x);
    const bool valid = b < pts.num_clouds;
    const int64_t n = valid ? pts.size(b) : 0;
    const int64_t rows = n > 0 ? real_node_count(n) : 0;
    // Inclusive warp scan + block combine (same pattern as the build init).
    const unsigned lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    int64_t x = rows;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(kFullMask, x, o);
      if (lane >= unsigned(o)) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    int64_t before = 0, total = 0;
    for (int w = 0; w < 8; ++w) {
      if (w < int(warp)) before += s_warp[w];
      total += s_warp[w];
    }
    if (valid) {
      CloudTree t{};
      t.n = n;
      t.leaf_level = ceil_log2_i64(n);
      t.row_off = carry + before + x - rows;
      table[b] = t;
    }
    carry += total;
    __syncthreads();
  }
}

template <int D, int K, bool kToDest>
cudaError_t launch_variant(const KnnArgs& a, unsigned blocks, cudaStream_t stream) {
  constexpr size_t smem = sizeof(KnnSmem<K>);
  static_assert(smem <= 227 * 1024, "traversal shared memory exceeds the per-block limit");
  if constexpr (smem > 48 * 1024) {
    // Opt in to more than the default 48 KB of dynamic shared memory. The
    // attribute belongs to the device's context, so set it on every device once.
    static bool set_on[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !set_on[dev]) {
      const cudaError_t e =
          cudaFuncSetAttribute(k_knn<D, K, kToDest>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
      if (e != cudaSuccess) return e;
      if (dev >= 0 && dev < 64) set_on[dev] = true;
    }
  }
  k_knn<D, K, kToDest><<<blocks, kKnnThreads, smem, stream>>>(a);
  count_launches(1);
  return cudaGetLastError();
}

template <int D, int K>
cudaError_t launch_typed(const KnnArgs& a, cudaStream_t stream) {
  const int64_t warps = (a.total_q + 31) / 32;
  const int64_t blocks = (warps + kKnnWarps - 1) / kKnnWarps;
  if (blocks <= 0) return cudaSuccess;
  if (a.num_dest > 0) return launch_variant<D, K, true>(a, unsigned(blocks), stream);
  return launch_variant<D, K, false>(a, unsigned(blocks), stream);
}

}  // namespace

cudaError_t launch_knn(const KnnLaunch& q, cudaStream_t stream) {
  KnnArgs a{};
  a.node_aabbs = q.node_aabbs;
  a.sorted = q.sorted_indices;
  a.queries = q.queries;
  a.order = q.order;
  a.out_idx = q.out_idx;
  a.out_dist = q.out_dist;
  a.pts = q.points;
  a.qry = q.queries_map;
  a.uni = q.uniform;
  a.uni_rows = q.uniform_rows;
  a.total_q = q.total_queries;
  a.src_points = q.source_points;
  a.out_pos = q.out_positions;
  a.spatial = q.spatial ? 1 : 0;
  a.num_dest = q.num_dest;
  a.dest_idx32 = q.dest_idx32 ? 1 : 0;
  a.dest_multimem = q.dest_multimem ? 1 : 0;
  for (int i = 0; i < kMaxDest; ++i) {
    a.dest_idx[i] = q.dest_idx[i];
    a.dest_dist[i] = q.dest_dist[i];
  }
  a.status = device_status_ptr();
  if (q.points.uniform_n > 0) {
    a.table = nullptr;
  } else {
    k_knn_table<<<1, 256, 0, stream>>>(q.points, q.table_scratch);
    count_launches(1);
    a.table = q.table_scratch;
  }
  const int D = q.dim;
  switch (q.k) {
    case 4: return D == 3 ? launch_typed<3, 4>(a, stream) : launch_typed<2, 4>(a, stream);
    case 8: return D == 3 ? launch_typed<3, 8>(a, stream) : launch_typed<2, 8>(a, stream);
    case 16: return D == 3 ? launch_typed<3, 16>(a, stream) : launch_typed<2, 16>(a, stream);
    case 32: return D == 3 ? launch_typed<3, 32>(a, stream) : launch_typed<2, 32>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace tbvh
