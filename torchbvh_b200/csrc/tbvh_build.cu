// BVH build for the B200 k-NN path: per-cloud scene bounds, Morton keys with
// fused digit histograms, a stable onesweep LSD radix sort (8-bit digits,
// decoupled look-back with bounded waits) and the implicit-tree AABB build.
//
// Replaces, for the k-NN path, torchbvh/csrc/bvh_build.cu:453-721 (bounds,
// Morton keys, CUB segmented sort, lower/upper AABB build, traversal arrays)
// and torchbvh/csrc/morton_sort.cu:43-81,212-287 (query Morton permutation).
// Fixed-size batches and ragged batches share one launch sequence; the cloud
// id enters the sort as the most significant digits of a composite key, so
// every cloud is sorted independently and stably by (Morton code, index).
#include <atomic>
#include <cstdio>

#include "tbvh_kernels.h"

namespace tbvh {

// Per-device status word. Kernels OR error bits into it instead of hanging or
// trapping; the host reads it with tbvh_device_status().
__device__ unsigned g_tbvh_status;

namespace {

constexpr int kMaxDevices = 64;
unsigned* g_status_ptr[kMaxDevices] = {};

__device__ __forceinline__ unsigned lane_id() { return threadIdx.x & 31u; }

// Exclusive scan of one value per thread over a 256-thread block. `s_warp`
// needs 8 entries. Returns the exclusive prefix; `total` gets the block sum.
template <typename T>
__device__ __forceinline__ T block_exclusive_scan_256(T v, T* s_warp, T& total) {
  const unsigned lane = lane_id();
  const unsigned warp = threadIdx.x >> 5;
  T x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T y = __shfl_up_sync(kFullMask, x, o);
    if (lane >= unsigned(o)) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    T w = lane < 8 ? s_warp[lane] : T(0);
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      const T y = __shfl_up_sync(kFullMask, w, o);
      if (lane >= unsigned(o)) w += y;
    }
    if (lane < 8) s_warp[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  total = s_warp[7];
  const T before = warp == 0 ? T(0) : s_warp[warp - 1];
  const T result = before + x - v;
  __syncthreads();  // s_warp may be reused by the caller
  return result;
}

__device__ __forceinline__ uint32_t composite_digit(uint32_t key, uint32_t cloud, int code_bits, int lo_bit) {
  const uint64_t comp = (uint64_t(cloud) << code_bits) | uint64_t(key);
  return uint32_t(comp >> lo_bit) & 0xffu;
}

__device__ __forceinline__ void device_error(unsigned* status, unsigned bits) {
  if (status) atomicOr(status, bits);
}

// ---------------------------------------------------------------------------
// Per-cloud tree facts (device side of cloud_tree_facts()).
// ---------------------------------------------------------------------------
__host__ __device__ inline CloudTree tree_facts(int64_t n) {
  CloudTree t{};
  t.n = n;
  t.leaf_level = n > 0 ? ceil_log2_i64(n) : 0;
  t.sub_level = t.leaf_level > kTreeSubLevels ? t.leaf_level - kTreeSubLevels : 0;
  return t;
}

__host__ __device__ inline int64_t tree_blocks_of(const CloudTree& t) {
  return t.n > 0 ? level_count(t.n, t.leaf_level, t.sub_level) : 0;
}

__host__ __device__ inline int64_t tree_counters_of(const CloudTree& t) {
  int64_t total = 0;
  int lv = t.sub_level;
  while (lv > 0) {
    const int lam = lv > kTreeHopLevels ? lv - kTreeHopLevels : 0;
    total += level_count(t.n, t.leaf_level, lam);
    lv = lam;
  }
  return total;
}

// ---------------------------------------------------------------------------
// Init: zero scratch ranges, seed the bounds reduction and (ragged) compute
// the per-cloud table with a block scan in block 0.
// ---------------------------------------------------------------------------
struct ZeroRange {
  uint32_t* ptr;
  int64_t words;
};

struct InitArgs {
  ZeroRange zero[4];
  uint32_t* bounds_enc;  // nullable
  int bounds_words;      // num_clouds * 2D
  int dim;
  CloudMap clouds;
  CloudTree* table;      // nullable
};

__global__ void __launch_bounds__(256) k_init(InitArgs a) {
  const int64_t gtid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t gstride = int64_t(gridDim.x) * blockDim.x;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    uint32_t* p = a.zero[r].ptr;
    const int64_t words = a.zero[r].words;
    if (p == nullptr) continue;
    for (int64_t i = gtid; i < words; i += gstride) p[i] = 0u;
  }
  if (a.bounds_enc) {
    const uint32_t enc_lo = float_to_ordered(1.0e30f);
    const uint32_t enc_hi = float_to_ordered(-1.0e30f);
    for (int64_t i = gtid; i < a.bounds_words; i += gstride) {
      const int within = int(i % (2 * a.dim));
      a.bounds_enc[i] = within < a.dim ? enc_lo : enc_hi;
    }
  }
  if (a.table && blockIdx.x == 0) {
    __shared__ int64_t s_warp[8];
    int64_t carry_rows = 0, carry_blocks = 0, carry_ctr = 0;
    for (int base = 0; base < a.clouds.num_clouds; base += 256) {
      const int b = base + int(threadIdx.x);
      const bool valid = b < a.clouds.num_clouds;
      const int64_t n = valid ? a.clouds.size(b) : 0;
      CloudTree t = tree_facts(n);
      const int64_t rows = n > 0 ? real_node_count(n) : 0;
      const int64_t blocks = tree_blocks_of(t);
      const int64_t ctrs = n > 0 ? tree_counters_of(t) : 0;
      int64_t tot_rows, tot_blocks, tot_ctrs;
      const int64_t ex_rows = block_exclusive_scan_256<int64_t>(rows, s_warp, tot_rows);
      const int64_t ex_blocks = block_exclusive_scan_256<int64_t>(blocks, s_warp, tot_blocks);
      const int64_t ex_ctrs = block_exclusive_scan_256<int64_t>(ctrs, s_warp, tot_ctrs);
      if (valid) {
        t.row_off = carry_rows + ex_rows;
        t.tree_cta = carry_blocks + ex_blocks;
        t.counter = carry_ctr + ex_ctrs;
        a.table[b] = t;
      }
      carry_rows += tot_rows;
      carry_blocks += tot_blocks;
      carry_ctr += tot_ctrs;
    }
  }
}

// ---------------------------------------------------------------------------
// Scene bounds: every block reduces a contiguous chunk; per-thread running
// boxes are flushed on cloud changes, combined per warp and per block, then
// merged into the per-cloud result with order-preserving atomics. Seeds and
// min/max semantics follow torchbvh/csrc/bvh_build.cu:453-494.
// ---------------------------------------------------------------------------
template <int D>
__device__ __forceinline__ void flush_box(uint32_t* enc, int cloud, const float* lo, const float* hi) {
#pragma unroll
  for (int a = 0; a < D; ++a) {
    atomicMin(enc + cloud * 2 * D + a, float_to_ordered(lo[a]));
    atomicMax(enc + cloud * 2 * D + D + a, float_to_ordered(hi[a]));
  }
}

// Points 4·qd .. 4·qd + 3 that lie below `end`. A quad of 3-D points is 48
// contiguous bytes (three float4), of 2-D points 32 (two float4): when the
// array is 16-byte aligned and the quad whole, it arrives in 128-bit loads;
// otherwise point by point (points at or past `end` read as 0 and are unused).
template <int D>
__device__ __forceinline__ void load_quad(const float* __restrict__ pts, int64_t qd, int64_t end, bool vec,
                                          float (&p)[4][D]) {
  const int64_t i0 = qd * 4;
  if (vec && i0 + 4 <= end) {
    const float4* v = reinterpret_cast<const float4*>(pts + i0 * D);
    float f[4 * D];
#pragma unroll
    for (int j = 0; j < D; ++j) {
      const float4 x = __ldg(v + j);
      f[4 * j] = x.x;
      f[4 * j + 1] = x.y;
      f[4 * j + 2] = x.z;
      f[4 * j + 3] = x.w;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int a = 0; a < D; ++a) p[u][a] = f[u * D + a];
  } else {
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int a = 0; a < D; ++a) p[u][a] = i0 + u < end ? __ldg(pts + (i0 + u) * D + a) : 0.0f;
  }
}

// Quads of points each k_keys thread has in flight (loaded before any is used).
// Measured on B200 (build ms, c4 / c2 / c5): 1 quad 1.583 / 0.198 / 1.166,
// 2 quads 1.592 / 0.198 / 1.190 (64 registers), scalar loads 1.598 / 0.206 / 1.219.
#ifndef TBVH_KEYS_QUADS
#define TBVH_KEYS_QUADS 1
#endif

__device__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

template <int D>
__global__ void __launch_bounds__(256) k_bounds(const float* __restrict__ pts, CloudMap cm, int64_t n,
                                                int64_t chunk, uint32_t* __restrict__ enc) {
  __shared__ int s_cloud[8];
  __shared__ float s_box[8][2 * D];
  const int64_t begin = int64_t(blockIdx.x) * chunk;
  const int64_t end = begin + chunk < n ? begin + chunk : n;
  int cur = -1;
  int64_t cur_end = -1;
  float lo[D], hi[D];
#pragma unroll
  for (int a = 0; a < D; ++a) { lo[a] = 1.0e30f; hi[a] = -1.0e30f; }
  // The chunk starts on a multiple of 256 points, so its quads are whole
  // quads of the array; each thread takes every 256th quad.
  const bool vec = aligned16(pts);
  for (int64_t qd = begin / 4 + threadIdx.x; qd * 4 < end; qd += blockDim.x) {
    float p[4][D];
    load_quad<D>(pts, qd, end, vec, p);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t i = qd * 4 + u;
      if (i >= end) break;
      if (i >= cur_end) {
        const int c = cm.find(i);
        if (cur >= 0 && c != cur) {
          flush_box<D>(enc, cur, lo, hi);
#pragma unroll
          for (int a = 0; a < D; ++a) { lo[a] = 1.0e30f; hi[a] = -1.0e30f; }
        }
        cur = c;
        cur_end = cm.start(c) + cm.size(c);
      }
#pragma unroll
      for (int a = 0; a < D; ++a) {
        lo[a] = fminf(lo[a], p[u][a]);
        hi[a] = fmaxf(hi[a], p[u][a]);
      }
    }
  }
  const unsigned lane = lane_id();
  const unsigned warp = threadIdx.x >> 5;
  const int c0 = __shfl_sync(kFullMask, cur, 0);
  // Threads without elements (cur == -1) carry the neutral box.
  const bool uniform = __all_sync(kFullMask, cur == c0 || cur == -1);
  int wc = __reduce_max_sync(kFullMask, uniform ? (cur < 0 ? -1 : cur) : -1);
  if (uniform) {
#pragma unroll
    for (int a = 0; a < D; ++a) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        lo[a] = fminf(lo[a], __shfl_xor_sync(kFullMask, lo[a], o));
        hi[a] = fmaxf(hi[a], __shfl_xor_sync(kFullMask, hi[a], o));
      }
    }
    if (lane == 0) {
      s_cloud[warp] = wc;
#pragma unroll
      for (int a = 0; a < D; ++a) { s_box[warp][a] = lo[a]; s_box[warp][D + a] = hi[a]; }
    }
  } else {
    if (cur >= 0) flush_box<D>(enc, cur, lo, hi);
    if (lane == 0) s_cloud[warp] = -1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc_cloud = -1;
    float alo[D], ahi[D];
    for (int w = 0; w < 8; ++w) {
      const int c = s_cloud[w];
      if (c < 0) continue;
      if (c != acc_cloud) {
        if (acc_cloud >= 0) flush_box<D>(enc, acc_cloud, alo, ahi);
        acc_cloud = c;
#pragma unroll
        for (int a = 0; a < D; ++a) { alo[a] = s_box[w][a]; ahi[a] = s_box[w][D + a]; }
      } else {
#pragma unroll
        for (int a = 0; a < D; ++a) {
          alo[a] = fminf(alo[a], s_box[w][a]);
          ahi[a] = fmaxf(ahi[a], s_box[w][D + a]);
        }
      }
    }
    if (acc_cloud >= 0) flush_box<D>(enc, acc_cloud, alo, ahi);
  }
}

// Scene box of one cloud from its order-preserving encoding (standalone bounds).
__global__ void k_bounds_decode(const uint32_t* __restrict__ enc, int dim, float* __restrict__ smin,
                                float* __restrict__ smax) {
  const int a = int(threadIdx.x);
  if (a < dim) {
    smin[a] = ordered_to_float(enc[a]);
    smax[a] = ordered_to_float(enc[dim + a]);
  }
}

// ---------------------------------------------------------------------------
// Morton keys + digit histograms for every sort pass (one read of the
// coordinates). Each lane counts its digits into the block's shared
// histograms (a digit the whole warp shares is counted once by one lane),
// which are then added to the global per-pass histograms.
// ---------------------------------------------------------------------------
template <int D, bool kEncodedBounds>
__global__ void __launch_bounds__(256) k_keys(const float* __restrict__ pts, CloudMap cm, int64_t n,
                                              const uint32_t* __restrict__ enc,
                                              const float* __restrict__ smin, const float* __restrict__ smax,
                                              uint32_t* __restrict__ keys, uint32_t* __restrict__ hist,
                                              int code_bits, int passes,
                                              float* __restrict__ out_min, float* __restrict__ out_max) {
  __shared__ uint32_t s_hist[kMaxSortPasses][kRadix];
  for (int i = threadIdx.x; i < kMaxSortPasses * kRadix; i += blockDim.x) (&s_hist[0][0])[i] = 0u;
  if (kEncodedBounds && blockIdx.x == 0) {
    const int words = cm.num_clouds * D;
    for (int i = threadIdx.x; i < words; i += blockDim.x) {
      const int b = i / D, a = i % D;
      out_min[i] = ordered_to_float(enc[b * 2 * D + a]);
      out_max[i] = ordered_to_float(enc[b * 2 * D + D + a]);
    }
  }
  __syncthreads();
  const unsigned lane = lane_id();
  // Each thread takes whole quads of 4 consecutive points (128-bit loads of
  // the coordinates, one 128-bit store of the 4 keys), two quads in flight.
  const int64_t nq = (n + 3) / 4;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const int64_t rounds = (nq + stride - 1) / stride;
  const bool vec = aligned16(pts);
  const bool vec_keys = aligned16(keys);
  int cur = -1;
  int64_t cur_end = -1;
  float lo[D], hi[D];
  constexpr int kGroup = TBVH_KEYS_QUADS;
  for (int64_t r0 = 0; r0 < rounds; r0 += kGroup) {
    float pg[kGroup][4][D];
#pragma unroll
    for (int u = 0; u < kGroup; ++u) {
      const int64_t qd = (r0 + u) * stride + int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
      if (r0 + u < rounds && qd < nq) load_quad<D>(pts, qd, n, vec, pg[u]);
    }
#pragma unroll
    for (int u = 0; u < kGroup; ++u) {
      if (r0 + u >= rounds) break;  // uniform across the grid
      const int64_t qd = (r0 + u) * stride + int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
      uint32_t code4[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const int64_t i = qd * 4 + v;
        const bool valid = qd < nq && i < n;
        uint32_t code = 0;
        int c = 0;
        if (valid) {
          if (i >= cur_end || cur < 0) {
            cur = cm.find(i);
            cur_end = cm.start(cur) + cm.size(cur);
#pragma unroll
            for (int a = 0; a < D; ++a) {
              if (kEncodedBounds) {
                lo[a] = ordered_to_float(enc[cur * 2 * D + a]);
                hi[a] = ordered_to_float(enc[cur * 2 * D + D + a]);
              } else {
                lo[a] = smin[cur * D + a];
                hi[a] = smax[cur * D + a];
              }
            }
          }
          c = cur;
          code = morton_code<D>(pg[u][v], lo, hi);
          code4[v] = code;
        }
        // Digits of Morton codes in input order are mostly distinct within a warp,
        // so each lane adds its own count. A digit that holds cloud-id bits is
        // often the same for the whole warp: it is added once, by one lane, to
        // avoid a 32-way conflict on one bin (passes of code bits only skip the test).
        for (int ps = 0; ps < passes; ++ps) {
          const uint32_t d = valid ? composite_digit(code, uint32_t(c), code_bits, 8 * ps) : 0x100u;
          if (8 * ps + 8 <= code_bits || cm.num_clouds == 1) {  // uniform across the grid
            if (d < 0x100u) atomicAdd(&s_hist[ps][d], 1u);
            continue;
          }
          const uint32_t d0 = __shfl_sync(kFullMask, d, 0);
          if (__all_sync(kFullMask, d == d0)) {
            if (lane == 0 && d0 < 0x100u) atomicAdd(&s_hist[ps][d0], 32u);
          } else if (d < 0x100u) {
            atomicAdd(&s_hist[ps][d], 1u);
          }
        }
      }
      if (qd < nq) {
        if (vec_keys && qd * 4 + 4 <= n) {
          reinterpret_cast<uint4*>(keys)[qd] = make_uint4(code4[0], code4[1], code4[2], code4[3]);
        } else {
#pragma unroll
          for (int v = 0; v < 4; ++v)
            if (qd * 4 + v < n) keys[qd * 4 + v] = code4[v];
        }
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < passes * kRadix; i += blockDim.x) {
    const uint32_t v = (&s_hist[0][0])[i];
    if (v) atomicAdd(hist + i, v);
  }
}

// ---------------------------------------------------------------------------
// One stable LSD pass over composite-key bits [lo_bit, lo_bit + 8).
//
// Tiles are claimed in launch order through an atomic ticket, so a tile only
// ever waits on tiles owned by blocks that are already running: the look-back
// makes progress without co-residency assumptions. Every wait is bounded; on
// expiry the kernel records kDevErrLookbackTimeout and carries on.
// ---------------------------------------------------------------------------
constexpr uint64_t kLbAggregate = 1ull << 62;
constexpr uint64_t kLbPrefix = 2ull << 62;
constexpr uint64_t kLbFlags = 3ull << 62;
constexpr int kLbSpinLimit = 1 << 22;

struct PassArgs {
  const uint32_t* keys_in;
  const uint32_t* vals_in;  // nullptr: value = element index
  uint32_t* keys_out;
  uint32_t* vals_out;
  int64_t* final_out;       // last pass: local (in-cloud) index as int64
  const uint32_t* hist;     // 256 counts for this pass
  uint64_t* lookback;       // this pass: tiles x 256
  uint64_t* lookback_next;  // next pass: tiles x 256 (cleared here), nullable
  uint32_t* tile_ctr;
  int64_t n;
  int lo_bit;
  int code_bits;
  int needs_cloud;
  CloudMap cm;
  unsigned* status;
  int spin_limit;           // polls of one look-back wait before it gives up
};

struct PassSmem {
  uint32_t keys[kSortTile];
  uint32_t vals[kSortTile];
  uint8_t dig[kSortTile];
  uint16_t whist[kSortThreads / 32][kRadix];
  uint32_t local_start[kRadix];
  int64_t gbase[kRadix];
  uint32_t scan_warp[8];
  int64_t scan_warp64[8];
  uint32_t tile;
};

__global__ void __launch_bounds__(kSortThreads) k_sort_pass(PassArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  PassSmem& s = *reinterpret_cast<PassSmem*>(smem_raw);
  const int tid = threadIdx.x;
  const unsigned lane = lane_id();
  const unsigned warp = threadIdx.x >> 5;
  const unsigned lt_mask = (1u << lane) - 1u;

  if (tid == 0) s.tile = atomicAdd(a.tile_ctr, 1u);
  for (int i = tid; i < (kSortThreads / 32) * kRadix; i += kSortThreads) (&s.whist[0][0])[i] = 0;
  // Global exclusive bin bases for this pass.
  uint32_t total_unused;
  const uint32_t bin_base = block_exclusive_scan_256<uint32_t>(a.hist[tid], s.scan_warp, total_unused);
  // (block_exclusive_scan_256 ends with __syncthreads, so s.tile / s.whist are visible.)
  const int64_t tile = s.tile;
  const int64_t tile_start = tile * kSortTile;
  const int tile_n = int(a.n - tile_start < kSortTile ? a.n - tile_start : kSortTile);
  if (a.lookback_next) a.lookback_next[tile * kRadix + tid] = 0ull;

  uint32_t key[kSortIpt], val[kSortIpt], packed[kSortIpt];  // packed = rank << 9 | digit
#pragma unroll
  for (int r = 0; r < kSortIpt; ++r) {
    const int idx = int(warp) * 32 * kSortIpt + r * 32 + int(lane);
    const bool valid = idx < tile_n;
    const int64_t e = tile_start + idx;
    key[r] = valid ? a.keys_in[e] : 0u;
    val[r] = valid ? (a.vals_in ? a.vals_in[e] : uint32_t(e)) : 0u;
  }
#pragma unroll
  for (int r = 0; r < kSortIpt; ++r) {
    const int idx = int(warp) * 32 * kSortIpt + r * 32 + int(lane);
    const bool valid = idx < tile_n;
    uint32_t d = 0x100u;
    if (valid) {
      const uint32_t cloud = a.needs_cloud ? uint32_t(a.cm.find(int64_t(val[r]))) : 0u;
      d = composite_digit(key[r], cloud, a.code_bits, a.lo_bit);
    }
    const unsigned peers = __match_any_sync(kFullMask, d);
    const int leader = __ffs(peers) - 1;
    uint32_t base = 0;
    if (int(lane) == leader && d < 0x100u) {
      base = s.whist[warp][d];
      s.whist[warp][d] = uint16_t(base + __popc(peers));
    }
    base = __shfl_sync(kFullMask, base, leader);
    packed[r] = ((base + __popc(peers & lt_mask)) << 9) | d;
    __syncwarp();
  }
  __syncthreads();

  // Per-digit: exclusive prefix over warps, tile count.
  const int d = tid;
  uint32_t run = 0;
#pragma unroll
  for (int w = 0; w < kSortThreads / 32; ++w) {
    const uint32_t c = s.whist[w][d];
    s.whist[w][d] = uint16_t(run);
    run += c;
  }
  const uint32_t tile_cnt = run;
  volatile uint64_t* lb = reinterpret_cast<volatile uint64_t*>(a.lookback);
  if (tile == 0) {
    lb[d] = kLbPrefix | uint64_t(tile_cnt);
  } else {
    lb[tile * kRadix + d] = kLbAggregate | uint64_t(tile_cnt);
  }
  int64_t excl = 0;
  if (tile > 0) {
    int64_t t = tile - 1;
    int spins = 0;
    while (t >= 0) {
      const uint64_t v = lb[t * kRadix + d];
      const uint64_t flag = v & kLbFlags;
      if (flag == 0) {
        if (++spins > a.spin_limit) {
          device_error(a.status, kDevErrLookbackTimeout);
          break;
        }
        if (spins > 64) __nanosleep(32);
        continue;
      }
      excl += int64_t(v & 0xffffffffull);
      if (flag == kLbPrefix) break;
      --t;
    }
    lb[tile * kRadix + d] = kLbPrefix | uint64_t(excl + tile_cnt);
  }
  uint32_t tile_total;
  const uint32_t local_start = block_exclusive_scan_256<uint32_t>(tile_cnt, s.scan_warp, tile_total);
  s.local_start[d] = local_start;
  s.gbase[d] = int64_t(bin_base) + excl - int64_t(local_start);
  __syncthreads();

  // Scatter into shared memory in digit order (stable within each digit).
#pragma unroll
  for (int r = 0; r < kSortIpt; ++r) {
    const uint32_t dg = packed[r] & 0x1ffu;
    if (dg < 0x100u) {
      const uint32_t lp = s.local_start[dg] + s.whist[warp][dg] + (packed[r] >> 9);
      s.keys[lp] = key[r];
      s.vals[lp] = val[r];
      s.dig[lp] = uint8_t(dg);
    }
  }
  __syncthreads();

  // Write out: consecutive shared slots of one digit land on consecutive
  // global positions, so the stores coalesce into runs.
  // The range checks only matter if an earlier pass gave up a bounded wait
  // (status bit set): they keep a corrupted permutation from writing out of bounds.
  if (a.final_out) {
    for (int i = tid; i < tile_n; i += kSortThreads) {
      const int64_t g = s.gbase[s.dig[i]] + i;
      const uint32_t v = s.vals[i];
      const int c = a.cm.find(int64_t(v));
      if (g >= 0 && g < a.n) a.final_out[g] = int64_t(v) - a.cm.start(c);
    }
  } else {
    for (int i = tid; i < tile_n; i += kSortThreads) {
      const int64_t g = s.gbase[s.dig[i]] + i;
      if (g >= 0 && g < a.n) {
        a.keys_out[g] = s.keys[i];
        a.vals_out[g] = s.vals[i];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Implicit-tree AABB build.
//
// Block (cloud, js) owns the subtree rooted at level Ls = max(L - 10, 0),
// index js: it gathers its <= 1024 sorted points, writes the leaf rows and
// merges upward (4 leaves per thread, then warp shuffles, then across warps),
// writing every real node row. Upper levels are merged in hops of 8 levels:
// the last block to finish inside a hop group (atomic ticket after a
// __threadfence) merges that group, exactly once. Node rows are written in
// the reference's memory order (level-major over real nodes) together with
// left_child_mem / right_child_mem / mem_to_leaf (bvh_build.cu:361-398).
// ---------------------------------------------------------------------------
struct TreeArgs {
  const float* points;
  const int64_t* sorted;
  float* node_aabbs;
  int32_t* left;
  int32_t* right;
  int32_t* m2l;
  int arrays_per_cloud;
  CloudMap cm;
  const CloudTree* table;  // ragged
  CloudTree uni;           // uniform clouds
  int64_t uni_blocks;      // blocks per uniform cloud
  int64_t uni_rows;        // rows per uniform cloud
  int64_t uni_counters;    // counters per uniform cloud
  uint32_t* counters;
  unsigned* status;
};

template <int D>
struct TreeCtx {
  const TreeArgs* a;
  const int64_t* cnt;     // shared, per level
  const int64_t* rowoff;  // shared, per level
  float* rows;            // cloud's first row
  int32_t* left;          // nullable, cloud's first entry
  int32_t* right;
  int32_t* m2l;
  int L;

  __device__ __forceinline__ void emit(int level, int64_t j, const float* lo, const float* hi) const {
    const int64_t row = rowoff[level] + j;
    float* r = rows + row * (2 * D);
    if constexpr (D == 3) {
      reinterpret_cast<float2*>(r)[0] = make_float2(lo[0], lo[1]);
      reinterpret_cast<float2*>(r)[1] = make_float2(lo[2], hi[0]);
      reinterpret_cast<float2*>(r)[2] = make_float2(hi[1], hi[2]);
    } else {
      reinterpret_cast<float4*>(r)[0] = make_float4(lo[0], lo[1], hi[0], hi[1]);
    }
    if (left) {
      if (level == L) {
        left[row] = -1;
        right[row] = -1;
        m2l[row] = int32_t(j);
      } else {
        const int64_t c0 = 2 * j;
        left[row] = int32_t(rowoff[level + 1] + c0);
        right[row] = c0 + 1 < cnt[level + 1] ? int32_t(rowoff[level + 1] + c0 + 1) : -1;
        m2l[row] = -1;
      }
    }
  }
};

template <int D>
__device__ __forceinline__ void merge_box(float* lo, float* hi, const float* olo, const float* ohi) {
#pragma unroll
  for (int a = 0; a < D; ++a) { lo[a] = fminf(lo[a], olo[a]); hi[a] = fmaxf(hi[a], ohi[a]); }
}

template <int D>
__device__ __forceinline__ void shfl_merge(float* lo, float* hi, int offset) {
#pragma unroll
  for (int a = 0; a < D; ++a) {
    lo[a] = fminf(lo[a], __shfl_down_sync(kFullMask, lo[a], offset));
    hi[a] = fmaxf(hi[a], __shfl_down_sync(kFullMask, hi[a], offset));
  }
}

template <int D>
__device__ __forceinline__ void load_row_cg(const float* rows, int64_t row, float* lo, float* hi) {
  const float* r = rows + row * (2 * D);
#pragma unroll
  for (int a = 0; a < D; ++a) { lo[a] = __ldcg(r + a); hi[a] = __ldcg(r + D + a); }
}

template <int D>
__global__ void __launch_bounds__(kTreeThreads) k_tree(TreeArgs a) {
  __shared__ int64_t s_cnt[34];
  __shared__ int64_t s_rowoff[34];
  __shared__ float s_wbox[kTreeThreads / 32][2 * D];
  __shared__ CloudTree s_t;
  __shared__ int64_t s_js;
  __shared__ int64_t s_ptoff;
  __shared__ int s_cloud;
  __shared__ int s_last;

  const int tid = threadIdx.x;
  const unsigned lane = lane_id();
  const unsigned warp = threadIdx.x >> 5;
  if (tid == 0) {
    int b;
    CloudTree t;
    int64_t js;
    if (a.table == nullptr) {
      b = int(int64_t(blockIdx.x) / a.uni_blocks);
      js = int64_t(blockIdx.x) - int64_t(b) * a.uni_blocks;
      t = a.uni;
      t.row_off = int64_t(b) * a.uni_rows;
      t.counter = int64_t(b) * a.uni_counters;
    } else {
      int lo = 0, hi = a.cm.num_clouds - 1;
      while (lo < hi) {  // last cloud whose first block <= blockIdx.x (skipping empty tail)
        const int mid = (lo + hi + 1) >> 1;
        if (a.table[mid].tree_cta <= int64_t(blockIdx.x)) lo = mid; else hi = mid - 1;
      }
      // Clouds own >= 1 block each (n >= 1), so `lo` is the owner.
      b = lo;
      t = a.table[b];
      js = int64_t(blockIdx.x) - t.tree_cta;
    }
    s_t = t;
    s_js = js;
    s_cloud = b;
    s_ptoff = a.cm.start(b);
  }
  __syncthreads();
  const CloudTree t = s_t;
  const int L = t.leaf_level;
  const int Ls = t.sub_level;
  const int64_t n = t.n;
  const int64_t js = s_js;
  const int64_t pt_off = s_ptoff;
  if (tid <= L) s_cnt[tid] = level_count(n, L, tid);
  __syncthreads();
  if (tid == 0) {
    int64_t acc = 0;
    for (int l = 0; l <= L; ++l) { s_rowoff[l] = acc; acc += s_cnt[l]; }
    s_rowoff[L + 1] = acc;
  }
  __syncthreads();

  TreeCtx<D> ctx;
  ctx.a = &a;
  ctx.cnt = s_cnt;
  ctx.rowoff = s_rowoff;
  ctx.rows = a.node_aabbs + t.row_off * (2 * D);
  ctx.L = L;
  const bool write_arrays = a.left != nullptr && (a.arrays_per_cloud || s_cloud == 0);
  const int64_t arr_base = a.arrays_per_cloud ? t.row_off : 0;
  ctx.left = write_arrays ? a.left + arr_base : nullptr;
  ctx.right = write_arrays ? a.right + arr_base : nullptr;
  ctx.m2l = write_arrays ? a.m2l + arr_base : nullptr;

  const int span = L - Ls;  // levels inside this block's subtree (<= 10)
  const int64_t base = js << span;
  const int64_t block_end = base + (int64_t(1) << span);
  const int64_t limit = block_end < n ? block_end : n;
  auto present = [&](int level, int64_t j) { return (j << (L - level)) < limit; };

  // Leaves: 4 consecutive sorted positions per thread. All four indices are
  // read, then all four points gathered, and only then are rows stored: the
  // stores could alias the points as far as the compiler knows, so mixing them
  // would serialise four round trips to DRAM per thread.
  float lo4[4][D], hi4[4][D];
  int64_t src4[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int64_t pos = base + 4 * tid + q;
    src4[q] = pos < limit ? __ldg(a.sorted + pt_off + pos) : -1;
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int64_t pos = base + 4 * tid + q;
    if (pos < limit) {
      int64_t src = src4[q];
      if (src < 0 || src >= n) {  // only reachable if the sort was corrupted; keep the read in bounds
        device_error(a.status, kDevErrBadIndex);
        src = 0;
      }
#pragma unroll
      for (int c = 0; c < D; ++c) {
        const float v = __ldg(a.points + (pt_off + src) * D + c);
        lo4[q][c] = v;
        hi4[q][c] = v;
      }
    } else {
#pragma unroll
      for (int c = 0; c < D; ++c) { lo4[q][c] = INFINITY; hi4[q][c] = -INFINITY; }
    }
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int64_t pos = base + 4 * tid + q;
    if (pos < limit) ctx.emit(L, pos, lo4[q], hi4[q]);
  }
  // Level L-1: two nodes per thread.
  float lo[D], hi[D];
  float lo2[2][D], hi2[2][D];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int c = 0; c < D; ++c) { lo2[h][c] = lo4[2 * h][c]; hi2[h][c] = hi4[2 * h][c]; }
    merge_box<D>(lo2[h], hi2[h], lo4[2 * h + 1], hi4[2 * h + 1]);
    if (L - 1 >= Ls) {
      const int64_t j = (base >> 1) + 2 * tid + h;
      if (present(L - 1, j)) ctx.emit(L - 1, j, lo2[h], hi2[h]);
    }
  }
  // Level L-2: one node per thread.
#pragma unroll
  for (int c = 0; c < D; ++c) { lo[c] = lo2[0][c]; hi[c] = hi2[0][c]; }
  merge_box<D>(lo, hi, lo2[1], hi2[1]);
  if (L - 2 >= Ls) {
    const int64_t j = (base >> 2) + tid;
    if (present(L - 2, j)) ctx.emit(L - 2, j, lo, hi);
  }
  // Levels L-3 .. L-7 inside the warp.
#pragma unroll
  for (int s = 1; s <= 5; ++s) {
    shfl_merge<D>(lo, hi, 1 << (s - 1));
    const int level = L - 2 - s;
    if (level >= Ls && (lane & ((1u << s) - 1u)) == 0u) {
      const int64_t j = (base >> (2 + s)) + (tid >> s);
      if (present(level, j)) ctx.emit(level, j, lo, hi);
    }
  }
  // Levels L-8 .. L-10 across the 8 warps.
  if (lane == 0) {
#pragma unroll
    for (int c = 0; c < D; ++c) { s_wbox[warp][c] = lo[c]; s_wbox[warp][D + c] = hi[c]; }
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int c = 0; c < D; ++c) {
      lo[c] = lane < 8 ? s_wbox[lane][c] : INFINITY;
      hi[c] = lane < 8 ? s_wbox[lane][D + c] : -INFINITY;
    }
#pragma unroll
    for (int s = 1; s <= 3; ++s) {
      shfl_merge<D>(lo, hi, 1 << (s - 1));
      const int level = L - 7 - s;
      if (level >= Ls && (lane & ((1u << s) - 1u)) == 0u) {
        const int64_t j = (base >> (7 + s)) + (lane >> s);
        if (present(level, j)) ctx.emit(level, j, lo, hi);
      }
    }
  }
  if (Ls == 0) return;

  // Upper levels: hop groups of 8 levels; last arriver merges the group.
  int lv = Ls;
  int64_t j = js;
  int64_t hop_base = 0;
  while (lv > 0) {
    const int lam = lv > kTreeHopLevels ? lv - kTreeHopLevels : 0;
    const int delta = lv - lam;
    const int64_t g = j >> delta;
    const int64_t first = g << delta;
    const int64_t group_end = (g + 1) << delta;
    const int64_t arrivals = (group_end < s_cnt[lv] ? group_end : s_cnt[lv]) - first;
    // The barrier orders every thread's row writes before thread 0's fence; the
    // fence is cumulative, so one thread publishes the whole block's rows
    // device-wide before taking the ticket (and, as the last arriver, orders
    // the other blocks' rows before the merge below reads them).
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      const uint32_t old = atomicAdd(a.counters + t.counter + hop_base + g, 1u);
      if (int64_t(old) >= arrivals) device_error(a.status, kDevErrTreeCounter);
      s_last = int64_t(old) == arrivals - 1 ? 1 : 0;
      __threadfence();
    }
    __syncthreads();
    if (!s_last) return;
    for (int m = lv - 1; m >= lam; --m) {
      const int64_t width = int64_t(1) << (m - lam);
      const int64_t jm = (g << (m - lam)) + tid;
      if (tid < width && jm < s_cnt[m]) {
        float clo[D], chi[D];
        load_row_cg<D>(ctx.rows, s_rowoff[m + 1] + 2 * jm, clo, chi);
        if (2 * jm + 1 < s_cnt[m + 1]) {
          float rlo[D], rhi[D];
          load_row_cg<D>(ctx.rows, s_rowoff[m + 1] + 2 * jm + 1, rlo, rhi);
          merge_box<D>(clo, chi, rlo, rhi);
        }
        ctx.emit(m, jm, clo, chi);
      }
      __syncthreads();  // the next level reads these rows (same block)
    }
    hop_base += s_cnt[lam];
    lv = lam;
    j = g;
  }
}

// ---------------------------------------------------------------------------
// Traversal arrays of the implicit layout of one cloud (left/right child row,
// leaf position), the values TreeCtx::emit writes. They depend only on the
// point count, so a build may leave them out and a caller compute them when
// they are first read.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_traversal_arrays(int64_t n, int L, int64_t rows, int32_t* left,
                                                           int32_t* right, int32_t* m2l) {
  __shared__ int64_t s_rowoff[34];
  __shared__ int64_t s_cnt[34];
  if (threadIdx.x <= unsigned(L)) s_cnt[threadIdx.x] = level_count(n, L, int(threadIdx.x));
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t acc = 0;
    for (int l = 0; l <= L; ++l) { s_rowoff[l] = acc; acc += s_cnt[l]; }
    s_rowoff[L + 1] = acc;
  }
  __syncthreads();
  for (int64_t row = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; row < rows;
       row += int64_t(gridDim.x) * blockDim.x) {
    int level = 0;
    while (level < L && s_rowoff[level + 1] <= row) ++level;
    const int64_t j = row - s_rowoff[level];
    if (level == L) {
      left[row] = -1;
      right[row] = -1;
      m2l[row] = int32_t(j);
    } else {
      const int64_t c0 = 2 * j;
      left[row] = int32_t(s_rowoff[level + 1] + c0);
      right[row] = c0 + 1 < s_cnt[level + 1] ? int32_t(s_rowoff[level + 1] + c0 + 1) : -1;
      m2l[row] = -1;
    }
  }
}

// Self-test set-up: a key pattern and a ticket counter that starts at 1, so
// no block of the following pass ever claims tile 0.
__global__ void __launch_bounds__(256) k_selftest_prepare(uint32_t* keys, int64_t n, uint32_t* tile_ctr) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    keys[i] = uint32_t(i) * 2654435761u;
  if (blockIdx.x == 0 && threadIdx.x == 0) *tile_ctr = 1u;
}

// ---------------------------------------------------------------------------
// One rank's share of the queries of one cloud (sharded single-cloud k-NN).
//
// The Morton-code range is cut at the granularity of its top kShareBits bits
// ("cells"): a histogram of the cells, then an ownership table that walks the
// cells in code order and hands consecutive runs of about `chunk` queries to
// the ranks in turn (one run per rank when chunk = M / world: contiguous
// Morton ranges; smaller chunks interleave the ranks over the whole cloud so
// that each rank sees every kind of region). Each rank then compacts only its
// own queries and sorts them by Morton code, instead of sorting all M. Every
// rank computes the same histogram and table, so no exchange is needed.
// ---------------------------------------------------------------------------
constexpr int kShareBits = 15;
constexpr int kShareCells = 1 << kShareBits;
constexpr int kShareThreads = 1024;

template <int D>
__global__ void __launch_bounds__(kShareThreads) k_share_cells(const float* __restrict__ q, int64_t m,
                                                               const float* __restrict__ smin,
                                                               const float* __restrict__ smax,
                                                               uint32_t* __restrict__ codes,
                                                               uint32_t* __restrict__ cell_count) {
  extern __shared__ uint32_t s_cells[];  // kShareCells counters
  for (int i = threadIdx.x; i < kShareCells; i += blockDim.x) s_cells[i] = 0u;
  float lo[D], hi[D];
#pragma unroll
  for (int a = 0; a < D; ++a) { lo[a] = smin[a]; hi[a] = smax[a]; }
  __syncthreads();
  constexpr int shift = morton_bits<D>() - kShareBits;
  // Whole quads of 4 consecutive queries per thread (128-bit loads and stores).
  const bool vec = aligned16(q), vec_codes = aligned16(codes);
  const int64_t nq = (m + 3) / 4;
  for (int64_t qd = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; qd < nq; qd += int64_t(gridDim.x) * blockDim.x) {
    float p[4][D];
    load_quad<D>(q, qd, m, vec, p);
    uint32_t code4[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      if (qd * 4 + v < m) {
        code4[v] = morton_code<D>(p[v], lo, hi);
        atomicAdd(&s_cells[code4[v] >> shift], 1u);
      }
    }
    if (vec_codes && qd * 4 + 4 <= m) {
      reinterpret_cast<uint4*>(codes)[qd] = make_uint4(code4[0], code4[1], code4[2], code4[3]);
    } else {
#pragma unroll
      for (int v = 0; v < 4; ++v)
        if (qd * 4 + v < m) codes[qd * 4 + v] = code4[v];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kShareCells; i += blockDim.x) {
    const uint32_t v = s_cells[i];
    if (v) atomicAdd(cell_count + i, v);
  }
}

// One block: exclusive scan of the cell counts in code order, owner of each
// cell = (queries before it / chunk) mod world, per-rank totals.
__global__ void __launch_bounds__(kShareThreads) k_share_owners(const uint32_t* __restrict__ cell_count,
                                                                int64_t chunk, int world,
                                                                uint8_t* __restrict__ owner,
                                                                int64_t* __restrict__ rank_count) {
  constexpr int per = kShareCells / kShareThreads;
  __shared__ int64_t s_warp[kShareThreads / 32];
  int64_t local[per];
  int64_t sum = 0;
#pragma unroll
  for (int j = 0; j < per; ++j) {
    local[j] = cell_count[threadIdx.x * per + j];
    sum += local[j];
  }
  // Block-wide exclusive scan of the per-thread sums.
  const unsigned lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  int64_t x = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t y = __shfl_up_sync(kFullMask, x, o);
    if (lane >= unsigned(o)) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int64_t w = s_warp[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(kFullMask, w, o);
      if (lane >= unsigned(o)) w += y;
    }
    s_warp[lane] = w;
  }
  __syncthreads();
  int64_t before = (warp == 0 ? 0 : s_warp[warp - 1]) + x - sum;
#pragma unroll
  for (int j = 0; j < per; ++j) {
    const int r = int((before / chunk) % world);
    owner[threadIdx.x * per + j] = uint8_t(r);
    if (local[j]) atomicAdd(reinterpret_cast<unsigned long long*>(rank_count + r),
                            static_cast<unsigned long long>(local[j]));
    before += local[j];
  }
}

// Appends this rank's queries (code, index) and accumulates the digit
// histograms of every sort pass over them. Warp-aggregated appends: the order
// among appended queries is arbitrary, which only decides the order of equal
// codes after the sort (each query's result does not depend on it).
template <int D>
__global__ void __launch_bounds__(256) k_share_compact(const uint32_t* __restrict__ codes, int64_t m,
                                                       const uint8_t* __restrict__ owner, int rank,
                                                       uint32_t* __restrict__ out_keys,
                                                       uint32_t* __restrict__ out_vals,
                                                       unsigned long long* __restrict__ counter,
                                                       uint32_t* __restrict__ hist, int passes,
                                                       int64_t capacity, unsigned* status) {
  __shared__ uint32_t s_hist[kMaxSortPasses][kRadix];
  for (int i = threadIdx.x; i < kMaxSortPasses * kRadix; i += blockDim.x) (&s_hist[0][0])[i] = 0u;
  __syncthreads();
  constexpr int shift = morton_bits<D>() - kShareBits;
  const unsigned lane = threadIdx.x & 31u;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const int64_t rounds = (m + stride - 1) / stride;
  for (int64_t r = 0; r < rounds; ++r) {
    const int64_t i = r * stride + int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    uint32_t code = 0;
    bool mine = false;
    if (i < m) {
      code = codes[i];
      mine = owner[code >> shift] == rank;
    }
    const unsigned take = __ballot_sync(kFullMask, mine);
    unsigned long long base = 0;
    if (lane == 0 && take) base = atomicAdd(counter, static_cast<unsigned long long>(__popc(take)));
    base = __shfl_sync(kFullMask, base, 0);
    if (mine) {
      const int64_t pos = int64_t(base) + __popc(take & ((1u << lane) - 1u));
      if (pos < capacity) {
        out_keys[pos] = code;
        out_vals[pos] = uint32_t(i);
        for (int ps = 0; ps < passes; ++ps) atomicAdd(&s_hist[ps][(code >> (8 * ps)) & 0xffu], 1u);
      } else {
        device_error(status, kDevErrBadIndex);
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < passes * kRadix; i += blockDim.x) {
    const uint32_t v = (&s_hist[0][0])[i];
    if (v) atomicAdd(hist + i, v);
  }
}

}  // namespace

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
constexpr int64_t kSelfTestElements = 4 * int64_t(kSortTile);

size_t selftest_scratch_bytes() { return sort_scratch_bytes(make_sort_plan(kSelfTestElements, 1, 3)); }

cudaError_t launch_lookback_selftest(void* scratch, int spin_limit, cudaStream_t stream) {
  const SortPlan p = make_sort_plan(kSelfTestElements, 1, 3);
  char* cur = static_cast<char*>(scratch);
  SortScratch ss;
  carve_sort_scratch(p, cur, ss);
  InitArgs ia{};
  ia.zero[0] = {ss.hist, int64_t(kMaxSortPasses) * kRadix};
  ia.zero[2] = {reinterpret_cast<uint32_t*>(ss.lookback[0]), p.tiles * kRadix * 2};
  k_init<<<8, 256, 0, stream>>>(ia);
  k_selftest_prepare<<<16, 256, 0, stream>>>(ss.keys[0], p.n, ss.tile_ctr);
  count_launches(2);
  PassArgs a{};
  a.keys_in = ss.keys[0];
  a.vals_in = nullptr;
  a.keys_out = ss.keys[1];
  a.vals_out = ss.vals[1];
  a.final_out = nullptr;
  a.hist = ss.hist;
  a.lookback = ss.lookback[0];
  a.lookback_next = nullptr;
  a.tile_ctr = ss.tile_ctr;
  a.n = p.n;
  a.lo_bit = 0;
  a.code_bits = p.code_bits;
  a.needs_cloud = 0;
  a.cm.offsets = nullptr;
  a.cm.uniform_n = p.n;
  a.cm.num_clouds = 1;
  a.status = device_status_ptr();
  a.spin_limit = spin_limit;
  // One block fewer than tiles: the blocks claim tickets 1 .. tiles-1, tile 0
  // never publishes, and tile 1's wait on it must give up after spin_limit polls.
  k_sort_pass<<<dim3(unsigned(p.tiles - 1)), kSortThreads, sizeof(PassSmem), stream>>>(a);
  count_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_traversal_arrays(int64_t n, int32_t* left, int32_t* right, int32_t* m2l, cudaStream_t stream) {
  const int L = ceil_log2_i64(n);
  const int64_t rows = real_node_count(n);
  int64_t grid = (rows + 255) / 256;
  if (grid > 148 * 16) grid = 148 * 16;
  k_traversal_arrays<<<unsigned(grid), 256, 0, stream>>>(n, L, rows, left, right, m2l);
  count_launches(1);
  return cudaGetLastError();
}

SortPlan make_sort_plan(int64_t n, int num_clouds, int dim) {
  SortPlan p;
  p.n = n;
  p.code_bits = dim == 3 ? 30 : 32;
  int cb = 0;
  while ((int64_t(1) << cb) < num_clouds) ++cb;
  p.cloud_bits = cb;
  p.passes = (p.code_bits + p.cloud_bits + 7) / 8;
  p.tiles = (n + kSortTile - 1) / kSortTile;
  return p;
}

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

size_t sort_scratch_bytes(const SortPlan& p) {
  size_t b = 0;
  b += 4 * align_up(size_t(p.n) * 4, 256);
  b += align_up(size_t(kMaxSortPasses) * kRadix * 4, 256);
  b += align_up(size_t(kMaxSortPasses) * 4, 256);
  b += 2 * align_up(size_t(p.tiles) * kRadix * 8, 256);
  return b;
}

void carve_sort_scratch(const SortPlan& p, char*& cur, SortScratch& s) {
  auto take = [&](size_t bytes) { char* r = cur; cur += align_up(bytes, 256); return r; };
  s.keys[0] = reinterpret_cast<uint32_t*>(take(size_t(p.n) * 4));
  s.keys[1] = reinterpret_cast<uint32_t*>(take(size_t(p.n) * 4));
  s.vals[0] = reinterpret_cast<uint32_t*>(take(size_t(p.n) * 4));
  s.vals[1] = reinterpret_cast<uint32_t*>(take(size_t(p.n) * 4));
  s.hist = reinterpret_cast<uint32_t*>(take(size_t(kMaxSortPasses) * kRadix * 4));
  s.tile_ctr = reinterpret_cast<uint32_t*>(take(size_t(kMaxSortPasses) * 4));
  s.lookback[0] = reinterpret_cast<uint64_t*>(take(size_t(p.tiles) * kRadix * 8));
  s.lookback[1] = reinterpret_cast<uint64_t*>(take(size_t(p.tiles) * kRadix * 8));
}

static std::atomic<uint64_t> g_launches{0};
void count_launches(int n) { g_launches.fetch_add(uint64_t(n), std::memory_order_relaxed); }
uint64_t launches_so_far() { return g_launches.load(std::memory_order_relaxed); }

CloudTree cloud_tree_facts(int64_t n) { return tree_facts(n); }
int64_t cloud_tree_blocks(const CloudTree& t) { return tree_blocks_of(t); }
int64_t cloud_tree_counters(const CloudTree& t) { return tree_counters_of(t); }

unsigned* device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  if (g_status_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_tbvh_status) != cudaSuccess) return nullptr;
    g_status_ptr[dev] = static_cast<unsigned*>(p);
  }
  return g_status_ptr[dev];
}

cudaError_t read_device_status(unsigned* out, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(out, g_tbvh_status, sizeof(unsigned));
  if (e != cudaSuccess) return e;
  if (clear) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_tbvh_status, &zero, sizeof(unsigned));
  }
  return e;
}

static int grid_for(int64_t work, int per_block, int cap) {
  int64_t g = (work + per_block - 1) / per_block;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return int(g);
}

// Runs the radix passes over keys already in ss.keys[0]; the values of the
// first pass are ss.vals[0] when explicit_vals, else the element index.
static cudaError_t run_sort_passes(const SortPlan& p, const SortScratch& ss, const CloudMap& cm,
                                   int64_t* final_out, cudaStream_t stream, bool explicit_vals = false) {
  const size_t smem = sizeof(PassSmem);
  static_assert(sizeof(PassSmem) <= 48 * 1024, "pass tile must fit the default dynamic shared memory limit");
  unsigned* status = device_status_ptr();
  int src = 0;
  for (int ps = 0; ps < p.passes; ++ps) {
    PassArgs a{};
    a.keys_in = ss.keys[src];
    a.vals_in = ps == 0 ? (explicit_vals ? ss.vals[0] : nullptr) : ss.vals[src];
    const bool last = ps == p.passes - 1;
    a.keys_out = last ? nullptr : ss.keys[src ^ 1];
    a.vals_out = last ? nullptr : ss.vals[src ^ 1];
    a.final_out = last ? final_out : nullptr;
    a.hist = ss.hist + ps * kRadix;
    a.lookback = ss.lookback[ps & 1];
    a.lookback_next = last ? nullptr : ss.lookback[(ps + 1) & 1];
    a.tile_ctr = ss.tile_ctr + ps;
    a.n = p.n;
    a.lo_bit = 8 * ps;
    a.code_bits = p.code_bits;
    a.needs_cloud = (8 * ps + 8 > p.code_bits && p.cloud_bits > 0) || (last && cm.num_clouds > 1) ? 1 : 0;
    a.cm = cm;
    a.status = status;
    a.spin_limit = kLbSpinLimit;
    k_sort_pass<<<dim3(unsigned(p.tiles)), kSortThreads, smem, stream>>>(a);
    count_launches(1);
    src ^= 1;
  }
  return cudaGetLastError();
}

cudaError_t launch_build(const BuildLaunch& b, cudaStream_t stream) {
  const int D = b.dim;
  const SortPlan& p = b.sort;
  const int64_t n = p.n;
  // 1. init
  InitArgs ia{};
  ia.zero[0] = {b.ss.hist, int64_t(kMaxSortPasses) * kRadix};
  ia.zero[1] = {b.ss.tile_ctr, int64_t(kMaxSortPasses)};
  ia.zero[2] = {reinterpret_cast<uint32_t*>(b.ss.lookback[0]), p.tiles * kRadix * 2};
  ia.zero[3] = {b.tree_counter, b.tree_counters};
  ia.bounds_enc = b.bounds_enc;
  ia.bounds_words = b.clouds.num_clouds * 2 * D;
  ia.dim = D;
  ia.clouds = b.clouds;
  ia.table = b.clouds.uniform_n > 0 ? nullptr : b.table;
  const int64_t init_work = p.tiles * kRadix * 2 > b.tree_counters ? p.tiles * kRadix * 2 : b.tree_counters;
  k_init<<<grid_for(init_work, 256 * 4, 1184), 256, 0, stream>>>(ia);
  count_launches(1);
  // 2. bounds
  const int64_t chunk = n / 1184 > 4096 ? ((n / 1184 + 255) / 256) * 256 : 4096;
  const int bgrid = int((n + chunk - 1) / chunk);
  if (D == 3) k_bounds<3><<<bgrid, 256, 0, stream>>>(b.points, b.clouds, n, chunk, b.bounds_enc);
  else k_bounds<2><<<bgrid, 256, 0, stream>>>(b.points, b.clouds, n, chunk, b.bounds_enc);
  count_launches(1);
  // 3. keys + histograms
  const int kgrid = grid_for((n + 3) / 4, 256, 148 * 8);  // one thread per quad of points
  if (D == 3)
    k_keys<3, true><<<kgrid, 256, 0, stream>>>(b.points, b.clouds, n, b.bounds_enc, nullptr, nullptr,
                                                b.ss.keys[0], b.ss.hist, p.code_bits, p.passes,
                                                b.scene_min, b.scene_max);
  else
    k_keys<2, true><<<kgrid, 256, 0, stream>>>(b.points, b.clouds, n, b.bounds_enc, nullptr, nullptr,
                                                b.ss.keys[0], b.ss.hist, p.code_bits, p.passes,
                                                b.scene_min, b.scene_max);
  count_launches(1);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // 4. radix passes -> sorted_indices
  e = run_sort_passes(p, b.ss, b.clouds, b.sorted_indices, stream);
  if (e != cudaSuccess) return e;
  // 5. tree
  TreeArgs ta{};
  ta.points = b.points;
  ta.sorted = b.sorted_indices;
  ta.node_aabbs = b.node_aabbs;
  ta.left = b.left_child;
  ta.right = b.right_child;
  ta.m2l = b.mem_to_leaf;
  ta.arrays_per_cloud = b.arrays_per_cloud ? 1 : 0;
  ta.cm = b.clouds;
  ta.table = b.clouds.uniform_n > 0 ? nullptr : b.table;
  ta.uni = b.uniform;
  ta.uni_blocks = b.clouds.uniform_n > 0 ? cloud_tree_blocks(b.uniform) : 0;
  ta.uni_rows = b.uniform_rows;
  ta.uni_counters = b.clouds.uniform_n > 0 ? cloud_tree_counters(b.uniform) : 0;
  ta.counters = b.tree_counter;
  ta.status = device_status_ptr();
  if (D == 3) k_tree<3><<<unsigned(b.tree_blocks), kTreeThreads, 0, stream>>>(ta);
  else k_tree<2><<<unsigned(b.tree_blocks), kTreeThreads, 0, stream>>>(ta);
  count_launches(1);
  return cudaGetLastError();
}

// The scene box of one cloud alone: the same seeds, chunks and reductions as
// the build's bounds step, so the result is bit-identical to the build's
// scene_min / scene_max for the same points (min / max are exact).
cudaError_t launch_scene_bounds(const float* points, int64_t n, int D, uint32_t* enc, float* smin, float* smax,
                                cudaStream_t stream) {
  CloudMap cm{};
  cm.offsets = nullptr;
  cm.uniform_n = n;
  cm.num_clouds = 1;
  InitArgs ia{};
  ia.bounds_enc = enc;
  ia.bounds_words = 2 * D;
  ia.dim = D;
  ia.clouds = cm;
  k_init<<<1, 256, 0, stream>>>(ia);
  const int64_t chunk = n / 1184 > 4096 ? ((n / 1184 + 255) / 256) * 256 : 4096;
  const int bgrid = int((n + chunk - 1) / chunk);
  if (D == 3) k_bounds<3><<<bgrid, 256, 0, stream>>>(points, cm, n, chunk, enc);
  else k_bounds<2><<<bgrid, 256, 0, stream>>>(points, cm, n, chunk, enc);
  k_bounds_decode<<<1, 32, 0, stream>>>(enc, D, smin, smax);
  count_launches(3);
  return cudaGetLastError();
}

cudaError_t launch_query_sort(const QuerySortLaunch& q, cudaStream_t stream) {
  const int D = q.dim;
  const SortPlan& p = q.sort;
  const int64_t n = p.n;
  InitArgs ia{};
  ia.zero[0] = {q.ss.hist, int64_t(kMaxSortPasses) * kRadix};
  ia.zero[1] = {q.ss.tile_ctr, int64_t(kMaxSortPasses)};
  ia.zero[2] = {reinterpret_cast<uint32_t*>(q.ss.lookback[0]), p.tiles * kRadix * 2};
  ia.dim = D;
  ia.clouds = q.clouds;
  k_init<<<grid_for(p.tiles * kRadix * 2, 256 * 4, 1184), 256, 0, stream>>>(ia);
  count_launches(1);
  const int kgrid = grid_for((n + 3) / 4, 256, 148 * 8);  // one thread per quad of points
  if (D == 3)
    k_keys<3, false><<<kgrid, 256, 0, stream>>>(q.queries, q.clouds, n, nullptr, q.scene_min, q.scene_max,
                                                 q.ss.keys[0], q.ss.hist, p.code_bits, p.passes, nullptr, nullptr);
  else
    k_keys<2, false><<<kgrid, 256, 0, stream>>>(q.queries, q.clouds, n, nullptr, q.scene_min, q.scene_max,
                                                 q.ss.keys[0], q.ss.hist, p.code_bits, p.passes, nullptr, nullptr);
  count_launches(1);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return run_sort_passes(p, q.ss, q.clouds, q.order_out, stream);
}

// ---- one rank's query share -------------------------------------------------
namespace {
constexpr int kShareMaxWorld = 256;

struct ShareScratch {
  uint32_t* codes;
  uint32_t* cell_count;
  uint8_t* owner;
  int64_t* rank_count;
  unsigned long long* counter;
  SortScratch ss;
};

void carve_share(int64_t m, int dim, char*& cur, ShareScratch& s) {
  auto take = [&](size_t bytes) { char* r = cur; cur += align_up(bytes, 256); return r; };
  s.codes = reinterpret_cast<uint32_t*>(take(size_t(m) * 4));
  s.cell_count = reinterpret_cast<uint32_t*>(take(size_t(kShareCells) * 4));
  s.owner = reinterpret_cast<uint8_t*>(take(size_t(kShareCells)));
  s.rank_count = reinterpret_cast<int64_t*>(take(size_t(kShareMaxWorld) * 8));
  s.counter = reinterpret_cast<unsigned long long*>(take(8));
  carve_sort_scratch(make_sort_plan(m, 1, dim), cur, s.ss);
}
}  // namespace

size_t share_scratch_bytes(int64_t m, int dim) {
  return align_up(size_t(m) * 4, 256) + align_up(size_t(kShareCells) * 4, 256) + align_up(size_t(kShareCells), 256) +
         align_up(size_t(kShareMaxWorld) * 8, 256) + align_up(8, 256) + sort_scratch_bytes(make_sort_plan(m, 1, dim));
}

cudaError_t launch_share_queries(const ShareLaunch& q, int64_t* count_out, cudaStream_t stream) {
  const int64_t m = q.num_queries;
  const int D = q.dim;
  char* cur = static_cast<char*>(q.workspace);
  ShareScratch s;
  carve_share(m, D, cur, s);
  const SortPlan full = make_sort_plan(m, 1, D);
  InitArgs ia{};
  ia.zero[0] = {s.cell_count, int64_t(kShareCells)};
  ia.zero[1] = {reinterpret_cast<uint32_t*>(s.rank_count), int64_t(kShareMaxWorld) * 2 + 2};  // + counter
  ia.zero[2] = {reinterpret_cast<uint32_t*>(s.ss.lookback[0]), full.tiles * kRadix * 2};
  ia.zero[3] = {s.ss.hist, int64_t(kMaxSortPasses) * kRadix + kMaxSortPasses};           // + tile counters
  k_init<<<grid_for(full.tiles * kRadix * 2, 256 * 4, 1184), 256, 0, stream>>>(ia);
  count_launches(1);
  const size_t cells_smem = size_t(kShareCells) * 4;
  // The shared-memory opt-in is per kernel (2-D and 3-D) and per device.
  static bool attr_set[2][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[D - 2][dev]) {
    cudaError_t e = D == 3 ? cudaFuncSetAttribute(k_share_cells<3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  int(cells_smem))
                           : cudaFuncSetAttribute(k_share_cells<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  int(cells_smem));
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[D - 2][dev] = true;
  }
  // Blocks of 1,024 threads with a 128 KB cell histogram each: about 128 K
  // queries per block keeps the per-block flush of the table cheap.
  const int cgrid = grid_for(m, kShareThreads * 128, 148 * 2);
  if (D == 3)
    k_share_cells<3><<<cgrid, kShareThreads, cells_smem, stream>>>(q.queries, m, q.scene_min, q.scene_max, s.codes,
                                                                    s.cell_count);
  else
    k_share_cells<2><<<cgrid, kShareThreads, cells_smem, stream>>>(q.queries, m, q.scene_min, q.scene_max, s.codes,
                                                                    s.cell_count);
  k_share_owners<<<1, kShareThreads, 0, stream>>>(s.cell_count, q.chunk, q.world, s.owner, s.rank_count);
  const int pgrid = grid_for(m, 256, 148 * 8);
  if (D == 3)
    k_share_compact<3><<<pgrid, 256, 0, stream>>>(s.codes, m, s.owner, q.rank, s.ss.keys[0], s.ss.vals[0],
                                                   s.counter, s.ss.hist, full.passes, m, device_status_ptr());
  else
    k_share_compact<2><<<pgrid, 256, 0, stream>>>(s.codes, m, s.owner, q.rank, s.ss.keys[0], s.ss.vals[0],
                                                   s.counter, s.ss.hist, full.passes, m, device_status_ptr());
  count_launches(3);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  int64_t count = 0;
  e = cudaMemcpyAsync(&count, s.rank_count + q.rank, sizeof(int64_t), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return e;
  if (count < 0 || count > m) count = 0;
  *count_out = count;
  if (count == 0) return cudaSuccess;
  SortPlan plan = make_sort_plan(count, 1, D);
  CloudMap cm{};
  cm.offsets = nullptr;
  cm.uniform_n = m;
  cm.num_clouds = 1;
  return run_sort_passes(plan, s.ss, cm, q.share_out, stream, /*explicit_vals=*/true);
}

}  // namespace tbvh
