// Shared device/host helpers for the B200 BVH k-NN path.
//
// Everything here is compiled with nvcc --use_fast_math (same floating-point
// mode as the reference extension, torchbvh/_extension.py:36) so that the
// Morton normalisation and the squared-distance arithmetic produce the same
// float32 bits as the reference kernels.
#pragma once

#include <cfloat>
#include <cstdint>
#include <cuda_runtime.h>

namespace tbvh {

// "No neighbour yet" distance. The reference initialises its top-k list with
// FLT_MAX and index -1 (torchbvh/csrc/knn_query.cu:13,85-88); a candidate only
// enters if it is strictly below the current k-th distance, so points whose
// squared distance overflows to +inf are never reported.
constexpr float kFar = FLT_MAX;
constexpr unsigned kFullMask = 0xffffffffu;

// Error bits OR-ed into the per-device status word by kernels that give up a
// bounded wait or detect an impossible state. Read back with
// tbvh_device_status().
enum DeviceErrorBits : unsigned {
  kDevErrLookbackTimeout = 1u,
  kDevErrStackOverflow = 2u,
  kDevErrTreeCounter = 4u,
  kDevErrBadIndex = 8u,
};

// ---------------------------------------------------------------------------
// Implicit tree geometry (own formulation of the layout of
// torchbvh/csrc/implicit_tree.cuh:21-120).
//
// A cloud of N points has leaf level L = ceil(log2 N). Level l (0 = root)
// holds cnt(l) = ceil(N / 2^(L-l)) real nodes; node j of level l covers sorted
// leaf positions [j << (L-l), (j+1) << (L-l)) clipped to N. Rows of
// node_aabbs are level-major over real nodes only, so row(l, j) =
// rowoff(l) + j with rowoff(l) = sum_{l'<l} cnt(l'). This equals the
// reference's memory_index() (implicit index minus the virtual nodes of the
// levels above), which the parity tests check.
// ---------------------------------------------------------------------------
__host__ __device__ inline int ceil_log2_i64(int64_t n) {
  int l = 0;
  while ((int64_t(1) << l) < n) ++l;
  return l;
}

__host__ __device__ inline int64_t level_count(int64_t n, int leaf_level, int level) {
  return ((n - 1) >> (leaf_level - level)) + 1;
}

__host__ __device__ inline int64_t level_row_offset(int64_t n, int leaf_level, int level) {
  int64_t off = 0;
  for (int l = 0; l < level; ++l) off += level_count(n, leaf_level, l);
  return off;
}

__host__ __device__ inline int64_t real_node_count(int64_t n) {
  const int L = ceil_log2_i64(n);
  return level_row_offset(n, L, L + 1);
}

// ---------------------------------------------------------------------------
// Morton codes (behaviour of torchbvh/csrc/morton.cuh:19-68): per axis the
// coordinate is normalised to the scene AABB, clamped to [0,1], scaled to the
// bin count (1024 in 3-D, 65536 in 2-D), truncated and clamped to bins-1; the
// per-axis integers are bit-interleaved x-lowest. The bit-spread steps are the
// standard published mask sequence.
// ---------------------------------------------------------------------------
__host__ __device__ inline float clamp_unit(float v) {
  return v < 0.0f ? 0.0f : (v > 1.0f ? 1.0f : v);
}

__host__ __device__ inline uint32_t quantize_axis(float x, float lo, float hi, uint32_t bins) {
  const float extent = hi - lo;
  float t;
  if (extent <= 0.0f) {
    t = 0.0f;
  } else {
    t = clamp_unit((x - lo) / extent);
  }
  const float scaled = clamp_unit(t) * static_cast<float>(bins);
  const uint32_t q = static_cast<uint32_t>(scaled);
  return q >= bins ? bins - 1 : q;
}

__host__ __device__ inline uint32_t spread_bits3(uint32_t v) {
  v &= 0x000003ffu;
  v = (v | (v << 16)) & 0x030000ffu;
  v = (v | (v << 8)) & 0x0300f00fu;
  v = (v | (v << 4)) & 0x030c30c3u;
  v = (v | (v << 2)) & 0x09249249u;
  return v;
}

__host__ __device__ inline uint32_t spread_bits2(uint32_t v) {
  v &= 0x0000ffffu;
  v = (v | (v << 8)) & 0x00ff00ffu;
  v = (v | (v << 4)) & 0x0f0f0f0fu;
  v = (v | (v << 2)) & 0x33333333u;
  v = (v | (v << 1)) & 0x55555555u;
  return v;
}

template <int D>
__host__ __device__ inline uint32_t morton_code(const float* p, const float* lo, const float* hi) {
  if constexpr (D == 3) {
    return spread_bits3(quantize_axis(p[0], lo[0], hi[0], 1024u)) |
           (spread_bits3(quantize_axis(p[1], lo[1], hi[1], 1024u)) << 1) |
           (spread_bits3(quantize_axis(p[2], lo[2], hi[2], 1024u)) << 2);
  } else {
    return spread_bits2(quantize_axis(p[0], lo[0], hi[0], 65536u)) |
           (spread_bits2(quantize_axis(p[1], lo[1], hi[1], 65536u)) << 1);
  }
}

template <int D>
__host__ __device__ constexpr int morton_bits() { return D == 3 ? 30 : 32; }

// ---------------------------------------------------------------------------
// Squared distances. Same float32 operation sequence as the reference's
// min_distance_sq_to_aabb (torchbvh/csrc/geometry.cuh:4-19) compiled with FMA
// contraction: per axis delta = max(lo - q, max(0, q - hi)), then
// d = delta0^2, d = fma(delta1, delta1, d), d = fma(delta2, delta2, d).
// For a leaf (lo == hi == p) delta is |p - q| exactly, so point_dist2 below
// gives bit-identical results.
// ---------------------------------------------------------------------------
template <int D>
__device__ __forceinline__ float box_dist2(const float* q, const float* lo, const float* hi) {
  float acc;
  {
    const float delta = fmaxf(lo[0] - q[0], fmaxf(0.0f, q[0] - hi[0]));
    acc = delta * delta;
  }
#pragma unroll
  for (int a = 1; a < D; ++a) {
    const float delta = fmaxf(lo[a] - q[a], fmaxf(0.0f, q[a] - hi[a]));
    acc = fmaf(delta, delta, acc);
  }
  return acc;
}

template <int D>
__device__ __forceinline__ float point_dist2(const float* q, float px, float py, float pz) {
  const float e0 = px - q[0];
  const float e1 = py - q[1];
  float acc = e0 * e0;
  acc = fmaf(e1, e1, acc);
  if constexpr (D == 3) {
    const float e2 = pz - q[2];
    acc = fmaf(e2, e2, acc);
  }
  return acc;
}

// Order-preserving float <-> uint32 map (total order with -0 < +0), used for
// atomicMin/atomicMax reductions of the scene bounds.
__device__ __forceinline__ uint32_t float_to_ordered(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ordered_to_float(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

// ---------------------------------------------------------------------------
// Packed clouds. Fixed-size batches are the uniform case (cloud b starts at
// b * uniform_n); ragged batches carry a device offsets array (B + 1 int64).
// ---------------------------------------------------------------------------
struct CloudMap {
  const int64_t* offsets;  // device, num_clouds + 1 entries; unused when uniform_n > 0
  int64_t uniform_n;       // > 0 for fixed-size clouds
  int num_clouds;

  __device__ __forceinline__ int64_t start(int b) const {
    return uniform_n > 0 ? int64_t(b) * uniform_n : offsets[b];
  }
  __device__ __forceinline__ int64_t size(int b) const {
    return uniform_n > 0 ? uniform_n : offsets[b + 1] - offsets[b];
  }
  // Cloud that owns packed element e (0 <= e < total). Totals are below 2^31
  // (checked by the host entry points), so the uniform case divides in 32 bits.
  __device__ __forceinline__ int find(int64_t e) const {
    if (num_clouds == 1) return 0;
    if (uniform_n > 0) return static_cast<int>(uint32_t(e) / uint32_t(uniform_n));
    int lo = 0, hi = num_clouds - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (offsets[mid] <= e) lo = mid; else hi = mid - 1;
    }
    return lo;
  }
};

// Per-cloud tree facts, either derived from a uniform size or read from the
// table that the init kernel writes for ragged batches.
struct CloudTree {
  int64_t n;          // points in the cloud
  int64_t row_off;    // first node_aabbs row of the cloud in the packed tensor
  int64_t tree_cta;   // first subtree block of the cloud in the build grid
  int64_t counter;    // first tree-climb counter of the cloud
  int leaf_level;     // L
  int sub_level;      // subtree-root level handled by one build block
};

}  // namespace tbvh
