/*
 * CPU oracle for the BVH k-NN path -- TEST INFRASTRUCTURE ONLY (see
 * tbvh_oracle.h). Every function names the reference code it restates.
 * Build: oracle/Makefile (gcc -O2 -mfma -ffp-contract=off).
 */
#include "tbvh_oracle.h"

#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <xmmintrin.h>

#define TBO_FAR FLT_MAX /* knn_query.cu:13 (kFloatInf is FLT_MAX) */

/* ---- floating-point mode: FTZ + DAZ like nvcc --use_fast_math ---------- */
static unsigned tbo_fp_enter(void) {
  unsigned old = _mm_getcsr();
  _mm_setcsr(old | 0x8040u); /* bit 15 FTZ, bit 6 DAZ */
  return old;
}
static void tbo_fp_leave(unsigned old) { _mm_setcsr(old); }

static double tbo_now(void) {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

/* ---- implicit tree sizes (implicit_tree.cuh:56-66,82-90) --------------- */
int tbo_leaf_level(int64_t n) {
  int l = 0;
  while (((int64_t)1 << l) < n) ++l;
  return l;
}

static int64_t tbo_level_count(int64_t n, int L, int l) { return ((n - 1) >> (L - l)) + 1; }

int64_t tbo_real_node_count(int64_t n) {
  if (n <= 0) return 0;
  const int L = tbo_leaf_level(n);
  int64_t total = 0;
  for (int l = 0; l <= L; ++l) total += tbo_level_count(n, L, l);
  return total;
}

/* ---- scene bounds (bvh_build.cu:453-494) ------------------------------- */
void tbo_scene_bounds(const float* pts, int64_t n, int d, float* lo, float* hi) {
  unsigned fp = tbo_fp_enter();
  for (int a = 0; a < d; ++a) {
    float l = 1.0e30f, h = -1.0e30f;
    for (int64_t i = 0; i < n; ++i) {
      const float v = pts[i * d + a];
      l = fminf(l, v);
      h = fmaxf(h, v);
    }
    lo[a] = l;
    hi[a] = h;
  }
  tbo_fp_leave(fp);
}

/* ---- Morton codes (morton.cuh:19-68) ------------------------------------ */
static float tbo_clamp01(float x) { return x < 0.0f ? 0.0f : (x > 1.0f ? 1.0f : x); }

static uint32_t tbo_quantize(float x, float lo, float hi, uint32_t bins) {
  const float extent = hi - lo;
  float t = 0.0f;
  if (!(extent <= 0.0f)) t = tbo_clamp01((x - lo) / extent);
  const float scaled = tbo_clamp01(t) * (float)bins;
  const uint32_t q = (uint32_t)scaled;
  return q >= bins ? bins - 1 : q;
}

static uint32_t tbo_spread3(uint32_t v) {
  v &= 0x000003ffu;
  v = (v | (v << 16)) & 0x030000ffu;
  v = (v | (v << 8)) & 0x0300f00fu;
  v = (v | (v << 4)) & 0x030c30c3u;
  v = (v | (v << 2)) & 0x09249249u;
  return v;
}

static uint32_t tbo_spread2(uint32_t v) {
  v &= 0x0000ffffu;
  v = (v | (v << 8)) & 0x00ff00ffu;
  v = (v | (v << 4)) & 0x0f0f0f0fu;
  v = (v | (v << 2)) & 0x33333333u;
  v = (v | (v << 1)) & 0x55555555u;
  return v;
}

void tbo_morton_codes(const float* pts, int64_t n, int d, const float* lo, const float* hi, uint32_t* codes) {
  unsigned fp = tbo_fp_enter();
  for (int64_t i = 0; i < n; ++i) {
    const float* p = pts + i * d;
    if (d == 3) {
      codes[i] = tbo_spread3(tbo_quantize(p[0], lo[0], hi[0], 1024u)) |
                 (tbo_spread3(tbo_quantize(p[1], lo[1], hi[1], 1024u)) << 1) |
                 (tbo_spread3(tbo_quantize(p[2], lo[2], hi[2], 1024u)) << 2);
    } else {
      codes[i] = tbo_spread2(tbo_quantize(p[0], lo[0], hi[0], 65536u)) |
                 (tbo_spread2(tbo_quantize(p[1], lo[1], hi[1], 65536u)) << 1);
    }
  }
  tbo_fp_leave(fp);
}

/* ---- stable argsort: LSD radix over 8-bit digits ------------------------ */
void tbo_stable_argsort_u32(const uint32_t* keys, int64_t n, int64_t* perm) {
  int64_t* tmp = (int64_t*)malloc((size_t)(n > 0 ? n : 1) * sizeof(int64_t));
  for (int64_t i = 0; i < n; ++i) perm[i] = i;
  int64_t* src = perm;
  int64_t* dst = tmp;
  for (int shift = 0; shift < 32; shift += 8) {
    int64_t count[257];
    memset(count, 0, sizeof(count));
    for (int64_t i = 0; i < n; ++i) count[((keys[src[i]] >> shift) & 0xffu) + 1]++;
    for (int b = 0; b < 256; ++b) count[b + 1] += count[b];
    for (int64_t i = 0; i < n; ++i) dst[count[(keys[src[i]] >> shift) & 0xffu]++] = src[i];
    int64_t* t = src;
    src = dst;
    dst = t;
  }
  /* four passes: result is back in perm */
  free(tmp);
}

/* ---- tree build (bvh_build.cu:241-398) ----------------------------------- */
void tbo_build_tree(const float* pts, const int64_t* sorted, int64_t n, int d, float* node_aabbs,
                    int32_t* left, int32_t* right, int32_t* mem_to_leaf) {
  unsigned fp = tbo_fp_enter();
  const int L = tbo_leaf_level(n);
  int64_t cnt[40], rowoff[41];
  int64_t acc = 0;
  for (int l = 0; l <= L; ++l) {
    cnt[l] = tbo_level_count(n, L, l);
    rowoff[l] = acc;
    acc += cnt[l];
  }
  rowoff[L + 1] = acc;
  const int w = 2 * d;
  for (int64_t j = 0; j < n; ++j) {
    float* r = node_aabbs + (rowoff[L] + j) * w;
    const float* p = pts + sorted[j] * d;
    for (int a = 0; a < d; ++a) {
      r[a] = p[a];
      r[d + a] = p[a];
    }
  }
  for (int l = L - 1; l >= 0; --l) {
    for (int64_t j = 0; j < cnt[l]; ++j) {
      float* r = node_aabbs + (rowoff[l] + j) * w;
      const float* c0 = node_aabbs + (rowoff[l + 1] + 2 * j) * w;
      if (2 * j + 1 < cnt[l + 1]) {
        const float* c1 = c0 + w;
        for (int a = 0; a < d; ++a) {
          r[a] = fminf(c0[a], c1[a]);
          r[d + a] = fmaxf(c0[d + a], c1[d + a]);
        }
      } else {
        memcpy(r, c0, sizeof(float) * (size_t)w);
      }
    }
  }
  if (left) {
    for (int l = 0; l <= L; ++l) {
      for (int64_t j = 0; j < cnt[l]; ++j) {
        const int64_t row = rowoff[l] + j;
        if (l == L) {
          left[row] = -1;
          right[row] = -1;
          mem_to_leaf[row] = (int32_t)j;
        } else {
          left[row] = (int32_t)(rowoff[l + 1] + 2 * j);
          right[row] = 2 * j + 1 < cnt[l + 1] ? (int32_t)(rowoff[l + 1] + 2 * j + 1) : -1;
          mem_to_leaf[row] = -1;
        }
      }
    }
  }
  tbo_fp_leave(fp);
}

void tbo_build(const float* pts, int64_t n, int d, float* node_aabbs, int64_t* sorted, float* scene_min,
               float* scene_max, int32_t* left, int32_t* right, int32_t* mem_to_leaf) {
  uint32_t* codes = (uint32_t*)malloc((size_t)n * sizeof(uint32_t));
  tbo_scene_bounds(pts, n, d, scene_min, scene_max);
  tbo_morton_codes(pts, n, d, scene_min, scene_max, codes);
  tbo_stable_argsort_u32(codes, n, sorted);
  free(codes);
  tbo_build_tree(pts, sorted, n, d, node_aabbs, left, right, mem_to_leaf);
}

/* ---- distances (geometry.cuh:4-19, FMA-contracted accumulation) -------- */
static float tbo_box_dist(const float* q, const float* box, int d) {
  float delta = fmaxf(box[0] - q[0], fmaxf(0.0f, q[0] - box[d]));
  float acc = delta * delta;
  for (int a = 1; a < d; ++a) {
    delta = fmaxf(box[a] - q[a], fmaxf(0.0f, q[a] - box[d + a]));
    acc = fmaf(delta, delta, acc);
  }
  return acc;
}

static float tbo_point_dist(const float* q, const float* p, int d) {
  float e = p[0] - q[0];
  float acc = e * e;
  for (int a = 1; a < d; ++a) {
    e = p[a] - q[a];
    acc = fmaf(e, e, acc);
  }
  return acc;
}

/* ---- reference traversal (knn_query.cu:20-154) --------------------------- */
static void tbo_insert_reference(int k, int64_t idx, float dist, int64_t* bi, float* bd) {
  if (dist >= bd[k - 1]) return;
  bd[k - 1] = dist;
  bi[k - 1] = idx;
  for (int i = k - 1; i >= 1; --i) {
    if (bd[i] < bd[i - 1]) {
      float td = bd[i - 1];
      int64_t ti = bi[i - 1];
      bd[i - 1] = bd[i];
      bi[i - 1] = bi[i];
      bd[i] = td;
      bi[i] = ti;
    }
  }
}

typedef struct {
  const float* node_aabbs;
  const int64_t* sorted;
  const float* pts;
  int64_t n;
  int d;
  const float* queries;
  int64_t m0, m1;
  int k;
  int64_t* out_idx;
  float* out_dist;
} tbo_job;

static void* tbo_reference_worker(void* arg) {
  tbo_job* job = (tbo_job*)arg;
  unsigned fp = tbo_fp_enter();
  const int d = job->d, k = job->k, w = 2 * d;
  const int64_t n = job->n;
  const int L = tbo_leaf_level(n);
  int64_t cnt[40], rowoff[41], acc = 0;
  for (int l = 0; l <= L; ++l) {
    cnt[l] = tbo_level_count(n, L, l);
    rowoff[l] = acc;
    acc += cnt[l];
  }
  int stack_level[64];
  int64_t stack_j[64];
  float stack_d[64];
  for (int64_t qi = job->m0; qi < job->m1; ++qi) {
    const float* q = job->queries + qi * d;
    int64_t* bi = job->out_idx + qi * k;
    float* bd = job->out_dist + qi * k;
    for (int i = 0; i < k; ++i) {
      bi[i] = -1;
      bd[i] = TBO_FAR;
    }
    int sp = 0, level = 0;
    int64_t j = 0;
    float node_dist = tbo_box_dist(q, job->node_aabbs, d);
    for (;;) {
      if (node_dist <= bd[k - 1]) {
        if (level == L) {
          tbo_insert_reference(k, job->sorted[j], node_dist, bi, bd);
        } else {
          const int cl = level + 1;
          const int64_t lj = 2 * j, rj = 2 * j + 1;
          const int right_real = rj < cnt[cl];
          const float ld = tbo_box_dist(q, job->node_aabbs + (rowoff[cl] + lj) * w, d);
          const float rd = right_real ? tbo_box_dist(q, job->node_aabbs + (rowoff[cl] + rj) * w, d) : TBO_FAR;
          const int left_near = ld <= rd;
          const int64_t near_j = left_near ? lj : rj, far_j = left_near ? rj : lj;
          const float near_d = left_near ? ld : rd, far_d = left_near ? rd : ld;
          const int near_real = left_near ? 1 : right_real, far_real = left_near ? right_real : 1;
          const float cutoff = bd[k - 1];
          if (far_real && far_d <= cutoff) {
            stack_level[sp] = cl;
            stack_j[sp] = far_j;
            stack_d[sp] = far_d;
            ++sp;
          }
          if (near_real && near_d <= cutoff) {
            level = cl;
            j = near_j;
            node_dist = near_d;
            continue;
          }
        }
      }
      if (sp == 0) break;
      --sp;
      level = stack_level[sp];
      j = stack_j[sp];
      node_dist = stack_d[sp];
    }
  }
  tbo_fp_leave(fp);
  return NULL;
}

/* ---- canonical brute force ---------------------------------------------- */
static void tbo_insert_canonical(int k, int64_t idx, float dist, int64_t* bi, float* bd) {
  if (!(dist < bd[k - 1] || (dist == bd[k - 1] && idx < bi[k - 1]))) return;
  bd[k - 1] = dist;
  bi[k - 1] = idx;
  for (int i = k - 1; i >= 1; --i) {
    if (bd[i] < bd[i - 1] || (bd[i] == bd[i - 1] && bi[i] < bi[i - 1])) {
      float td = bd[i - 1];
      int64_t ti = bi[i - 1];
      bd[i - 1] = bd[i];
      bi[i - 1] = bi[i];
      bd[i] = td;
      bi[i] = ti;
    }
  }
}

static void* tbo_brute_worker(void* arg) {
  tbo_job* job = (tbo_job*)arg;
  unsigned fp = tbo_fp_enter();
  const int d = job->d, k = job->k;
  for (int64_t qi = job->m0; qi < job->m1; ++qi) {
    const float* q = job->queries + qi * d;
    int64_t* bi = job->out_idx + qi * k;
    float* bd = job->out_dist + qi * k;
    for (int i = 0; i < k; ++i) {
      bi[i] = -1;
      bd[i] = TBO_FAR;
    }
    for (int64_t p = 0; p < job->n; ++p) {
      const float dist = tbo_point_dist(q, job->pts + p * d, d);
      tbo_insert_canonical(k, p, dist, bi, bd);
    }
  }
  tbo_fp_leave(fp);
  return NULL;
}

static void tbo_run(void* (*fn)(void*), tbo_job base, int64_t m, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if ((int64_t)threads > m) threads = m > 0 ? (int)m : 1;
  pthread_t tid[256];
  tbo_job jobs[256];
  for (int t = 0; t < threads; ++t) {
    jobs[t] = base;
    jobs[t].m0 = m * t / threads;
    jobs[t].m1 = m * (t + 1) / threads;
  }
  if (threads == 1) {
    fn(&jobs[0]);
    return;
  }
  for (int t = 0; t < threads; ++t) pthread_create(&tid[t], NULL, fn, &jobs[t]);
  for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
}

void tbo_knn_reference(const float* node_aabbs, const int64_t* sorted, int64_t n, int d, const float* queries,
                       int64_t m, int k, int64_t* out_idx, float* out_dist, int threads) {
  tbo_job job = {node_aabbs, sorted, NULL, n, d, queries, 0, m, k, out_idx, out_dist};
  tbo_run(tbo_reference_worker, job, m, threads);
}

void tbo_knn_bruteforce(const float* pts, int64_t n, int d, const float* queries, int64_t m, int k,
                        int64_t* out_idx, float* out_dist, int threads) {
  tbo_job job = {NULL, NULL, pts, n, d, queries, 0, m, k, out_idx, out_dist};
  tbo_run(tbo_brute_worker, job, m, threads);
}

void tbo_pair_distances(const float* pts, int64_t n, int d, const float* queries, int64_t m, int k,
                        const int64_t* idx, float* out) {
  unsigned fp = tbo_fp_enter();
  for (int64_t qi = 0; qi < m; ++qi) {
    for (int j = 0; j < k; ++j) {
      const int64_t p = idx[qi * k + j];
      out[qi * k + j] = (p < 0 || p >= n) ? TBO_FAR : tbo_point_dist(queries + qi * d, pts + p * d, d);
    }
  }
  tbo_fp_leave(fp);
}

/* ---- multi-cloud build + query (CPU baseline) ----------------------------- */
typedef struct {
  const float* pts;
  const int64_t* off;
  int64_t c0, c1;
  int d;
  float** trees;
  int64_t** sorted;
} tbo_build_job;

static void* tbo_build_worker(void* arg) {
  tbo_build_job* job = (tbo_build_job*)arg;
  for (int64_t c = job->c0; c < job->c1; ++c) {
    const int64_t n = job->off[c + 1] - job->off[c];
    const int64_t nr = tbo_real_node_count(n);
    job->trees[c] = (float*)malloc((size_t)nr * 2 * job->d * sizeof(float));
    job->sorted[c] = (int64_t*)malloc((size_t)n * sizeof(int64_t));
    float lo[3], hi[3];
    tbo_build(job->pts + job->off[c] * job->d, n, job->d, job->trees[c], job->sorted[c], lo, hi, NULL, NULL, NULL);
  }
  return NULL;
}

void tbo_build_and_query(const float* pts, const int64_t* pt_offsets, const float* queries, const int64_t* q_offsets,
                         int64_t clouds, int d, int k, int64_t* out_idx, float* out_dist, int threads,
                         double* build_seconds, double* query_seconds) {
  float** trees = (float**)calloc((size_t)clouds, sizeof(float*));
  int64_t** sorted = (int64_t**)calloc((size_t)clouds, sizeof(int64_t*));
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  const double t0 = tbo_now();
  {
    int nt = (int64_t)threads > clouds ? (int)clouds : threads;
    pthread_t tid[256];
    tbo_build_job jobs[256];
    for (int t = 0; t < nt; ++t) {
      jobs[t].pts = pts;
      jobs[t].off = pt_offsets;
      jobs[t].c0 = clouds * t / nt;
      jobs[t].c1 = clouds * (t + 1) / nt;
      jobs[t].d = d;
      jobs[t].trees = trees;
      jobs[t].sorted = sorted;
    }
    if (nt == 1) {
      tbo_build_worker(&jobs[0]);
    } else {
      for (int t = 0; t < nt; ++t) pthread_create(&tid[t], NULL, tbo_build_worker, &jobs[t]);
      for (int t = 0; t < nt; ++t) pthread_join(tid[t], NULL);
    }
  }
  const double t1 = tbo_now();
  for (int64_t c = 0; c < clouds; ++c) {
    const int64_t n = pt_offsets[c + 1] - pt_offsets[c];
    const int64_t m = q_offsets[c + 1] - q_offsets[c];
    tbo_knn_reference(trees[c], sorted[c], n, d, queries + q_offsets[c] * d, m, k, out_idx + q_offsets[c] * k,
                      out_dist + q_offsets[c] * k, threads);
  }
  const double t2 = tbo_now();
  for (int64_t c = 0; c < clouds; ++c) {
    free(trees[c]);
    free(sorted[c]);
  }
  free(trees);
  free(sorted);
  if (build_seconds) *build_seconds = t1 - t0;
  if (query_seconds) *query_seconds = t2 - t1;
}
