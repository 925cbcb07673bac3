/*
 * CPU oracle for the DSA lightning-indexer top-K path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the shipped library links or calls
 * this file; it is used by tests/, by __graft_entry__.smoke() and by the
 * cpu_baseline leg of bench.py, always as the checker and never as the thing
 * measured for the GPU arm.
 *
 * It restates, in plain C, the semantics of the reference operator
 * `dsa_topk_indexer_fp8_h64_d128_topk2048_ps64`:
 *
 *   - page format (reference methodology/framework/CLAUDE (16).md:493-537 and
 *     solution/cuda/kernel.cu:22-25): one physical page is 8448 bytes; bytes
 *     [0,8192) hold 64 tokens x 128 FP8 e4m3 values (token-major), bytes
 *     [8192,8448) hold the 64 per-token fp32 scales.
 *   - dequantisation (CLAUDE (16).md:505-517): K_deq = f32(fp8) * scale,
 *     rounded to fp32 per element.
 *   - score (methodology/checkpoints/kernel_naive.cu:103-106):
 *     score[t] = sum_h w[h] * relu(q_h . K_deq[t]) for t < seq_len.
 *   - selection (solution/cuda/kernel.cu:472-530): descending score; ties
 *     broken by ascending logical position (the order a stable descending
 *     radix sort yields); actual_topk = min(seq_len, 2048).
 *   - output (kernel.cu:513-529): rank r < actual_topk holds the physical
 *     slot block_table[b, pos >> 6] * 64 + (pos & 63); the other ranks hold
 *     -1. seq_len <= 0 gives a row of -1.
 *
 * Floating point: the e4m3 decode is exact; dot products accumulate in fp32
 * with eight partial sums (the reference path accumulates in fp32 as well,
 * in an unspecified order); the head reduction accumulates in fp32.
 *
 * Sequences longer than max_pages * 64 are clamped to max_pages * 64 (the
 * reference would read past its block-table row there); the GPU path clamps
 * identically and raises a status bit.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_H 64
#define ORC_D 128
#define ORC_PAGE 64
#define ORC_PAGE_BYTES 8448
#define ORC_PAGE_DATA 8192
#define ORC_TOPK 2048

/* e4m3 (OCP FP8, bias 7, no infinities, S.1111.111 is NaN). */
float oracle_e4m3_to_f32(uint8_t b) {
  const int s = b >> 7, e = (b >> 3) & 15, m = b & 7;
  float v;
  if (e == 15 && m == 7) return NAN;
  if (e == 0)
    v = ldexpf((float)m, -9); /* subnormal: m/8 * 2^-6 */
  else
    v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
  return s ? -v : v;
}

static float g_lut[256];
static int g_lut_ready = 0;
static void lut_init(void) {
  if (g_lut_ready) return;
  for (int i = 0; i < 256; ++i) g_lut[i] = oracle_e4m3_to_f32((uint8_t)i);
  g_lut_ready = 1;
}

/* Monotone map of an fp32 bit pattern to uint32 (larger float -> larger
 * uint); the same order a radix sort over float keys uses. */
static inline uint32_t ordered_u32(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

/* Sort key: score order first, then smaller position first. Unique per
 * position, so the selection has no ties left to break. */
static inline uint64_t pack_key(float score, int32_t pos) {
  return ((uint64_t)ordered_u32(score) << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)pos);
}

static int clamp_len(int32_t sl, int64_t max_pages) {
  if (sl <= 0) return 0;
  const int64_t cap = max_pages * ORC_PAGE;
  return (int)(sl > cap ? cap : sl);
}

/* Scores of one request: out[t] for t < len. q_f: [64][128] fp32. */
static void score_row(const float* q_f, const uint8_t* kcache, const float* w,
                      const int32_t* bt_row, int len, float* out) {
  float kd[ORC_D];
  for (int t = 0; t < len; ++t) {
    const int64_t page = bt_row[t / ORC_PAGE];
    const int off = t % ORC_PAGE;
    const uint8_t* pg = kcache + page * ORC_PAGE_BYTES;
    const uint8_t* row = pg + off * ORC_D;
    float scale;
    memcpy(&scale, pg + ORC_PAGE_DATA + off * 4, 4);
    for (int d = 0; d < ORC_D; ++d) kd[d] = g_lut[row[d]] * scale;
    float acc = 0.0f;
    for (int h = 0; h < ORC_H; ++h) {
      const float* qh = q_f + h * ORC_D;
      float p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int d = 0; d < ORC_D; d += 8)
        for (int l = 0; l < 8; ++l) p[l] += qh[d + l] * kd[d + l];
      const float dot = ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
      acc += w[h] * (dot > 0.0f ? dot : 0.0f);
    }
    out[t] = acc;
  }
}

static int cmp_desc_u64(const void* a, const void* b) {
  const uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
  return (x < y) - (x > y);
}

/* In-place selection: moves the k largest keys to keys[0..k) (unordered). */
static void select_top(uint64_t* keys, int n, int k) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const uint64_t pivot = keys[lo + (hi - lo) / 2];
    int i = lo, j = hi;
    while (i <= j) {
      while (keys[i] > pivot) ++i;
      while (keys[j] < pivot) --j;
      if (i <= j) {
        const uint64_t t = keys[i];
        keys[i] = keys[j];
        keys[j] = t;
        ++i;
        --j;
      }
    }
    if (k - 1 <= j)
      hi = j;
    else if (k - 1 >= i)
      lo = i;
    else
      break;
  }
}

/* Top-K of one score row; writes 2048 int32 (slots, then -1). */
static void topk_row(const float* scores, int len, const int32_t* bt_row,
                     uint64_t* scratch, int32_t* out) {
  const int k = len < ORC_TOPK ? len : ORC_TOPK;
  for (int t = 0; t < len; ++t) scratch[t] = pack_key(scores[t], t);
  if (len > k) select_top(scratch, len, k);
  qsort(scratch, (size_t)k, sizeof(uint64_t), cmp_desc_u64);
  for (int r = 0; r < ORC_TOPK; ++r) {
    if (r < k) {
      const int32_t pos = (int32_t)(0xFFFFFFFFu - (uint32_t)(scratch[r] & 0xFFFFFFFFu));
      out[r] = bt_row[pos / ORC_PAGE] * ORC_PAGE + (pos % ORC_PAGE);
    } else {
      out[r] = -1;
    }
  }
}

/*
 * scores: [B][score_stride] fp32; entries t >= len are set to -inf (the
 * reference's mask value, kernel.cu:433-434).
 */
int oracle_scores(const uint8_t* q, const uint8_t* kcache, const float* w,
                  const int32_t* seq_lens, const int32_t* block_table, int64_t B,
                  int64_t max_pages, float* scores, int64_t score_stride, int nthreads) {
  lut_init();
  if (nthreads <= 0) nthreads = 1;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads)
  for (int64_t b = 0; b < B; ++b) {
    float q_f[ORC_H * ORC_D];
    for (int i = 0; i < ORC_H * ORC_D; ++i) q_f[i] = g_lut[q[b * ORC_H * ORC_D + i]];
    const int len = clamp_len(seq_lens[b], max_pages);
    float* row = scores + b * score_stride;
    const int64_t lim = len < score_stride ? len : score_stride;
    score_row(q_f, kcache, w + b * ORC_H, block_table + b * max_pages, (int)lim, row);
    for (int64_t t = lim; t < score_stride; ++t) row[t] = -INFINITY;
  }
  return 0;
}

/* Top-K from precomputed scores (used to check the selection alone). */
int oracle_topk_from_scores(const float* scores, int64_t score_stride, const int32_t* seq_lens,
                            const int32_t* block_table, int64_t B, int64_t max_pages,
                            int32_t* out, int nthreads) {
  if (nthreads <= 0) nthreads = 1;
  int err = 0;
#pragma omp parallel num_threads(nthreads)
  {
    uint64_t* scratch = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)(score_stride > 0 ? score_stride : 1));
    if (!scratch) {
#pragma omp atomic write
      err = 1;
    } else {
#pragma omp for schedule(dynamic, 1)
      for (int64_t b = 0; b < B; ++b) {
        int len = clamp_len(seq_lens[b], max_pages);
        if (len > score_stride) len = (int)score_stride;
        topk_row(scores + b * score_stride, len, block_table + b * max_pages, scratch, out + b * ORC_TOPK);
      }
      free(scratch);
    }
  }
  return err;
}

/* The whole operator: scores + top-K + translation, one request per task. */
int oracle_indexer(const uint8_t* q, const uint8_t* kcache, const float* w,
                   const int32_t* seq_lens, const int32_t* block_table, int64_t B,
                   int64_t max_pages, int32_t* out, int nthreads) {
  lut_init();
  if (nthreads <= 0) nthreads = 1;
  const int64_t cap = max_pages * ORC_PAGE;
  int err = 0;
#pragma omp parallel num_threads(nthreads)
  {
    float* sc = (float*)malloc(sizeof(float) * (size_t)(cap > 0 ? cap : 1));
    uint64_t* scratch = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)(cap > 0 ? cap : 1));
    float* q_f = (float*)malloc(sizeof(float) * ORC_H * ORC_D);
    if (!sc || !scratch || !q_f) {
#pragma omp atomic write
      err = 1;
    } else {
#pragma omp for schedule(dynamic, 1)
      for (int64_t b = 0; b < B; ++b) {
        for (int i = 0; i < ORC_H * ORC_D; ++i) q_f[i] = g_lut[q[b * ORC_H * ORC_D + i]];
        const int len = clamp_len(seq_lens[b], max_pages);
        const int32_t* bt_row = block_table + b * max_pages;
        score_row(q_f, kcache, w + b * ORC_H, bt_row, len, sc);
        topk_row(sc, len, bt_row, scratch, out + b * ORC_TOPK);
      }
    }
    free(sc);
    free(scratch);
    free(q_f);
  }
  return err;
}

/* Raw MMA-level product for known-answer tests: d[m][n] = sum_k a[m][k]*b[n][k]
 * over e4m3 bytes (a: [M][128], b: [N][128]). */
void oracle_fp8_gemm_nt(const uint8_t* a, const uint8_t* b, int M, int N, float* d) {
  lut_init();
  for (int m = 0; m < M; ++m)
    for (int n = 0; n < N; ++n) {
      double acc = 0.0;
      for (int k = 0; k < ORC_D; ++k) acc += (double)g_lut[a[m * ORC_D + k]] * (double)g_lut[b[n * ORC_D + k]];
      d[m * N + n] = (float)acc;
    }
}
