/*
 * CPU restatement of the bit-exact integer path of Spark-H3 routing.
 * TEST INFRASTRUCTURE ONLY: this file is the checker the tests, the smoke check and
 * bench.py's CPU-baseline leg compare against.  The product never links or calls it.
 *
 * It follows, with the arithmetic order fixed so results are reproducible bit for bit:
 *   - query block centroids: h3_sparse_attention/spark_integration.py:111-127
 *     (_sol_topk_policy_scores: fp32 block sum / rows in block)
 *   - key block centroids:   sol_attn/preprocess.py:16-52 (_reduce_kc_kernel: fp32 sum
 *     over the block / rows, stored in the key dtype)
 *   - scores:                spark_integration.py:127-129 (einsum * D^-1/2 * log2(e))
 *   - Top-K + packing:       spark_integration.py:136-175 (_sol_topk_route_from_scores),
 *     head_budget.py:11 (stable descending order: ties go to the lower index) and
 *     sol_topk_cutoff.py:19-44 (bit kb % 32 of word kb / 32)
 *
 * Canonical order (shared with the CUDA kernels): a block sum is the in-order fp32 sum of
 * its 64-row sub-blocks, each an in-order fp32 sum of its rows starting from 0; a score is
 * a sequential fused multiply-add chain over d = 0 .. D-1 starting from 0, then one fp32
 * multiply by scale_log2.  Compile with -ffp-contract=off so no other contraction occurs.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static float bf16_to_f(uint16_t x) {
  uint32_t u = (uint32_t)x << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static uint16_t f_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40u);
  const uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

static float load_elem(const void* x, int dtype, int64_t i) {
  return dtype == 1 ? bf16_to_f(((const uint16_t*)x)[i]) : ((const float*)x)[i];
}

/* Block means of x [B, T, H, D] -> out [B, NB, H, D] fp32.  Blocks are independent, so they
 * are spread over OpenMP threads; each element's sum keeps the canonical order. */
void orc_block_means(const void* x, int dtype, int B, int T, int H, int D, int block, float* out) {
  const int NB = (T + block - 1) / block;
  const int64_t HD = (int64_t)H * D;
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
  for (int b = 0; b < B; ++b)
    for (int j = 0; j < NB; ++j) {
      const int row0 = j * block;
      const int rows = T - row0 < block ? T - row0 : block;
      float* total = out + ((int64_t)b * NB + j) * HD;
      float* acc = (float*)malloc(sizeof(float) * (size_t)HD);
      for (int64_t c = 0; c < HD; ++c) total[c] = 0.f;
      for (int s = 0; s < rows; s += 64) {
        const int sub = rows - s < 64 ? rows - s : 64;
        for (int64_t c = 0; c < HD; ++c) acc[c] = 0.f;
        /* rows outer, columns inner: every column's chain still adds its rows in order */
        for (int r = 0; r < sub; ++r) {
          const int64_t base = ((int64_t)b * T + row0 + s + r) * HD;
          for (int64_t c = 0; c < HD; ++c) acc[c] = acc[c] + load_elem(x, dtype, base + c);
        }
        for (int64_t c = 0; c < HD; ++c) total[c] = total[c] + acc[c];
      }
      for (int64_t c = 0; c < HD; ++c) total[c] = total[c] / (float)rows;
      free(acc);
    }
}

/* Round fp32 values to bf16 in place (returns them as floats). */
void orc_round_bf16(float* x, int64_t n) {
  for (int64_t i = 0; i < n; ++i) x[i] = bf16_to_f(f_to_bf16(x[i]));
}

/* Global anchor from query block means: sum_j qc[j] * block / (prefix * block). */
void orc_anchor(const float* qc, int B, int NB, int H, int D, int block, int prefix_blocks, float* out) {
  const int64_t HD = (int64_t)H * D;
  for (int b = 0; b < B; ++b)
    for (int64_t c = 0; c < HD; ++c) {
      float acc = 0.f;
      for (int j = 0; j < prefix_blocks; ++j) acc = acc + qc[((int64_t)b * NB + j) * HD + c] * (float)block;
      out[(int64_t)b * HD + c] = acc / ((float)prefix_blocks * (float)block);
    }
}

/* scores [B, QB, H, C] from qc [B, NB, H, D] and kc (already at key precision, fp32).
 * Eight candidates at a time keep eight independent fma chains in flight; each chain is
 * still the sequential one over d. */
void orc_scores(const float* qc, const float* kc, int B, int QB, int NB, int H, int D, int C, float scale_log2,
                float* scores) {
#pragma omp parallel for collapse(3) schedule(static)
  for (int b = 0; b < B; ++b)
    for (int i = 0; i < QB; ++i)
      for (int h = 0; h < H; ++h) {
        const float* q = qc + (((int64_t)b * NB + i) * H + h) * D;
        float* row = scores + (((int64_t)b * QB + i) * H + h) * C;
        for (int j0 = 0; j0 < C; j0 += 8) {
          const int n = C - j0 < 8 ? C - j0 : 8;
          const float* k[8];
          float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          for (int u = 0; u < 8; ++u) k[u] = kc + (((int64_t)b * NB + j0 + (u < n ? u : 0)) * H + h) * D;
          for (int d = 0; d < D; ++d) {
            const float qd = q[d];
            for (int u = 0; u < 8; ++u) s[u] = fmaf(qd, k[u][d], s[u]);
          }
          for (int u = 0; u < n; ++u) row[j0 + u] = s[u] * scale_log2;
        }
      }
}

typedef struct {
  float v;
  int i;
} Entry;

static int entry_cmp(const void* a, const void* b) {
  const Entry* x = (const Entry*)a;
  const Entry* y = (const Entry*)b;
  if (x->v > y->v) return -1;
  if (x->v < y->v) return 1;
  return x->i < y->i ? -1 : (x->i > y->i ? 1 : 0);
}

static int int_cmp(const void* a, const void* b) {
  const int x = *(const int*)a, y = *(const int*)b;
  return x < y ? -1 : (x > y ? 1 : 0);
}

/* One row: keep the k largest of C scores (ties -> lower index), 0 <= k <= C.  Writes the k
 * ascending indices into idx[0 .. k) and the packed words. */
static void topk_row(const float* score, int C, int k, int words, Entry* e, int* sel, int32_t* idx, int32_t* w) {
  for (int j = 0; j < C; ++j) {
    e[j].v = score[j];
    e[j].i = j;
  }
  qsort(e, (size_t)C, sizeof(Entry), entry_cmp);
  for (int t = 0; t < k; ++t) sel[t] = e[t].i;
  qsort(sel, (size_t)k, sizeof(int), int_cmp);
  memset(w, 0, sizeof(int32_t) * (size_t)words);
  for (int t = 0; t < k; ++t) {
    idx[t] = sel[t];
    w[sel[t] >> 5] = (int32_t)((uint32_t)w[sel[t] >> 5] | (1u << (sel[t] & 31)));
  }
}

/* Per row: keep the topk largest scores (ties -> lower index).  Writes ascending indices
 * [rows, topk] and packed words [rows, words]. */
void orc_topk(const float* scores, int64_t rows, int C, int topk, int words, int32_t* indices, int32_t* packed) {
#pragma omp parallel
  {
    Entry* e = (Entry*)malloc(sizeof(Entry) * (size_t)C);
    int* sel = (int*)malloc(sizeof(int) * (size_t)C);
#pragma omp for schedule(dynamic, 64)
    for (int64_t r = 0; r < rows; ++r)
      topk_row(scores + r * C, C, topk, words, e, sel, indices + r * topk, packed + r * words);
    free(e);
    free(sel);
  }
}

/* Per-head budgets (head_budget.py:7-19, route_with_head_budgets): row r of the
 * [B, QB, H] rows keeps the budget[r % H] largest scores in stable descending order, the
 * budget clamped to [0, C].  indices rows are `width` wide; entries past a row's budget
 * (or past width) are -1. */
void orc_topk_head_budgets(const float* scores, int64_t rows, int H, int C, const int32_t* budget, int width,
                           int words, int32_t* indices, int32_t* packed) {
#pragma omp parallel
  {
    Entry* e = (Entry*)malloc(sizeof(Entry) * (size_t)C);
    int* sel = (int*)malloc(sizeof(int) * (size_t)C);
    int32_t* idx = (int32_t*)malloc(sizeof(int32_t) * (size_t)C);
#pragma omp for schedule(dynamic, 64)
    for (int64_t r = 0; r < rows; ++r) {
      int k = budget[r % H];
      k = k < 0 ? 0 : (k > C ? C : k);
      topk_row(scores + r * C, C, k, words, e, sel, idx, packed + r * words);
      for (int t = 0; t < width; ++t) indices[r * width + t] = t < k ? idx[t] : -1;
    }
    free(e);
    free(sel);
    free(idx);
  }
}
