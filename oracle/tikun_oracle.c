/*
 * tikun oracle — TEST INFRASTRUCTURE ONLY (see tikun_oracle.h).
 *
 * CPU restatement of the reference's optimizer-step arithmetic:
 *   - Tier 1 global L2 norm and clip scale: crates/tikun-cpu/src/lib.rs:79-125
 *     (x86 branch: f64 scalar accumulation per leaf, :106-113).
 *   - Tier 2 pointwise AdamW / Lion / SGD: lib.rs:144-272 (x86 scalar update
 *     :258-270), :274-359 (scalar :347-358), :361-428 (scalar :419-427), and
 *     the CustomDAG fallback rule :429-440.
 *   - Bias corrections: lib.rs:152-154 (f32 powi of a clamped step).
 *   - Newton-Schulz polar step: crates/tikun-cpu/src/tensor_engine.rs:12-77,
 *     non-macOS GEMM loops :130-142 (gemm_fast) and :177-190 (gemm_trans).
 *   - LayoutPlan::from_shapes: crates/tikun-core/src/arena.rs:34-57.
 *
 * Build with -ffp-contract=off: the reference (Rust) never fuses a*b+c into an
 * FMA, and every multiply, add, divide and square root here must round the
 * way the reference's scalar f32 code does.
 */
#include "tikun_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* bf16 <-> f32                                                               */
/* ------------------------------------------------------------------------ */
float tko_bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

uint16_t tko_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

static inline float load_elem(const void* base, uint64_t i, int32_t dtype) {
  if (dtype == TKO_BF16) return tko_bf16_to_f32(((const uint16_t*)base)[i]);
  return ((const float*)base)[i];
}

static inline void store_elem(void* base, uint64_t i, int32_t dtype, float x) {
  if (dtype == TKO_BF16)
    ((uint16_t*)base)[i] = tko_f32_to_bf16(x);
  else
    ((float*)base)[i] = x;
}

/* ------------------------------------------------------------------------ */
/* powi: binary exponentiation in f32, the routine a runtime-exponent        */
/* f32::powi lowers to on x86-64.                                             */
/* ------------------------------------------------------------------------ */
float tko_powi(float a, int32_t b) {
  int recip = b < 0;
  uint32_t e = recip ? (uint32_t)(-(int64_t)b) : (uint32_t)b;
  float r = 1.0f;
  for (;;) {
    if (e & 1u) r *= a;
    e >>= 1;
    if (e == 0) break;
    a *= a;
  }
  return recip ? 1.0f / r : r;
}

/* ------------------------------------------------------------------------ */
/* Tier 1                                                                     */
/* ------------------------------------------------------------------------ */
double tko_leaf_sumsq(const tko_leaf* leaf) {
  double s = 0.0;
  for (uint64_t i = 0; i < leaf->n; ++i) {
    double g = (double)load_elem(leaf->g, i, leaf->g_dtype);
    s += g * g;
  }
  return s;
}

float tko_clip_scale(double total_sumsq, float max_norm) {
  float global_norm = (float)sqrt(total_sumsq);
  if (global_norm > max_norm && max_norm > 0.0f) return max_norm / (global_norm + 1e-6f);
  return 1.0f;
}

/* ------------------------------------------------------------------------ */
/* Tier 2                                                                     */
/* ------------------------------------------------------------------------ */
void tko_pointwise_leaf(const tko_leaf* leaf, int32_t kind, const tko_hparams* hp,
                        uint64_t step, float clip_scale) {
  const uint64_t n = leaf->n;
  float* m1 = leaf->m;
  float* m2 = leaf->v;
  if (kind == TKO_LION) {
    /* lib.rs:347-358 */
    const float lr = hp->lr, b1 = hp->beta1, b2 = hp->beta2, decay = hp->decay;
    for (uint64_t i = 0; i < n; ++i) {
      float g = load_elem(leaf->g, i, leaf->g_dtype) * clip_scale;
      float m = m1[i];
      float c = b1 * m + (1.0f - b1) * g;
      float sign_c = c > 0.0f ? 1.0f : (c < 0.0f ? -1.0f : 0.0f);
      float p = load_elem(leaf->p, i, leaf->p_dtype);
      p = p - lr * (sign_c + decay * p);
      store_elem(leaf->p, i, leaf->p_dtype, p);
      m1[i] = b2 * m + (1.0f - b2) * g;
    }
    return;
  }
  if (kind == TKO_CUSTOM) {
    /* lib.rs:429-440: PointwiseOp::CustomDAG runs one fixed rule whatever its
     * primitives; the hyperparameters and m2 are not read */
    for (uint64_t i = 0; i < n; ++i) {
      float g = load_elem(leaf->g, i, leaf->g_dtype) * clip_scale;
      m1[i] = 0.9f * m1[i] + 0.1f * g;
      float p = load_elem(leaf->p, i, leaf->p_dtype);
      p = p - 1e-3f * m1[i];
      store_elem(leaf->p, i, leaf->p_dtype, p);
    }
    return;
  }
  if (kind == TKO_SGD) {
    /* lib.rs:419-427; momentum is the b1 argument (tikun-py/src/lib.rs:201-205) */
    const float lr = hp->lr, mom = hp->beta1, decay = hp->decay;
    for (uint64_t i = 0; i < n; ++i) {
      float g = load_elem(leaf->g, i, leaf->g_dtype) * clip_scale;
      m1[i] = mom * m1[i] + g;
      float p = load_elem(leaf->p, i, leaf->p_dtype);
      float update = m1[i] + decay * p;
      p = p - lr * update;
      store_elem(leaf->p, i, leaf->p_dtype, p);
    }
    return;
  }
  /* AdamW: crates/tikun-cpu/src/lib.rs:152-154 then :258-270 */
  const float lr = hp->lr, b1 = hp->beta1, b2 = hp->beta2, eps = hp->eps, decay = hp->decay;
  int32_t step_val = (int32_t)(step < 1 ? 1 : step);
  float bias_corr1 = 1.0f - tko_powi(b1, step_val);
  float bias_corr2 = 1.0f - tko_powi(b2, step_val);
  for (uint64_t i = 0; i < n; ++i) {
    float g = load_elem(leaf->g, i, leaf->g_dtype) * clip_scale;
    m1[i] = b1 * m1[i] + (1.0f - b1) * g;
    m2[i] = b2 * m2[i] + (1.0f - b2) * g * g;
    float m_hat = m1[i] / bias_corr1;
    float m_hat2 = m2[i] / bias_corr2;
    float p = load_elem(leaf->p, i, leaf->p_dtype);
    float step_update = (m_hat / (sqrtf(m_hat2) + eps)) + (decay * p);
    p -= lr * step_update;
    store_elem(leaf->p, i, leaf->p_dtype, p);
  }
}

/* ------------------------------------------------------------------------ */
/* A minimal work-sharing pool: items are claimed one at a time from an       */
/* atomic counter, the granularity rayon's par_iter over leaves has.          */
/* ------------------------------------------------------------------------ */
typedef void (*item_fn)(void* ctx, size_t item);
typedef struct {
  item_fn fn;
  void* ctx;
  size_t n_items;
  atomic_size_t next;
} pool_job;

static void* pool_worker(void* arg) {
  pool_job* job = (pool_job*)arg;
  for (;;) {
    size_t i = atomic_fetch_add(&job->next, 1);
    if (i >= job->n_items) break;
    job->fn(job->ctx, i);
  }
  return NULL;
}

static void run_parallel(item_fn fn, void* ctx, size_t n_items, int nthreads) {
  if (n_items == 0) return;
  if (nthreads <= 1 || n_items == 1) {
    for (size_t i = 0; i < n_items; ++i) fn(ctx, i);
    return;
  }
  if ((size_t)nthreads > n_items) nthreads = (int)n_items;
  pool_job job;
  job.fn = fn;
  job.ctx = ctx;
  job.n_items = n_items;
  atomic_init(&job.next, 0);
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)(nthreads - 1));
  int started = 0;
  for (int t = 0; t < nthreads - 1; ++t) {
    if (pthread_create(&th[t], NULL, pool_worker, &job) == 0) ++started;
  }
  pool_worker(&job);
  for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
  free(th);
}

typedef struct {
  const tko_leaf* leaves;
  double* sums;
} norm_ctx;

static void norm_item(void* c, size_t i) {
  norm_ctx* ctx = (norm_ctx*)c;
  ctx->sums[i] = tko_leaf_sumsq(&ctx->leaves[i]);
}

typedef struct {
  const tko_leaf* leaves;
  int32_t kind;
  const tko_hparams* hp;
  uint64_t step;
  float scale;
} update_ctx;

static void update_item(void* c, size_t i) {
  update_ctx* ctx = (update_ctx*)c;
  tko_pointwise_leaf(&ctx->leaves[i], ctx->kind, ctx->hp, ctx->step, ctx->scale);
}

float tko_step_two_tier(const tko_leaf* leaves, size_t n_leaves, int32_t kind,
                        const tko_hparams* hp, uint64_t step, float max_norm,
                        int nthreads) {
  float scale = 1.0f;
  if (max_norm > 0.0f) {
    double* sums = (double*)calloc(n_leaves ? n_leaves : 1, sizeof(double));
    norm_ctx nc = {leaves, sums};
    run_parallel(norm_item, &nc, n_leaves, nthreads);
    double total = 0.0;
    for (size_t i = 0; i < n_leaves; ++i) total += sums[i];
    free(sums);
    scale = tko_clip_scale(total, max_norm);
  }
  update_ctx uc = {leaves, kind, hp, step, scale};
  run_parallel(update_item, &uc, n_leaves, nthreads);
  return scale;
}

/* ------------------------------------------------------------------------ */
/* Newton-Schulz                                                              */
/* ------------------------------------------------------------------------ */
static const float NS_A = 3.4445f;
static const float NS_B = -4.7750f;
static const float NS_C = 2.0315f;

typedef struct {
  const float* a;
  const float* b;
  float* out;
  uint64_t m, k, n;
} gemm_ctx;

/* gemm_fast row i: out = a (m x k) * b (k x n), tensor_engine.rs:132-141 */
static void gemm_fast_row(void* c, size_t i) {
  gemm_ctx* g = (gemm_ctx*)c;
  float* out_row = g->out + i * g->n;
  for (uint64_t j = 0; j < g->n; ++j) out_row[j] = 0.0f;
  for (uint64_t p = 0; p < g->k; ++p) {
    float a_val = g->a[i * g->k + p];
    const float* b_row = g->b + p * g->n;
    for (uint64_t j = 0; j < g->n; ++j) out_row[j] += a_val * b_row[j];
  }
}

/* gemm_trans row i: out = a (m x k) * b^T (b is n x k), tensor_engine.rs:179-189 */
static void gemm_trans_row(void* c, size_t i) {
  gemm_ctx* g = (gemm_ctx*)c;
  const float* a_row = g->a + i * g->k;
  float* out_row = g->out + i * g->n;
  for (uint64_t j = 0; j < g->n; ++j) {
    const float* b_row = g->b + j * g->k;
    float sum = 0.0f;
    for (uint64_t p = 0; p < g->k; ++p) sum += a_row[p] * b_row[p];
    out_row[j] = sum;
  }
}

void tko_polar_step(float* matrix, uint64_t rows, uint64_t cols, uint64_t steps,
                    int nthreads) {
  if (rows == 0 || cols == 0) return;
  if (rows > cols) {
    /* tensor_engine.rs:18-34: work on the transpose (cols x rows) */
    float* t = (float*)malloc(sizeof(float) * rows * cols);
    for (uint64_t r = 0; r < rows; ++r)
      for (uint64_t c = 0; c < cols; ++c) t[c * rows + r] = matrix[r * cols + c];
    tko_polar_step(t, cols, rows, steps, nthreads);
    for (uint64_t r = 0; r < rows; ++r)
      for (uint64_t c = 0; c < cols; ++c) matrix[r * cols + c] = t[c * rows + r];
    free(t);
    return;
  }
  /* tensor_engine.rs:37-44 */
  double sum_sq = 0.0;
  for (uint64_t i = 0; i < rows * cols; ++i) sum_sq += (double)matrix[i] * (double)matrix[i];
  float nrm = (float)sqrt(sum_sq);
  float inv_norm = 1.0f / fmaxf(nrm, 1e-7f);
  for (uint64_t i = 0; i < rows * cols; ++i) matrix[i] *= inv_norm;

  const uint64_t r2 = rows * rows;
  float* a_mat = (float*)calloc(r2, sizeof(float));
  float* b_mat = (float*)calloc(r2, sizeof(float));
  float* poly = (float*)calloc(r2, sizeof(float));
  float* next_x = (float*)calloc(rows * cols, sizeof(float));
  for (uint64_t s = 0; s < steps; ++s) {
    gemm_ctx g1 = {matrix, matrix, a_mat, rows, cols, rows};
    run_parallel(gemm_trans_row, &g1, rows, nthreads);
    gemm_ctx g2 = {a_mat, a_mat, b_mat, rows, rows, rows};
    run_parallel(gemm_fast_row, &g2, rows, nthreads);
    /* tensor_engine.rs:61-70 */
    for (uint64_t i = 0; i < rows; ++i)
      for (uint64_t j = 0; j < rows; ++j) {
        float eye = (i == j) ? 1.0f : 0.0f;
        uint64_t idx = i * rows + j;
        poly[idx] = NS_A * eye + NS_B * a_mat[idx] + NS_C * b_mat[idx];
      }
    gemm_ctx g3 = {poly, matrix, next_x, rows, rows, cols};
    run_parallel(gemm_fast_row, &g3, rows, nthreads);
    memcpy(matrix, next_x, sizeof(float) * rows * cols);
  }
  free(a_mat);
  free(b_mat);
  free(poly);
  free(next_x);
}

void tko_polar_batched(float* tensor, uint64_t heads, uint64_t out, uint64_t in,
                       uint64_t steps, int nthreads) {
  uint64_t slice = out * in;
  for (uint64_t h = 0; h < heads; ++h) tko_polar_step(tensor + h * slice, out, in, steps, nthreads);
}

/* ------------------------------------------------------------------------ */
/* Layout                                                                     */
/* ------------------------------------------------------------------------ */
void tko_layout_from_shapes(const uint64_t* shapes, size_t n, uint64_t* byte_offsets,
                            uint64_t* total_bytes) {
  uint64_t cur = 0;
  const uint64_t line = 64;
  for (size_t i = 0; i < n; ++i) {
    uint64_t rem = cur % line;
    if (rem != 0) cur += line - rem;
    byte_offsets[i] = cur;
    cur += shapes[i] * 4u;
  }
  *total_bytes = cur;
}
