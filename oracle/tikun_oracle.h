/*
 * tikun oracle — TEST INFRASTRUCTURE ONLY.
 *
 * A CPU restatement of the reference engine's arithmetic for the optimizer-step
 * hot path (tikun-cpu, x86 scalar branch), used as the checker for the CUDA
 * path and as the timed CPU baseline.  Only tests/, __graft_entry__.smoke()
 * and bench.py (its cpu_baseline leg and its reference arm) may load it.  The
 * product library never links or calls anything in this directory.
 *
 * Parity status: pinned against the reference's own known-answer checks
 * (torch AdamW over 10 steps, examples/verify_exact_math_parity.py:16-72; the
 * reference's torch Newton-Schulz, python/tikun/muon.py:10-32; the 4x4 polar
 * identity test, crates/tikun-cpu/src/tensor_engine.rs:198-210; the 64-byte
 * slot alignment test, crates/tikun-core/src/arena.rs:109-118).  The
 * reference itself (Rust) cannot be built in this environment.
 */
#ifndef TIKUN_ORACLE_H
#define TIKUN_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { TKO_F32 = 0, TKO_BF16 = 1 };
enum { TKO_ADAMW = 0, TKO_LION = 1, TKO_SGD = 2, TKO_CUSTOM = 3 };

/* One leaf of the step: the reference's TensorBuffer
 * (crates/tikun-cpu/src/lib.rs:25-32) plus element types for p and g.
 * m and v are always f32. */
typedef struct {
  void* p;
  const void* g;
  float* m;
  float* v;
  uint64_t n;
  int32_t p_dtype;
  int32_t g_dtype;
} tko_leaf;

typedef struct {
  float lr, beta1, beta2, eps, decay;
} tko_hparams;

/* Rust f32::powi for a runtime exponent (binary exponentiation in f32). */
float tko_powi(float a, int32_t b);

/* Tier 1: sequential f64 sum of g*g over one leaf (lib.rs:106-113). */
double tko_leaf_sumsq(const tko_leaf* leaf);

/* Clip scale from the global sum of squares (lib.rs:117-122). */
float tko_clip_scale(double total_sumsq, float max_norm);

/* Tier 2 over one leaf with a given clip scale (lib.rs:143-428). */
void tko_pointwise_leaf(const tko_leaf* leaf, int32_t kind, const tko_hparams* hp,
                        uint64_t step, float clip_scale);

/* Whole two-tier step (lib.rs:68-445).  nthreads <= 1 runs on the calling
 * thread; otherwise leaves are spread over a pool, as rayon's par_iter over
 * leaves does.  Returns the clip scale. */
float tko_step_two_tier(const tko_leaf* leaves, size_t n_leaves, int32_t kind,
                        const tko_hparams* hp, uint64_t step, float max_norm,
                        int nthreads);

/* Newton-Schulz polar step in f32 (tensor_engine.rs:12-77), row-parallel GEMMs
 * over nthreads (tensor_engine.rs:130-142, 177-190). */
void tko_polar_step(float* matrix, uint64_t rows, uint64_t cols, uint64_t steps,
                    int nthreads);

/* Batched polar over heads (tensor_engine.rs:79-96). */
void tko_polar_batched(float* tensor, uint64_t heads, uint64_t out, uint64_t in,
                       uint64_t steps, int nthreads);

/* LayoutPlan::from_shapes (crates/tikun-core/src/arena.rs:34-57). */
void tko_layout_from_shapes(const uint64_t* shapes, size_t n, uint64_t* byte_offsets,
                            uint64_t* total_bytes);

/* bf16 helpers (round to nearest even, NaN kept quiet). */
float tko_bf16_to_f32(uint16_t h);
uint16_t tko_f32_to_bf16(float f);

#ifdef __cplusplus
}
#endif
#endif
