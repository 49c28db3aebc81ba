// Element-wise arithmetic and table helpers shared by the pointwise kernels
// (tk_pointwise.cu, tk_pointwise_bulk.cu).  Every multiply, add, divide and
// square root is a separately rounded IEEE f32 operation, in the reference's
// order, so every kernel that uses these gives tikun-cpu's bits.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "tk_internal.h"

namespace tk {
namespace pw {

// ------------------------------------------------------------------ dtypes
__device__ __forceinline__ float bf16_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

__device__ __forceinline__ uint32_t f32_to_bf16(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return ((u >> 16) | 0x40u) & 0xffffu;  // quiet NaN
  u += 0x7fffu + ((u >> 16) & 1u);                                              // nearest even
  return u >> 16;
}

// ------------------------------------------------------------------ update rules
// AdamW, crates/tikun-cpu/src/lib.rs:258-270 (g already scaled by the caller).
__device__ __forceinline__ void adamw(float& p, float g, float& m, float& v,
                                      const PointwiseConsts& k) {
  m = __fadd_rn(__fmul_rn(k.b1, m), __fmul_rn(k.omb1, g));
  v = __fadd_rn(__fmul_rn(k.b2, v), __fmul_rn(__fmul_rn(k.omb2, g), g));
  const float m_hat = __fdiv_rn(m, k.bc1);
  const float m_hat2 = __fdiv_rn(v, k.bc2);
  const float step_update =
      __fadd_rn(__fdiv_rn(m_hat, __fadd_rn(__fsqrt_rn(m_hat2), k.eps)), __fmul_rn(k.decay, p));
  p = __fsub_rn(p, __fmul_rn(k.lr, step_update));
}

// Lion, lib.rs:347-358.
__device__ __forceinline__ void lion(float& p, float g, float& m, const PointwiseConsts& k) {
  const float c = __fadd_rn(__fmul_rn(k.b1, m), __fmul_rn(k.omb1, g));
  const float sign_c = c > 0.0f ? 1.0f : (c < 0.0f ? -1.0f : 0.0f);
  p = __fsub_rn(p, __fmul_rn(k.lr, __fadd_rn(sign_c, __fmul_rn(k.decay, p))));
  m = __fadd_rn(__fmul_rn(k.b2, m), __fmul_rn(k.omb2, g));
}

// SGD with momentum, lib.rs:419-427 (momentum carried in b1).
__device__ __forceinline__ void sgd(float& p, float g, float& m, const PointwiseConsts& k) {
  m = __fadd_rn(__fmul_rn(k.b1, m), g);
  const float update = __fadd_rn(m, __fmul_rn(k.decay, p));
  p = __fsub_rn(p, __fmul_rn(k.lr, update));
}

// PointwiseOp::CustomDAG, lib.rs:429-440: one fixed rule, whatever the
// primitives: m = 0.9 m + 0.1 g; p -= 1e-3 m (f32 literals).
__device__ __forceinline__ void custom_dag(float& p, float g, float& m) {
  m = __fadd_rn(__fmul_rn(0.9f, m), __fmul_rn(0.1f, g));
  p = __fsub_rn(p, __fmul_rn(1e-3f, m));
}

template <int KIND>
__device__ __forceinline__ void apply(float& p, float g, float& m, float& v,
                                      const PointwiseConsts& k) {
  if constexpr (KIND == TK_ADAMW) adamw(p, g, m, v, k);
  else if constexpr (KIND == TK_LION) lion(p, g, m, k);
  else if constexpr (KIND == TK_SGD) sgd(p, g, m, k);
  else custom_dag(p, g, m);
}

// ------------------------------------------------------------------ reductions
// Deterministic block sum: fixed shuffle tree per warp, then warp 0 adds the
// warp totals in warp order.  Result valid in thread 0.
template <int NT>
__device__ __forceinline__ double block_sum(double x) {
  __shared__ double warp_tot[NT / 32];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) x += __shfl_down_sync(0xffffffffu, x, off);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) warp_tot[wid] = x;
  __syncthreads();
  double t = 0.0;
  if (wid == 0) {
    t = lane < (NT / 32) ? warp_tot[lane] : 0.0;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) t += __shfl_down_sync(0xffffffffu, t, off);
  }
  __syncthreads();
  return t;
}

// lib.rs:117-122: norm rounded to f32, scale only if it exceeds max_norm > 0.
__device__ __forceinline__ float clip_from_sumsq(double total, float max_norm) {
  const float norm = __double2float_rn(sqrt(total));
  if (norm > max_norm && max_norm > 0.0f) return __fdiv_rn(max_norm, __fadd_rn(norm, 1e-6f));
  return 1.0f;
}

__device__ __forceinline__ int find_leaf(const LeafTable& t, uint64_t q) {
  int lo = 0, hi = t.n_leaves - 1;  // last leaf with q_begin <= q
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (t.leaf[mid].q_begin <= q) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ uint64_t leaf_quads(const LeafDesc& L) { return (L.n + 3) >> 2; }

}  // namespace pw
}  // namespace tk
