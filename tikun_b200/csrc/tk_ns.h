// Internal interface of the Newton-Schulz engine (tk_ns.cu) used by the C-ABI
// layer (tk_ns_api.cpp).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace tk {
namespace ns {

// Scratch layout of one batch of same-shape matrices (R x C each; m = min,
// n = max; X is m x n, X^T is n x m, A and B are m x m, all half precision
// with rows padded to a multiple of 64 elements).
struct GroupLayout {
  int64_t R, C, m, n, batch;
  bool tall;
  int64_t ldx, ldm;
  size_t x_bytes, xt_bytes, a_bytes;
  int nblk;
  size_t scratch_bytes;
};

GroupLayout group_layout(int64_t rows, int64_t cols, int64_t batch);

// Inputs and outputs of one batch (host arrays of device pointers).
struct GroupIO {
  const void* const* src;  // NS input, or the Muon gradient
  void* const* dst;        // NS output (may equal src), or the Muon parameter
  float* const* mom;       // Muon momentum (f32), or nullptr for plain NS
  int src_dtype, dst_dtype;
  int update;              // 0: dst = O;  1: dst = dst + upd_scale * O
  float upd_scale;
  float mu, om;            // momentum and (1 - momentum) in f32
  int nesterov;
};

struct PrepArgs {
  const void* const* src;
  void* const* dst;
  float* const* mom;
  int64_t rows, cols;
  float mu, om;
  int nesterov;
  uint16_t* x;
  int64_t x_ld, x_bs;
  uint16_t* xt;
  int64_t xt_ld, xt_bs;
  float prescale;
  int steps;
  int dst_dtype;
  int update;
  float upd_scale;
};

// Enqueues the whole iteration for one batch on stream s.  scratch holds
// layout.scratch_bytes; err_dev is a device int a kernel sets when a bounded
// wait expires.
int run_group(const GroupLayout& layout, const GroupIO& io, int steps, int fmt, void* scratch,
              int* err_dev, cudaStream_t s);

// D = alpha * P Q^T (batched, half precision), for the GEMM kernel's tests.
int plain_gemm(const uint16_t* P, const uint16_t* Q, uint16_t* D, int batch, int M, int N, int K,
               int64_t ldp, int64_t ldq, int64_t ldd, float alpha, int fmt, int* err_dev,
               cudaStream_t s);

}  // namespace ns
}  // namespace tk
