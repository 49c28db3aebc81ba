// Internal interface of the Newton-Schulz engine (tk_ns.cu) used by the C-ABI
// layer (tk_ns_api.cpp).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "tk_internal.h"

namespace tk {
namespace ns {

// Matrices per batch (one launch sequence).  Their pointers travel in the
// kernels' parameter space, so a batch needs no device-side table.
constexpr int kMaxBatch = 256;

// Scratch layout of one batch of matrices that are all m x n or n x m
// (m <= n): two X^T buffers (ping-pong) are n x m, and A, A' and B are m x m,
// all half precision with rows padded to a multiple of 64 elements (ldm).  No
// m x n copy of X exists: X X^T reads X^T MN-major.  With split operands
// (format 2) each row holds ldm hi values followed by ldm lo values: row
// stride rsm = 2 ldm.
struct GroupLayout {
  int64_t m, n, batch;
  int64_t ldm;
  int64_t rsm;
  bool split;
  size_t xt_bytes, a_bytes;
  int nblk;
  size_t scratch_bytes;
};

GroupLayout group_layout(int64_t m, int64_t n, int64_t batch, bool split = false);

// Inputs and outputs of one batch (host arrays of device pointers, length
// batch <= kMaxBatch).  A "tall" matrix is stored n x m (rows > cols).
struct GroupIO {
  const void* const* src;  // NS input, or the Muon gradient
  void* const* dst;        // NS output (may equal src), or the Muon parameter
  float* const* mom;       // Muon momentum (f32), or nullptr for plain NS
  const uint8_t* tall;
  int src_dtype, dst_dtype;
  int update;              // 0: dst = O;  1: dst = dst + scale * O
  float upd_scale_wide, upd_scale_tall;
  float mu, om;            // momentum and (1 - momentum) in f32
  int nesterov;
  const PeerSet* peers = nullptr;  // the final parameters also go to these peers
};

struct PrepArgs {
  const void* src[kMaxBatch];
  void* dst[kMaxBatch];
  float* mom[kMaxBatch];
  uint64_t tall[kMaxBatch / 64];
  int64_t m, n;
  float mu, om;
  int nesterov;
  uint16_t* xt;
  int64_t xt_ld, xt_bs, xt_lo;  // xt_lo: offset of the lo values (split operands)
  float prescale;
  int steps;
  int dst_dtype;
  int update;
  float upd_scale_wide, upd_scale_tall;
};

// Enqueues the whole iteration for one batch on stream s.  scratch holds
// layout.scratch_bytes; err_dev is a device int a kernel sets when a bounded
// wait expires.
int run_group(const GroupLayout& layout, const GroupIO& io, int steps, int fmt, void* scratch,
              int* err_dev, cudaStream_t s);

// Newton-Schulz GEMM grids leave this many SMs free (per calling thread), for
// a copy kernel running beside them.
void set_gemm_reserved_sms(int n);

// Copies of finished parameters into the peers' copies by an SM kernel (16-byte
// loads once, a store per peer): the entries' 16-byte units are split evenly
// over `blocks` CTAs.  src must be 16-byte aligned and every delta a multiple
// of 16.
struct PeerCopyList {
  int n;
  const uint8_t* src[kMaxBatch];
  uint64_t bytes[kMaxBatch];
  uint64_t unit0[kMaxBatch + 1];  // first 16-byte unit of each entry; unit0[n] = total
};
int launch_peer_copy(const PeerCopyList& list, const PeerSet& peers, int blocks, cudaStream_t s);

// D = alpha * P Q^T (batched, half precision), for the GEMM kernel's tests.
int plain_gemm(const uint16_t* P, const uint16_t* Q, uint16_t* D, int batch, int M, int N, int K,
               int64_t ldp, int64_t ldq, int64_t ldd, float alpha, int fmt, int* err_dev,
               cudaStream_t s);

// Test hook: a kernel whose only wait can never complete gives up after
// limit_ms and records code 9 in *err_dev.
int bounded_wait_probe(int* err_dev, int limit_ms, cudaStream_t s);

}  // namespace ns
}  // namespace tk
