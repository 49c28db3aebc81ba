// Internal declarations shared by the C-ABI layer (tk_api.cpp) and the CUDA
// kernels.  Nothing here is part of the public ABI.
#pragma once

#include <cuda_runtime.h>

#include <nvtx3/nvToolsExt.h>

#include <cstdint>
#include <string>

#include "../../include/tikun_cuda.h"

namespace tk {

// ---------------------------------------------------------------- errors
int set_error(int code, const char* fmt, ...);
void clear_error();
int cuda_error(cudaError_t e, const char* what);

#define TK_CUDA_TRY(expr)                                     \
  do {                                                        \
    cudaError_t _e = (expr);                                  \
    if (_e != cudaSuccess) return ::tk::cuda_error(_e, #expr); \
  } while (0)

#define TK_TRY(expr)               \
  do {                             \
    int _s = (expr);               \
    if (_s != TK_OK) return _s;    \
  } while (0)

// ---------------------------------------------------------------- tracing
// An NVTX range over the enqueueing of one phase (Tier 1, Tier 2, a
// Newton-Schulz iteration, an exchange); profilers project it onto the GPU
// work launched inside.  Costs a function-pointer test when no tool is
// attached.
class NvtxRange {
 public:
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

// ---------------------------------------------------------------- scratch
// Stream-ordered device scratch from a per-device memory pool that keeps its
// memory cached between calls.  Freed (stream-ordered) by the destructor.
class Scratch {
 public:
  Scratch() = default;
  ~Scratch();
  Scratch(const Scratch&) = delete;
  Scratch& operator=(const Scratch&) = delete;
  int alloc(size_t bytes, cudaStream_t s);
  void* get() const { return ptr_; }

 private:
  void* ptr_ = nullptr;
  cudaStream_t stream_ = nullptr;
};

int sm_count(int* out);

// In-place ncclAllReduce(sum) of count doubles over an ncclComm_t (NCCL
// resolved at run time; tk_shard.cpp).
int nccl_allreduce_sum_f64(double* buf, size_t count, void* comm, cudaStream_t s);

// Records the calling thread's update start/stop event (tk_set_update_events)
// on s, if one is set.
int record_update_event(bool start, cudaStream_t s);

// SMs the pointwise kernels leave free (tk_set_reserved_sms); grids are sized
// for the remaining ones.
int pointwise_sms(int* out);

// Where a pointer lives (cudaPointerGetAttributes); device memory of another
// device is an error.
enum class Residency { kNone, kDevice, kHost };
int classify_pointer(const void* ptr, Residency* r, int dev);

// A persistent per-device status word that kernels set when a bounded wait
// expires (0 = fine).
int device_status_word(int** out);

// ---------------------------------------------------------------- pointwise
constexpr int kMaxLeavesPerLaunch = 224;

struct LeafDesc {
  void* p;
  const void* g;
  float* m;
  float* v;
  uint64_t n;        // elements
  uint64_t q_begin;  // first quad (4-element group) of this leaf in the launch
  uint32_t vec_ok;   // p, g, m, v aligned for vector access of a whole quad
  uint32_t reserved;
};

struct LeafTable {
  int32_t n_leaves;
  int32_t reserved;
  uint64_t total_quads;
  LeafDesc leaf[kMaxLeavesPerLaunch];
};

// Other GPUs' copies of the same parameter layout, mapped into this process:
// a parameter at address a is also stored at a + delta[i] (bytes).
constexpr int kMaxPeers = 7;
struct PeerSet {
  int32_t n;
  int32_t reserved;
  int64_t delta[kMaxPeers];
};

struct PointwiseConsts {
  float lr, b1, b2, eps, decay;
  float omb1, omb2;  // 1 - b1, 1 - b2 in f32
  float bc1, bc2;    // AdamW bias corrections
};

// The update's constants for optimizer `kind` at `step`, formed in f32 as the
// reference does (crates/tikun-cpu/src/lib.rs:152-154): every entry point
// builds them here, so all give the same bits.
PointwiseConsts make_consts(int kind, const tk_hparams& hp, uint64_t step);

// A byte range of one leaf buffer; writable for p, m and v.
struct ByteRange {
  uintptr_t lo, hi;
  bool writable;
};

// Sorts `ranges` in place and fails with TK_ERR_INVALID if a range the step
// writes shares memory with any other range.  Allocates nothing.
int check_overlaps(ByteRange* ranges, size_t n);

// Launchers (tk_pointwise.cu).  Tables hold leaves of one (p, g) dtype pair.
int launch_sumsq_partials(const LeafTable& t, int g_dtype, double* partials, int n_blocks,
                          cudaStream_t s);
int sumsq_blocks_for(uint64_t total_quads);
int launch_sumsq_reduce(const double* partials, int n_partials, double* total,
                        cudaStream_t s);
int launch_clip_scale(const double* sumsq, int n_partials, float max_norm, float* scale_out,
                      cudaStream_t s);
// Tier 2.  If partials != nullptr every CTA folds partials[0..n_partials) into
// the clip scale itself (same order in every CTA); else scale_dev (or 1.0).
// Tier 2 for a table of f32 leaves whose four pointers are 16-byte aligned,
// through the bulk-copy pipeline (tk_pointwise_bulk.cu).  Same results.
int launch_pointwise_bulk(const LeafTable& t, int kind, const PointwiseConsts& c,
                          const double* partials, int n_partials, float max_norm,
                          const float* scale_dev, float* scale_out, cudaStream_t s);
int launch_pointwise(const LeafTable& t, int kind, int p_dtype, int g_dtype,
                     const PointwiseConsts& c, const double* partials, int n_partials,
                     float max_norm, const float* scale_dev, float* scale_out,
                     cudaStream_t s, const PeerSet* peers = nullptr);

}  // namespace tk
