/*
 * tikun-cuda: B200 (sm_100a) optimizer-step engine behind a C ABI.
 *
 * Plain C: pointers, sizes and enums only.  Every entry point returns an int
 * status (TK_OK == 0); on failure tk_last_error() returns a message for the
 * calling thread.  No entry point aborts the process.
 *
 * Buffers are owned by the caller.  p, m, v (and the Newton-Schulz matrix) are
 * updated in place; g is read only.  Device pointers and host pointers are
 * both accepted by tk_step_buffers (all leaves of one call must be of one
 * kind): host leaves are staged through device memory, so a caller of the
 * reference's CPU engine keeps its buffers where they are.
 *
 * Streams are passed as void* (a cudaStream_t; NULL is the legacy default
 * stream).  Calls are stream-ordered; the synchronous variants return after
 * the result they report is on the host.
 */
#ifndef TIKUN_CUDA_H
#define TIKUN_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TK_ABI_VERSION 1

#if defined(__GNUC__)
#define TK_API __attribute__((visibility("default")))
#else
#define TK_API
#endif

/* status codes */
enum {
  TK_OK = 0,
  TK_ERR_INVALID = 1,     /* bad argument: null pointer, size, dtype, aliasing */
  TK_ERR_VERIFY = 2,      /* static verification of the schedule failed */
  TK_ERR_CUDA = 3,        /* a CUDA runtime call failed */
  TK_ERR_ALLOC = 4,       /* device or pinned memory could not be obtained */
  TK_ERR_UNSUPPORTED = 5, /* combination not implemented */
  TK_ERR_DEVICE = 6       /* a kernel reported an error status (bounded wait expired),
                             or a step missed its deadline (tk_stream_wait_deadline) */
};

/* element types */
enum { TK_F32 = 0, TK_BF16 = 1, TK_F16 = 2 };

/* pointwise optimizers: the reference's PointwiseOp (crates/tikun-core/src/ir.rs:74-97).
 * TK_CUSTOM is PointwiseOp::CustomDAG, which the reference executes as one fixed
 * rule whatever its primitives (crates/tikun-cpu/src/lib.rs:429-440):
 * m = 0.9 m + 0.1 g;  p -= 1e-3 m  (g clip-scaled; hparams and v unused). */
enum { TK_ADAMW = 0, TK_LION = 1, TK_SGD = 2, TK_CUSTOM = 3 };

/* schedule roles: WorkloadRole (crates/tikun-core/src/ir.rs:5-12) */
enum { TK_ROLE_LOAD = 0, TK_ROLE_COMPUTE = 1, TK_ROLE_STORE = 2 };

/* Newton-Schulz tensor-core operands (accumulation is always f32):
 *   TK_NS_F16    f16 operands (the default);
 *   TK_NS_BF16   bf16 operands;
 *   TK_NS_F16X3  every operand value v held as an f16 pair, hi = f16(v) and
 *                lo = f16(v - hi), each product formed as hi*hi + hi*lo + lo*hi:
 *                about 22 significant bits at three times the tensor-core work
 *                and twice the scratch; Newton-Schulz within a few 1e-6 of f32
 *                (for callers whose parameters are stored in bf16 and must stay
 *                within 1e-3 of the f32 result over many steps, and for inputs
 *                with strong directions over a noise floor near 1e-3 of the
 *                largest, where 16-bit operands end 3 % (f16) or 25 % (bf16)
 *                from the f32 result and split f16 ends within 1e-3);
 *   TK_NS_F16X2  X held as f16 pairs and each iteration's update B' X formed
 *                as B' X_hi + B' X_lo, the m x m matrices (X X^T, B') in f16,
 *                X X^T from X_hi: 1.4 to 1.5 times the f16 time (measured
 *                on 2 x 4096 x 14336; TK_NS_F16X3: 3 times), and the same
 *                accuracy as f16 on random inputs without its loss over a noise
 *                floor (matrices under 256 rows run as TK_NS_F16X3). */
enum { TK_NS_F16 = 0, TK_NS_BF16 = 1, TK_NS_F16X3 = 2, TK_NS_F16X2 = 3 };

/* One schedule node: ScheduleIRNode (crates/tikun-core/src/ir.rs:16-36). */
typedef struct {
  const char* name;
  int32_t role;
  uint64_t tile_size;
  uint64_t unroll_factor;
  uint64_t vector_width;
  uint64_t prefetch_distance;
} tk_schedule_node;

/* SchedulePipeline (crates/tikun-core/src/ir.rs:101-110).  max_norm > 0 means
 * the pipeline carries GlobalReduction::GlobalL2Norm { max_norm }. */
typedef struct {
  const tk_schedule_node* nodes;
  size_t n_nodes;
  float max_norm;
} tk_pipeline;

/* One leaf: TensorBuffer (crates/tikun-cpu/src/lib.rs:25-32) with element
 * types.  m and v are f32.  v may be NULL unless the optimizer is AdamW
 * (tikun-py/src/lib.rs:178 passes 0 when the m2 list is empty). */
typedef struct {
  void* p;
  const void* g;
  float* m;
  float* v;
  uint64_t n;
  int32_t p_dtype; /* TK_F32 or TK_BF16 */
  int32_t g_dtype; /* TK_F32 or TK_BF16 */
} tk_leaf;

/* Pointwise hyperparameters (PointwiseOp fields).  For SGD, beta1 is the
 * momentum (tikun-py/src/lib.rs:201-205); Lion ignores eps. */
typedef struct {
  float lr;
  float beta1;
  float beta2;
  float eps;
  float decay;
} tk_hparams;

/* ---------------------------------------------------------------------- */
/* library                                                                 */
/* ---------------------------------------------------------------------- */

/* Message of the last failing call on this thread ("" if none). */
TK_API const char* tk_last_error(void);

/* TK_ABI_VERSION of the loaded library. */
TK_API int tk_abi_version(void);

/* Static verification: Verifier::verify (crates/tikun-core/src/verifier.rs:14-45).
 * Empty pipeline, tile_size % 64 != 0, vector_width not a power of two or < 4
 * fail with TK_ERR_VERIFY and the message "Static verification failed: [...]"
 * (crates/tikun-cpu/src/lib.rs:74). */
TK_API int tk_verify(const tk_pipeline* pipeline);

/* LayoutPlan::from_shapes (crates/tikun-core/src/arena.rs:34-57): f32 leaves
 * packed at 64-byte-aligned byte offsets. */
TK_API int tk_layout_from_shapes(const uint64_t* num_elements, size_t n_leaves,
                          uint64_t* byte_offsets, uint64_t* total_bytes);

/* ---------------------------------------------------------------------- */
/* two-tier pointwise step (Tier 1 global L2 norm, Tier 2 update)          */
/* ---------------------------------------------------------------------- */

/* CpuLowering::step_two_tier (crates/tikun-cpu/src/lib.rs:68-445): verify the
 * pipeline, compute the clip scale if it carries a GlobalL2Norm, apply the
 * optimizer to every leaf.  step is the AdamW step count (clamped to >= 1,
 * lib.rs:152).  *clip_scale_out (host) receives the scale; the call returns
 * after it is known. */
TK_API int tk_step_two_tier(const tk_pipeline* pipeline, const tk_leaf* leaves, size_t n_leaves,
                     int32_t kind, const tk_hparams* hp, uint64_t step,
                     float* clip_scale_out, void* stream);

/* CpuLowering::step_arena (crates/tikun-cpu/src/lib.rs:39-65): the two-tier
 * step over the slots of four f32 arenas (MemoryArena, crates/tikun-core/src/
 * arena.rs:69-103): slot i is slot_elems[i] elements at byte offset
 * slot_offsets[i] of every arena (tk_layout_from_shapes gives the reference's
 * 64-byte-aligned offsets).  Each arena holds arena_bytes bytes; a slot that
 * does not fit, or an offset that is not a multiple of 4, is TK_ERR_INVALID.
 * The padding between slots is not touched.  m2_arena may be NULL unless kind
 * is TK_ADAMW.  Verifies the pipeline, then runs as tk_step_two_tier over the
 * slots (device or host arenas); *clip_scale_out (host, may be NULL) receives
 * the scale and the call returns after it is known. */
TK_API int tk_step_arena(const tk_pipeline* pipeline, float* params_arena,
                         const float* grads_arena, float* m1_arena, float* m2_arena,
                         uint64_t arena_bytes, const uint64_t* slot_offsets,
                         const uint64_t* slot_elems, size_t n_slots, int32_t kind,
                         const tk_hparams* hp, uint64_t step, float* clip_scale_out, void* stream);

/* step_fast_buffers (crates/tikun-py/src/lib.rs:155-222): builds the
 * reference's three-node pipeline (load_g / fma_opt / store_p, vector width 8)
 * with a GlobalL2Norm when max_norm > 0 and runs tk_step_two_tier.  Accepts
 * device leaves or host leaves.  clip_scale_out may be NULL. */
TK_API int tk_step_buffers(const tk_leaf* leaves, size_t n_leaves, int32_t kind,
                    const tk_hparams* hp, uint64_t step, float max_norm,
                    float* clip_scale_out, void* stream);

/* As tk_step_buffers for device leaves, without waiting: the clip scale is
 * written to clip_scale_dev (device memory, may be NULL) in stream order. */
TK_API int tk_step_buffers_async(const tk_leaf* leaves, size_t n_leaves, int32_t kind,
                          const tk_hparams* hp, uint64_t step, float max_norm,
                          float* clip_scale_dev, void* stream);

/* tk_step_buffers for callers that cannot allocate device memory (an
 * application that owns a fixed memory budget, or a host runtime whose
 * allocator must not be re-entered from an optimizer hook).  No counterpart
 * in the reference.  The norm's partial sums and the clip scale live in a
 * fixed 64 KB device array per GPU (8192 f64 slots plus the scale) instead of
 * pool memory; no cudaMalloc, cudaFree or other allocating routine is called.
 * Device leaves only, at most 224 leaves and 8192 norm blocks per call, else
 * TK_ERR_INVALID.  All calls on a device share the array: calls that overlap
 * on the GPU race.  The first call on each device, and the first after a
 * cudaDeviceReset, looks up the array's address (do it before any stream
 * capture).  With clip_scale_out non-NULL the call waits for the stream and
 * returns the scale; with NULL it returns once its kernels are enqueued (a
 * kernel error then surfaces at the caller's next synchronisation).  Its leaf
 * tables and overlap check live on the calling thread's stack: about 72 KB. */
TK_API int tk_step_buffers_noalloc(const tk_leaf* leaves, size_t n_leaves, int32_t kind,
                                   const tk_hparams* hp, uint64_t step, float max_norm,
                                   float* clip_scale_out, void* stream);

/* The pieces of the step, for callers that shard it (ZeRO-1 over ranks):
 *   tk_grad_sumsq       sum over the leaves of g*g in f64 -> *sumsq_dev
 *   tk_clip_scale       *scale_dev = clip scale of *sumsq_dev
 *                       (crates/tikun-cpu/src/lib.rs:117-122)
 *   tk_apply_pointwise  Tier 2 over the leaves with the scale at scale_dev
 *                       (NULL: no clipping)
 * The caller may all-reduce *sumsq_dev between the first two. */
TK_API int tk_grad_sumsq(const tk_leaf* leaves, size_t n_leaves, double* sumsq_dev, void* stream);
TK_API int tk_clip_scale(const double* sumsq_dev, float max_norm, float* scale_dev, void* stream);
TK_API int tk_apply_pointwise(const tk_leaf* leaves, size_t n_leaves, int32_t kind,
                       const tk_hparams* hp, uint64_t step, const float* scale_dev,
                       void* stream);

/* ---------------------------------------------------------------------- */
/* Newton-Schulz (Muon)                                                    */
/* ---------------------------------------------------------------------- */

/* TensorEngine::polar_step (crates/tikun-cpu/src/tensor_engine.rs:12-77) in
 * place on a row-major rows x cols matrix of dtype TK_F32 or TK_BF16:
 * transpose when rows > cols, divide by max(||X||_F, 1e-7), then `steps`
 * iterations of A = X X^T, B = b A + c A A, X = a X + B X with
 * (a, b, c) = (3.4445, -4.7750, 2.0315).  The GEMMs run on the tensor cores
 * with TK_NS_F16 or TK_NS_BF16 operands and f32 accumulation.  Device or host
 * pointer; returns after the result is in place (newton_schulz_2d_ffi,
 * crates/tikun-py/src/lib.rs:224-237). */
TK_API int tk_newton_schulz_2d(void* matrix, int64_t rows, int64_t cols, int32_t steps,
                               int32_t dtype, int32_t precision, void* stream);

/* TensorEngine::polar_batched (tensor_engine.rs:79-96): num_heads contiguous
 * head_dim_out x head_dim_in matrices (newton_schulz_3d_ffi,
 * crates/tikun-py/src/lib.rs:239-254). */
TK_API int tk_newton_schulz_3d(void* tensor, int64_t num_heads, int64_t head_dim_out,
                               int64_t head_dim_in, int32_t steps, int32_t dtype,
                               int32_t precision, void* stream);

/* One Muon leaf: heads (0 or 1 for a matrix) contiguous rows x cols matrices
 * of parameters p, gradients g and f32 momentum: device memory, or (for
 * tk_muon_step only) host memory. */
typedef struct {
  void* p;
  const void* g;
  float* momentum;
  int64_t heads;
  int64_t rows;
  int64_t cols;
  int32_t p_dtype; /* TK_F32 or TK_BF16 */
  int32_t g_dtype; /* TK_F32 or TK_BF16 */
} tk_muon_leaf;

typedef struct {
  double lr;         /* learning rate */
  double momentum;   /* mu; (1 - mu) is formed in double, then rounded to f32 */
  int32_t nesterov;  /* 1: Newton-Schulz of mu*buf + (1-mu)*g, 0: of buf */
  int32_t ns_steps;  /* Newton-Schulz iterations (5) */
  int32_t precision; /* TK_NS_F16 or TK_NS_BF16 */
} tk_muon_hparams;

/* The MuonND update of every 2-D (and head-batched) leaf
 * (python/tikun/muon_nd.py:104-126, :129-160):
 *   buf = mu*buf + (1-mu)*g;  U = mu*buf + (1-mu)*g (Nesterov) or buf;
 *   U = NS(U);  p = p - lr*sqrt(max(1, rows/cols))*U
 * fused into one prologue kernel pass, the tensor-core iteration, and the
 * parameter update in the last GEMM's epilogue.  Same-shape matrices are
 * batched.  Device leaves: stream-ordered, does not wait; a kernel that gives
 * up on a bounded wait sets the device status word (tk_device_status).
 * Host leaves (all leaves of one call on one side; pinned memory overlaps
 * best), the reference's calling convention (muon_nd.py keeps momentum in
 * NumPy arrays): whole matrices stream through three device slots of
 * TIKUN_MUON_STAGE_MB (default 2048) -- g, momentum and p in, p and momentum
 * out -- overlapping both copy directions with the tensor-core work, and the
 * call returns when the results are back in host memory (TK_ERR_DEVICE if a
 * kernel gave up on a bounded wait). */
TK_API int tk_muon_step(const tk_muon_leaf* leaves, size_t n_leaves,
                        const tk_muon_hparams* hp, void* stream);

/* Waits for the device, then reads and clears its status word (0: no kernel
 * reported a problem). */
TK_API int tk_device_status(int* status_out);

/* tk_muon_step for a Muon group sharded by matrix across GPUs: the final
 * Newton-Schulz GEMM's epilogue stores each updated parameter both locally
 * and into n_peers (<= 7) other GPUs' copies at byte offset peer_deltas[i]
 * (a multiple of 16) from the local address (peer memory mapped with
 * tk_ipc_import), so the
 * parameter exchange overlaps the tensor-core work.  The stores are visible
 * system-wide when the kernels end; order the peers' reads after them with a
 * cross-GPU barrier (an all-reduce).  No reference counterpart: the
 * reference's Muon (python/tikun/muon_nd.py:94-160) is single-process. */
TK_API int tk_muon_step_peers(const tk_muon_leaf* leaves, size_t n_leaves,
                              const tk_muon_hparams* hp, const int64_t* peer_deltas, int n_peers,
                              void* stream);

/* The same exchange overlapped with the next batch's tensor-core work: shape
 * groups run largest first, and after each batch of matrices finishes, a copy
 * kernel on a side stream -- on SMs the Newton-Schulz GEMMs leave free
 * (TIKUN_MUON_COPY_SMS, default 16) -- loads each parameter once and stores
 * it into every peer's copy over NVLink, while the next batch computes.  With
 * TIKUN_MUON_COPY_ENGINE=1 the copy engines do it instead (one stream per
 * peer).  The caller's stream waits for every copy before the call's work
 * completes. */
TK_API int tk_muon_step_copy(const tk_muon_leaf* leaves, size_t n_leaves,
                             const tk_muon_hparams* hp, const int64_t* peer_deltas, int n_peers,
                             void* stream);

/* tk_muon_step_copy whose copies may still be running when the call's other
 * work completes -- for a step issued in several calls (a layer at a time in
 * backward order): the copies of every call run in order on the device's copy
 * stream(s), and tk_muon_copy_join makes `stream` wait for all of them. */
TK_API int tk_muon_step_copy_deferred(const tk_muon_leaf* leaves, size_t n_leaves,
                                      const tk_muon_hparams* hp, const int64_t* peer_deltas,
                                      int n_peers, void* stream);
TK_API int tk_muon_copy_join(void* stream);

/* tk_apply_pointwise for ZeRO-1 without a separate all-gather: the updated
 * parameters of these leaves are also stored into n_peers (<= 7) other GPUs'
 * copies of the same layout, at byte offset peer_deltas[i] from each local
 * parameter address (peer memory mapped into this process, tk_ipc_import);
 * each delta must be a multiple of 16 bytes (TK_ERR_INVALID otherwise).
 * The stores are made visible system-wide before the kernel ends; a caller
 * orders the peers' later reads after it with any cross-GPU barrier (an
 * all-reduce).  Device leaves only. */
TK_API int tk_apply_pointwise_peers(const tk_leaf* leaves, size_t n_leaves, int32_t kind,
                                    const tk_hparams* hp, uint64_t step, const float* scale_dev,
                                    const int64_t* peer_deltas, int n_peers, void* stream);

/* CUDA IPC for the peer copies: tk_ipc_export writes the 64-byte handle of
 * the device allocation holding ptr and ptr's offset in it; another process
 * maps it with tk_ipc_import (returning the address of the same byte) and
 * unmaps it with tk_ipc_close. */
TK_API int tk_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out);
TK_API int tk_ipc_import(const void* handle, uint64_t offset, void** ptr_out);
TK_API int tk_ipc_close(void* ptr);

/* ---------------------------------------------------------------------- */
/* ZeRO-1 over NCCL (one process per GPU)                                  */
/* ---------------------------------------------------------------------- */

/* The multi-GPU form of tk_step_buffers (the reference's step_fast_buffers,
 * tikun-py/src/lib.rs:155-222, has no multi-GPU counterpart; this follows
 * the sharding of its arena, crates/tikun-core/src/arena.rs:34-103).  Every
 * rank holds the full f32 parameter and gradient arenas, leaf i at element
 * offset leaf_offsets[i] with leaf_sizes[i] elements (ascending, disjoint;
 * padding between leaves is never touched).  Rank r of W owns elements
 * [r*n/W, (r+1)*n/W) -- n_elems must be a multiple of 16*W -- and keeps the
 * optimizer state for those only.  tk_shard_step: Tier 1 on the owned
 * elements, one f64 ncclAllReduce, the clip scale, Tier 2 on the owned
 * elements, then the exchange of the updated parameters:
 *   TK_SHARD_PEERS      the update kernel also stores them into every other
 *                       rank's arena (CUDA IPC mappings; all ranks on one
 *                       node, W <= 8) and an 8-byte all-reduce closes the
 *                       step;
 *   TK_SHARD_COPY       the update runs in chunks of ~4M elements and the copy
 *                       engines copy each finished chunk into every other
 *                       rank's arena (one stream per peer, CUDA IPC), then
 *                       an 8-byte all-reduce closes the step;
 *   TK_SHARD_ALLGATHER  an in-place ncclAllGather follows the update.
 * All calls are collective over nccl_comm (an ncclComm_t; from PyTorch,
 * ProcessGroupNCCL._comm_ptr()), made on the communicator's device, in the
 * same order on every rank.  clip_scale_out (host, may be NULL) receives the
 * step's clip scale (1 without clipping) and makes the call synchronous.
 * NCCL is resolved at run time from the libnccl.so.2 loaded in the process. */
typedef struct tk_shard tk_shard;
enum { TK_SHARD_ALLGATHER = 0, TK_SHARD_PEERS = 1, TK_SHARD_COPY = 2 };

/* tk_step_buffers for one rank's share of a PyTree split across the ranks of
 * nccl_comm (any split: whole leaves or pieces of leaves, each element on one
 * rank): the Tier-1 f64 sum is all-reduced over the communicator before the
 * clip scale is formed, so every rank clips with the global norm.  Leaves may
 * be device or host buffers as for tk_step_buffers (pinned host leaves stream
 * through the copy engines).  Collective when max_norm > 0; a rank holding no
 * elements still calls it.  No parameter exchange: ranks whose leaves live in
 * one shared host arena need none. */
TK_API int tk_step_buffers_sharded(const tk_leaf* leaves, size_t n_leaves, int32_t kind,
                                   const tk_hparams* hp, uint64_t step, float max_norm,
                                   float* clip_scale_out, void* nccl_comm, void* stream);
#define TK_NCCL_ID_BYTES 128

TK_API int tk_shard_init(void* nccl_comm, float* p_arena, const float* g_arena, uint64_t n_elems,
                         const uint64_t* leaf_offsets, const uint64_t* leaf_sizes,
                         size_t n_leaves, int32_t kind, int32_t exchange, void* stream,
                         tk_shard** out);
TK_API int tk_shard_step(tk_shard* shard, const tk_hparams* hp, uint64_t step, float max_norm,
                         float* clip_scale_out, void* stream);
/* The owned element range and its optimizer state (v is NULL unless AdamW). */
TK_API int tk_shard_info(const tk_shard* shard, uint64_t* lo, uint64_t* hi, float** m, float** v);
/* Collective; waits for the stream, then unmaps the peers and frees the state. */
TK_API int tk_shard_destroy(tk_shard* shard, void* stream);

/* Muon across the ranks of nccl_comm (no reference counterpart; the
 * reference's Muon, python/tikun/muon_nd.py:94-160, is single-process).
 * tk_muon_layout assigns whole matrices to ranks -- longest-processing-time
 * bin-packing on their dense Newton-Schulz FLOPs 5(4 m^2 n + 2 m^3), largest
 * first (ties: lower index), each to the least-loaded rank (ties: lower rank)
 * -- and lays the parameters out owner-major: rank r's matrices, in index
 * order at 64-element-aligned offsets, in [r*extent, (r+1)*extent).  The
 * caller allocates the parameter arena (world * extent elements of p_dtype,
 * replicated on every rank) and tk_muon_shard_init keeps momentum for the
 * rank's own matrices.  tk_muon_shard_step reads grads[i] (device, g_dtype)
 * of the rank's own matrices, runs the Muon step on them and exchanges the
 * parameters (TK_SHARD_COPY: a copy kernel beside the next batch;
 * TK_SHARD_PEERS: the last GEMM's epilogue; TK_SHARD_ALLGATHER: an
 * ncclAllGather of the arena).  Calls other than tk_muon_layout are
 * collective over nccl_comm. */
typedef struct tk_muon_shard tk_muon_shard;
TK_API int tk_muon_layout(size_t n_mats, const int64_t* rows, const int64_t* cols, int world,
                          int32_t* owner_out, uint64_t* offset_out, uint64_t* extent_out);
TK_API int tk_muon_shard_init(void* nccl_comm, size_t n_mats, const int64_t* rows,
                              const int64_t* cols, void* p_arena, int32_t p_dtype,
                              const tk_muon_hparams* hp, int32_t exchange, void* stream,
                              tk_muon_shard** out);
TK_API int tk_muon_shard_info(const tk_muon_shard* shard, int32_t* owner_out, uint64_t* offset_out,
                              uint64_t* extent_out);
TK_API int tk_muon_shard_step(tk_muon_shard* shard, const void* const* grads, int32_t g_dtype,
                              void* stream);
TK_API int tk_muon_shard_destroy(tk_muon_shard* shard, void* stream);

/* A communicator without PyTorch: rank 0 makes the id (TK_NCCL_ID_BYTES),
 * every rank passes the same bytes to tk_nccl_comm_init. */
TK_API int tk_nccl_unique_id(void* id_out);
TK_API int tk_nccl_comm_init(const void* id, int world, int rank, void** comm_out);
TK_API int tk_nccl_comm_destroy(void* comm);

/* Failure detection for a communicator (no reference counterpart: the
 * reference is single-process).
 *   tk_nccl_comm_async_error  *result_out = the communicator's asynchronous
 *                             error (an ncclResult_t; 0 = none)
 *   tk_nccl_comm_abort        ncclCommAbort: ends its collectives, including
 *                             kernels waiting for a peer that is gone, and
 *                             releases it (use instead of _destroy)
 *   tk_stream_wait_deadline   waits on the host for the work on `stream`,
 *                             at most timeout_ms, polling the communicator's
 *                             asynchronous error when `comm` is given; on an
 *                             error or at the deadline it aborts `comm` (if
 *                             given) and returns TK_ERR_DEVICE.  Results of
 *                             that step are then not valid.  Give only a
 *                             communicator this caller owns (PyTorch aborts
 *                             its own through its watchdog). */
TK_API int tk_nccl_comm_async_error(void* comm, int32_t* result_out);
TK_API int tk_nccl_comm_abort(void* comm);
TK_API int tk_stream_wait_deadline(void* stream, int32_t timeout_ms, void* comm);

/* Leaves `sms` SMs of every device free of pointwise (Tier 1 / Tier 2) CTAs,
 * so that kernels launched concurrently on other streams -- NCCL all-gathers
 * overlapping a sharded update -- can run at the same time.  Process-wide;
 * 0 (the default) lets the pointwise kernels use every SM. */
TK_API int tk_set_reserved_sms(int sms);

/* ---------------------------------------------------------------------- */
/* measurement                                                             */
/* ---------------------------------------------------------------------- */

/* While set (two cudaEvent_t handles), every step call made by this thread
 * records start_event on its stream just before its first Tier-2 (update)
 * launch and stop_event just after its last, so a caller can time the update
 * kernels alone inside a running loop.  Pass NULLs to clear. */
TK_API int tk_set_update_events(void* start_event, void* stop_event);

#ifdef __cplusplus
}
#endif
#endif /* TIKUN_CUDA_H */
