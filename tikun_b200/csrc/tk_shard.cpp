// ZeRO-1 pointwise step over NCCL: the multi-GPU form of step_fast_buffers.
//
// Every rank holds the full f32 parameter and gradient arenas (leaf i at
// element offset offsets[i], sizes[i] elements -- the LayoutPlan layout of
// crates/tikun-core/src/arena.rs:34-57).  Rank r of W owns the contiguous
// element range [r*n/W, (r+1)*n/W), keeps optimizer state for it only, and
// per step
//   1. Tier 1 on its range -> one f64, ncclAllReduce(sum) -> the clip scale
//      (crates/tikun-cpu/src/lib.rs:79-125 over the global sum);
//   2. Tier 2 on its range (lib.rs:144-428), and
//   3. the exchange of the updated parameters: either the update kernel
//      stores them into every peer's arena over NVLink (CUDA IPC mappings,
//      TK_SHARD_PEERS) and an 8-byte all-reduce closes the step, or an
//      in-place ncclAllGather follows the update (TK_SHARD_ALLGATHER).
// The update is element-wise, so every rank ends with the parameters the
// single-GPU step produces (the f64 sum order of the norm aside).
//
// NCCL is not linked: its entry points are resolved at run time from the
// libnccl.so.2 already loaded in the process (the one that made the caller's
// communicator, e.g. PyTorch's), else from the system library.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "tk_internal.h"

namespace tk {
namespace {

struct Nccl {
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*CommCount)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*CommUserRank)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*CommCuDevice)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

int nccl(const Nccl** out) {
  static Nccl fns;
  static int status = -1;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (status < 0) {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    status = 1;
    if (h != nullptr) {
      bool ok = true;
      auto sym = [&](auto& fn, const char* name) {
        void* p = dlsym(h, name);
        if (p == nullptr) ok = false;
        fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(p);
      };
      sym(fns.AllReduce, "ncclAllReduce");
      sym(fns.AllGather, "ncclAllGather");
      sym(fns.CommCount, "ncclCommCount");
      sym(fns.CommUserRank, "ncclCommUserRank");
      sym(fns.CommCuDevice, "ncclCommCuDevice");
      sym(fns.GetUniqueId, "ncclGetUniqueId");
      sym(fns.CommInitRank, "ncclCommInitRank");
      sym(fns.CommDestroy, "ncclCommDestroy");
      sym(fns.CommAbort, "ncclCommAbort");
      sym(fns.CommGetAsyncError, "ncclCommGetAsyncError");
      sym(fns.GetErrorString, "ncclGetErrorString");
      if (ok) status = 0;
    }
  }
  if (status != 0) return set_error(TK_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
  *out = &fns;
  return TK_OK;
}

#define TK_NCCL_TRY(N, expr)                                                               \
  do {                                                                                     \
    ncclResult_t _r = (expr);                                                              \
    if (_r != ncclSuccess)                                                                 \
      return set_error(TK_ERR_CUDA, "%s failed: %s", #expr, (N)->GetErrorString(_r));      \
  } while (0)

// What one rank tells the others at init.
struct PeerInfo {
  unsigned char handle[64];
  uint64_t offset;   // byte offset of the arena in its allocation
  uint64_t n_elems;  // arena length (must agree)
  int64_t exchange;  // exchange mode (must agree)
};

}  // namespace

int nccl_allreduce_sum_f64(double* buf, size_t count, void* comm, cudaStream_t s) {
  const Nccl* N = nullptr;
  TK_TRY(nccl(&N));
  TK_NCCL_TRY(N, N->AllReduce(buf, buf, count, ncclFloat64, ncclSum, static_cast<ncclComm_t>(comm), s));
  return TK_OK;
}

}  // namespace tk

using namespace tk;

struct tk_shard {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, device = 0;
  int32_t kind = TK_ADAMW, exchange = TK_SHARD_ALLGATHER;
  float* p = nullptr;
  uint64_t n = 0, lo = 0, hi = 0;
  float* m = nullptr;  // owned range only
  float* v = nullptr;
  double* sumsq = nullptr;  // [0] norm sum, [1] barrier word
  float* scale = nullptr;
  std::vector<tk_leaf> leaves;  // owned segments of the leaves
  std::vector<void*> peer_ptrs;
  std::vector<int64_t> deltas;
  // TK_SHARD_COPY: the owned range in chunks, each updated then copied to
  // every peer by the copy engines (one stream per peer)
  std::vector<std::vector<tk_leaf>> chunk_leaves;
  std::vector<std::pair<uint64_t, uint64_t>> chunk_range;
  std::vector<cudaEvent_t> chunk_done;
  std::vector<cudaStream_t> peer_streams;
  std::vector<cudaEvent_t> peer_done;
};

extern "C" {

int tk_nccl_unique_id(void* id_out) {
  clear_error();
  if (id_out == nullptr) return set_error(TK_ERR_INVALID, "id_out is NULL");
  const Nccl* N = nullptr;
  TK_TRY(nccl(&N));
  ncclUniqueId id;
  TK_NCCL_TRY(N, N->GetUniqueId(&id));
  static_assert(sizeof(id) == TK_NCCL_ID_BYTES, "NCCL unique ids are 128 bytes");
  std::memcpy(id_out, &id, sizeof(id));
  return TK_OK;
}

int tk_nccl_comm_init(const void* id, int world, int rank, void** comm_out) {
  clear_error();
  if (id == nullptr || comm_out == nullptr) return set_error(TK_ERR_INVALID, "null argument");
  if (world < 1 || rank < 0 || rank >= world)
    return set_error(TK_ERR_INVALID, "rank %d of world %d", rank, world);
  const Nccl* N = nullptr;
  TK_TRY(nccl(&N));
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclComm_t c = nullptr;
  TK_NCCL_TRY(N, N->CommInitRank(&c, world, uid, rank));
  *comm_out = c;
  return TK_OK;
}

int tk_nccl_comm_destroy(void* comm) {
  clear_error();
  if (comm == nullptr) return TK_OK;
  const Nccl* N = nullptr;
  TK_TRY(nccl(&N));
  TK_NCCL_TRY(N, N->CommDestroy(static_cast<ncclComm_t>(comm)));
  return TK_OK;
}

int tk_nccl_comm_async_error(void* comm, int32_t* result_out) {
  clear_error();
  if (comm == nullptr || result_out == nullptr) return set_error(TK_ERR_INVALID, "null argument");
  const Nccl* N = nullptr;
  TK_TRY(nccl(&N));
  ncclResult_t r = ncclSuccess;
  TK_NCCL_TRY(N, N->CommGetAsyncError(static_cast<ncclComm_t>(comm), &r));
  *result_out = (int32_t)r;
  return TK_OK;
}

int tk_nccl_comm_abort(void* comm) {
  clear_error();
  if (comm == nullptr) return TK_OK;
  const Nccl* N = nullptr;
  TK_TRY(nccl(&N));
  TK_NCCL_TRY(N, N->CommAbort(static_cast<ncclComm_t>(comm)));
  return TK_OK;
}

int tk_stream_wait_deadline(void* stream, int32_t timeout_ms, void* comm) {
  clear_error();
  if (timeout_ms < 0) return set_error(TK_ERR_INVALID, "negative timeout %d ms", timeout_ms);
  const Nccl* N = nullptr;
  if (comm != nullptr) TK_TRY(nccl(&N));
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t e = cudaStreamQuery(s);
    if (e == cudaSuccess) return TK_OK;
    if (e != cudaErrorNotReady) return cuda_error(e, "cudaStreamQuery");
    if (N != nullptr) {
      ncclResult_t r = ncclSuccess;
      const ncclResult_t q = N->CommGetAsyncError(c, &r);
      if (q != ncclSuccess || (r != ncclSuccess && r != ncclInProgress)) {
        const char* why = N->GetErrorString(q != ncclSuccess ? q : r);
        N->CommAbort(c);
        return set_error(TK_ERR_DEVICE, "the communicator reported an error (%s) and was aborted",
                         why);
      }
    }
    const auto waited = std::chrono::duration_cast<std::chrono::milliseconds>(
        std::chrono::steady_clock::now() - t0);
    if (waited.count() > timeout_ms) {
      if (N != nullptr) {
        N->CommAbort(c);
        return set_error(TK_ERR_DEVICE,
                         "the stream's work did not finish within %d ms; the communicator was "
                         "aborted",
                         timeout_ms);
      }
      return set_error(TK_ERR_DEVICE, "the stream's work did not finish within %d ms",
                       timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

// Both free functions keep the thread's error message: they run on failure
// paths, and closing a peer mapping through the public entry point clears it.
static void shard_free(tk_shard* sh) {
  const std::string err = tk_last_error();
  for (cudaEvent_t e : sh->chunk_done) cudaEventDestroy(e);
  for (cudaEvent_t e : sh->peer_done) cudaEventDestroy(e);
  for (cudaStream_t q : sh->peer_streams) cudaStreamDestroy(q);
  for (void* p : sh->peer_ptrs) tk_ipc_close(p);
  if (sh->m) cudaFree(sh->m);
  if (sh->v) cudaFree(sh->v);
  if (sh->sumsq) cudaFree(sh->sumsq);
  delete sh;
  if (!err.empty()) set_error(TK_OK, "%s", err.c_str());
}

int tk_shard_init(void* nccl_comm, float* p_arena, const float* g_arena, uint64_t n_elems,
                  const uint64_t* leaf_offsets, const uint64_t* leaf_sizes, size_t n_leaves,
                  int32_t kind, int32_t exchange, void* stream, tk_shard** out) {
  clear_error();
  if (out == nullptr) return set_error(TK_ERR_INVALID, "out is NULL");
  *out = nullptr;
  if (nccl_comm == nullptr || p_arena == nullptr || g_arena == nullptr)
    return set_error(TK_ERR_INVALID, "null communicator or arena");
  if (n_leaves > 0 && (leaf_offsets == nullptr || leaf_sizes == nullptr))
    return set_error(TK_ERR_INVALID, "null leaf offsets or sizes");
  if (kind != TK_ADAMW && kind != TK_LION && kind != TK_SGD && kind != TK_CUSTOM)
    return set_error(TK_ERR_INVALID, "unknown optimizer kind %d", kind);
  if (exchange != TK_SHARD_ALLGATHER && exchange != TK_SHARD_PEERS && exchange != TK_SHARD_COPY)
    return set_error(TK_ERR_INVALID, "unknown exchange mode %d", exchange);
  const Nccl* N = nullptr;
  TK_TRY(nccl(&N));
  ncclComm_t comm = static_cast<ncclComm_t>(nccl_comm);
  int world = 0, rank = 0, cdev = 0, dev = 0;
  TK_NCCL_TRY(N, N->CommCount(comm, &world));
  TK_NCCL_TRY(N, N->CommUserRank(comm, &rank));
  TK_NCCL_TRY(N, N->CommCuDevice(comm, &cdev));
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (cdev != dev)
    return set_error(TK_ERR_INVALID, "the communicator is on device %d, the current device is %d",
                     cdev, dev);
  if (exchange != TK_SHARD_ALLGATHER && world > 1 + kMaxPeers)
    return set_error(TK_ERR_UNSUPPORTED, "peer stores reach at most %d peers", kMaxPeers);
  if (n_elems == 0 || n_elems % (16ull * (uint64_t)world) != 0)
    return set_error(TK_ERR_INVALID,
                     "arena of %llu elements is not a positive multiple of 16 x %d ranks",
                     (unsigned long long)n_elems, world);
  for (size_t i = 0; i < n_leaves; ++i)
    if (leaf_offsets[i] > n_elems || leaf_sizes[i] > n_elems - leaf_offsets[i] ||
        (i > 0 && leaf_offsets[i] < leaf_offsets[i - 1] + leaf_sizes[i - 1]))
      return set_error(TK_ERR_INVALID, "leaf %zu [%llu, +%llu) is outside the arena or "
                       "overlaps the previous leaf", i, (unsigned long long)leaf_offsets[i],
                       (unsigned long long)leaf_sizes[i]);
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  tk_shard* sh = new tk_shard();
  sh->comm = comm;
  sh->rank = rank;
  sh->world = world;
  sh->device = dev;
  sh->kind = kind;
  sh->exchange = exchange;
  sh->p = p_arena;
  sh->n = n_elems;
  const uint64_t per = n_elems / (uint64_t)world;
  sh->lo = per * (uint64_t)rank;
  sh->hi = sh->lo + per;
  auto fail = [&](int code) {
    shard_free(sh);
    return code;
  };
  const size_t state_bytes = sizeof(float) * (size_t)per;
  if (cudaMalloc(&sh->m, state_bytes) != cudaSuccess ||
      (kind == TK_ADAMW && cudaMalloc(&sh->v, state_bytes) != cudaSuccess) ||
      cudaMalloc(&sh->sumsq, 4 * sizeof(double)) != cudaSuccess) {
    cudaGetLastError();
    return fail(set_error(TK_ERR_ALLOC, "could not allocate %zu bytes of optimizer state",
                          state_bytes * (kind == TK_ADAMW ? 2 : 1)));
  }
  sh->scale = reinterpret_cast<float*>(sh->sumsq + 2);
  if (cudaMemsetAsync(sh->m, 0, state_bytes, s) != cudaSuccess ||
      (sh->v && cudaMemsetAsync(sh->v, 0, state_bytes, s) != cudaSuccess) ||
      cudaMemsetAsync(sh->sumsq, 0, 4 * sizeof(double), s) != cudaSuccess)
    return fail(set_error(TK_ERR_CUDA, "could not clear the optimizer state"));
  // owned segments of every leaf
  for (size_t i = 0; i < n_leaves; ++i) {
    const uint64_t a = std::max(leaf_offsets[i], sh->lo);
    const uint64_t b = std::min(leaf_offsets[i] + leaf_sizes[i], sh->hi);
    if (a >= b) continue;
    tk_leaf L;
    std::memset(&L, 0, sizeof(L));
    L.p = p_arena + a;
    L.g = g_arena + a;
    L.m = sh->m + (a - sh->lo);
    L.v = sh->v ? sh->v + (a - sh->lo) : nullptr;
    L.n = b - a;
    L.p_dtype = TK_F32;
    L.g_dtype = TK_F32;
    sh->leaves.push_back(L);
  }
  // every rank's arena description, gathered through NCCL
  PeerInfo mine;
  std::memset(&mine, 0, sizeof(mine));
  mine.n_elems = n_elems;
  mine.exchange = exchange;
  if (exchange != TK_SHARD_ALLGATHER && world > 1) {
    int st = tk_ipc_export(p_arena, mine.handle, &mine.offset);
    if (st != TK_OK) return fail(st);
  }
  std::vector<PeerInfo> all((size_t)world);
  void* buf = nullptr;
  if (cudaMalloc(&buf, sizeof(PeerInfo) * (size_t)(world + 1)) != cudaSuccess) {
    cudaGetLastError();
    return fail(set_error(TK_ERR_ALLOC, "could not allocate the init exchange buffer"));
  }
  char* gathered = static_cast<char*>(buf) + sizeof(PeerInfo);
  int st = TK_OK;
  ncclResult_t nr = ncclSuccess;
  if (cudaMemcpyAsync(buf, &mine, sizeof(mine), cudaMemcpyHostToDevice, s) != cudaSuccess)
    st = set_error(TK_ERR_CUDA, "init exchange copy failed");
  if (st == TK_OK) {
    nr = N->AllGather(buf, gathered, sizeof(PeerInfo), ncclUint8, comm, s);
    if (nr != ncclSuccess)
      st = set_error(TK_ERR_CUDA, "ncclAllGather of the arena descriptions failed: %s",
                     N->GetErrorString(nr));
  }
  if (st == TK_OK &&
      (cudaMemcpyAsync(all.data(), gathered, sizeof(PeerInfo) * (size_t)world,
                       cudaMemcpyDeviceToHost, s) != cudaSuccess ||
       cudaStreamSynchronize(s) != cudaSuccess))
    st = set_error(TK_ERR_CUDA, "init exchange read-back failed");
  cudaFree(buf);
  if (st != TK_OK) return fail(st);
  for (int r = 0; r < world; ++r)
    if (all[(size_t)r].n_elems != n_elems || all[(size_t)r].exchange != exchange)
      return fail(set_error(TK_ERR_INVALID,
                            "rank %d has an arena of %llu elements and exchange %lld; this rank "
                            "%llu and %d", r, (unsigned long long)all[(size_t)r].n_elems,
                            (long long)all[(size_t)r].exchange, (unsigned long long)n_elems,
                            exchange));
  if (exchange != TK_SHARD_ALLGATHER)
    for (int r = 0; r < world; ++r) {
      if (r == rank) continue;
      void* ptr = nullptr;
      int ist = tk_ipc_import(all[(size_t)r].handle, all[(size_t)r].offset, &ptr);
      if (ist != TK_OK) return fail(ist);
      sh->peer_ptrs.push_back(ptr);
      sh->deltas.push_back((int64_t)((char*)ptr - (char*)p_arena));
      if (sh->deltas.back() % 16 != 0)
        return fail(set_error(TK_ERR_UNSUPPORTED,
                              "rank %d's arena is not at the same address modulo 16 bytes as "
                              "this rank's; use TK_SHARD_ALLGATHER", r));
    }
  if (exchange == TK_SHARD_COPY && world > 1) {
    // chunks of about kChunkElems, on 16-element boundaries
    constexpr uint64_t kChunkElems = 4ull << 20;
    const uint64_t k = std::max<uint64_t>(1, (per + kChunkElems - 1) / kChunkElems);
    const uint64_t len = ((per + k - 1) / k + 15) / 16 * 16;
    for (uint64_t a = sh->lo; a < sh->hi; a += len) {
      const uint64_t b = std::min(a + len, sh->hi);
      std::vector<tk_leaf> cl;
      for (const tk_leaf& L : sh->leaves) {
        const uint64_t l0 = (uint64_t)(static_cast<float*>(L.p) - p_arena), l1 = l0 + L.n;
        const uint64_t x = std::max(l0, a), y = std::min(l1, b);
        if (x >= y) continue;
        tk_leaf c = L;
        c.p = static_cast<float*>(L.p) + (x - l0);
        c.g = static_cast<const float*>(L.g) + (x - l0);
        c.m = L.m + (x - l0);
        c.v = L.v ? L.v + (x - l0) : nullptr;
        c.n = y - x;
        cl.push_back(c);
      }
      sh->chunk_leaves.push_back(cl);
      sh->chunk_range.emplace_back(a, b);
      cudaEvent_t e;
      if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
        return fail(set_error(TK_ERR_CUDA, "could not create the chunk events"));
      sh->chunk_done.push_back(e);
    }
    for (size_t j = 0; j < sh->peer_ptrs.size(); ++j) {
      cudaStream_t q;
      cudaEvent_t e;
      if (cudaStreamCreateWithFlags(&q, cudaStreamNonBlocking) != cudaSuccess)
        return fail(set_error(TK_ERR_CUDA, "could not create the copy streams"));
      sh->peer_streams.push_back(q);
      if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
        return fail(set_error(TK_ERR_CUDA, "could not create the copy events"));
      sh->peer_done.push_back(e);
    }
  }
  *out = sh;
  return TK_OK;
}

int tk_shard_step(tk_shard* sh, const tk_hparams* hp, uint64_t step, float max_norm,
                  float* clip_scale_out, void* stream) {
  clear_error();
  if (sh == nullptr || hp == nullptr) return set_error(TK_ERR_INVALID, "null shard or hparams");
  const Nccl* N = nullptr;
  TK_TRY(nccl(&N));
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev != sh->device)
    return set_error(TK_ERR_INVALID, "the shard lives on device %d, the current device is %d",
                     sh->device, dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const tk_leaf* L = sh->leaves.empty() ? nullptr : sh->leaves.data();
  const size_t nl = sh->leaves.size();
  const bool clip = max_norm > 0.f;
  const bool peers = sh->exchange == TK_SHARD_PEERS && sh->world > 1;
  const bool copy = sh->exchange == TK_SHARD_COPY && sh->world > 1;
  NvtxRange range("tikun/shard_step");
  if (clip) {
    if (nl > 0) TK_TRY(tk_grad_sumsq(L, nl, sh->sumsq, s));
    else TK_CUDA_TRY(cudaMemsetAsync(sh->sumsq, 0, sizeof(double), s));
    TK_NCCL_TRY(N, N->AllReduce(sh->sumsq, sh->sumsq, 1, ncclFloat64, ncclSum, sh->comm, s));
    TK_TRY(tk_clip_scale(sh->sumsq, max_norm, sh->scale, s));
  } else if (peers || copy) {
    // orders this step's stores into the peers' arenas after their reads of
    // the previous parameters (the norm all-reduce does it when clipping)
    TK_NCCL_TRY(N, N->AllReduce(sh->sumsq + 1, sh->sumsq + 1, 1, ncclFloat64, ncclSum, sh->comm, s));
  }
  const float* scale = clip ? sh->scale : nullptr;
  TK_TRY(record_update_event(true, s));
  if (copy) {
    for (size_t c = 0; c < sh->chunk_leaves.size(); ++c) {
      const std::vector<tk_leaf>& cl = sh->chunk_leaves[c];
      if (!cl.empty()) TK_TRY(tk_apply_pointwise(cl.data(), cl.size(), sh->kind, hp, step, scale, s));
      TK_CUDA_TRY(cudaEventRecord(sh->chunk_done[c], s));
      const uint64_t a = sh->chunk_range[c].first, b = sh->chunk_range[c].second;
      for (size_t j = 0; j < sh->peer_streams.size(); ++j) {
        TK_CUDA_TRY(cudaStreamWaitEvent(sh->peer_streams[j], sh->chunk_done[c], 0));
        TK_CUDA_TRY(cudaMemcpyAsync(reinterpret_cast<char*>(sh->p + a) + sh->deltas[j], sh->p + a,
                                    (b - a) * sizeof(float), cudaMemcpyDeviceToDevice,
                                    sh->peer_streams[j]));
      }
    }
    TK_TRY(record_update_event(false, s));
    for (size_t j = 0; j < sh->peer_streams.size(); ++j) {
      TK_CUDA_TRY(cudaEventRecord(sh->peer_done[j], sh->peer_streams[j]));
      TK_CUDA_TRY(cudaStreamWaitEvent(s, sh->peer_done[j], 0));
    }
    // every peer's copies into this arena have landed once this completes
    TK_NCCL_TRY(N, N->AllReduce(sh->sumsq + 1, sh->sumsq + 1, 1, ncclFloat64, ncclSum, sh->comm, s));
  } else if (peers) {
    if (nl > 0)
      TK_TRY(tk_apply_pointwise_peers(L, nl, sh->kind, hp, step, scale, sh->deltas.data(),
                                      (int)sh->deltas.size(), s));
    TK_TRY(record_update_event(false, s));
    // every peer has finished writing into this arena once this completes
    TK_NCCL_TRY(N, N->AllReduce(sh->sumsq + 1, sh->sumsq + 1, 1, ncclFloat64, ncclSum, sh->comm, s));
  } else {
    if (nl > 0) TK_TRY(tk_apply_pointwise(L, nl, sh->kind, hp, step, scale, s));
    TK_TRY(record_update_event(false, s));
    if (sh->world > 1)
      TK_NCCL_TRY(N, N->AllGather(sh->p + sh->lo, sh->p, sh->hi - sh->lo, ncclFloat32, sh->comm, s));
  }
  if (clip_scale_out != nullptr) {
    if (clip) {
      TK_CUDA_TRY(cudaMemcpyAsync(clip_scale_out, sh->scale, sizeof(float), cudaMemcpyDeviceToHost, s));
      TK_CUDA_TRY(cudaStreamSynchronize(s));
    } else {
      *clip_scale_out = 1.0f;
    }
  }
  return TK_OK;
}

int tk_shard_info(const tk_shard* sh, uint64_t* lo, uint64_t* hi, float** m, float** v) {
  clear_error();
  if (sh == nullptr) return set_error(TK_ERR_INVALID, "shard is NULL");
  if (lo) *lo = sh->lo;
  if (hi) *hi = sh->hi;
  if (m) *m = sh->m;
  if (v) *v = sh->v;
  return TK_OK;
}

int tk_shard_destroy(tk_shard* sh, void* stream) {
  clear_error();
  if (sh == nullptr) return TK_OK;
  int st = TK_OK;
  if (!sh->peer_ptrs.empty()) {
    // no peer may still be writing through a mapping this rank is closing
    const Nccl* N = nullptr;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    st = nccl(&N);
    if (st == TK_OK) {
      ncclResult_t r = N->AllReduce(sh->sumsq + 1, sh->sumsq + 1, 1, ncclFloat64, ncclSum,
                                    sh->comm, s);
      if (r != ncclSuccess)
        st = set_error(TK_ERR_CUDA, "end-of-life barrier failed: %s", N->GetErrorString(r));
      else if (cudaStreamSynchronize(s) != cudaSuccess)
        st = set_error(TK_ERR_CUDA, "end-of-life barrier did not complete");
    }
  } else {
    cudaDeviceSynchronize();
  }
  shard_free(sh);
  return st;
}

}  // extern "C"

// ---------------------------------------------------------------- Muon shards
// Whole matrices are owned by one rank each: longest-processing-time
// bin-packing on their dense Newton-Schulz FLOPs 5(4 m^2 n + 2 m^3) (m = min,
// n = max) -- largest first (ties: lower index), each to the least-loaded rank
// (ties: lower rank) -- and an owner-major parameter arena: rank r's matrices,
// in index order at 64-element-aligned offsets, fill [r*E, (r+1)*E) with the
// extent E equal for every rank.
namespace {

uint64_t ns_flops(int64_t r, int64_t c) {
  const uint64_t m = (uint64_t)std::min(r, c), n = (uint64_t)std::max(r, c);
  return 5ull * (4ull * m * m * n + 2ull * m * m * m);
}

}  // namespace

struct tk_muon_shard {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, device = 0;
  int32_t p_dtype = TK_BF16, exchange = TK_SHARD_COPY;
  tk_muon_hparams hp{};
  char* p = nullptr;  // owner-major arena
  std::vector<int64_t> rows, cols;
  std::vector<int32_t> owner;
  std::vector<uint64_t> offset;
  uint64_t extent = 0;
  std::vector<size_t> mine;
  std::vector<uint64_t> mom_off;  // per own matrix, elements into mom
  float* mom = nullptr;
  double* barrier = nullptr;
  std::vector<void*> peer_ptrs;
  std::vector<int64_t> deltas;
};

extern "C" {

int tk_muon_layout(size_t n_mats, const int64_t* rows, const int64_t* cols, int world,
                   int32_t* owner_out, uint64_t* offset_out, uint64_t* extent_out) {
  clear_error();
  if (world < 1) return set_error(TK_ERR_INVALID, "world %d < 1", world);
  if (n_mats > 0 && (rows == nullptr || cols == nullptr || owner_out == nullptr ||
                     offset_out == nullptr))
    return set_error(TK_ERR_INVALID, "null argument");
  if (extent_out == nullptr) return set_error(TK_ERR_INVALID, "extent_out is NULL");
  for (size_t i = 0; i < n_mats; ++i)
    if (rows[i] <= 0 || cols[i] <= 0)
      return set_error(TK_ERR_INVALID, "matrix %zu has shape %lld x %lld", i,
                       (long long)rows[i], (long long)cols[i]);
  std::vector<size_t> order(n_mats);
  for (size_t i = 0; i < n_mats; ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) {
    return ns_flops(rows[a], cols[a]) > ns_flops(rows[b], cols[b]);
  });
  std::vector<uint64_t> load((size_t)world, 0);
  for (size_t i : order) {
    int best = 0;
    for (int r = 1; r < world; ++r)
      if (load[(size_t)r] < load[(size_t)best]) best = r;
    owner_out[i] = best;
    load[(size_t)best] += ns_flops(rows[i], cols[i]);
  }
  std::vector<uint64_t> cursor((size_t)world, 0);
  for (size_t i = 0; i < n_mats; ++i) {
    const uint64_t sz = (uint64_t)rows[i] * (uint64_t)cols[i];
    offset_out[i] = cursor[(size_t)owner_out[i]];
    cursor[(size_t)owner_out[i]] += (sz + 63) / 64 * 64;
  }
  uint64_t extent = 64;
  for (uint64_t c : cursor) extent = std::max(extent, c);
  extent = (extent + 63) / 64 * 64;
  for (size_t i = 0; i < n_mats; ++i) offset_out[i] += (uint64_t)owner_out[i] * extent;
  *extent_out = extent;
  return TK_OK;
}

static void muon_shard_free(tk_muon_shard* sh) {
  const std::string err = tk_last_error();
  for (void* p : sh->peer_ptrs) tk_ipc_close(p);
  if (sh->mom) cudaFree(sh->mom);
  if (sh->barrier) cudaFree(sh->barrier);
  delete sh;
  if (!err.empty()) set_error(TK_OK, "%s", err.c_str());
}

int tk_muon_shard_init(void* nccl_comm, size_t n_mats, const int64_t* rows, const int64_t* cols,
                       void* p_arena, int32_t p_dtype, const tk_muon_hparams* hp,
                       int32_t exchange, void* stream, tk_muon_shard** out) {
  clear_error();
  if (out == nullptr) return set_error(TK_ERR_INVALID, "out is NULL");
  *out = nullptr;
  if (nccl_comm == nullptr || p_arena == nullptr || hp == nullptr)
    return set_error(TK_ERR_INVALID, "null communicator, arena or hparams");
  if (p_dtype != TK_F32 && p_dtype != TK_BF16)
    return set_error(TK_ERR_INVALID, "parameter dtype %d is not f32 or bf16", p_dtype);
  if (exchange != TK_SHARD_ALLGATHER && exchange != TK_SHARD_PEERS && exchange != TK_SHARD_COPY)
    return set_error(TK_ERR_INVALID, "unknown exchange mode %d", exchange);
  const Nccl* N = nullptr;
  TK_TRY(nccl(&N));
  ncclComm_t comm = static_cast<ncclComm_t>(nccl_comm);
  int world = 0, rank = 0, cdev = 0, dev = 0;
  TK_NCCL_TRY(N, N->CommCount(comm, &world));
  TK_NCCL_TRY(N, N->CommUserRank(comm, &rank));
  TK_NCCL_TRY(N, N->CommCuDevice(comm, &cdev));
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (cdev != dev)
    return set_error(TK_ERR_INVALID, "the communicator is on device %d, the current device is %d",
                     cdev, dev);
  if (exchange != TK_SHARD_ALLGATHER && world > 1 + kMaxPeers)
    return set_error(TK_ERR_UNSUPPORTED, "peer stores reach at most %d peers", kMaxPeers);
  tk_muon_shard* sh = new tk_muon_shard();
  auto fail = [&](int code) {
    muon_shard_free(sh);
    return code;
  };
  sh->comm = comm;
  sh->rank = rank;
  sh->world = world;
  sh->device = dev;
  sh->p_dtype = p_dtype;
  sh->exchange = exchange;
  sh->hp = *hp;
  sh->p = static_cast<char*>(p_arena);
  sh->rows.assign(rows, rows + n_mats);
  sh->cols.assign(cols, cols + n_mats);
  sh->owner.resize(n_mats);
  sh->offset.resize(n_mats);
  int st = tk_muon_layout(n_mats, rows, cols, world, sh->owner.data(), sh->offset.data(),
                          &sh->extent);
  if (st != TK_OK) return fail(st);
  uint64_t mom_elems = 0;
  for (size_t i = 0; i < n_mats; ++i)
    if (sh->owner[i] == rank) {
      sh->mine.push_back(i);
      sh->mom_off.push_back(mom_elems);
      mom_elems += (uint64_t)rows[i] * (uint64_t)cols[i];
    }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMalloc(&sh->barrier, 256) != cudaSuccess ||
      (mom_elems > 0 && cudaMalloc(&sh->mom, sizeof(float) * mom_elems) != cudaSuccess)) {
    cudaGetLastError();
    return fail(set_error(TK_ERR_ALLOC, "could not allocate the Muon momentum"));
  }
  if (cudaMemsetAsync(sh->barrier, 0, 256, s) != cudaSuccess ||
      (sh->mom && cudaMemsetAsync(sh->mom, 0, sizeof(float) * mom_elems, s) != cudaSuccess))
    return fail(set_error(TK_ERR_CUDA, "could not clear the Muon momentum"));
  if (exchange != TK_SHARD_ALLGATHER && world > 1) {
    // every rank's arena, gathered through NCCL, then mapped
    PeerInfo mine;
    std::memset(&mine, 0, sizeof(mine));
    mine.n_elems = sh->extent * (uint64_t)world;
    mine.exchange = exchange;
    st = tk_ipc_export(p_arena, mine.handle, &mine.offset);
    if (st != TK_OK) return fail(st);
    std::vector<PeerInfo> all((size_t)world);
    void* buf = nullptr;
    if (cudaMalloc(&buf, sizeof(PeerInfo) * (size_t)(world + 1)) != cudaSuccess) {
      cudaGetLastError();
      return fail(set_error(TK_ERR_ALLOC, "could not allocate the init exchange buffer"));
    }
    char* gathered = static_cast<char*>(buf) + sizeof(PeerInfo);
    if (cudaMemcpyAsync(buf, &mine, sizeof(mine), cudaMemcpyHostToDevice, s) != cudaSuccess)
      st = set_error(TK_ERR_CUDA, "init exchange copy failed");
    ncclResult_t nr = ncclSuccess;
    if (st == TK_OK) {
      nr = N->AllGather(buf, gathered, sizeof(PeerInfo), ncclUint8, comm, s);
      if (nr != ncclSuccess)
        st = set_error(TK_ERR_CUDA, "ncclAllGather of the arena descriptions failed: %s",
                       N->GetErrorString(nr));
    }
    if (st == TK_OK &&
        (cudaMemcpyAsync(all.data(), gathered, sizeof(PeerInfo) * (size_t)world,
                         cudaMemcpyDeviceToHost, s) != cudaSuccess ||
         cudaStreamSynchronize(s) != cudaSuccess))
      st = set_error(TK_ERR_CUDA, "init exchange read-back failed");
    cudaFree(buf);
    if (st != TK_OK) return fail(st);
    for (int r = 0; r < world; ++r) {
      if (all[(size_t)r].n_elems != mine.n_elems || all[(size_t)r].exchange != exchange)
        return fail(set_error(TK_ERR_INVALID, "rank %d has another layout or exchange", r));
      if (r == rank) continue;
      void* ptr = nullptr;
      st = tk_ipc_import(all[(size_t)r].handle, all[(size_t)r].offset, &ptr);
      if (st != TK_OK) return fail(st);
      sh->peer_ptrs.push_back(ptr);
      sh->deltas.push_back((int64_t)(static_cast<char*>(ptr) - sh->p));
      if (sh->deltas.back() % 16 != 0)
        return fail(set_error(TK_ERR_UNSUPPORTED,
                              "rank %d's arena is not at the same address modulo 16 bytes as "
                              "this rank's; use TK_SHARD_ALLGATHER", r));
    }
  }
  *out = sh;
  return TK_OK;
}

int tk_muon_shard_info(const tk_muon_shard* sh, int32_t* owner_out, uint64_t* offset_out,
                       uint64_t* extent_out) {
  clear_error();
  if (sh == nullptr) return set_error(TK_ERR_INVALID, "shard is NULL");
  if (owner_out) std::copy(sh->owner.begin(), sh->owner.end(), owner_out);
  if (offset_out) std::copy(sh->offset.begin(), sh->offset.end(), offset_out);
  if (extent_out) *extent_out = sh->extent;
  return TK_OK;
}

int tk_muon_shard_step(tk_muon_shard* sh, const void* const* grads, int32_t g_dtype,
                       void* stream) {
  clear_error();
  if (sh == nullptr) return set_error(TK_ERR_INVALID, "shard is NULL");
  if (g_dtype != TK_F32 && g_dtype != TK_BF16)
    return set_error(TK_ERR_INVALID, "gradient dtype %d is not f32 or bf16", g_dtype);
  if (!sh->mine.empty() && grads == nullptr) return set_error(TK_ERR_INVALID, "grads is NULL");
  const Nccl* N = nullptr;
  TK_TRY(nccl(&N));
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev != sh->device)
    return set_error(TK_ERR_INVALID, "the shard lives on device %d, the current device is %d",
                     sh->device, dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t esz = sh->p_dtype == TK_F32 ? 4 : 2;
  std::vector<tk_muon_leaf> leaves;
  for (size_t k = 0; k < sh->mine.size(); ++k) {
    const size_t i = sh->mine[k];
    if (grads[i] == nullptr) return set_error(TK_ERR_INVALID, "gradient %zu is NULL", i);
    tk_muon_leaf L;
    std::memset(&L, 0, sizeof(L));
    L.p = sh->p + sh->offset[i] * esz;
    L.g = grads[i];
    L.momentum = sh->mom + sh->mom_off[k];
    L.heads = 1;
    L.rows = sh->rows[i];
    L.cols = sh->cols[i];
    L.p_dtype = sh->p_dtype;
    L.g_dtype = g_dtype;
    leaves.push_back(L);
  }
  const tk_muon_leaf* lp = leaves.empty() ? nullptr : leaves.data();
  const bool peers = sh->world > 1 && sh->exchange != TK_SHARD_ALLGATHER;
  NvtxRange range("tikun/muon_shard_step");
  if (peers)  // the peers are done reading this step's destination ranges
    TK_NCCL_TRY(N, N->AllReduce(sh->barrier, sh->barrier, 1, ncclFloat64, ncclSum, sh->comm, s));
  if (peers && sh->exchange == TK_SHARD_PEERS)
    TK_TRY(tk_muon_step_peers(lp, leaves.size(), &sh->hp, sh->deltas.data(),
                              (int)sh->deltas.size(), s));
  else if (peers)
    TK_TRY(tk_muon_step_copy(lp, leaves.size(), &sh->hp, sh->deltas.data(),
                             (int)sh->deltas.size(), s));
  else
    TK_TRY(tk_muon_step(lp, leaves.size(), &sh->hp, s));
  if (peers)
    TK_NCCL_TRY(N, N->AllReduce(sh->barrier, sh->barrier, 1, ncclFloat64, ncclSum, sh->comm, s));
  else if (sh->world > 1)
    TK_NCCL_TRY(N, N->AllGather(sh->p + (uint64_t)sh->rank * sh->extent * esz, sh->p,
                                sh->extent * esz, ncclUint8, sh->comm, s));
  return TK_OK;
}

int tk_muon_shard_destroy(tk_muon_shard* sh, void* stream) {
  clear_error();
  if (sh == nullptr) return TK_OK;
  int st = TK_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!sh->peer_ptrs.empty()) {
    const Nccl* N = nullptr;
    st = nccl(&N);
    if (st == TK_OK) {
      ncclResult_t r = N->AllReduce(sh->barrier, sh->barrier, 1, ncclFloat64, ncclSum, sh->comm, s);
      if (r != ncclSuccess)
        st = set_error(TK_ERR_CUDA, "end-of-life barrier failed: %s", N->GetErrorString(r));
      else if (cudaStreamSynchronize(s) != cudaSuccess)
        st = set_error(TK_ERR_CUDA, "end-of-life barrier did not complete");
    }
  } else {
    cudaDeviceSynchronize();
  }
  muon_shard_free(sh);
  return st;
}

}  // extern "C"
