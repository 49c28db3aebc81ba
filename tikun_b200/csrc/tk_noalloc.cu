// tk_step_buffers_noalloc: the two-tier pointwise step for callers that must
// not allocate device memory.
//
// Who needs it: code that runs where cudaMalloc (or a framework's caching
// allocator) is off limits — an embedding application that hands this
// library a fixed memory budget and owns every allocation itself, a runtime
// whose allocator must not be re-entered from inside an optimizer hook, or a
// caller that has reserved the whole device for its own pool.  Every other
// entry point takes its norm scratch from a stream-ordered pool, which
// allocates on first use and whenever a call needs more.
//
// This variant keeps the Tier-1 partial sums and the clip scale in one
// file-scope device array of fixed size instead.  Limits and rules:
//   * device leaves only, at most kNoallocMaxLeaves leaves per call (one
//     launch table per element-type pair), and at most kNoallocMaxPartials
//     norm blocks in total; larger calls are rejected with TK_ERR_INVALID;
//   * the array is shared by every call on a device and keeps the last call's
//     contents; every slot a call reads is written earlier in the same call,
//     so nothing needs clearing, but calls whose kernels overlap on the GPU
//     (different streams, no ordering between them) race on it;
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress) with that device current; make that first call
//     before any stream capture.  The address is kept per device together
//     with the id of the CUDA context it was looked up in; after
//     cudaDeviceReset the next call sees a new context id and looks it up
//     again (do that call outside a stream capture too).
//   * with clip_scale_out NULL the call returns once its kernels are
//     enqueued: a kernel error then surfaces at the caller's next
//     synchronisation, not from this call.
// No cudaMalloc, cudaFree or other allocating routine is called.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "tk_internal.h"

namespace tk {
namespace {

constexpr int kNoallocMaxLeaves = kMaxLeavesPerLaunch;  // 224
constexpr int kNoallocMaxPartials = 8192;               // f64 norm partials
// slots [0, kNoallocMaxPartials): partials; then the clip scale (f32)
constexpr int kNoallocSlots = kNoallocMaxPartials + 32;

static __device__ __align__(256) double g_noalloc_scratch[kNoallocSlots];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
struct CachedAddress {
  double* addr = nullptr;
  unsigned long long ctx_id = 0;  // the CUDA context the address belongs to
};
CachedAddress g_scratch_addr[kMaxDevices];

// The id of the current CUDA context (cuCtxGetCurrent + cuCtxGetId, from the
// driver through the runtime's entry-point query; no link to libcuda).
int current_context_id(unsigned long long* id) {
  using GetCurrentFn = CUresult (*)(CUcontext*);
  using GetIdFn = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrentFn get_current = nullptr;
  static GetIdFn get_id = nullptr;
  if (get_current == nullptr || get_id == nullptr) {
    void* a = nullptr;
    void* b = nullptr;
    cudaDriverEntryPointQueryResult qa, qb;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &a, 12000, cudaEnableDefault, &qa) !=
            cudaSuccess ||
        qa != cudaDriverEntryPointSuccess ||
        cudaGetDriverEntryPointByVersion("cuCtxGetId", &b, 12000, cudaEnableDefault, &qb) !=
            cudaSuccess ||
        qb != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return set_error(TK_ERR_CUDA, "cuCtxGetCurrent / cuCtxGetId are not available from the driver");
    }
    get_current = reinterpret_cast<GetCurrentFn>(a);
    get_id = reinterpret_cast<GetIdFn>(b);
  }
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr || get_id(ctx, id) != CUDA_SUCCESS)
    return set_error(TK_ERR_CUDA, "could not identify the current CUDA context");
  return TK_OK;
}

int scratch_for_current_device(double** out) {
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return set_error(TK_ERR_CUDA, "device index %d out of range", dev);
  TK_CUDA_TRY(cudaSetDevice(dev));  // binds the device's primary context to this thread
  unsigned long long ctx = 0;
  TK_TRY(current_context_id(&ctx));
  std::lock_guard<std::mutex> lock(g_setup_mu);
  CachedAddress& c = g_scratch_addr[dev];
  if (c.addr == nullptr || c.ctx_id != ctx) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(TK_ERR_CUDA, "cudaGetSymbolAddress of the fixed scratch failed: %s",
                       cudaGetErrorString(e));
    c.addr = static_cast<double*>(p);
    c.ctx_id = ctx;
  }
  *out = c.addr;
  return TK_OK;
}

size_t na_esize(int dt) { return dt == TK_F32 ? 4 : 2; }

// Same checks as the allocating entry points, on fixed-size stack storage.
int validate(const tk_leaf* leaves, size_t n, int kind) {
  if (n > (size_t)kNoallocMaxLeaves)
    return set_error(TK_ERR_INVALID,
                     "tk_step_buffers_noalloc takes at most %d leaves per call (got %zu); "
                     "split the call or use tk_step_buffers",
                     kNoallocMaxLeaves, n);
  if (n > 0 && leaves == nullptr) return set_error(TK_ERR_INVALID, "leaves is NULL");
  if (kind != TK_ADAMW && kind != TK_LION && kind != TK_SGD && kind != TK_CUSTOM)
    return set_error(TK_ERR_INVALID, "unknown optimizer kind %d", kind);
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  ByteRange ranges[4 * kNoallocMaxLeaves];
  size_t nr = 0;
  for (size_t i = 0; i < n; ++i) {
    const tk_leaf& L = leaves[i];
    if ((L.p_dtype != TK_F32 && L.p_dtype != TK_BF16) || (L.g_dtype != TK_F32 && L.g_dtype != TK_BF16))
      return set_error(TK_ERR_INVALID, "leaf %zu: p and g must be f32 or bf16", i);
    if (L.n == 0) continue;
    if (L.p == nullptr || L.g == nullptr || L.m == nullptr)
      return set_error(TK_ERR_INVALID, "leaf %zu: null p, g or m pointer", i);
    if (kind == TK_ADAMW && L.v == nullptr)
      return set_error(TK_ERR_INVALID, "leaf %zu: AdamW needs a second-moment (m2) buffer", i);
    ranges[nr++] = {(uintptr_t)L.p, (uintptr_t)L.p + L.n * na_esize(L.p_dtype), true};
    ranges[nr++] = {(uintptr_t)L.g, (uintptr_t)L.g + L.n * na_esize(L.g_dtype), false};
    ranges[nr++] = {(uintptr_t)L.m, (uintptr_t)L.m + L.n * 4, true};
    if (kind == TK_ADAMW) ranges[nr++] = {(uintptr_t)L.v, (uintptr_t)L.v + L.n * 4, true};
    const void* ptrs[4] = {L.p, L.g, L.m, kind == TK_ADAMW ? (const void*)L.v : nullptr};
    for (const void* ptr : ptrs) {
      if (ptr == nullptr) continue;
      Residency r;
      TK_TRY(classify_pointer(ptr, &r, dev));
      if (r != Residency::kDevice)
        return set_error(TK_ERR_INVALID,
                         "leaf %zu: tk_step_buffers_noalloc takes device buffers only "
                         "(host buffers would need device staging memory)",
                         i);
    }
  }
  return check_overlaps(ranges, nr);
}

}  // namespace
}  // namespace tk

using namespace tk;

extern "C" int tk_step_buffers_noalloc(const tk_leaf* leaves, size_t n_leaves, int32_t kind,
                                       const tk_hparams* hp, uint64_t step, float max_norm,
                                       float* clip_scale_out, void* stream) {
  clear_error();
  if (hp == nullptr) return set_error(TK_ERR_INVALID, "hparams is NULL");
  TK_TRY(validate(leaves, n_leaves, kind));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  double* scratch = nullptr;
  TK_TRY(scratch_for_current_device(&scratch));
  float* scale_dev = reinterpret_cast<float*>(scratch + kNoallocMaxPartials);

  // one table per (p, g) element-type pair: n_leaves <= 224 fits one each
  // (on the stack: about 50 KB)
  LeafTable tables[4];
  int pdt[4], gdt[4], n_tables = 0;
  const int dts[2] = {TK_F32, TK_BF16};
  for (int pd : dts)
    for (int gd : dts) {
      LeafTable& t = tables[n_tables];
      std::memset(&t, 0, sizeof(t));
      for (size_t i = 0; i < n_leaves; ++i) {
        const tk_leaf& L = leaves[i];
        if (L.n == 0 || L.p_dtype != pd || L.g_dtype != gd) continue;
        LeafDesc& d = t.leaf[t.n_leaves++];
        d.p = L.p;
        d.g = L.g;
        d.m = L.m;
        d.v = kind == TK_ADAMW ? L.v : nullptr;
        d.n = L.n;
        d.q_begin = t.total_quads;
        d.vec_ok = ((uintptr_t)L.p % (4 * na_esize(pd)) == 0) && ((uintptr_t)L.g % (4 * na_esize(gd)) == 0) &&
                   ((uintptr_t)L.m % 16 == 0) && (kind != TK_ADAMW || (uintptr_t)L.v % 16 == 0);
        t.total_quads += (L.n + 3) / 4;
      }
      if (t.n_leaves > 0) {
        pdt[n_tables] = pd;
        gdt[n_tables] = gd;
        ++n_tables;
      }
    }

  const PointwiseConsts c = make_consts(kind, *hp, step);

  const bool clip = max_norm > 0.0f && n_tables > 0;
  int n_partials = 0;
  if (clip) {
    int blocks[4];
    for (int i = 0; i < n_tables; ++i) {
      blocks[i] = sumsq_blocks_for(tables[i].total_quads);
      if (blocks[i] <= 0) return set_error(TK_ERR_CUDA, "could not size the norm grid");
      n_partials += blocks[i];
    }
    if (n_partials > kNoallocMaxPartials)
      return set_error(TK_ERR_INVALID, "the norm needs %d partial sums; the fixed scratch holds %d",
                       n_partials, kNoallocMaxPartials);
    int off = 0;
    for (int i = 0; i < n_tables; ++i) {
      TK_TRY(launch_sumsq_partials(tables[i], gdt[i], scratch + off, blocks[i], s));
      off += blocks[i];
    }
  }
  for (int i = 0; i < n_tables; ++i)
    TK_TRY(launch_pointwise(tables[i], kind, pdt[i], gdt[i], c, clip ? scratch : nullptr,
                            n_partials, max_norm, nullptr, (clip && i == 0) ? scale_dev : nullptr, s));
  if (clip_scale_out != nullptr) {
    float scale = 1.0f;
    if (clip) TK_CUDA_TRY(cudaMemcpyAsync(&scale, scale_dev, sizeof(float), cudaMemcpyDeviceToHost, s));
    TK_CUDA_TRY(cudaStreamSynchronize(s));
    *clip_scale_out = scale;
  }
  return TK_OK;
}
