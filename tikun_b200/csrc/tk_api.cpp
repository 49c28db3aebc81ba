// C-ABI entry points of the pointwise step (include/tikun_cuda.h): the static
// verifier, the layout plan, leaf validation and the Tier 1 / Tier 2
// orchestration over the CUDA kernels in tk_pointwise.cu.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "tk_internal.h"
#include "tk_testing.h"

namespace tk {

// ------------------------------------------------------------------ errors
static thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

void clear_error() { g_last_error.clear(); }

int cuda_error(cudaError_t e, const char* what) {
  return set_error(TK_ERR_CUDA, "CUDA error %s (%s) in %s", cudaGetErrorName(e),
                   cudaGetErrorString(e), what);
}

// ------------------------------------------------------------------ device info
int sm_count(int* out) {
  static int cached[64] = {0};
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(TK_ERR_CUDA, "device index %d out of range", dev);
  if (cached[dev] == 0) {
    int n = 0;
    TK_CUDA_TRY(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    cached[dev] = n;
  }
  *out = cached[dev];
  return TK_OK;
}

static std::atomic<int> g_reserved_sms{0};

int pointwise_sms(int* out) {
  int sms = 0;
  TK_TRY(sm_count(&sms));
  *out = std::max(1, sms - g_reserved_sms.load());
  return TK_OK;
}

// ------------------------------------------------------------------ scratch pool
static std::mutex g_pool_mu;
static cudaMemPool_t g_pools[64] = {};

static int device_pool(cudaMemPool_t* out) {
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(TK_ERR_CUDA, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_pool_mu);
  if (g_pools[dev] == nullptr) {
    cudaMemPoolProps props;
    std::memset(&props, 0, sizeof(props));
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool;
    TK_CUDA_TRY(cudaMemPoolCreate(&pool, &props));
    uint64_t keep = UINT64_MAX;  // keep freed scratch cached for the next step
    TK_CUDA_TRY(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
    g_pools[dev] = pool;
  }
  *out = g_pools[dev];
  return TK_OK;
}

static int* g_status[64] = {};

int device_status_word(int** out) {
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(TK_ERR_CUDA, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_pool_mu);
  if (g_status[dev] == nullptr) {
    int* p = nullptr;
    TK_CUDA_TRY(cudaMalloc(&p, 256));
    TK_CUDA_TRY(cudaMemset(p, 0, 256));
    g_status[dev] = p;
  }
  *out = g_status[dev];
  return TK_OK;
}

Scratch::~Scratch() {
  if (ptr_ != nullptr) cudaFreeAsync(ptr_, stream_);
}

int Scratch::alloc(size_t bytes, cudaStream_t s) {
  if (ptr_ != nullptr) return set_error(TK_ERR_INVALID, "scratch allocated twice");
  cudaMemPool_t pool;
  TK_TRY(device_pool(&pool));
  stream_ = s;
  cudaError_t e = cudaMallocFromPoolAsync(&ptr_, bytes ? bytes : 16, pool, s);
  if (e != cudaSuccess) {
    ptr_ = nullptr;
    return set_error(TK_ERR_ALLOC, "could not allocate %zu bytes of device scratch: %s", bytes,
                     cudaGetErrorString(e));
  }
  return TK_OK;
}

// ------------------------------------------------------------------ verifier
// Verifier::verify, crates/tikun-core/src/verifier.rs:14-45, with the error
// text of `format!("Static verification failed: {:?}", violations)`
// (crates/tikun-cpu/src/lib.rs:74).
static bool is_pow2(uint64_t x) { return x != 0 && (x & (x - 1)) == 0; }

// Rust's Debug text of a string (str::escape_debug) for the characters a C
// string can hold: \t \r \n \\ \" escaped by name, other ASCII control
// characters as \u{hex}, everything else (UTF-8 bytes included) as is.
static std::string rust_debug_str(const char* s) {
  std::string out = "\"";
  for (const char* c = s ? s : ""; *c; ++c) {
    const unsigned char u = static_cast<unsigned char>(*c);
    switch (u) {
      case '\t': out += "\\t"; break;
      case '\r': out += "\\r"; break;
      case '\n': out += "\\n"; break;
      case '\\': out += "\\\\"; break;
      case '"': out += "\\\""; break;
      default:
        if (u < 0x20 || u == 0x7f) {
          char buf[16];
          std::snprintf(buf, sizeof(buf), "\\u{%x}", u);
          out += buf;
        } else {
          out += *c;
        }
    }
  }
  return out + "\"";
}

static int verify_pipeline(const tk_pipeline* pl) {
  if (pl == nullptr) return set_error(TK_ERR_INVALID, "pipeline is NULL");
  if (pl->n_nodes == 0) return set_error(TK_ERR_VERIFY, "Static verification failed: [EmptyPipeline]");
  if (pl->nodes == nullptr) return set_error(TK_ERR_INVALID, "pipeline nodes are NULL");
  std::vector<std::string> errs;
  for (size_t i = 0; i < pl->n_nodes; ++i) {
    const tk_schedule_node& n = pl->nodes[i];
    if (n.tile_size % 64 != 0)
      errs.push_back("MisalignedCacheLine { node_name: " + rust_debug_str(n.name) +
                     ", tile_size: " + std::to_string(n.tile_size) + " }");
    if (!is_pow2(n.vector_width) || n.vector_width < 4)
      errs.push_back("InvalidVectorWidth { node_name: " + rust_debug_str(n.name) +
                     ", width: " + std::to_string(n.vector_width) + " }");
  }
  if (errs.empty()) return TK_OK;
  std::string msg = "Static verification failed: [";
  for (size_t i = 0; i < errs.size(); ++i) msg += (i ? ", " : "") + errs[i];
  msg += "]";
  return set_error(TK_ERR_VERIFY, "%s", msg.c_str());
}

// ------------------------------------------------------------------ leaves
static size_t esize(int dt) { return dt == TK_F32 ? 4 : 2; }

int classify_pointer(const void* ptr, Residency* r, int dev) {
  cudaPointerAttributes a;
  cudaError_t e = cudaPointerGetAttributes(&a, ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(TK_ERR_INVALID, "cannot classify pointer %p: %s", ptr, cudaGetErrorString(e));
  }
  if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) {
    if (a.type == cudaMemoryTypeDevice && a.device != dev)
      return set_error(TK_ERR_INVALID, "pointer %p lives on device %d, the current device is %d",
                       ptr, a.device, dev);
    *r = Residency::kDevice;
  } else {
    *r = Residency::kHost;
  }
  return TK_OK;
}

int check_overlaps(ByteRange* ranges, size_t n) {
  std::sort(ranges, ranges + n,
            [](const ByteRange& a, const ByteRange& b) { return a.lo < b.lo; });
  uintptr_t max_any = 0, max_w = 0;
  for (size_t i = 0; i < n; ++i) {
    const ByteRange& r = ranges[i];
    if ((r.writable && max_any > r.lo) || max_w > r.lo)
      return set_error(TK_ERR_INVALID,
                       "leaf buffers overlap at %p: a buffer the step writes (p, m or v) "
                       "shares memory with another buffer",
                       (void*)r.lo);
    max_any = std::max(max_any, r.hi);
    if (r.writable) max_w = std::max(max_w, r.hi);
  }
  return TK_OK;
}

// Rejects null or mismatched fields, bad dtypes, any overlap between a range
// the step writes (p, m, v) and any other range, and a mix of host and device
// leaves.  Reports where the leaves live.
static int validate_leaves_full(const tk_leaf* leaves, size_t n, int kind, Residency* where);

// A training loop steps the same leaf table every time; classifying its
// pointers costs one driver query per buffer (four per leaf), which for a
// few hundred leaves is a good part of a sub-millisecond step's host time.
// The last table that passed on this thread (with its device and kind) is
// remembered, and an identical table is accepted without the queries.
struct ValidatedTable {
  bool valid = false;
  int dev = -1, kind = -1;
  std::vector<tk_leaf> leaves;
  Residency where = Residency::kNone;
};
static thread_local ValidatedTable g_validated;

static int validate_leaves(const tk_leaf* leaves, size_t n, int kind, Residency* where) {
  int dev = 0;
  if (n > 0 && leaves != nullptr) {
    TK_CUDA_TRY(cudaGetDevice(&dev));
    const ValidatedTable& v = g_validated;
    if (v.valid && v.dev == dev && v.kind == kind && v.leaves.size() == n &&
        std::memcmp(v.leaves.data(), leaves, n * sizeof(tk_leaf)) == 0) {
      *where = v.where;
      return TK_OK;
    }
  }
  const int st = validate_leaves_full(leaves, n, kind, where);
  if (st == TK_OK && n > 0) {
    g_validated.valid = true;
    g_validated.dev = dev;
    g_validated.kind = kind;
    g_validated.leaves.assign(leaves, leaves + n);
    g_validated.where = *where;
  }
  return st;
}

static int validate_leaves_full(const tk_leaf* leaves, size_t n, int kind, Residency* where) {
  *where = Residency::kNone;
  if (n == 0) return TK_OK;
  if (leaves == nullptr) return set_error(TK_ERR_INVALID, "leaves is NULL with n_leaves=%zu", n);
  if (kind != TK_ADAMW && kind != TK_LION && kind != TK_SGD && kind != TK_CUSTOM)
    return set_error(TK_ERR_INVALID, "unknown optimizer kind %d", kind);
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  std::vector<ByteRange> ranges;
  ranges.reserve(n * 4);
  for (size_t i = 0; i < n; ++i) {
    const tk_leaf& L = leaves[i];
    if (L.p_dtype != TK_F32 && L.p_dtype != TK_BF16)
      return set_error(TK_ERR_INVALID, "leaf %zu: p_dtype %d is not f32 or bf16", i, L.p_dtype);
    if (L.g_dtype != TK_F32 && L.g_dtype != TK_BF16)
      return set_error(TK_ERR_INVALID, "leaf %zu: g_dtype %d is not f32 or bf16", i, L.g_dtype);
    if (L.n == 0) continue;
    if (L.p == nullptr || L.g == nullptr || L.m == nullptr)
      return set_error(TK_ERR_INVALID, "leaf %zu: null p, g or m pointer", i);
    if (kind == TK_ADAMW && L.v == nullptr)
      return set_error(TK_ERR_INVALID, "leaf %zu: AdamW needs a second-moment (m2) buffer", i);
    const uintptr_t p = (uintptr_t)L.p, g = (uintptr_t)L.g, m = (uintptr_t)L.m;
    ranges.push_back({p, p + L.n * esize(L.p_dtype), true});
    ranges.push_back({g, g + L.n * esize(L.g_dtype), false});
    ranges.push_back({m, m + L.n * 4, true});
    if (kind == TK_ADAMW) ranges.push_back({(uintptr_t)L.v, (uintptr_t)L.v + L.n * 4, true});
    const void* ptrs[4] = {L.p, L.g, L.m, kind == TK_ADAMW ? (const void*)L.v : nullptr};
    for (const void* ptr : ptrs) {
      if (ptr == nullptr) continue;
      Residency r;
      TK_TRY(classify_pointer(ptr, &r, dev));
      if (*where == Residency::kNone) *where = r;
      else if (*where != r)
        return set_error(TK_ERR_INVALID,
                         "leaf %zu: host and device buffers are mixed in one call", i);
    }
  }
  return check_overlaps(ranges.data(), ranges.size());
}

static bool aligned(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }

static bool leaf_vec_ok(const tk_leaf& L, int kind) {
  return aligned(L.p, 4 * esize(L.p_dtype)) && aligned(L.g, 4 * esize(L.g_dtype)) &&
         aligned(L.m, 16) && (kind != TK_ADAMW || aligned(L.v, 16));
}

// Splits the non-empty leaves with one (p, g) dtype pair into launch tables;
// `want_vec` selects leaves whose pointers are (1) or are not (0) aligned for
// whole-group access, -1 takes both.
static void build_tables(const tk_leaf* leaves, size_t n, int kind, int pdt, int gdt,
                         std::vector<LeafTable>* out, int want_vec = -1) {
  LeafTable* t = nullptr;
  for (size_t i = 0; i < n; ++i) {
    const tk_leaf& L = leaves[i];
    if (L.n == 0 || L.p_dtype != pdt || L.g_dtype != gdt) continue;
    if (want_vec >= 0 && (int)leaf_vec_ok(L, kind) != want_vec) continue;
    if (t == nullptr || t->n_leaves == kMaxLeavesPerLaunch) {
      out->emplace_back();
      t = &out->back();
      std::memset(t, 0, sizeof(*t));
    }
    LeafDesc& d = t->leaf[t->n_leaves++];
    d.p = L.p;
    d.g = L.g;
    d.m = L.m;
    d.v = kind == TK_ADAMW ? L.v : nullptr;
    d.n = L.n;
    d.q_begin = t->total_quads;
    d.vec_ok = leaf_vec_ok(L, kind);
    t->total_quads += (L.n + 3) / 4;
  }
}

// Rust f32::powi with a runtime exponent: binary exponentiation in f32.
static float powi_f32(float a, int32_t b) {
  const bool recip = b < 0;
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

PointwiseConsts make_consts(int kind, const tk_hparams& hp, uint64_t step) {
  PointwiseConsts c;
  c.lr = hp.lr;
  c.b1 = hp.beta1;
  c.b2 = hp.beta2;
  c.eps = hp.eps;
  c.decay = hp.decay;
  volatile float one = 1.0f;  // keep 1 - b in f32, as the reference does
  c.omb1 = one - hp.beta1;
  c.omb2 = one - hp.beta2;
  c.bc1 = c.bc2 = 1.0f;
  if (kind == TK_ADAMW) {
    // lib.rs:152-154
    const int32_t step_val = (int32_t)(step < 1 ? 1 : (step > INT32_MAX ? INT32_MAX : step));
    c.bc1 = one - powi_f32(hp.beta1, step_val);
    c.bc2 = one - powi_f32(hp.beta2, step_val);
  }
  return c;
}

struct Plan {
  std::vector<LeafTable> tables;
  std::vector<int> pdt, gdt;
  std::vector<char> bulk;  // table goes through the bulk-copy kernel
};

// With TIKUN_PW_BULK=1 in the environment, f32 leaves with aligned pointers
// form tables for the bulk-copy pipeline kernel and every other leaf goes to
// the register kernel.  Off by default: on B200 the bulk pipeline at its best
// tile/ring shape only ties the register kernel (both near 0.87 of the copy
// bandwidth, bound by the exact divide/square-root chain), and the register
// kernel alone carries the peer stores.
static bool bulk_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("TIKUN_PW_BULK");
    return e != nullptr && e[0] == '1';
  }();
  return on;
}

static void make_plan(const tk_leaf* leaves, size_t n, int kind, Plan* plan) {
  const int dts[2] = {TK_F32, TK_BF16};
  for (int pd : dts)
    for (int gd : dts) {
      const bool f32 = bulk_enabled() && pd == TK_F32 && gd == TK_F32;
      for (int pass = 0; pass < (f32 ? 2 : 1); ++pass) {
        size_t before = plan->tables.size();
        build_tables(leaves, n, kind, pd, gd, &plan->tables, f32 ? (pass == 0 ? 1 : 0) : -1);
        for (size_t i = before; i < plan->tables.size(); ++i) {
          plan->pdt.push_back(pd);
          plan->gdt.push_back(gd);
          plan->bulk.push_back(f32 && pass == 0);
        }
      }
    }
}

static int launch_table(const Plan& plan, size_t i, int kind, const PointwiseConsts& c,
                        const double* partials, int n_partials, float max_norm,
                        const float* scale_dev, float* scale_out, cudaStream_t s) {
  if (plan.bulk[i])
    return launch_pointwise_bulk(plan.tables[i], kind, c, partials, n_partials, max_norm,
                                 scale_dev, scale_out, s);
  return launch_pointwise(plan.tables[i], kind, plan.pdt[i], plan.gdt[i], c, partials, n_partials,
                          max_norm, scale_dev, scale_out, s);
}

// Tier 1 partials for every table into one buffer; returns the block count.
// With a communicator (the leaves are this rank's share of a sharded PyTree)
// the partials are summed into one f64, all-reduced over it, and that global
// sum is returned as the single partial.
static int launch_norm(const Plan& plan, Scratch* scratch, double** partials, int* n_partials,
                       cudaStream_t s, void* comm = nullptr) {
  std::vector<int> blocks;
  int total = 0;
  for (const LeafTable& t : plan.tables) {
    const int b = sumsq_blocks_for(t.total_quads);
    if (b <= 0) return set_error(TK_ERR_CUDA, "could not size the norm grid");
    blocks.push_back(b);
    total += b;
  }
  TK_TRY(scratch->alloc(sizeof(double) * (size_t)std::max(total, 1) + 64, s));
  double* base = static_cast<double*>(scratch->get());
  int off = 0;
  for (size_t i = 0; i < plan.tables.size(); ++i) {
    TK_TRY(launch_sumsq_partials(plan.tables[i], plan.gdt[i], base + off, blocks[i], s));
    off += blocks[i];
  }
  *partials = base;
  *n_partials = total;
  if (comm != nullptr) {
    double* sum = base + total;  // inside the 64 spare bytes
    if (total > 0) TK_TRY(launch_sumsq_reduce(base, total, sum, s));
    else TK_CUDA_TRY(cudaMemsetAsync(sum, 0, sizeof(double), s));
    TK_TRY(nccl_allreduce_sum_f64(sum, 1, comm, s));
    *partials = sum;
    *n_partials = 1;
  }
  return TK_OK;
}

// Measurement hook (tk_set_update_events).
static thread_local cudaEvent_t g_update_start = nullptr;
static thread_local cudaEvent_t g_update_stop = nullptr;

int record_update_event(bool start, cudaStream_t s) {
  cudaEvent_t e = start ? g_update_start : g_update_stop;
  if (e) TK_CUDA_TRY(cudaEventRecord(e, s));
  return TK_OK;
}

// The device-resident step.  scale_dev (may be null) receives the clip scale.
static int step_device(const tk_leaf* leaves, size_t n, int kind, const tk_hparams& hp,
                       uint64_t step, float max_norm, float* scale_dev, bool* scale_written,
                       cudaStream_t s, void* comm = nullptr) {
  *scale_written = false;
  Plan plan;
  make_plan(leaves, n, kind, &plan);
  const bool join = comm != nullptr && max_norm > 0.0f;  // the norm all-reduce is collective
  if (plan.tables.empty() && !join) return TK_OK;  // nothing to update; the scale is 1
  const PointwiseConsts c = make_consts(kind, hp, step);
  Scratch norm_scratch;
  double* partials = nullptr;
  int n_partials = 0;
  if (max_norm > 0.0f) {
    NvtxRange r("tikun/tier1_norm");
    TK_TRY(launch_norm(plan, &norm_scratch, &partials, &n_partials, s, comm));
  }
  if (plan.tables.empty()) {  // a rank holding no elements still reports the global scale
    if (scale_dev != nullptr) {
      TK_TRY(launch_clip_scale(partials, n_partials, max_norm, scale_dev, s));
      *scale_written = true;
    }
    return TK_OK;
  }
  NvtxRange r("tikun/tier2_update");
  if (g_update_start) TK_CUDA_TRY(cudaEventRecord(g_update_start, s));
  for (size_t i = 0; i < plan.tables.size(); ++i)
    TK_TRY(launch_table(plan, i, kind, c, partials, n_partials, max_norm, nullptr,
                        i == 0 ? scale_dev : nullptr, s));
  if (g_update_stop) TK_CUDA_TRY(cudaEventRecord(g_update_stop, s));
  *scale_written = partials != nullptr && scale_dev != nullptr;
  return TK_OK;
}

// ---- host leaves through the copy engines ----------------------------------
// Per-device side streams and events for the pipelined host step.
struct HostPipe {
  std::mutex mu;  // one host-buffer step at a time per device (shared streams/events)
  cudaStream_t h2d = nullptr, d2h = nullptr;
  static constexpr int kSlots = 3;
  cudaEvent_t start = nullptr, g_ready = nullptr, end = nullptr;
  cudaEvent_t in_ready[kSlots] = {}, done[kSlots] = {}, out_done[kSlots] = {};
};

static int host_pipe(HostPipe** out) {
  static HostPipe pipes[64];
  static bool ready[64] = {};
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(TK_ERR_CUDA, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_pool_mu);
  if (!ready[dev]) {
    HostPipe& P = pipes[dev];
    TK_CUDA_TRY(cudaStreamCreateWithFlags(&P.h2d, cudaStreamNonBlocking));
    TK_CUDA_TRY(cudaStreamCreateWithFlags(&P.d2h, cudaStreamNonBlocking));
    for (cudaEvent_t* e : {&P.start, &P.g_ready, &P.end})
      TK_CUDA_TRY(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
    for (int k = 0; k < HostPipe::kSlots; ++k)
      for (cudaEvent_t* e : {&P.in_ready[k], &P.done[k], &P.out_done[k]})
        TK_CUDA_TRY(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
    ready[dev] = true;
  }
  *out = &pipes[dev];
  return TK_OK;
}

static bool all_pinned(const tk_leaf* leaves, size_t n, int kind) {
  for (size_t i = 0; i < n; ++i) {
    const tk_leaf& L = leaves[i];
    if (L.n == 0) continue;
    const void* ptrs[4] = {L.p, L.g, L.m, kind == TK_ADAMW ? (const void*)L.v : nullptr};
    for (const void* p : ptrs) {
      if (p == nullptr) continue;
      cudaPointerAttributes a;
      if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
      }
      if (a.type != cudaMemoryTypeHost) return false;
    }
  }
  return true;
}

// A piece of one leaf: elements [off, off + cnt).
struct Piece {
  size_t leaf;
  uint64_t off, cnt;
};

// Pinned host leaves.  The elements are cut into chunks of at most
// kChunkElems (whole small leaves share a chunk); chunk c moves through a ring
// of three device slots: the H2D stream copies its p, m, v (and g, when not
// clipping) into slot c % 3, the caller's stream updates it, the D2H stream
// copies p, m, v back, so both copy directions and the update overlap.  With a
// clip, all of g is copied first and Tier 1 runs on it before any update.
static int step_host_pipelined(const tk_leaf* leaves, size_t n, int kind, const tk_hparams& hp,
                               uint64_t step, float max_norm, float* clip_scale_out,
                               cudaStream_t s, void* comm = nullptr) {
  constexpr uint64_t kChunkElems = 8u << 20;
  constexpr int kMaxPieces = kMaxLeavesPerLaunch;
  NvtxRange range("tikun/host_pipeline");
  HostPipe* P = nullptr;
  TK_TRY(host_pipe(&P));
  std::lock_guard<std::mutex> serial(P->mu);
  const bool clip = max_norm > 0.0f;
  const bool adam = kind == TK_ADAMW;

  // chunks of pieces
  std::vector<std::vector<Piece>> chunks;
  std::vector<uint64_t> chunk_elems;
  for (size_t i = 0; i < n; ++i) {
    uint64_t off = 0;
    while (off < leaves[i].n) {
      if (chunks.empty() || chunk_elems.back() >= kChunkElems ||
          (int)chunks.back().size() >= kMaxPieces) {
        chunks.emplace_back();
        chunk_elems.push_back(0);
      }
      const uint64_t take = std::min(leaves[i].n - off, kChunkElems - chunk_elems.back());
      chunks.back().push_back({i, off, take});
      chunk_elems.back() += (take + 63) / 64 * 64;
      off += take;
    }
  }
  if (chunks.empty()) {
    if (comm != nullptr && clip) {  // join the collective norm; nothing to update
      Scratch sc, norm_scratch;
      TK_TRY(sc.alloc(64, s));
      float* scale_dev = static_cast<float*>(sc.get());
      double* partials = nullptr;
      int n_partials = 0;
      TK_TRY(launch_norm(Plan(), &norm_scratch, &partials, &n_partials, s, comm));
      TK_TRY(launch_clip_scale(partials, n_partials, max_norm, scale_dev, s));
      float scale = 1.0f;
      TK_CUDA_TRY(cudaMemcpyAsync(&scale, scale_dev, 4, cudaMemcpyDeviceToHost, s));
      TK_CUDA_TRY(cudaStreamSynchronize(s));
      if (clip_scale_out) *clip_scale_out = scale;
      return TK_OK;
    }
    if (clip_scale_out) *clip_scale_out = 1.0f;
    return TK_OK;
  }
  // device memory: g for every leaf when clipping; three slots of
  // (p, g unless clipping, m, v) for kChunkElems (+ padding) elements each
  size_t gbytes = 0;
  std::vector<size_t> goff(n, 0);
  if (clip)
    for (size_t i = 0; i < n; ++i) {
      goff[i] = gbytes;
      gbytes += (leaves[i].n * esize(leaves[i].g_dtype) + 255) / 256 * 256;
    }
  const uint64_t slot_elems = kChunkElems + 64 * (uint64_t)kMaxPieces;
  const size_t arr_bytes = slot_elems * 4;
  const int arrays = 2 + (adam ? 1 : 0) + (clip ? 0 : 1);  // p, m, [v], [g]
  const size_t slot_bytes = arr_bytes * arrays;
  Scratch sc;
  TK_TRY(sc.alloc(256 + gbytes + slot_bytes * HostPipe::kSlots, s));
  // On an early return the scratch goes back to the pool in s's order while
  // copies on the side streams may still use it: s first waits for both.
  // (Destroyed before sc; disarmed once s has joined them on the normal path.)
  struct JoinSideStreams {
    HostPipe* P;
    cudaStream_t s;
    bool armed = true;
    ~JoinSideStreams() {
      if (!armed) return;
      if (cudaEventRecord(P->g_ready, P->h2d) == cudaSuccess) cudaStreamWaitEvent(s, P->g_ready, 0);
      if (cudaEventRecord(P->end, P->d2h) == cudaSuccess) cudaStreamWaitEvent(s, P->end, 0);
    }
  } join_guard{P, s};
  char* base = static_cast<char*>(sc.get());
  float* scale_dev = reinterpret_cast<float*>(base);
  char* gdev = base + 256;
  char* slots = gdev + gbytes;

  const PointwiseConsts c = make_consts(kind, hp, step);
  // everything starts after the caller's earlier work on s
  TK_CUDA_TRY(cudaEventRecord(P->start, s));
  TK_CUDA_TRY(cudaStreamWaitEvent(P->h2d, P->start, 0));
  TK_CUDA_TRY(cudaStreamWaitEvent(P->d2h, P->start, 0));

  Scratch norm_scratch;
  double* partials = nullptr;
  int n_partials = 0;
  if (clip) {
    for (size_t i = 0; i < n; ++i)
      if (leaves[i].n)
        TK_CUDA_TRY(cudaMemcpyAsync(gdev + goff[i], leaves[i].g, leaves[i].n * esize(leaves[i].g_dtype),
                                    cudaMemcpyHostToDevice, P->h2d));
    TK_CUDA_TRY(cudaEventRecord(P->g_ready, P->h2d));
    TK_CUDA_TRY(cudaStreamWaitEvent(s, P->g_ready, 0));
    std::vector<tk_leaf> gl(leaves, leaves + n);
    for (size_t i = 0; i < n; ++i) gl[i].g = gdev + goff[i];
    Plan plan;
    make_plan(gl.data(), n, TK_SGD, &plan);  // Tier 1 reads g only
    TK_TRY(launch_norm(plan, &norm_scratch, &partials, &n_partials, s, comm));
  }

  for (size_t ci = 0; ci < chunks.size(); ++ci) {
    const int k = (int)(ci % HostPipe::kSlots);
    char* slot = slots + k * slot_bytes;
    char* pbase = slot;  // each array: slot_elems elements of up to 4 bytes
    char* mbase = slot + arr_bytes;
    char* vbase = slot + 2 * arr_bytes;
    char* gbase = slot + (adam ? 3 : 2) * arr_bytes;
    if (ci >= (size_t)HostPipe::kSlots) TK_CUDA_TRY(cudaStreamWaitEvent(P->h2d, P->out_done[k], 0));
    std::vector<tk_leaf> dl;
    uint64_t at = 0;
    for (const Piece& pc : chunks[ci]) {
      const tk_leaf& L = leaves[pc.leaf];
      const size_t pe = esize(L.p_dtype), ge = esize(L.g_dtype);
      tk_leaf d = L;
      d.n = pc.cnt;
      d.p = pbase + at * 4;
      d.m = reinterpret_cast<float*>(mbase + at * 4);
      d.v = adam ? reinterpret_cast<float*>(vbase + at * 4) : nullptr;
      TK_CUDA_TRY(cudaMemcpyAsync(d.p, static_cast<const char*>(L.p) + pc.off * pe, pc.cnt * pe,
                                  cudaMemcpyHostToDevice, P->h2d));
      TK_CUDA_TRY(cudaMemcpyAsync(d.m, L.m + pc.off, pc.cnt * 4, cudaMemcpyHostToDevice, P->h2d));
      if (adam)
        TK_CUDA_TRY(cudaMemcpyAsync(d.v, L.v + pc.off, pc.cnt * 4, cudaMemcpyHostToDevice, P->h2d));
      if (clip) {
        d.g = gdev + goff[pc.leaf] + pc.off * ge;
      } else {
        d.g = gbase + at * 4;
        TK_CUDA_TRY(cudaMemcpyAsync(const_cast<void*>(d.g), static_cast<const char*>(L.g) + pc.off * ge,
                                    pc.cnt * ge, cudaMemcpyHostToDevice, P->h2d));
      }
      dl.push_back(d);
      at += (pc.cnt + 63) / 64 * 64;
    }
    TK_CUDA_TRY(cudaEventRecord(P->in_ready[k], P->h2d));
    TK_CUDA_TRY(cudaStreamWaitEvent(s, P->in_ready[k], 0));
    Plan plan;
    make_plan(dl.data(), dl.size(), kind, &plan);
    for (size_t t = 0; t < plan.tables.size(); ++t)
      TK_TRY(launch_table(plan, t, kind, c, partials, n_partials, max_norm, nullptr,
                          (clip && ci == 0 && t == 0) ? scale_dev : nullptr, s));
    TK_CUDA_TRY(cudaEventRecord(P->done[k], s));
    TK_CUDA_TRY(cudaStreamWaitEvent(P->d2h, P->done[k], 0));
    size_t j = 0;
    for (const Piece& pc : chunks[ci]) {
      const tk_leaf& L = leaves[pc.leaf];
      const tk_leaf& d = dl[j++];
      const size_t pe = esize(L.p_dtype);
      TK_CUDA_TRY(cudaMemcpyAsync(static_cast<char*>(L.p) + pc.off * pe, d.p, pc.cnt * pe,
                                  cudaMemcpyDeviceToHost, P->d2h));
      TK_CUDA_TRY(cudaMemcpyAsync(L.m + pc.off, d.m, pc.cnt * 4, cudaMemcpyDeviceToHost, P->d2h));
      if (adam)
        TK_CUDA_TRY(cudaMemcpyAsync(L.v + pc.off, d.v, pc.cnt * 4, cudaMemcpyDeviceToHost, P->d2h));
    }
    TK_CUDA_TRY(cudaEventRecord(P->out_done[k], P->d2h));
  }
  // the caller's stream (and the scratch it frees) waits for the last copies
  TK_CUDA_TRY(cudaEventRecord(P->end, P->d2h));
  TK_CUDA_TRY(cudaStreamWaitEvent(s, P->end, 0));
  join_guard.armed = false;
  float scale = 1.0f;
  if (clip) TK_CUDA_TRY(cudaMemcpyAsync(&scale, scale_dev, 4, cudaMemcpyDeviceToHost, s));
  TK_CUDA_TRY(cudaStreamSynchronize(s));
  if (clip_scale_out) *clip_scale_out = scale;
  return TK_OK;
}

// Pinned host leaves, many of them small: every leaf costs the copy engines
// seven transfers with a fixed cost each (about 60 us per leaf, measured), so
// f32 leaves of at most kSmallElems elements are gathered on the host into one
// pinned staging block per array, each at a 64-element-aligned offset with
// zeros in between, and the block goes through the pipeline as one leaf.  The
// update is element-wise and zeros stay zero (g = m = v = 0 leaves p = 0), so
// the result is the per-leaf step; Tier 1 sums the same squares plus zeros.
// p, m and v are copied back to the caller's leaves afterwards.
static int step_host_staged(const tk_leaf* leaves, size_t n, int kind, const tk_hparams& hp,
                            uint64_t step, float max_norm, float* clip_scale_out,
                            cudaStream_t s, void* comm) {
  constexpr uint64_t kSmallElems = 64u << 10;
  const bool adam = kind == TK_ADAMW;
  std::vector<size_t> small;
  std::vector<tk_leaf> rest;
  uint64_t total = 0;
  for (size_t i = 0; i < n; ++i) {
    const tk_leaf& L = leaves[i];
    if (L.n > 0 && L.n <= kSmallElems && L.p_dtype == TK_F32 && L.g_dtype == TK_F32) {
      small.push_back(i);
      total += (L.n + 63) / 64 * 64;
    } else {
      rest.push_back(L);
    }
  }
  if (small.size() < 2)
    return step_host_pipelined(leaves, n, kind, hp, step, max_norm, clip_scale_out, s, comm);
  // per-device pinned staging, grown on demand; one staged step at a time
  struct Stage {
    std::mutex mu;
    float* buf = nullptr;
    uint64_t elems = 0;  // per array
  };
  static Stage stages[64];
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(TK_ERR_CUDA, "device index %d out of range", dev);
  Stage& st = stages[dev];
  std::lock_guard<std::mutex> lock(st.mu);
  if (st.elems < total) {
    if (st.buf) cudaFreeHost(st.buf);
    st.buf = nullptr;
    st.elems = 0;
    if (cudaHostAlloc(reinterpret_cast<void**>(&st.buf), sizeof(float) * 4 * total,
                      cudaHostAllocDefault) != cudaSuccess) {
      cudaGetLastError();
      return set_error(TK_ERR_ALLOC, "could not allocate %llu bytes of pinned staging",
                       (unsigned long long)(sizeof(float) * 4 * total));
    }
    st.elems = total;
  }
  float* P = st.buf;
  float* G = P + total;
  float* M = G + total;
  float* V = M + total;
  std::vector<uint64_t> off(small.size());
  uint64_t at = 0;
  for (size_t k = 0; k < small.size(); ++k) {
    const tk_leaf& L = leaves[small[k]];
    const uint64_t len = (L.n + 63) / 64 * 64;
    off[k] = at;
    std::memcpy(P + at, L.p, L.n * 4);
    std::memcpy(G + at, L.g, L.n * 4);
    std::memcpy(M + at, L.m, L.n * 4);
    if (adam) std::memcpy(V + at, L.v, L.n * 4);
    if (len > L.n) {
      for (float* a : {P, G, M, V}) std::memset(a + at + L.n, 0, (len - L.n) * 4);
    }
    at += len;
  }
  tk_leaf block;
  std::memset(&block, 0, sizeof(block));
  block.p = P;
  block.g = G;
  block.m = M;
  block.v = adam ? V : nullptr;
  block.n = total;
  block.p_dtype = TK_F32;
  block.g_dtype = TK_F32;
  rest.insert(rest.begin(), block);
  TK_TRY(step_host_pipelined(rest.data(), rest.size(), kind, hp, step, max_norm, clip_scale_out,
                             s, comm));
  for (size_t k = 0; k < small.size(); ++k) {
    const tk_leaf& L = leaves[small[k]];
    std::memcpy(L.p, P + off[k], L.n * 4);
    std::memcpy(L.m, M + off[k], L.n * 4);
    if (adam) std::memcpy(L.v, V + off[k], L.n * 4);
  }
  return TK_OK;
}

// Pageable host leaves: copy everything the step touches into device scratch,
// run the device step there and copy p, m, v back.  Synchronous.
static int step_host(const tk_leaf* leaves, size_t n, int kind, const tk_hparams& hp,
                     uint64_t step, float max_norm, float* clip_scale_out, cudaStream_t s,
                     void* comm = nullptr) {
  size_t bytes = 64;
  for (size_t i = 0; i < n; ++i) {
    const tk_leaf& L = leaves[i];
    if (L.n == 0) continue;
    bytes += (L.n * esize(L.p_dtype) + 255) / 256 * 256;
    bytes += (L.n * esize(L.g_dtype) + 255) / 256 * 256;
    bytes += (L.n * 4 + 255) / 256 * 256 * (kind == TK_ADAMW ? 2 : 1);
  }
  Scratch stage;
  TK_TRY(stage.alloc(bytes, s));
  char* cur = static_cast<char*>(stage.get());
  float* scale_dev = reinterpret_cast<float*>(cur);
  cur += 64;
  std::vector<tk_leaf> dev(leaves, leaves + n);
  for (size_t i = 0; i < n; ++i) {
    const tk_leaf& L = leaves[i];
    if (L.n == 0) continue;
    auto take = [&](size_t b) {
      char* r = cur;
      cur += (b + 255) / 256 * 256;
      return r;
    };
    char* gdev = take(L.n * esize(L.g_dtype));
    dev[i].p = take(L.n * esize(L.p_dtype));
    dev[i].g = gdev;
    dev[i].m = reinterpret_cast<float*>(take(L.n * 4));
    dev[i].v = kind == TK_ADAMW ? reinterpret_cast<float*>(take(L.n * 4)) : nullptr;
    TK_CUDA_TRY(cudaMemcpyAsync(gdev, L.g, L.n * esize(L.g_dtype), cudaMemcpyHostToDevice, s));
    TK_CUDA_TRY(cudaMemcpyAsync(dev[i].p, L.p, L.n * esize(L.p_dtype), cudaMemcpyHostToDevice, s));
    TK_CUDA_TRY(cudaMemcpyAsync(dev[i].m, L.m, L.n * 4, cudaMemcpyHostToDevice, s));
    if (kind == TK_ADAMW)
      TK_CUDA_TRY(cudaMemcpyAsync(dev[i].v, L.v, L.n * 4, cudaMemcpyHostToDevice, s));
  }
  bool written = false;
  TK_TRY(step_device(dev.data(), n, kind, hp, step, max_norm, scale_dev, &written, s, comm));
  for (size_t i = 0; i < n; ++i) {
    const tk_leaf& L = leaves[i];
    if (L.n == 0) continue;
    TK_CUDA_TRY(cudaMemcpyAsync(L.p, dev[i].p, L.n * esize(L.p_dtype), cudaMemcpyDeviceToHost, s));
    TK_CUDA_TRY(cudaMemcpyAsync(L.m, dev[i].m, L.n * 4, cudaMemcpyDeviceToHost, s));
    if (kind == TK_ADAMW)
      TK_CUDA_TRY(cudaMemcpyAsync(L.v, dev[i].v, L.n * 4, cudaMemcpyDeviceToHost, s));
  }
  float scale = 1.0f;
  if (written) TK_CUDA_TRY(cudaMemcpyAsync(&scale, scale_dev, 4, cudaMemcpyDeviceToHost, s));
  TK_CUDA_TRY(cudaStreamSynchronize(s));
  if (clip_scale_out) *clip_scale_out = scale;
  return TK_OK;
}

static int step_entry(const tk_leaf* leaves, size_t n, int kind, const tk_hparams* hp,
                      uint64_t step, float max_norm, float* clip_scale_out, float* scale_dev,
                      bool sync, cudaStream_t s, void* comm = nullptr) {
  if (hp == nullptr) return set_error(TK_ERR_INVALID, "hparams is NULL");
  Residency where;
  TK_TRY(validate_leaves(leaves, n, kind, &where));
  if (where == Residency::kHost) {
    if (!sync)
      return set_error(TK_ERR_INVALID, "the asynchronous step takes device buffers only");
    if (all_pinned(leaves, n, kind))
      return step_host_staged(leaves, n, kind, *hp, step, max_norm, clip_scale_out, s, comm);
    return step_host(leaves, n, kind, *hp, step, max_norm, clip_scale_out, s, comm);
  }
  if (!sync) {
    bool written = false;
    TK_TRY(step_device(leaves, n, kind, *hp, step, max_norm, scale_dev, &written, s));
    if (scale_dev != nullptr && !written) {
      const float one = 1.0f;
      TK_CUDA_TRY(cudaMemcpyAsync(scale_dev, &one, 4, cudaMemcpyHostToDevice, s));
    }
    return TK_OK;
  }
  Scratch sc;
  float* dscale = nullptr;
  if (clip_scale_out != nullptr && max_norm > 0.0f) {
    TK_TRY(sc.alloc(64, s));
    dscale = static_cast<float*>(sc.get());
  }
  bool written = false;
  TK_TRY(step_device(leaves, n, kind, *hp, step, max_norm, dscale, &written, s, comm));
  float scale = 1.0f;
  if (written) TK_CUDA_TRY(cudaMemcpyAsync(&scale, dscale, 4, cudaMemcpyDeviceToHost, s));
  TK_CUDA_TRY(cudaStreamSynchronize(s));
  if (clip_scale_out) *clip_scale_out = scale;
  return TK_OK;
}

}  // namespace tk

using namespace tk;

extern "C" {

const char* tk_last_error(void) { return g_last_error.c_str(); }

int tk_abi_version(void) { return TK_ABI_VERSION; }

int tk_testing_library_device_bytes(uint64_t* bytes_out) {
  g_last_error.clear();
  if (bytes_out == nullptr) return set_error(TK_ERR_INVALID, "bytes_out is NULL");
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(TK_ERR_CUDA, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_pool_mu);
  uint64_t bytes = 0;
  if (g_pools[dev] != nullptr) {
    cuuint64_t reserved = 0;
    TK_CUDA_TRY(cudaMemPoolGetAttribute(g_pools[dev], cudaMemPoolAttrReservedMemCurrent, &reserved));
    bytes += reserved;
  }
  if (g_status[dev] != nullptr) bytes += 256;
  *bytes_out = bytes;
  return TK_OK;
}

int tk_verify(const tk_pipeline* pipeline) {
  g_last_error.clear();
  return verify_pipeline(pipeline);
}

int tk_layout_from_shapes(const uint64_t* num_elements, size_t n_leaves, uint64_t* byte_offsets,
                          uint64_t* total_bytes) {
  g_last_error.clear();
  if (n_leaves > 0 && (num_elements == nullptr || byte_offsets == nullptr))
    return set_error(TK_ERR_INVALID, "null shape or offset array");
  if (total_bytes == nullptr) return set_error(TK_ERR_INVALID, "total_bytes is NULL");
  // arena.rs:34-57: pad each offset up to a 64-byte cache line
  uint64_t cur = 0;
  for (size_t i = 0; i < n_leaves; ++i) {
    const uint64_t rem = cur % 64;
    if (rem) cur += 64 - rem;
    byte_offsets[i] = cur;
    cur += num_elements[i] * 4;
  }
  *total_bytes = cur;
  return TK_OK;
}

int tk_step_two_tier(const tk_pipeline* pipeline, const tk_leaf* leaves, size_t n_leaves,
                     int32_t kind, const tk_hparams* hp, uint64_t step, float* clip_scale_out,
                     void* stream) {
  g_last_error.clear();
  TK_TRY(verify_pipeline(pipeline));
  return step_entry(leaves, n_leaves, kind, hp, step, pipeline->max_norm, clip_scale_out,
                    nullptr, true, static_cast<cudaStream_t>(stream));
}

int tk_step_arena(const tk_pipeline* pipeline, float* params_arena, const float* grads_arena,
                  float* m1_arena, float* m2_arena, uint64_t arena_bytes,
                  const uint64_t* slot_offsets, const uint64_t* slot_elems, size_t n_slots,
                  int32_t kind, const tk_hparams* hp, uint64_t step, float* clip_scale_out,
                  void* stream) {
  g_last_error.clear();
  if (n_slots > 0 && (slot_offsets == nullptr || slot_elems == nullptr))
    return set_error(TK_ERR_INVALID, "null slot offsets or sizes");
  if (params_arena == nullptr || grads_arena == nullptr || m1_arena == nullptr ||
      (kind == TK_ADAMW && m2_arena == nullptr))
    return set_error(TK_ERR_INVALID, "null arena");
  // lib.rs:47-62: one TensorBuffer per slot, at the same byte offset in every arena
  std::vector<tk_leaf> leaves(n_slots);
  for (size_t i = 0; i < n_slots; ++i) {
    const uint64_t off = slot_offsets[i], n = slot_elems[i];
    if (off % 4 != 0)
      return set_error(TK_ERR_INVALID, "slot %zu: byte offset %llu is not a multiple of 4", i,
                       (unsigned long long)off);
    if (off > arena_bytes || n > (arena_bytes - off) / 4)
      return set_error(TK_ERR_INVALID, "slot %zu (%llu elements at byte %llu) does not fit an "
                       "arena of %llu bytes", i, (unsigned long long)n, (unsigned long long)off,
                       (unsigned long long)arena_bytes);
    const uint64_t e = off / 4;
    leaves[i] = {params_arena + e, grads_arena + e, m1_arena + e,
                 m2_arena ? m2_arena + e : nullptr, n, TK_F32, TK_F32};
  }
  return tk_step_two_tier(pipeline, leaves.data(), n_slots, kind, hp, step, clip_scale_out,
                          stream);
}

// The pipeline step_fast_buffers builds (crates/tikun-py/src/lib.rs:183-192).
static const tk_schedule_node kFastNodes[3] = {
    {"load_g", TK_ROLE_LOAD, 64, 4, 8, 2},
    {"fma_opt", TK_ROLE_COMPUTE, 64, 4, 8, 2},
    {"store_p", TK_ROLE_STORE, 64, 4, 8, 2},
};

int tk_step_buffers(const tk_leaf* leaves, size_t n_leaves, int32_t kind, const tk_hparams* hp,
                    uint64_t step, float max_norm, float* clip_scale_out, void* stream) {
  const tk_pipeline pl = {kFastNodes, 3, max_norm > 0.0f ? max_norm : 0.0f};
  return tk_step_two_tier(&pl, leaves, n_leaves, kind, hp, step, clip_scale_out, stream);
}

int tk_step_buffers_sharded(const tk_leaf* leaves, size_t n_leaves, int32_t kind,
                            const tk_hparams* hp, uint64_t step, float max_norm,
                            float* clip_scale_out, void* nccl_comm, void* stream) {
  g_last_error.clear();
  if (nccl_comm == nullptr) return set_error(TK_ERR_INVALID, "nccl_comm is NULL");
  const tk_pipeline pl = {kFastNodes, 3, max_norm > 0.0f ? max_norm : 0.0f};
  TK_TRY(verify_pipeline(&pl));
  return step_entry(leaves, n_leaves, kind, hp, step, max_norm > 0.0f ? max_norm : 0.0f,
                    clip_scale_out, nullptr, true, static_cast<cudaStream_t>(stream), nccl_comm);
}

int tk_step_buffers_async(const tk_leaf* leaves, size_t n_leaves, int32_t kind,
                          const tk_hparams* hp, uint64_t step, float max_norm,
                          float* clip_scale_dev, void* stream) {
  g_last_error.clear();
  const tk_pipeline pl = {kFastNodes, 3, max_norm};
  TK_TRY(verify_pipeline(&pl));
  return step_entry(leaves, n_leaves, kind, hp, step, max_norm > 0.0f ? max_norm : 0.0f,
                    nullptr, clip_scale_dev, false, static_cast<cudaStream_t>(stream));
}

int tk_set_reserved_sms(int sms) {
  g_last_error.clear();
  if (sms < 0 || sms > 1024) return set_error(TK_ERR_INVALID, "reserved SM count %d out of range", sms);
  g_reserved_sms.store(sms);
  return TK_OK;
}

int tk_set_update_events(void* start_event, void* stop_event) {
  g_last_error.clear();
  if ((start_event == nullptr) != (stop_event == nullptr))
    return set_error(TK_ERR_INVALID, "set both events or neither");
  g_update_start = static_cast<cudaEvent_t>(start_event);
  g_update_stop = static_cast<cudaEvent_t>(stop_event);
  return TK_OK;
}

int tk_apply_pointwise_peers(const tk_leaf* leaves, size_t n_leaves, int32_t kind,
                             const tk_hparams* hp, uint64_t step, const float* scale_dev,
                             const int64_t* peer_deltas, int n_peers, void* stream) {
  g_last_error.clear();
  if (hp == nullptr) return set_error(TK_ERR_INVALID, "hparams is NULL");
  if (n_peers < 0 || n_peers > kMaxPeers || (n_peers > 0 && peer_deltas == nullptr))
    return set_error(TK_ERR_INVALID, "n_peers must be 0..%d with a delta for each", kMaxPeers);
  for (int i = 0; i < n_peers; ++i)  // the kernel's vector stores keep their alignment
    if (peer_deltas[i] % 16 != 0)
      return set_error(TK_ERR_INVALID, "peer delta %lld is not a multiple of 16 bytes",
                       (long long)peer_deltas[i]);
  Residency where;
  TK_TRY(validate_leaves(leaves, n_leaves, kind, &where));
  if (where == Residency::kHost)
    return set_error(TK_ERR_INVALID, "tk_apply_pointwise_peers takes device buffers");
  PeerSet peers;
  std::memset(&peers, 0, sizeof(peers));
  peers.n = n_peers;
  for (int i = 0; i < n_peers; ++i) peers.delta[i] = peer_deltas[i];
  // every leaf through the register kernel, which carries the peer stores
  Plan plan;
  const int dts[2] = {TK_F32, TK_BF16};
  for (int pd : dts)
    for (int gd : dts) {
      size_t before = plan.tables.size();
      build_tables(leaves, n_leaves, kind, pd, gd, &plan.tables);
      for (size_t i = before; i < plan.tables.size(); ++i) {
        plan.pdt.push_back(pd);
        plan.gdt.push_back(gd);
      }
    }
  const PointwiseConsts c = make_consts(kind, *hp, step);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (size_t i = 0; i < plan.tables.size(); ++i)
    TK_TRY(launch_pointwise(plan.tables[i], kind, plan.pdt[i], plan.gdt[i], c, nullptr, 0, 0.f,
                            scale_dev, nullptr, s, &peers));
  return TK_OK;
}

typedef CUresult (*GetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

static int alloc_base(const void* ptr, char** base) {
  static GetAddressRangeFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000,
                                                     cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess)
      return set_error(TK_ERR_CUDA, "cuMemGetAddressRange is not available from the driver");
    fn = (GetAddressRangeFn)p;
  }
  CUdeviceptr b = 0;
  size_t sz = 0;
  if (fn(&b, &sz, (CUdeviceptr)(uintptr_t)ptr) != CUDA_SUCCESS)
    return set_error(TK_ERR_INVALID, "%p is not inside a device allocation", ptr);
  *base = reinterpret_cast<char*>((uintptr_t)b);
  return TK_OK;
}

static std::mutex g_ipc_mu;
static std::vector<std::pair<char*, char*>> g_ipc_open;  // (returned pointer, mapped base)

int tk_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out) {
  g_last_error.clear();
  if (ptr == nullptr || handle_out == nullptr || offset_out == nullptr)
    return set_error(TK_ERR_INVALID, "null argument");
  char* base = nullptr;
  TK_TRY(alloc_base(ptr, &base));
  cudaIpcMemHandle_t h;
  TK_CUDA_TRY(cudaIpcGetMemHandle(&h, base));
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = (uint64_t)(static_cast<const char*>(ptr) - base);
  return TK_OK;
}

int tk_ipc_import(const void* handle, uint64_t offset, void** ptr_out) {
  g_last_error.clear();
  if (handle == nullptr || ptr_out == nullptr) return set_error(TK_ERR_INVALID, "null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  TK_CUDA_TRY(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
  char* p = static_cast<char*>(base) + offset;
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  g_ipc_open.emplace_back(p, static_cast<char*>(base));
  *ptr_out = p;
  return TK_OK;
}

int tk_ipc_close(void* ptr) {
  g_last_error.clear();
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  for (size_t i = 0; i < g_ipc_open.size(); ++i)
    if (g_ipc_open[i].first == ptr) {
      char* base = g_ipc_open[i].second;
      g_ipc_open.erase(g_ipc_open.begin() + (long)i);
      TK_CUDA_TRY(cudaIpcCloseMemHandle(base));
      return TK_OK;
    }
  return set_error(TK_ERR_INVALID, "%p was not returned by tk_ipc_import", ptr);
}

int tk_grad_sumsq(const tk_leaf* leaves, size_t n_leaves, double* sumsq_dev, void* stream) {
  g_last_error.clear();
  if (sumsq_dev == nullptr) return set_error(TK_ERR_INVALID, "sumsq_dev is NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Residency where;
  TK_TRY(validate_leaves(leaves, n_leaves, TK_SGD, &where));
  if (where == Residency::kHost) return set_error(TK_ERR_INVALID, "tk_grad_sumsq takes device buffers");
  Plan plan;
  make_plan(leaves, n_leaves, TK_SGD, &plan);
  if (plan.tables.empty()) {
    TK_CUDA_TRY(cudaMemsetAsync(sumsq_dev, 0, sizeof(double), s));
    return TK_OK;
  }
  Scratch sc;
  double* partials = nullptr;
  int n_partials = 0;
  TK_TRY(launch_norm(plan, &sc, &partials, &n_partials, s));
  return launch_sumsq_reduce(partials, n_partials, sumsq_dev, s);
}

int tk_clip_scale(const double* sumsq_dev, float max_norm, float* scale_dev, void* stream) {
  g_last_error.clear();
  if (sumsq_dev == nullptr || scale_dev == nullptr)
    return set_error(TK_ERR_INVALID, "null sumsq or scale pointer");
  return launch_clip_scale(sumsq_dev, 1, max_norm, scale_dev, static_cast<cudaStream_t>(stream));
}

int tk_apply_pointwise(const tk_leaf* leaves, size_t n_leaves, int32_t kind, const tk_hparams* hp,
                       uint64_t step, const float* scale_dev, void* stream) {
  g_last_error.clear();
  if (hp == nullptr) return set_error(TK_ERR_INVALID, "hparams is NULL");
  Residency where;
  TK_TRY(validate_leaves(leaves, n_leaves, kind, &where));
  if (where == Residency::kHost)
    return set_error(TK_ERR_INVALID, "tk_apply_pointwise takes device buffers");
  Plan plan;
  make_plan(leaves, n_leaves, kind, &plan);
  const PointwiseConsts c = make_consts(kind, *hp, step);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (size_t i = 0; i < plan.tables.size(); ++i)
    TK_TRY(launch_table(plan, i, kind, c, nullptr, 0, 0.f, scale_dev, nullptr, s));
  return TK_OK;
}

}  // extern "C"
