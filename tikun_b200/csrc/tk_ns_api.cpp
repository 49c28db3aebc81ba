// C-ABI entry points of the Newton-Schulz engine (include/tikun_cuda.h):
// tk_newton_schulz_2d / _3d (the reference's newton_schulz_2d_ffi and
// newton_schulz_3d_ffi) and tk_muon_step (momentum, Nesterov, Newton-Schulz
// and the scaled update of python/tikun/muon_nd.py:104-160 in one call).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "tk_internal.h"
#include "tk_ns.h"
#include "tk_testing.h"

namespace tk {

static size_t ns_scratch_budget() {
  const char* e = std::getenv("TIKUN_NS_SCRATCH_GB");
  double gb = e ? std::atof(e) : 8.0;
  if (!(gb > 0.0)) gb = 8.0;
  return (size_t)(gb * (1ull << 30));
}

// Operand format of the Newton-Schulz kernels: 0 f16, 1 bf16, 2 f16 pairs,
// 3 f16 pairs for X only.  Formats 2 and 3 use the split scratch layout.
static int fmt_of(int precision) {
  switch (precision) {
    case TK_NS_F16: return 0;
    case TK_NS_BF16: return 1;
    case TK_NS_F16X3: return 2;
    case TK_NS_F16X2: return 3;
  }
  return -1;
}

// Reads and clears the device status word after the stream has drained.
static int check_status(cudaStream_t s) {
  int* status = nullptr;
  TK_TRY(device_status_word(&status));
  int h = 0;
  TK_CUDA_TRY(cudaStreamSynchronize(s));
  TK_CUDA_TRY(cudaMemcpy(&h, status, sizeof(int), cudaMemcpyDeviceToHost));
  if (h != 0) {
    TK_CUDA_TRY(cudaMemset(status, 0, sizeof(int)));
    return set_error(TK_ERR_DEVICE,
                     "a Newton-Schulz kernel gave up on a bounded wait (code %d); results of "
                     "this call are not valid",
                     h);
  }
  return TK_OK;
}

// Copy-engine exchange of finished parameters: one non-blocking stream per
// peer (per device), fed after each wave of a Muon step.
// By default the copies are made by an SM kernel on a side stream (stream[0])
// that runs on SMs the Newton-Schulz GEMMs leave free; with
// TIKUN_MUON_COPY_ENGINE=1, by the copy engines, one stream per peer.
struct PeerCopy {
  int n = 0;
  const int64_t* delta = nullptr;
  bool engines = false;
  bool join = true;  // the caller's stream waits for the copies at the end of the call
  int sms = 0;       // SMs left to the copy kernel
  cudaStream_t stream[kMaxPeers] = {};
  cudaEvent_t wave_done = nullptr;
  cudaEvent_t done[kMaxPeers] = {};
};

static int peer_copy_streams(PeerCopy* pc) {
  struct PerDevice {
    bool ready = false;
    cudaStream_t stream[kMaxPeers];
    cudaEvent_t wave_done;
    cudaEvent_t done[kMaxPeers];
  };
  static PerDevice devs[64];
  static std::mutex mu;
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(TK_ERR_CUDA, "device index %d out of range", dev);
  const char* e = std::getenv("TIKUN_MUON_COPY_ENGINE");
  pc->engines = e != nullptr && e[0] == '1';
  const char* k = std::getenv("TIKUN_MUON_COPY_SMS");
  pc->sms = k ? std::max(1, std::atoi(k)) : 16;
  std::lock_guard<std::mutex> lock(mu);
  PerDevice& d = devs[dev];
  if (!d.ready) {
    for (int j = 0; j < kMaxPeers; ++j) {
      TK_CUDA_TRY(cudaStreamCreateWithFlags(&d.stream[j], cudaStreamNonBlocking));
      TK_CUDA_TRY(cudaEventCreateWithFlags(&d.done[j], cudaEventDisableTiming));
    }
    TK_CUDA_TRY(cudaEventCreateWithFlags(&d.wave_done, cudaEventDisableTiming));
    d.ready = true;
  }
  for (int j = 0; j < kMaxPeers; ++j) {
    pc->stream[j] = d.stream[j];
    pc->done[j] = d.done[j];
  }
  pc->wave_done = d.wave_done;
  return TK_OK;
}

// Shape groups of one call run concurrently on side streams: a persistent
// GEMM launch of one group leaves SMs idle in its first and last waves, and
// another group's launch fills them.  That pays for calls of modest work (the
// GPT-2 and 1.3B shapes: 3 % and 10 % per clock) but not for the 8B shapes,
// whose launches are many waves long (4 % slower per clock), so calls under
// 50 dense TFLOP use 2 streams and larger ones 1; TIKUN_NS_STREAMS (1..4)
// overrides.
struct GroupStreams {
  std::mutex mu;  // serialises the enqueueing, not the device work
  bool ready = false;
  cudaStream_t st[4] = {};
  cudaEvent_t fork = nullptr;
  cudaEvent_t join[4] = {};
  unsigned calls = 0;  // successive calls take successive pairs of streams, so
                       // calls from different caller streams can overlap too
};

static int ns_streams(double call_flops) {
  static const int forced = [] {
    const char* e = std::getenv("TIKUN_NS_STREAMS");
    return e ? std::max(1, std::min(std::atoi(e), 4)) : 0;
  }();
  if (forced) return forced;
  return call_flops < 50e12 ? 2 : 1;
}

static int group_streams(GroupStreams** out) {
  static GroupStreams devs[64];
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(TK_ERR_CUDA, "device index %d out of range", dev);
  *out = &devs[dev];
  return TK_OK;
}

// Runs NS over matrices that are all m x n or n x m, in waves that fit the
// scratch budget and the per-launch pointer capacity.  With `copy`, each
// wave's finished parameters are copied into the peers' copies by the copy
// engines while the next wave computes.
static int run_batches(int64_t m, int64_t n, const std::vector<const void*>& src,
                       const std::vector<void*>& dst, const std::vector<float*>* mom,
                       const std::vector<uint8_t>& tall, int src_dtype, int dst_dtype, int update,
                       float scale_wide, float scale_tall, float mu, float om, int nesterov,
                       int steps, int fmt, cudaStream_t s, const PeerSet* peers = nullptr,
                       PeerCopy* copy = nullptr) {
  const int64_t count = (int64_t)src.size();
  const ns::GroupLayout one = ns::group_layout(m, n, 1, fmt >= 2);
  int64_t per_wave = std::max<int64_t>(
      1, std::min<int64_t>({count, (int64_t)(ns_scratch_budget() / one.scratch_bytes),
                            (int64_t)ns::kMaxBatch}));
  // With a copy exchange, a group runs in at least three waves: the copies of
  // one wave's parameters then cross NVLink while the next waves compute,
  // instead of all after the group's last GEMM.
  if (copy != nullptr && copy->n > 0) per_wave = std::max<int64_t>(1, std::min(per_wave, (count + 2) / 3));
  int* status = nullptr;
  TK_TRY(device_status_word(&status));
  for (int64_t first = 0; first < count; first += per_wave) {
    const int64_t nb = std::min(per_wave, count - first);
    const ns::GroupLayout L = ns::group_layout(m, n, nb, fmt >= 2);
    Scratch scratch;
    TK_TRY(scratch.alloc(L.scratch_bytes, s));
    ns::GroupIO io;
    io.src = src.data() + first;
    io.dst = dst.data() + first;
    io.mom = mom ? mom->data() + first : nullptr;
    io.tall = tall.data() + first;
    io.src_dtype = src_dtype;
    io.dst_dtype = dst_dtype;
    io.update = update;
    io.upd_scale_wide = scale_wide;
    io.upd_scale_tall = scale_tall;
    io.mu = mu;
    io.om = om;
    io.nesterov = nesterov;
    io.peers = peers;
    TK_TRY(ns::run_group(L, io, steps, fmt, scratch.get(), status, s));
    if (copy != nullptr && copy->n > 0) {
      const size_t bytes = (size_t)m * (size_t)n * (dst_dtype == TK_F32 ? 4 : 2);
      TK_CUDA_TRY(cudaEventRecord(copy->wave_done, s));
      if (copy->engines) {
        for (int j = 0; j < copy->n; ++j) {
          TK_CUDA_TRY(cudaStreamWaitEvent(copy->stream[j], copy->wave_done, 0));
          for (int64_t i = first; i < first + nb; ++i)
            TK_CUDA_TRY(cudaMemcpyAsync(static_cast<char*>(dst[i]) + copy->delta[j], dst[i],
                                        bytes, cudaMemcpyDeviceToDevice, copy->stream[j]));
        }
      } else {
        cudaStream_t cs = copy->stream[0];
        TK_CUDA_TRY(cudaStreamWaitEvent(cs, copy->wave_done, 0));
        static thread_local ns::PeerCopyList list;
        list.n = 0;
        list.unit0[0] = 0;
        PeerSet peers;
        std::memset(&peers, 0, sizeof(peers));
        peers.n = copy->n;
        for (int j = 0; j < copy->n; ++j) peers.delta[j] = copy->delta[j];
        for (int64_t i = first; i < first + nb; ++i) {
          const uint8_t* src = static_cast<const uint8_t*>(dst[i]);
          if ((reinterpret_cast<uintptr_t>(src) & 15) != 0) {  // rare: the engines copy it
            for (int j = 0; j < copy->n; ++j)
              TK_CUDA_TRY(cudaMemcpyAsync(static_cast<char*>(dst[i]) + copy->delta[j], dst[i],
                                          bytes, cudaMemcpyDeviceToDevice, cs));
            continue;
          }
          list.src[list.n] = src;
          list.bytes[list.n] = bytes;
          list.unit0[list.n + 1] = list.unit0[list.n] + (bytes + 15) / 16;
          ++list.n;
        }
        TK_TRY(ns::launch_peer_copy(list, peers, 2 * copy->sms, cs));
      }
    }
  }
  return TK_OK;
}

static size_t dt_size(int dt) { return dt == TK_F32 ? 4 : 2; }

static int ns_entry(void* base, int64_t heads, int64_t rows, int64_t cols, int32_t steps,
                    int32_t dtype, int32_t precision, cudaStream_t s) {
  if (heads < 0 || rows < 0 || cols < 0 || steps < 0)
    return set_error(TK_ERR_INVALID, "negative size or step count");
  if (dtype != TK_F32 && dtype != TK_BF16)
    return set_error(TK_ERR_INVALID, "matrix dtype %d is not f32 or bf16", dtype);
  const int fmt = fmt_of(precision);
  if (fmt < 0) return set_error(TK_ERR_INVALID, "unknown Newton-Schulz precision %d", precision);
  // tensor_engine.rs:13-15: empty matrices are left alone
  if (heads == 0 || rows == 0 || cols == 0) return TK_OK;
  if (base == nullptr) return set_error(TK_ERR_INVALID, "matrix pointer is NULL");
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  Residency where;
  TK_TRY(classify_pointer(base, &where, dev));
  const size_t esz = dt_size(dtype);
  const size_t bytes = (size_t)heads * rows * cols * esz;
  Scratch stage;
  char* dbase = static_cast<char*>(base);
  if (where == Residency::kHost) {
    TK_TRY(stage.alloc(bytes, s));
    dbase = static_cast<char*>(stage.get());
    TK_CUDA_TRY(cudaMemcpyAsync(dbase, base, bytes, cudaMemcpyHostToDevice, s));
  }
  std::vector<const void*> src(heads);
  std::vector<void*> dst(heads);
  std::vector<uint8_t> tall(heads, rows > cols ? 1 : 0);
  for (int64_t h = 0; h < heads; ++h) {
    dst[h] = dbase + (size_t)h * rows * cols * esz;
    src[h] = dst[h];
  }
  TK_TRY(run_batches(std::min(rows, cols), std::max(rows, cols), src, dst, nullptr, tall, dtype,
                     dtype, 0, 0.f, 0.f, 0.f, 0.f, 0, steps, fmt, s));
  if (where == Residency::kHost)
    TK_CUDA_TRY(cudaMemcpyAsync(base, dbase, bytes, cudaMemcpyDeviceToHost, s));
  return check_status(s);
}

// Host Muon leaves (the reference's calling convention: MuonND keeps its
// momentum in NumPy arrays and hands host buffers to the engine,
// python/tikun/muon_nd.py:96-126).  Every shape group is cut into chunks of
// whole matrices that fit one device slot (TIKUN_MUON_STAGE_MB, default
// 2048 MB, at least one matrix); chunk c moves through a ring of three slots:
// the H2D stream copies its g, momentum and p into slot c % 3, the caller's
// stream runs the fused Muon step on them (momentum, Nesterov, Newton-Schulz,
// update), and the D2H stream copies p and momentum back, so both copy
// directions overlap the tensor-core work.  Synchronous, like the reference.
struct HostGroup {
  int64_t m = 0, n = 0;
  int p_dtype = TK_F32, g_dtype = TK_F32;
  std::vector<const void*> g;
  std::vector<void*> p;
  std::vector<float*> mom;
  std::vector<uint8_t> tall;
};

struct MuonHostPipe {
  std::mutex mu;  // one host-buffer Muon step at a time per device
  cudaStream_t h2d = nullptr, d2h = nullptr;
  static constexpr int kSlots = 3;
  cudaEvent_t start = nullptr, end = nullptr;
  cudaEvent_t in_ready[kSlots] = {}, done[kSlots] = {}, out_done[kSlots] = {};
};

static int muon_host_pipe(MuonHostPipe** out) {
  static MuonHostPipe pipes[64];
  static bool ready[64] = {};
  static std::mutex init_mu;
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(TK_ERR_CUDA, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(init_mu);
  if (!ready[dev]) {
    MuonHostPipe& P = pipes[dev];
    TK_CUDA_TRY(cudaStreamCreateWithFlags(&P.h2d, cudaStreamNonBlocking));
    TK_CUDA_TRY(cudaStreamCreateWithFlags(&P.d2h, cudaStreamNonBlocking));
    for (cudaEvent_t* e : {&P.start, &P.end})
      TK_CUDA_TRY(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
    for (int k = 0; k < MuonHostPipe::kSlots; ++k)
      for (cudaEvent_t* e : {&P.in_ready[k], &P.done[k], &P.out_done[k]})
        TK_CUDA_TRY(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
    ready[dev] = true;
  }
  *out = &pipes[dev];
  return TK_OK;
}

static size_t muon_stage_budget() {
  const char* e = std::getenv("TIKUN_MUON_STAGE_MB");
  double mb = e ? std::atof(e) : 2048.0;
  if (!(mb > 0.0)) mb = 2048.0;
  return (size_t)(mb * (1ull << 20));
}

static int muon_step_host(const std::vector<HostGroup>& groups, const tk_muon_hparams& hp,
                          float mu, float om, int fmt, cudaStream_t s) {
  NvtxRange range("tikun/muon_host_pipeline");
  MuonHostPipe* P = nullptr;
  TK_TRY(muon_host_pipe(&P));
  std::lock_guard<std::mutex> serial(P->mu);
  struct Chunk {
    size_t group;
    size_t first, count;
  };
  const size_t budget = muon_stage_budget();
  auto a256 = [](size_t b) { return (b + 255) / 256 * 256; };
  std::vector<Chunk> chunks;
  size_t slot_bytes = 0;
  for (size_t gi = 0; gi < groups.size(); ++gi) {
    const HostGroup& G = groups[gi];
    const size_t mat = (size_t)G.m * (size_t)G.n;
    const size_t per = a256(mat * dt_size(G.p_dtype)) + a256(mat * dt_size(G.g_dtype)) + a256(mat * 4);
    const size_t fit = std::max<size_t>(1, budget / per);
    for (size_t first = 0; first < G.g.size(); first += fit) {
      const size_t cnt = std::min(fit, G.g.size() - first);
      chunks.push_back({gi, first, cnt});
      slot_bytes = std::max(slot_bytes, cnt * per);
    }
  }
  if (chunks.empty()) return TK_OK;
  Scratch sc;
  TK_TRY(sc.alloc(slot_bytes * MuonHostPipe::kSlots, s));
  // On an early return the slots go back to the pool in s's order while copies
  // on the side streams may still use them: s first waits for both.
  struct JoinSideStreams {
    MuonHostPipe* P;
    cudaStream_t s;
    bool armed = true;
    ~JoinSideStreams() {
      if (!armed) return;
      if (cudaEventRecord(P->start, P->h2d) == cudaSuccess) cudaStreamWaitEvent(s, P->start, 0);
      if (cudaEventRecord(P->end, P->d2h) == cudaSuccess) cudaStreamWaitEvent(s, P->end, 0);
    }
  } join_guard{P, s};
  char* slots = static_cast<char*>(sc.get());
  // everything starts after the caller's earlier work on s
  TK_CUDA_TRY(cudaEventRecord(P->start, s));
  TK_CUDA_TRY(cudaStreamWaitEvent(P->h2d, P->start, 0));
  TK_CUDA_TRY(cudaStreamWaitEvent(P->d2h, P->start, 0));
  for (size_t ci = 0; ci < chunks.size(); ++ci) {
    const Chunk& C = chunks[ci];
    const HostGroup& G = groups[C.group];
    const int k = (int)(ci % MuonHostPipe::kSlots);
    char* at = slots + (size_t)k * slot_bytes;
    if (ci >= (size_t)MuonHostPipe::kSlots)
      TK_CUDA_TRY(cudaStreamWaitEvent(P->h2d, P->out_done[k], 0));
    const size_t mat = (size_t)G.m * (size_t)G.n;
    const size_t pb = mat * dt_size(G.p_dtype), gb = mat * dt_size(G.g_dtype), mb = mat * 4;
    std::vector<const void*> dg(C.count);
    std::vector<void*> dp(C.count);
    std::vector<float*> dm(C.count);
    std::vector<uint8_t> tall(G.tall.begin() + C.first, G.tall.begin() + C.first + C.count);
    for (size_t j = 0; j < C.count; ++j) {
      const size_t i = C.first + j;
      dp[j] = at;
      at += a256(pb);
      dg[j] = at;
      at += a256(gb);
      dm[j] = reinterpret_cast<float*>(at);
      at += a256(mb);
      TK_CUDA_TRY(cudaMemcpyAsync(const_cast<void*>(dg[j]), G.g[i], gb, cudaMemcpyHostToDevice, P->h2d));
      TK_CUDA_TRY(cudaMemcpyAsync(dm[j], G.mom[i], mb, cudaMemcpyHostToDevice, P->h2d));
      TK_CUDA_TRY(cudaMemcpyAsync(dp[j], G.p[i], pb, cudaMemcpyHostToDevice, P->h2d));
    }
    TK_CUDA_TRY(cudaEventRecord(P->in_ready[k], P->h2d));
    TK_CUDA_TRY(cudaStreamWaitEvent(s, P->in_ready[k], 0));
    const float upd_wide = (float)(-hp.lr * std::sqrt(std::max(1.0, (double)G.m / (double)G.n)));
    const float upd_tall = (float)(-hp.lr * std::sqrt(std::max(1.0, (double)G.n / (double)G.m)));
    TK_TRY(run_batches(G.m, G.n, dg, dp, &dm, tall, G.g_dtype, G.p_dtype, 1, upd_wide, upd_tall,
                       mu, om, hp.nesterov ? 1 : 0, hp.ns_steps, fmt, s));
    TK_CUDA_TRY(cudaEventRecord(P->done[k], s));
    TK_CUDA_TRY(cudaStreamWaitEvent(P->d2h, P->done[k], 0));
    for (size_t j = 0; j < C.count; ++j) {
      const size_t i = C.first + j;
      TK_CUDA_TRY(cudaMemcpyAsync(G.p[i], dp[j], pb, cudaMemcpyDeviceToHost, P->d2h));
      TK_CUDA_TRY(cudaMemcpyAsync(G.mom[i], dm[j], mb, cudaMemcpyDeviceToHost, P->d2h));
    }
    TK_CUDA_TRY(cudaEventRecord(P->out_done[k], P->d2h));
  }
  // the caller's stream (and the slots it frees) waits for the last copies
  TK_CUDA_TRY(cudaEventRecord(P->end, P->d2h));
  TK_CUDA_TRY(cudaStreamWaitEvent(s, P->end, 0));
  join_guard.armed = false;
  return check_status(s);
}

}  // namespace tk

using namespace tk;

extern "C" {

int tk_newton_schulz_2d(void* matrix, int64_t rows, int64_t cols, int32_t steps, int32_t dtype,
                        int32_t precision, void* stream) {
  clear_error();
  return ns_entry(matrix, 1, rows, cols, steps, dtype, precision,
                  static_cast<cudaStream_t>(stream));
}

int tk_newton_schulz_3d(void* tensor, int64_t num_heads, int64_t head_dim_out,
                        int64_t head_dim_in, int32_t steps, int32_t dtype, int32_t precision,
                        void* stream) {
  clear_error();
  return ns_entry(tensor, num_heads, head_dim_out, head_dim_in, steps, dtype, precision,
                  static_cast<cudaStream_t>(stream));
}

static int muon_step(const tk_muon_leaf* leaves, size_t n_leaves, const tk_muon_hparams* hp,
                     const PeerSet* peers, PeerCopy* copy, void* stream) {
  if (hp == nullptr) return set_error(TK_ERR_INVALID, "hparams is NULL");
  if (n_leaves > 0 && leaves == nullptr) return set_error(TK_ERR_INVALID, "leaves is NULL");
  const int fmt = fmt_of(hp->precision);
  if (fmt < 0) return set_error(TK_ERR_INVALID, "unknown Newton-Schulz precision %d", hp->precision);
  if (hp->ns_steps < 0) return set_error(TK_ERR_INVALID, "negative Newton-Schulz step count");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));

  struct Range {
    uintptr_t lo, hi;
    bool w;
  };
  std::vector<Range> ranges;
  // group by (rows, cols, p dtype, g dtype): every head of every leaf of a
  // group is one matrix of one batch
  struct Batch {
    std::vector<const void*> g;
    std::vector<void*> p;
    std::vector<float*> mom;
    std::vector<uint8_t> tall;
  };
  std::map<std::tuple<int64_t, int64_t, int, int>, Batch> groups;
  Residency where = Residency::kNone;
  for (size_t i = 0; i < n_leaves; ++i) {
    const tk_muon_leaf& L = leaves[i];
    if (L.heads < 0 || L.rows < 0 || L.cols < 0)
      return set_error(TK_ERR_INVALID, "leaf %zu: negative shape", i);
    if ((L.p_dtype != TK_F32 && L.p_dtype != TK_BF16) || (L.g_dtype != TK_F32 && L.g_dtype != TK_BF16))
      return set_error(TK_ERR_INVALID, "leaf %zu: p and g must be f32 or bf16", i);
    const int64_t heads = L.heads == 0 ? 1 : L.heads;
    if (L.rows == 0 || L.cols == 0) continue;
    if (L.p == nullptr || L.g == nullptr || L.momentum == nullptr)
      return set_error(TK_ERR_INVALID, "leaf %zu: null p, g or momentum", i);
    const size_t n = (size_t)heads * L.rows * L.cols;
    ranges.push_back({(uintptr_t)L.p, (uintptr_t)L.p + n * dt_size(L.p_dtype), true});
    ranges.push_back({(uintptr_t)L.g, (uintptr_t)L.g + n * dt_size(L.g_dtype), false});
    ranges.push_back({(uintptr_t)L.momentum, (uintptr_t)L.momentum + n * 4, true});
    for (const void* ptr : {(const void*)L.p, L.g, (const void*)L.momentum}) {
      Residency r;
      TK_TRY(classify_pointer(ptr, &r, dev));
      if (where == Residency::kNone) where = r;
      if (r != where)
        return set_error(TK_ERR_INVALID,
                         "leaf %zu: host and device buffers are mixed in one Muon call", i);
      if (r == Residency::kHost && (peers != nullptr || copy != nullptr))
        return set_error(TK_ERR_INVALID,
                         "leaf %zu: the multi-GPU Muon steps take device buffers", i);
    }
    // an m x n and an n x m matrix share one batch (m = min, n = max)
    Batch& b = groups[std::make_tuple(std::min(L.rows, L.cols), std::max(L.rows, L.cols),
                                      L.p_dtype, L.g_dtype)];
    const size_t mat = (size_t)L.rows * L.cols;
    for (int64_t h = 0; h < heads; ++h) {
      b.g.push_back(static_cast<const char*>(L.g) + h * mat * dt_size(L.g_dtype));
      b.p.push_back(static_cast<char*>(L.p) + h * mat * dt_size(L.p_dtype));
      b.mom.push_back(L.momentum + h * mat);
      b.tall.push_back(L.rows > L.cols ? 1 : 0);
    }
  }
  std::sort(ranges.begin(), ranges.end(), [](const Range& a, const Range& b) { return a.lo < b.lo; });
  uintptr_t max_any = 0, max_w = 0;
  for (const Range& r : ranges) {
    if ((r.w && max_any > r.lo) || max_w > r.lo)
      return set_error(TK_ERR_INVALID, "Muon leaf buffers overlap at %p", (void*)r.lo);
    max_any = std::max(max_any, r.hi);
    if (r.w) max_w = std::max(max_w, r.hi);
  }
  // muon_nd.py: buf *= momentum; buf += (1.0 - momentum) * g  (NumPy float32 with
  // Python-float scalars rounded once), scale = max(1, rows/cols) ** 0.5,
  // p += (-lr * scale) * U
  const float mu = (float)hp->momentum;
  const float om = (float)(1.0 - hp->momentum);
  // largest groups first, so that with a copy-engine exchange the bulk of
  // the parameters crosses NVLink while the smaller groups compute
  std::vector<std::pair<double, decltype(groups)::iterator>> order;
  for (auto it = groups.begin(); it != groups.end(); ++it) {
    const double m = (double)std::get<0>(it->first), n = (double)std::get<1>(it->first);
    order.emplace_back(-(double)it->second.g.size() * (4.0 * m * m * n + 2.0 * m * m * m), it);
  }
  std::stable_sort(order.begin(), order.end(),
                   [](const auto& a, const auto& b) { return a.first < b.first; });
  if (where == Residency::kHost) {
    std::vector<HostGroup> hg;
    for (const auto& o : order) {
      const auto& key = o.second->first;
      const Batch& b = o.second->second;
      HostGroup h;
      h.m = std::get<0>(key);
      h.n = std::get<1>(key);
      h.p_dtype = std::get<2>(key);
      h.g_dtype = std::get<3>(key);
      h.g = b.g;
      h.p = b.p;
      h.mom = b.mom;
      h.tall = b.tall;
      hg.push_back(std::move(h));
    }
    return muon_step_host(hg, *hp, mu, om, fmt, s);
  }
  double call_flops = 0.0;
  for (const auto& o : order) call_flops -= o.first * (double)hp->ns_steps;
  const int ks = std::min<int>(ns_streams(call_flops), (int)order.size());
  GroupStreams* GS = nullptr;
  std::unique_lock<std::mutex> gs_lock;
  if (ks > 1) {
    TK_TRY(group_streams(&GS));
    gs_lock = std::unique_lock<std::mutex>(GS->mu);
    if (!GS->ready) {
      for (int j = 0; j < 4; ++j) {
        TK_CUDA_TRY(cudaStreamCreateWithFlags(&GS->st[j], cudaStreamNonBlocking));
        TK_CUDA_TRY(cudaEventCreateWithFlags(&GS->join[j], cudaEventDisableTiming));
      }
      TK_CUDA_TRY(cudaEventCreateWithFlags(&GS->fork, cudaEventDisableTiming));
      GS->ready = true;
    }
    TK_CUDA_TRY(cudaEventRecord(GS->fork, s));
  }
  const int base = ks > 1 ? (int)((GS->calls++ * (unsigned)ks) % 4u) : 0;
  auto sidx = [&](int j) { return (base + j) % 4; };
  if (ks > 1)
    for (int j = 0; j < ks; ++j) TK_CUDA_TRY(cudaStreamWaitEvent(GS->st[sidx(j)], GS->fork, 0));
  NvtxRange range("tikun/muon_step");
  for (size_t gi = 0; gi < order.size(); ++gi) {
    auto& kv = *order[gi].second;
    cudaStream_t gs = ks > 1 ? GS->st[sidx((int)(gi % (size_t)ks))] : s;
    const int64_t m = std::get<0>(kv.first), n = std::get<1>(kv.first);
    const int pdt = std::get<2>(kv.first), gdt = std::get<3>(kv.first);
    // rows/cols is m/n (<= 1) for a wide matrix and n/m for a tall one
    const float upd_wide = (float)(-hp->lr * std::sqrt(std::max(1.0, (double)m / (double)n)));
    const float upd_tall = (float)(-hp->lr * std::sqrt(std::max(1.0, (double)n / (double)m)));
    TK_TRY(run_batches(m, n, kv.second.g, kv.second.p, &kv.second.mom, kv.second.tall, gdt, pdt,
                       1, upd_wide, upd_tall, mu, om, hp->nesterov ? 1 : 0, hp->ns_steps, fmt, gs,
                       peers, copy));
  }
  if (ks > 1)  // the caller's stream waits for every group
    for (int j = 0; j < ks; ++j) {
      TK_CUDA_TRY(cudaEventRecord(GS->join[sidx(j)], GS->st[sidx(j)]));
      TK_CUDA_TRY(cudaStreamWaitEvent(s, GS->join[sidx(j)], 0));
    }
  if (copy != nullptr && copy->join) {
    const int streams = copy->engines ? copy->n : (copy->n > 0 ? 1 : 0);
    for (int j = 0; j < streams; ++j) {  // the caller's stream waits for every copy
      TK_CUDA_TRY(cudaEventRecord(copy->done[j], copy->stream[j]));
      TK_CUDA_TRY(cudaStreamWaitEvent(s, copy->done[j], 0));
    }
  }
  return TK_OK;
}

int tk_muon_step(const tk_muon_leaf* leaves, size_t n_leaves, const tk_muon_hparams* hp,
                 void* stream) {
  clear_error();
  return muon_step(leaves, n_leaves, hp, nullptr, nullptr, stream);
}

int tk_muon_step_peers(const tk_muon_leaf* leaves, size_t n_leaves, const tk_muon_hparams* hp,
                       const int64_t* peer_deltas, int n_peers, void* stream) {
  clear_error();
  if (n_peers < 0 || n_peers > kMaxPeers || (n_peers > 0 && peer_deltas == nullptr))
    return set_error(TK_ERR_INVALID, "n_peers must be 0..%d with a delta for each", kMaxPeers);
  for (int i = 0; i < n_peers; ++i)  // vector stores into the peers keep their alignment
    if (peer_deltas[i] % 16 != 0)
      return set_error(TK_ERR_INVALID, "peer delta %lld is not a multiple of 16 bytes",
                       (long long)peer_deltas[i]);
  PeerSet peers;
  std::memset(&peers, 0, sizeof(peers));
  peers.n = n_peers;
  for (int i = 0; i < n_peers; ++i) peers.delta[i] = peer_deltas[i];
  return muon_step(leaves, n_leaves, hp, &peers, nullptr, stream);
}

static int muon_step_copy(const tk_muon_leaf* leaves, size_t n_leaves, const tk_muon_hparams* hp,
                          const int64_t* peer_deltas, int n_peers, bool join, void* stream) {
  clear_error();
  if (n_peers < 0 || n_peers > kMaxPeers || (n_peers > 0 && peer_deltas == nullptr))
    return set_error(TK_ERR_INVALID, "n_peers must be 0..%d with a delta for each", kMaxPeers);
  for (int i = 0; i < n_peers; ++i)  // vector stores into the peers keep their alignment
    if (peer_deltas[i] % 16 != 0)
      return set_error(TK_ERR_INVALID, "peer delta %lld is not a multiple of 16 bytes",
                       (long long)peer_deltas[i]);
  PeerCopy copy;
  TK_TRY(peer_copy_streams(&copy));
  copy.n = n_peers;
  copy.delta = peer_deltas;
  copy.join = join;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the copy streams start after the caller's earlier work
  TK_CUDA_TRY(cudaEventRecord(copy.wave_done, s));
  for (int j = 0; j < n_peers; ++j) TK_CUDA_TRY(cudaStreamWaitEvent(copy.stream[j], copy.wave_done, 0));
  // the GEMMs leave SMs free for the copy kernel
  if (!copy.engines && n_peers > 0) ns::set_gemm_reserved_sms(copy.sms);
  const int st = muon_step(leaves, n_leaves, hp, nullptr, &copy, stream);
  ns::set_gemm_reserved_sms(0);
  return st;
}

int tk_muon_step_copy(const tk_muon_leaf* leaves, size_t n_leaves, const tk_muon_hparams* hp,
                      const int64_t* peer_deltas, int n_peers, void* stream) {
  return muon_step_copy(leaves, n_leaves, hp, peer_deltas, n_peers, true, stream);
}

int tk_muon_step_copy_deferred(const tk_muon_leaf* leaves, size_t n_leaves,
                               const tk_muon_hparams* hp, const int64_t* peer_deltas, int n_peers,
                               void* stream) {
  return muon_step_copy(leaves, n_leaves, hp, peer_deltas, n_peers, false, stream);
}

int tk_muon_copy_join(void* stream) {
  clear_error();
  PeerCopy copy;
  TK_TRY(peer_copy_streams(&copy));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int j = 0; j < kMaxPeers; ++j) {
    TK_CUDA_TRY(cudaEventRecord(copy.done[j], copy.stream[j]));
    TK_CUDA_TRY(cudaStreamWaitEvent(s, copy.done[j], 0));
  }
  return TK_OK;
}

int tk_device_status(int* status_out) {
  clear_error();
  if (status_out == nullptr) return set_error(TK_ERR_INVALID, "status_out is NULL");
  int* status = nullptr;
  TK_TRY(device_status_word(&status));
  TK_CUDA_TRY(cudaDeviceSynchronize());
  TK_CUDA_TRY(cudaMemcpy(status_out, status, sizeof(int), cudaMemcpyDeviceToHost));
  if (*status_out != 0) TK_CUDA_TRY(cudaMemset(status, 0, sizeof(int)));
  return TK_OK;
}

int tk_testing_gemm_tn(const void* P, const void* Q, void* D, int batch, int M, int N, int K,
                       int64_t ldp, int64_t ldq, int64_t ldd, float alpha, int fmt, void* stream) {
  clear_error();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* status = nullptr;
  TK_TRY(device_status_word(&status));
  TK_TRY(ns::plain_gemm(static_cast<const uint16_t*>(P), static_cast<const uint16_t*>(Q),
                        static_cast<uint16_t*>(D), batch, M, N, K, ldp, ldq, ldd, alpha, fmt,
                        status, s));
  return check_status(s);
}

int tk_testing_bounded_wait(int limit_ms, void* stream) {
  clear_error();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* status = nullptr;
  TK_TRY(device_status_word(&status));
  TK_TRY(ns::bounded_wait_probe(status, limit_ms, s));
  return check_status(s);
}

}  // extern "C"
