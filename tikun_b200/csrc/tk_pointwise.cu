// Tier 1 (global L2 norm -> clip scale) and Tier 2 (AdamW / Lion / SGD) for
// sm_100a.  Memory-bound streaming kernels over a table of leaves.
//
// Work split: the leaves of one launch form one index space of "quads"
// (4-element groups, a leaf's last quad may be partial).  Every CTA takes an
// equal contiguous slice of that space, so the grid is balanced whatever the
// leaf sizes (a 38.6M-element embedding next to 768-element LayerNorms), and
// each CTA streams contiguous memory.  A quad is one 128-bit access per f32
// array (64-bit for bf16) when the leaf's pointers are aligned for it.
//
// Arithmetic follows the reference's x86 scalar code element by element
// (crates/tikun-cpu/src/lib.rs:258-270, :347-358, :419-427): every multiply,
// add, divide and square root is a separately rounded IEEE f32 operation
// (__fmul_rn & co. are never contracted into FMAs), denormals are kept, so the
// results are bit-identical to tikun-cpu's.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>

#include "tk_internal.h"
#include "tk_pointwise_math.cuh"

namespace tk {
namespace {

using namespace pw;

// Tuning knobs (compile time): quads each thread keeps in flight per loop
// trip, the minimum resident CTAs per SM the register budget must allow,
// whether the loop is software-pipelined (TK_PW_PIPE below), and the cache
// policy of the streaming accesses (0: default, 1: evict-first).  Measured on
// B200 (AdamW update, CUDA events, SM clock 1965 MHz), all settings giving
// the same bits:
//   all-f32 leaves: pipelined, 5 quads per trip, 1 CTA of 256 threads per SM
//     (GPT-2-small table 0.595 -> 0.579 ms = 6022 GB/s, flat 100M elements
//     0.478 -> 0.455 ms = 6150 GB/s); unpipelined the best was 4 quads with 2
//     CTAs per SM; 6 pipelined quads spill and fall to 4500 GB/s;
//   leaves with a bf16 p or g: 1 quad per trip, 6 CTAs per SM, not pipelined
//     (flat 100M bf16 p and g 0.491 -> 0.420 ms = 5235 GB/s; 2 quads with 3
//     CTAs per SM before).
#ifndef TK_PW_UNROLL
#define TK_PW_UNROLL 5
#endif
#ifndef TK_PW_MINBLOCKS
#define TK_PW_MINBLOCKS 1
#endif
#ifndef TK_PW_UNROLL_BF16
#define TK_PW_UNROLL_BF16 1
#endif
#ifndef TK_PW_MINBLOCKS_BF16
#define TK_PW_MINBLOCKS_BF16 6
#endif
#ifndef TK_PW_STREAMING
#define TK_PW_STREAMING 0
#endif
// Grid sizing: 0 = one wave of resident CTAs, each with a long contiguous
// slice; 1 = one short slice (kThreads * kUnroll groups) per CTA, many waves,
// so the CTAs sweep memory together.
#ifndef TK_PW_OVERSUB
#define TK_PW_OVERSUB 0
#endif
// Software pipelining of the vector loop: 1 = each thread issues the loads of
// its next trip's quads before it computes and stores the current ones, so a
// warp's memory requests stay in flight through its arithmetic.
#ifndef TK_PW_PIPE
#define TK_PW_PIPE 1
#endif
#ifndef TK_PW_PIPE_BF16
#define TK_PW_PIPE_BF16 0
#endif
constexpr int kThreads = 256;

// PEER: the instantiation launched when updated parameters also go to the
// peers' copies over NVLink.  It keeps the settings measured for it before
// the local update was retuned (4 quads with 2 CTAs per SM for f32, 2 quads
// with 3 CTAs for bf16, not pipelined): with 6 CTAs of 40 registers the bf16
// variant's seven peer stores per quad spilled, and the 2-GPU Muon+AdamW step
// lost 9 ms to it.  Both instantiations keep the (runtime) peer-store loop:
// compiled without it, the pipelined f32 loop was scheduled into 224
// registers instead of 235 and ran 8 % slower.
template <int PDT, int GDT, bool PEER = false>
struct Tune {
  static constexpr bool all_f32 = PDT == TK_F32 && GDT == TK_F32;
  static constexpr int unroll = PEER ? (all_f32 ? 4 : 2) : (all_f32 ? TK_PW_UNROLL : TK_PW_UNROLL_BF16);
  static constexpr int minblocks =
      PEER ? (all_f32 ? 2 : 3) : (all_f32 ? TK_PW_MINBLOCKS : TK_PW_MINBLOCKS_BF16);
  static constexpr bool pipe = PEER ? false : (all_f32 ? TK_PW_PIPE != 0 : TK_PW_PIPE_BF16 != 0);
};

// One trip's quads of one thread: quad lq + u*kThreads for u < U, the ones
// below `end` active.
template <int U>
struct Batch {
  float P[U][4], G[U][4], M[U][4], V[U][4];
  bool act[U];
};

template <typename T>
__device__ __forceinline__ T ld_stream(const T* p) {
  if constexpr (TK_PW_STREAMING) return __ldcs(p);
  else return *p;
}

template <typename T>
__device__ __forceinline__ void st_stream(T* p, const T& v) {
  if constexpr (TK_PW_STREAMING) __stcs(p, v);
  else *p = v;
}

template <int DT>
__device__ __forceinline__ void load_quad(const void* base, uint64_t e, float (&x)[4]) {
  if constexpr (DT == TK_F32) {
    const float4 q = ld_stream(reinterpret_cast<const float4*>(static_cast<const float*>(base) + e));
    x[0] = q.x; x[1] = q.y; x[2] = q.z; x[3] = q.w;
  } else {
    const uint2 q = ld_stream(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(base) + e));
    x[0] = bf16_to_f32(q.x & 0xffffu); x[1] = bf16_to_f32(q.x >> 16);
    x[2] = bf16_to_f32(q.y & 0xffffu); x[3] = bf16_to_f32(q.y >> 16);
  }
}

template <int DT>
__device__ __forceinline__ void store_quad(void* base, uint64_t e, const float (&x)[4]) {
  if constexpr (DT == TK_F32) {
    st_stream(reinterpret_cast<float4*>(static_cast<float*>(base) + e), make_float4(x[0], x[1], x[2], x[3]));
  } else {
    uint2 q;
    q.x = f32_to_bf16(x[0]) | (f32_to_bf16(x[1]) << 16);
    q.y = f32_to_bf16(x[2]) | (f32_to_bf16(x[3]) << 16);
    st_stream(reinterpret_cast<uint2*>(static_cast<uint16_t*>(base) + e), q);
  }
}

template <int DT>
__device__ __forceinline__ float load1(const void* base, uint64_t e) {
  if constexpr (DT == TK_F32) return static_cast<const float*>(base)[e];
  else return bf16_to_f32(static_cast<const uint16_t*>(base)[e]);
}

template <int DT>
__device__ __forceinline__ void store1(void* base, uint64_t e, float x) {
  if constexpr (DT == TK_F32) static_cast<float*>(base)[e] = x;
  else static_cast<uint16_t*>(base)[e] = static_cast<uint16_t>(f32_to_bf16(x));
}

// ------------------------------------------------------------------ Tier 1
template <int GDT>
__global__ void __launch_bounds__(kThreads)
sumsq_partials_kernel(const __grid_constant__ LeafTable t, double* __restrict__ partials) {
  const uint64_t total = t.total_quads;
  const uint64_t q0 = total * blockIdx.x / gridDim.x;
  const uint64_t q1 = total * (blockIdx.x + 1) / gridDim.x;
  // four independent accumulators, one per quad of a loop trip, so that four
  // loads per thread are in flight; summed in a fixed order at the end
  constexpr int kU = 4;
  double acc[kU] = {0.0, 0.0, 0.0, 0.0};
  if (q0 < q1) {
    int li = find_leaf(t, q0);
    uint64_t q = q0;
    while (q < q1) {
      const LeafDesc& L = t.leaf[li];
      const uint64_t seg_end = min(q1, L.q_begin + leaf_quads(L));
      const uint64_t a = q - L.q_begin, b = seg_end - L.q_begin;
      // quads [a, full_end) are whole and vector-accessible; the rest go scalar
      const uint64_t full_end = L.vec_ok ? min(b, L.n >> 2) : a;
      for (uint64_t lq = a + threadIdx.x; lq < full_end; lq += (uint64_t)kThreads * kU) {
        float x[kU][4];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const uint64_t qq = lq + (uint64_t)u * kThreads;
          if (qq < full_end) load_quad<GDT>(L.g, qq * 4, x[u]);
          else x[u][0] = x[u][1] = x[u][2] = x[u][3] = 0.0f;
        }
#pragma unroll
        for (int u = 0; u < kU; ++u)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[u] = fma((double)x[u][j], (double)x[u][j], acc[u]);
      }
      for (uint64_t lq = max(a, full_end) + threadIdx.x; lq < b; lq += kThreads) {
        for (uint64_t j = lq * 4; j < min(lq * 4 + 4, L.n); ++j) {
          const double x = load1<GDT>(L.g, j);
          acc[0] = fma(x, x, acc[0]);
        }
      }
      q = seg_end;
      ++li;
    }
  }
  // x*x of an f32 value is exact in f64, so fma == multiply-then-add here.
  const double s = block_sum<kThreads>((acc[0] + acc[1]) + (acc[2] + acc[3]));
  if (threadIdx.x == 0) partials[blockIdx.x] = s;
}

__global__ void __launch_bounds__(kThreads)
sumsq_reduce_kernel(const double* __restrict__ partials, int n, double* __restrict__ total) {
  double acc = 0.0;
  for (int i = threadIdx.x; i < n; i += kThreads) acc += partials[i];
  const double s = block_sum<kThreads>(acc);
  if (threadIdx.x == 0) *total = s;
}

__global__ void __launch_bounds__(kThreads)
clip_scale_kernel(const double* __restrict__ partials, int n, float max_norm,
                  float* __restrict__ scale_out) {
  double acc = 0.0;
  for (int i = threadIdx.x; i < n; i += kThreads) acc += partials[i];
  const double s = block_sum<kThreads>(acc);
  if (threadIdx.x == 0) *scale_out = clip_from_sumsq(s, max_norm);
}

// ------------------------------------------------------------------ Tier 2
// SCALE: 0 = no clipping, 1 = fold partials in every CTA, 2 = read scale_dev.
template <int KIND, int PDT, int GDT, int SCALE, bool PEER>
__global__ void __launch_bounds__(kThreads, (Tune<PDT, GDT, PEER>::minblocks))
pointwise_kernel(const __grid_constant__ LeafTable t, const PointwiseConsts k,
                 const double* __restrict__ partials, int n_partials, float max_norm,
                 const float* __restrict__ scale_dev, float* __restrict__ scale_out,
                 const PeerSet peers) {
  float scale = 1.0f;
  if constexpr (SCALE == 1) {
    __shared__ float s_scale;
    double acc = 0.0;
    for (int i = threadIdx.x; i < n_partials; i += kThreads) acc += partials[i];
    const double s = block_sum<kThreads>(acc);
    if (threadIdx.x == 0) {
      const float sc = clip_from_sumsq(s, max_norm);
      s_scale = sc;
      if (blockIdx.x == 0 && scale_out != nullptr) *scale_out = sc;
    }
    __syncthreads();
    scale = s_scale;
  } else if constexpr (SCALE == 2) {
    scale = *scale_dev;
  }

  const uint64_t total = t.total_quads;
  const uint64_t q0 = total * blockIdx.x / gridDim.x;
  const uint64_t q1 = total * (blockIdx.x + 1) / gridDim.x;
  if (q0 >= q1) return;
  int li = find_leaf(t, q0);
  uint64_t q = q0;
  while (q < q1) {
    const LeafDesc& L = t.leaf[li];
    const uint64_t nq = leaf_quads(L);
    const uint64_t seg_end = min(q1, L.q_begin + nq);
    const uint64_t a = q - L.q_begin, b = seg_end - L.q_begin;
    // quads [a, full_end) are whole and vector-accessible; the rest go scalar
    const uint64_t full_end = L.vec_ok ? min(b, L.n >> 2) : a;
    constexpr int kUnroll = Tune<PDT, GDT, PEER>::unroll;
    constexpr uint64_t kStride = (uint64_t)kThreads * kUnroll;
    auto load_batch = [&](uint64_t lq, Batch<kUnroll>& B) {
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const uint64_t qq = lq + (uint64_t)u * kThreads;
        B.act[u] = qq < full_end;
        if (B.act[u]) {
          const uint64_t e = qq * 4;
          load_quad<GDT>(L.g, e, B.G[u]);
          load_quad<PDT>(L.p, e, B.P[u]);
          load_quad<TK_F32>(L.m, e, B.M[u]);
          if constexpr (KIND == TK_ADAMW) load_quad<TK_F32>(L.v, e, B.V[u]);
        }
      }
    };
    auto update_store = [&](uint64_t lq, Batch<kUnroll>& B) {
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (!B.act[u]) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float g = B.G[u][j];
          if constexpr (SCALE != 0) g = __fmul_rn(g, scale);
          apply<KIND>(B.P[u][j], g, B.M[u][j], B.V[u][j], k);
        }
        const uint64_t e = (lq + (uint64_t)u * kThreads) * 4;
        store_quad<PDT>(L.p, e, B.P[u]);
#pragma unroll
        for (int r = 0; r < kMaxPeers; ++r)  // the updated parameters, into each peer's copy
          if (r < peers.n) store_quad<PDT>(static_cast<char*>(L.p) + peers.delta[r], e, B.P[u]);
        store_quad<TK_F32>(L.m, e, B.M[u]);
        if constexpr (KIND == TK_ADAMW) store_quad<TK_F32>(L.v, e, B.V[u]);
      }
    };
    if constexpr (Tune<PDT, GDT, PEER>::pipe) {
      uint64_t lq = a + threadIdx.x;
      Batch<kUnroll> cur;
      if (lq < full_end) load_batch(lq, cur);
      for (; lq < full_end; lq += kStride) {
        Batch<kUnroll> nxt;
        const bool more = lq + kStride < full_end;
        if (more) load_batch(lq + kStride, nxt);
        update_store(lq, cur);
        if (more) cur = nxt;
      }
    } else {
      for (uint64_t lq = a + threadIdx.x; lq < full_end; lq += kStride) {
        Batch<kUnroll> cur;
        load_batch(lq, cur);
        update_store(lq, cur);
      }
    }
    // ragged tail or unaligned leaf: element by element
    for (uint64_t lq = max(a, full_end) + threadIdx.x; lq < b; lq += kThreads) {
      for (uint64_t e = lq * 4; e < min(lq * 4 + 4, L.n); ++e) {
        float p = load1<PDT>(L.p, e);
        float g = load1<GDT>(L.g, e);
        if constexpr (SCALE != 0) g = __fmul_rn(g, scale);
        float m = L.m[e];
        float v = 0.0f;
        if constexpr (KIND == TK_ADAMW) v = L.v[e];
        apply<KIND>(p, g, m, v, k);
        store1<PDT>(L.p, e, p);
#pragma unroll
        for (int r = 0; r < kMaxPeers; ++r)
          if (r < peers.n) store1<PDT>(static_cast<char*>(L.p) + peers.delta[r], e, p);
        L.m[e] = m;
        if constexpr (KIND == TK_ADAMW) L.v[e] = v;
      }
    }
    q = seg_end;
    ++li;
  }
  if (peers.n) __threadfence_system();  // peer stores visible before the kernel ends
}

template <int KIND, int PDT, int GDT, int SCALE, bool PEER>
int occupancy_grid(uint64_t total_quads) {
  static int per_sm = 0;
  if (per_sm == 0) {
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &occ, pointwise_kernel<KIND, PDT, GDT, SCALE, PEER>, kThreads, 0) != cudaSuccess ||
        occ < 1)
      occ = 1;
    per_sm = occ;
  }
  int sms = 0;
  if (pointwise_sms(&sms) != TK_OK) return 0;
  const int cap = sms * per_sm;
  constexpr int kUnroll = Tune<PDT, GDT, PEER>::unroll;
  const uint64_t want = (total_quads + kThreads * kUnroll - 1) / (kThreads * kUnroll);
  if (TK_PW_OVERSUB) return (int)std::min<uint64_t>(want ? want : 1, 1u << 30);
  return (int)(want < (uint64_t)cap ? (want ? want : 1) : cap);
}

template <int KIND, int PDT, int GDT, int SCALE>
int launch_t(const LeafTable& t, const PointwiseConsts& c, const double* partials,
             int n_partials, float max_norm, const float* scale_dev, float* scale_out,
             cudaStream_t s, const PeerSet& peers) {
  if (peers.n > 0) {
    const int grid = occupancy_grid<KIND, PDT, GDT, SCALE, true>(t.total_quads);
    if (grid <= 0) return set_error(TK_ERR_CUDA, "could not size the pointwise grid");
    pointwise_kernel<KIND, PDT, GDT, SCALE, true><<<grid, kThreads, 0, s>>>(
        t, c, partials, n_partials, max_norm, scale_dev, scale_out, peers);
  } else {
    const int grid = occupancy_grid<KIND, PDT, GDT, SCALE, false>(t.total_quads);
    if (grid <= 0) return set_error(TK_ERR_CUDA, "could not size the pointwise grid");
    pointwise_kernel<KIND, PDT, GDT, SCALE, false><<<grid, kThreads, 0, s>>>(
        t, c, partials, n_partials, max_norm, scale_dev, scale_out, peers);
  }
  TK_CUDA_TRY(cudaGetLastError());
  return TK_OK;
}

template <int KIND, int PDT, int GDT>
int launch_scale(const LeafTable& t, const PointwiseConsts& c, const double* partials,
                 int n_partials, float max_norm, const float* scale_dev, float* scale_out,
                 cudaStream_t s, const PeerSet& pr) {
  if (partials) return launch_t<KIND, PDT, GDT, 1>(t, c, partials, n_partials, max_norm, nullptr, scale_out, s, pr);
  if (scale_dev) return launch_t<KIND, PDT, GDT, 2>(t, c, nullptr, 0, 0.f, scale_dev, nullptr, s, pr);
  return launch_t<KIND, PDT, GDT, 0>(t, c, nullptr, 0, 0.f, nullptr, nullptr, s, pr);
}

template <int KIND>
int launch_kind(const LeafTable& t, int pdt, int gdt, const PointwiseConsts& c,
                const double* partials, int n_partials, float max_norm, const float* scale_dev,
                float* scale_out, cudaStream_t s, const PeerSet& pr) {
  if (pdt == TK_F32 && gdt == TK_F32) return launch_scale<KIND, TK_F32, TK_F32>(t, c, partials, n_partials, max_norm, scale_dev, scale_out, s, pr);
  if (pdt == TK_F32 && gdt == TK_BF16) return launch_scale<KIND, TK_F32, TK_BF16>(t, c, partials, n_partials, max_norm, scale_dev, scale_out, s, pr);
  if (pdt == TK_BF16 && gdt == TK_F32) return launch_scale<KIND, TK_BF16, TK_F32>(t, c, partials, n_partials, max_norm, scale_dev, scale_out, s, pr);
  if (pdt == TK_BF16 && gdt == TK_BF16) return launch_scale<KIND, TK_BF16, TK_BF16>(t, c, partials, n_partials, max_norm, scale_dev, scale_out, s, pr);
  return set_error(TK_ERR_INVALID, "unsupported dtype pair p=%d g=%d", pdt, gdt);
}

}  // namespace

int sumsq_blocks_for(uint64_t total_quads) {
  static int per_sm = 0;
  if (per_sm == 0) {
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, sumsq_partials_kernel<TK_F32>,
                                                      kThreads, 0) != cudaSuccess || occ < 1)
      occ = 1;
    per_sm = occ;
  }
  int sms = 0;
  if (pointwise_sms(&sms) != TK_OK) return 0;
  const int cap = sms * per_sm;
  const uint64_t want = (total_quads + kThreads - 1) / kThreads;
  return (int)(want < (uint64_t)cap ? (want ? want : 1) : cap);
}

int launch_sumsq_partials(const LeafTable& t, int g_dtype, double* partials, int n_blocks,
                          cudaStream_t s) {
  if (g_dtype == TK_F32) sumsq_partials_kernel<TK_F32><<<n_blocks, kThreads, 0, s>>>(t, partials);
  else if (g_dtype == TK_BF16) sumsq_partials_kernel<TK_BF16><<<n_blocks, kThreads, 0, s>>>(t, partials);
  else return set_error(TK_ERR_INVALID, "unsupported gradient dtype %d", g_dtype);
  TK_CUDA_TRY(cudaGetLastError());
  return TK_OK;
}

int launch_sumsq_reduce(const double* partials, int n_partials, double* total, cudaStream_t s) {
  sumsq_reduce_kernel<<<1, kThreads, 0, s>>>(partials, n_partials, total);
  TK_CUDA_TRY(cudaGetLastError());
  return TK_OK;
}

int launch_clip_scale(const double* sumsq, int n_partials, float max_norm, float* scale_out,
                      cudaStream_t s) {
  clip_scale_kernel<<<1, kThreads, 0, s>>>(sumsq, n_partials, max_norm, scale_out);
  TK_CUDA_TRY(cudaGetLastError());
  return TK_OK;
}

int launch_pointwise(const LeafTable& t, int kind, int p_dtype, int g_dtype,
                     const PointwiseConsts& c, const double* partials, int n_partials,
                     float max_norm, const float* scale_dev, float* scale_out, cudaStream_t s,
                     const PeerSet* peers) {
  PeerSet none;
  std::memset(&none, 0, sizeof(none));
  const PeerSet& pr = peers ? *peers : none;
  switch (kind) {
    case TK_ADAMW: return launch_kind<TK_ADAMW>(t, p_dtype, g_dtype, c, partials, n_partials, max_norm, scale_dev, scale_out, s, pr);
    case TK_LION: return launch_kind<TK_LION>(t, p_dtype, g_dtype, c, partials, n_partials, max_norm, scale_dev, scale_out, s, pr);
    case TK_SGD: return launch_kind<TK_SGD>(t, p_dtype, g_dtype, c, partials, n_partials, max_norm, scale_dev, scale_out, s, pr);
    case TK_CUSTOM: return launch_kind<TK_CUSTOM>(t, p_dtype, g_dtype, c, partials, n_partials, max_norm, scale_dev, scale_out, s, pr);
    default: return set_error(TK_ERR_INVALID, "unknown optimizer kind %d", kind);
  }
}

}  // namespace tk
