// Tier 2 for f32 leaves through a bulk-copy pipeline in shared memory.
//
// One CTA per SM, 10 warps.  Warp 0 streams tiles of p, g, m (and v) --
// 1024 aligned 4-element groups of one leaf, 16 KB per array -- into a 3-stage
// shared-memory ring with cp.async.bulk (completion counted on the stage's
// mbarrier); warps 2-9 apply the update in shared memory; warp 1 writes p, m
// (and v) back with bulk stores and frees the stage once they have read it.
// Loads, arithmetic and stores of different tiles overlap, so HBM stays busy
// while the divide/square-root chain of each element runs.  Each CTA takes an
// equal contiguous slice of the launch's group index space (as the register
// kernel does); the partial last group of a leaf is done element by element.
//
// Leaves with misaligned pointers or bf16 p/g go to the register kernel
// (tk_pointwise.cu); the arithmetic (tk_pointwise_math.cuh) is the same.
#include <cuda_runtime.h>

#include <cstdint>

#include "tk_internal.h"
#include "tk_pointwise_math.cuh"
#include "tk_sm100.cuh"

namespace tk {
namespace {

using namespace pw;
using namespace sm100;

// Tile size (4-element groups per array), ring depth, and how many tiles'
// bulk stores may still be reading shared memory before the store warp frees
// their stages.
#ifndef TK_BULK_TILE_QUADS
#define TK_BULK_TILE_QUADS 1024
#endif
#ifndef TK_BULK_STAGES
#define TK_BULK_STAGES 3
#endif
#ifndef TK_BULK_STORE_LAG
#define TK_BULK_STORE_LAG 1
#endif
constexpr int kTileQuads = TK_BULK_TILE_QUADS;
constexpr int kTileBytes = kTileQuads * 16;  // per array
constexpr int kStages = TK_BULK_STAGES;
constexpr int kStoreLag = TK_BULK_STORE_LAG;
static_assert(kStoreLag >= 0 && kStoreLag < kStages, "store lag must leave a free stage");
constexpr int kArrays = 4;
constexpr int kComputeWarps = 8;
constexpr int kComputeThreads = 32 * kComputeWarps;
constexpr int kThreadsB = 32 * (2 + kComputeWarps);
constexpr int kRingBytes = kStages * kArrays * kTileBytes;  // 192 KB
constexpr int kSmemBytesB = kRingBytes + 3 * kStages * 8 + 256;

struct Tile {
  int li;
  uint64_t lq;   // first group within the leaf
  uint32_t cnt;  // groups
};

// Walks the whole 4-element groups of [q, q1) leaf by leaf in tiles of at
// most kTileQuads groups; a leaf's partial last group is skipped (done apart).
struct TileIter {
  const LeafTable* t;
  uint64_t q, q1;
  int li;
  __device__ void init(const LeafTable& tab, uint64_t q0, uint64_t qe) {
    t = &tab;
    q = q0;
    q1 = qe;
    li = q0 < qe ? find_leaf(tab, q0) : 0;
  }
  __device__ bool next(Tile& out) {
    while (q < q1) {
      const LeafDesc& L = t->leaf[li];
      const uint64_t full_end = L.q_begin + (L.n >> 2);
      if (q >= full_end) {
        const uint64_t leaf_end = L.q_begin + leaf_quads(L);
        if (leaf_end > q) q = leaf_end;
        ++li;
        continue;
      }
      const uint64_t end = full_end < q1 ? full_end : q1;
      const uint64_t cnt = end - q < (uint64_t)kTileQuads ? end - q : (uint64_t)kTileQuads;
      out.li = li;
      out.lq = q - L.q_begin;
      out.cnt = (uint32_t)cnt;
      q += cnt;
      return true;
    }
    return false;
  }
};

template <int KIND, int SCALE>
__global__ void __launch_bounds__(kThreadsB, 1)
pointwise_bulk_kernel(const __grid_constant__ LeafTable t, const PointwiseConsts k,
                      const double* __restrict__ partials, int n_partials, float max_norm,
                      const float* __restrict__ scale_dev, float* __restrict__ scale_out,
                      int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                             ~static_cast<uintptr_t>(127));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRingBytes);
  uint64_t* computed = full + kStages;
  uint64_t* empty = computed + kStages;
  __shared__ float s_scale;
  __shared__ int s_abort;
  constexpr int NA = KIND == TK_ADAMW ? 4 : 3;  // p, g, m (, v)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&computed[s], kComputeWarps);
      mbar_init(&empty[s], 1);
    }
    s_abort = 0;
    fence_barrier_init();
  }
  float scale = 1.0f;
  if constexpr (SCALE == 1) {
    // every CTA folds the Tier-1 partials in the same fixed order
    double acc = 0.0;
    for (int i = threadIdx.x; i < n_partials; i += kThreadsB) acc += partials[i];
    const double tot = block_sum<kThreadsB>(acc);
    if (threadIdx.x == 0) {
      const float sc = clip_from_sumsq(tot, max_norm);
      s_scale = sc;
      if (blockIdx.x == 0 && scale_out != nullptr) *scale_out = sc;
    }
  }
  __syncthreads();
  if constexpr (SCALE == 1) scale = s_scale;
  else if constexpr (SCALE == 2) scale = *scale_dev;

  const uint64_t total = t.total_quads;
  const uint64_t q0 = total * blockIdx.x / gridDim.x;
  const uint64_t q1 = total * (blockIdx.x + 1) / gridDim.x;
  volatile int* abort_flag = &s_abort;
  auto buf = [&](int stage, int a) -> float* {
    return reinterpret_cast<float*>(smem + (size_t)(stage * kArrays + a) * kTileBytes);
  };

  if (warp == 0) {
    if (lane == 0) {  // ---- loads
      TileIter it;
      it.init(t, q0, q1);
      Tile tl;
      int stage = 0;
      uint32_t phase = 0;
      while (it.next(tl)) {
        if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, err, 21)) break;
        const LeafDesc& L = t.leaf[tl.li];
        const uint32_t bytes = tl.cnt * 16;
        const uint64_t e = tl.lq * 4;
        mbar_arrive_expect_tx(&full[stage], bytes * NA);
        bulk_load(buf(stage, 0), static_cast<const float*>(L.p) + e, bytes, &full[stage]);
        bulk_load(buf(stage, 1), static_cast<const float*>(L.g) + e, bytes, &full[stage]);
        bulk_load(buf(stage, 2), L.m + e, bytes, &full[stage]);
        if constexpr (NA == 4) bulk_load(buf(stage, 3), L.v + e, bytes, &full[stage]);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- stores
      TileIter it;
      it.init(t, q0, q1);
      Tile tl;
      int stage = 0;
      uint32_t phase = 0;
      uint64_t n_done = 0;  // tiles whose stores have been committed
      while (it.next(tl)) {
        if (!mbar_wait(&computed[stage], phase, abort_flag, err, 22)) break;
        const LeafDesc& L = t.leaf[tl.li];
        const uint32_t bytes = tl.cnt * 16;
        const uint64_t e = tl.lq * 4;
        bulk_store(static_cast<float*>(L.p) + e, buf(stage, 0), bytes);
        bulk_store(L.m + e, buf(stage, 2), bytes);
        if constexpr (NA == 4) bulk_store(L.v + e, buf(stage, 3), bytes);
        bulk_commit();
        ++n_done;
        // the tile kStoreLag back has been read out of shared memory: its
        // stage may be refilled
        bulk_wait_read<kStoreLag>();
        if (n_done > (uint64_t)kStoreLag)
          mbar_arrive(&empty[(int)((n_done - 1 - kStoreLag) % kStages)]);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      bulk_wait_all();
    }
  } else {  // ---- arithmetic, warps 2..9
    const int ct = threadIdx.x - 64;
    TileIter it;
    it.init(t, q0, q1);
    Tile tl;
    int stage = 0;
    uint32_t phase = 0;
    while (it.next(tl)) {
      if (!mbar_wait(&full[stage], phase, abort_flag, err, 23)) break;
      float4* P = reinterpret_cast<float4*>(buf(stage, 0));
      const float4* G = reinterpret_cast<const float4*>(buf(stage, 1));
      float4* M = reinterpret_cast<float4*>(buf(stage, 2));
      float4* V = reinterpret_cast<float4*>(buf(stage, 3));
      for (uint32_t j = ct; j < tl.cnt; j += kComputeThreads) {
        float p[4], g[4], m[4], v[4] = {0.f, 0.f, 0.f, 0.f};
        const float4 p4 = P[j], g4 = G[j], m4 = M[j];
        p[0] = p4.x; p[1] = p4.y; p[2] = p4.z; p[3] = p4.w;
        g[0] = g4.x; g[1] = g4.y; g[2] = g4.z; g[3] = g4.w;
        m[0] = m4.x; m[1] = m4.y; m[2] = m4.z; m[3] = m4.w;
        if constexpr (NA == 4) {
          const float4 v4 = V[j];
          v[0] = v4.x; v[1] = v4.y; v[2] = v4.z; v[3] = v4.w;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float gq = g[q];
          if constexpr (SCALE != 0) gq = __fmul_rn(gq, scale);
          apply<KIND>(p[q], gq, m[q], v[q], k);
        }
        P[j] = make_float4(p[0], p[1], p[2], p[3]);
        M[j] = make_float4(m[0], m[1], m[2], m[3]);
        if constexpr (NA == 4) V[j] = make_float4(v[0], v[1], v[2], v[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&computed[stage]);
      if (++stage == kStages) {
        stage = 0;
        phase ^= 1;
      }
    }
    // the partial last group of each leaf in this CTA's slice, element-wise
    if (ct == 0 && q0 < q1) {
      for (int li = find_leaf(t, q0); li < t.n_leaves && t.leaf[li].q_begin < q1; ++li) {
        const LeafDesc& L = t.leaf[li];
        if ((L.n & 3) == 0) continue;
        const uint64_t tq = L.q_begin + (L.n >> 2);
        if (tq < q0 || tq >= q1) continue;
        float* pp = static_cast<float*>(L.p);
        const float* gg = static_cast<const float*>(L.g);
        for (uint64_t e = (L.n >> 2) * 4; e < L.n; ++e) {
          float p = pp[e], g = gg[e], m = L.m[e], v = NA == 4 ? L.v[e] : 0.f;
          if constexpr (SCALE != 0) g = __fmul_rn(g, scale);
          apply<KIND>(p, g, m, v, k);
          pp[e] = p;
          L.m[e] = m;
          if constexpr (NA == 4) L.v[e] = v;
        }
      }
    }
  }
  __syncthreads();
}

template <int KIND, int SCALE>
int launch_bulk_t(const LeafTable& t, const PointwiseConsts& c, const double* partials,
                  int n_partials, float max_norm, const float* scale_dev, float* scale_out,
                  cudaStream_t s) {
  static bool attr_set[64] = {};
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(TK_ERR_CUDA, "device index %d out of range", dev);
  if (!attr_set[dev]) {
    TK_CUDA_TRY(cudaFuncSetAttribute(pointwise_bulk_kernel<KIND, SCALE>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytesB));
    attr_set[dev] = true;
  }
  int sms = 0;
  TK_TRY(pointwise_sms(&sms));
  int* status = nullptr;
  TK_TRY(device_status_word(&status));
  const uint64_t tiles = (t.total_quads + kTileQuads - 1) / kTileQuads;
  const int grid = (int)(tiles < (uint64_t)sms ? (tiles ? tiles : 1) : sms);
  pointwise_bulk_kernel<KIND, SCALE><<<grid, kThreadsB, kSmemBytesB, s>>>(
      t, c, partials, n_partials, max_norm, scale_dev, scale_out, status);
  TK_CUDA_TRY(cudaGetLastError());
  return TK_OK;
}

template <int KIND>
int launch_bulk_kind(const LeafTable& t, const PointwiseConsts& c, const double* partials,
                     int n_partials, float max_norm, const float* scale_dev, float* scale_out,
                     cudaStream_t s) {
  if (partials) return launch_bulk_t<KIND, 1>(t, c, partials, n_partials, max_norm, nullptr, scale_out, s);
  if (scale_dev) return launch_bulk_t<KIND, 2>(t, c, nullptr, 0, 0.f, scale_dev, nullptr, s);
  return launch_bulk_t<KIND, 0>(t, c, nullptr, 0, 0.f, nullptr, nullptr, s);
}

}  // namespace

int launch_pointwise_bulk(const LeafTable& t, int kind, const PointwiseConsts& c,
                          const double* partials, int n_partials, float max_norm,
                          const float* scale_dev, float* scale_out, cudaStream_t s) {
  switch (kind) {
    case TK_ADAMW: return launch_bulk_kind<TK_ADAMW>(t, c, partials, n_partials, max_norm, scale_dev, scale_out, s);
    case TK_LION: return launch_bulk_kind<TK_LION>(t, c, partials, n_partials, max_norm, scale_dev, scale_out, s);
    case TK_SGD: return launch_bulk_kind<TK_SGD>(t, c, partials, n_partials, max_norm, scale_dev, scale_out, s);
    case TK_CUSTOM: return launch_bulk_kind<TK_CUSTOM>(t, c, partials, n_partials, max_norm, scale_dev, scale_out, s);
    default: return set_error(TK_ERR_INVALID, "unknown optimizer kind %d", kind);
  }
}

}  // namespace tk
