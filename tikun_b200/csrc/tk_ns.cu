// Muon Newton-Schulz on sm_100a: tcgen05 tensor-core GEMMs fed by TMA, with the
// momentum / Nesterov prologue, the Frobenius normalisation and the scaled
// parameter update fused around them.
//
// The quintic iteration of crates/tikun-cpu/src/tensor_engine.rs:12-77,
//     A = X X^T;  B = b A + c A A;  X <- a X + B X       (a, b, c) = (3.4445, -4.7750, 2.0315)
// on X (m x n, m <= n; a tall input is transposed first, :18-34) runs as three
// "TN" GEMMs, D[M x N] = P[M x K] * Q[N x K]^T, whose operands are all K-major
// row-major arrays in HBM:
//   GEMM1  D = X X^T           P = Q = X          symmetric: upper tiles only
//   GEMM2  D = A A = A A^T     P = Q = A          symmetric: upper tiles only
//   GEMM3  D = X^T B  (= (B X)^T)                 P = X^T, Q = B
// GEMM3 produces X_new^T directly; its epilogue stores both X_new^T and X_new
// (a transposed store, which the one-row-per-thread TMEM layout makes
// coalesced), so no operand ever needs the MN-major layout.  Symmetric tiles
// store each element above the diagonal twice (at (r, c) and (c, r)), which
// keeps A and B exactly symmetric in storage.
//
// Kernel: persistent, one CTA per SM, 192 threads.  Warp 0 issues TMA loads of
// 128x64 and 256x64 operand tiles (128-byte swizzle) into a 4-stage ring; warp
// 1 allocates 512 TMEM columns (two 128x256 f32 accumulators) and one thread
// issues tcgen05.mma (M=128, N=256, K=16); warps 2-5 drain an accumulator with
// tcgen05.ld while the next tile accumulates into the other one.
//
// Operands are f16 (default) or bf16, accumulation f32.  In f16 mode the first
// iterate is pre-scaled by a power of two 2^k (undone exactly in the GEMM1 and
// GEMM3 epilogues of the first iteration) so the normalised matrix does not
// sit in the f16 subnormal range.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <vector>

#include "tk_internal.h"
#include "tk_ns.h"
#include "tk_sm100.cuh"

namespace tk {
namespace ns {

using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_TILE_BYTES = BM * BK * 2;
constexpr int B_TILE_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_TILE_BYTES + B_TILE_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;

constexpr float NS_A = 3.4445f, NS_B = -4.7750f, NS_C = 2.0315f;

enum Epi { EPI_PLAIN = 0, EPI_GRAM = 1, EPI_POLY = 2, EPI_XUPD = 3, EPI_FINAL = 4 };

struct GemmArgs {
  int M, N, K;
  int batch;
  int tiles_m, tiles_n, tiles_per_mat;
  int symmetric;
  float alpha, beta;
  const uint16_t* aux;  // GEMM2: A; GEMM3: X^T (current)
  int64_t aux_ld, aux_bs;
  uint16_t* out;  // GEMM1: A; GEMM2: B; GEMM3: X^T (next)
  int64_t out_ld, out_bs;
  uint16_t* out2;  // GEMM3: X (transposed store)
  int64_t out2_ld, out2_bs;
  // final iteration: per-matrix destination (NS output or parameter)
  void* const* fin_ptrs;
  int fin_dtype;       // TK_F32 / TK_BF16
  int fin_update;      // 0: store O; 1: p = p + fin_scale * O
  int fin_transposed;  // 1: O[c][r] (row length fin_ld); 0: O[r][c]
  int64_t fin_ld;
  float fin_scale;
  int* err;
};

// ------------------------------------------------------------------ helpers
template <int FMT>
__device__ __forceinline__ uint16_t to_half_bits(float x) {
  if constexpr (FMT == 0) return __half_as_ushort(__float2half_rn(x));
  else return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

template <int FMT>
__device__ __forceinline__ float from_half_bits(uint16_t h) {
  if constexpr (FMT == 0) return __half2float(__ushort_as_half(h));
  else return __bfloat162float(__ushort_as_bfloat16(h));
}

__device__ __forceinline__ void decode_tile(const GemmArgs& a, int t, int& b, int& tm, int& tn) {
  b = t / a.tiles_per_mat;
  int r = t - b * a.tiles_per_mat;
  if (!a.symmetric) {
    tm = r / a.tiles_n;
    tn = r - tm * a.tiles_n;
    return;
  }
  // row block i holds column blocks floor(i/2) .. tiles_n-1: the 128x256
  // tiles that touch the diagonal or lie above it
  for (int i = 0; i < a.tiles_m; ++i) {
    const int cnt = a.tiles_n - (i >> 1);
    if (r < cnt) {
      tm = i;
      tn = (i >> 1) + r;
      return;
    }
    r -= cnt;
  }
  tm = a.tiles_m;  // unreachable for a valid tile index
  tn = 0;
}

__host__ __device__ inline int sym_tiles(int tiles_m, int tiles_n) {
  int s = 0;
  for (int i = 0; i < tiles_m; ++i) s += tiles_n - (i >> 1);
  return s;
}

__device__ __forceinline__ bool wait_no_abort(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitLimitNs) return false;
  }
  return true;
}

// ------------------------------------------------------------------ epilogue
template <int EPI, int FMT>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& a, int b, int r, int c0,
                                               const uint32_t (&v)[32]) {
  if (r >= a.M) return;
  float acc[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) acc[j] = __uint_as_float(v[j]);
  const bool full = c0 + 32 <= a.N;

  if constexpr (EPI == EPI_PLAIN) {
    uint16_t* dst = a.out + (int64_t)b * a.out_bs + (int64_t)r * a.out_ld + c0;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (full || c0 + j < a.N) dst[j] = to_half_bits<FMT>(a.alpha * acc[j]);
    return;
  }

  if constexpr (EPI == EPI_GRAM || EPI == EPI_POLY) {
    float o[32];
    if constexpr (EPI == EPI_POLY) {
      const uint16_t* src = a.aux + (int64_t)b * a.aux_bs + (int64_t)r * a.aux_ld + c0;
      if (full) {
        uint4 raw[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) raw[q] = reinterpret_cast<const uint4*>(src)[q];
        const uint16_t* h = reinterpret_cast<const uint16_t*>(raw);
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = a.beta * from_half_bits<FMT>(h[j]) + a.alpha * acc[j];
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          o[j] = (c0 + j < a.N) ? a.beta * from_half_bits<FMT>(src[j]) + a.alpha * acc[j] : 0.f;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) o[j] = a.alpha * acc[j];
    }
    uint16_t* base = a.out + (int64_t)b * a.out_bs;
    uint16_t hb[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) hb[j] = to_half_bits<FMT>(o[j]);
    if (full && c0 >= r) {
      uint4* dst = reinterpret_cast<uint4*>(base + (int64_t)r * a.out_ld + c0);
#pragma unroll
      for (int q = 0; q < 4; ++q) dst[q] = reinterpret_cast<const uint4*>(hb)[q];
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c0 + j < a.N && c0 + j >= r) base[(int64_t)r * a.out_ld + c0 + j] = hb[j];
    }
    // mirror: (c, r) for c > r; consecutive lanes write consecutive r
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (c0 + j < a.N && c0 + j > r) base[(int64_t)(c0 + j) * a.out_ld + r] = hb[j];
    return;
  }

  if constexpr (EPI == EPI_XUPD || EPI == EPI_FINAL) {
    const uint16_t* src = a.aux + (int64_t)b * a.aux_bs + (int64_t)r * a.aux_ld + c0;
    float o[32];
    if (full) {
      uint4 raw[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) raw[q] = reinterpret_cast<const uint4*>(src)[q];
      const uint16_t* h = reinterpret_cast<const uint16_t*>(raw);
#pragma unroll
      for (int j = 0; j < 32; ++j) o[j] = a.alpha * acc[j] + a.beta * from_half_bits<FMT>(h[j]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        o[j] = (c0 + j < a.N) ? a.alpha * acc[j] + a.beta * from_half_bits<FMT>(src[j]) : 0.f;
    }
    if constexpr (EPI == EPI_XUPD) {
      uint16_t hb[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) hb[j] = to_half_bits<FMT>(o[j]);
      uint16_t* d1 = a.out + (int64_t)b * a.out_bs + (int64_t)r * a.out_ld + c0;
      if (full) {
#pragma unroll
        for (int q = 0; q < 4; ++q) reinterpret_cast<uint4*>(d1)[q] = reinterpret_cast<const uint4*>(hb)[q];
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < a.N) d1[j] = hb[j];
      }
      uint16_t* d2 = a.out2 + (int64_t)b * a.out2_bs;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c0 + j < a.N) d2[(int64_t)(c0 + j) * a.out2_ld + r] = hb[j];
    } else {
      void* dst = a.fin_ptrs[b];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (!(c0 + j < a.N)) continue;
        const int64_t idx = a.fin_transposed ? (int64_t)(c0 + j) * a.fin_ld + r
                                             : (int64_t)r * a.fin_ld + c0 + j;
        if (a.fin_dtype == TK_F32) {
          float* p = static_cast<float*>(dst) + idx;
          *p = a.fin_update ? __fadd_rn(*p, __fmul_rn(a.fin_scale, o[j])) : o[j];
        } else {
          __nv_bfloat16* p = static_cast<__nv_bfloat16*>(dst) + idx;
          const float cur = a.fin_update ? __bfloat162float(*p) : 0.f;
          *p = __float2bfloat16_rn(a.fin_update ? __fadd_rn(cur, __fmul_rn(a.fin_scale, o[j]))
                                                : o[j]);
        }
      }
    }
  }
}

// ------------------------------------------------------------------ GEMM kernel
template <int EPI, int FMT>
__global__ void __launch_bounds__(THREADS, 1)
gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_tiles = args.batch * args.tiles_per_mat;
  const int num_kb = (args.K + BK - 1) / BK;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued = 0;         // stages that have received a copy
      uint32_t issued_parity = 0;  // phase parity of each stage's last copy
      for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x) {
        int b, tm, tn;
        decode_tile(args, t, b, tm, tn);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, args.err, 1)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_3d(st, &tmA, &full[stage], kb * BK, tm * BM, b);
          tma_load_3d(st + A_TILE_BYTES, &tmB, &full[stage], kb * BK, tn * BN, b);
          issued |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // give up: let the copies already issued land (bounded) before the
        // CTA's shared memory is released
        for (int st = 0; st < STAGES; ++st)
          if (issued & (1u << st)) wait_no_abort(&full[st], (issued_parity >> st) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t IDESC = idesc_f16(FMT, BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x, ++it) {
        const int acc = it & 1;
        const uint32_t use = static_cast<uint32_t>(it >> 1);
        if (!mbar_wait(&tempty[acc], (use & 1) ^ 1, abort_flag, args.err, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, args.err, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint64_t da = smem_desc_k_sw128(sa);
          const uint64_t db = smem_desc_k_sw128(sa + A_TILE_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(d, da + 2 * k, db + 2 * k, IDESC, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) umma_commit(&tfull[acc]);
      }
      // every issued MMA has finished before TMEM is released
      umma_commit(drain);
      if (!wait_no_abort(drain, 0) && args.err) atomicCAS(args.err, 0, 4);
    }
  } else {
    // ---------------- epilogue: warps 2..5, one accumulator row per thread
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    int it = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t use = static_cast<uint32_t>(it >> 1);
      if (!mbar_wait(&tfull[acc], use & 1, abort_flag, args.err, 5)) break;
      tc_fence_after();
      int b, tm, tn;
      decode_tile(args, t, b, tm, tn);
      const int r = tm * BM + row_in_tile;
      const int c_base = tn * BN;
      for (int cc = 0; cc < BN; cc += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem_base + static_cast<uint32_t>(acc * BN + cc) +
                               (static_cast<uint32_t>(q * 32) << 16),
                           v);
        tmem_ld_wait();
        if (c_base + cc < args.N) epilogue_chunk<EPI, FMT>(args, b, r, c_base + cc, v);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ prologue
// Pass 1: per matrix, optional Muon momentum update, f64 sum of squares of the
// matrix handed to Newton-Schulz.  grid (nblk, batch).
template <int SDT, bool MUON>
__global__ void __launch_bounds__(256)
prep_stats_kernel(const PrepArgs a, double* __restrict__ partials) {
  const int b = blockIdx.y;
  const int64_t total = a.rows * a.cols;
  const int64_t chunk = (total + gridDim.x - 1) / gridDim.x;
  const int64_t lo = blockIdx.x * chunk, hi = min(total, lo + chunk);
  const void* src = a.src[b];
  float* mom = MUON ? a.mom[b] : nullptr;
  double s = 0.0;
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float g = SDT == TK_F32 ? static_cast<const float*>(src)[i]
                                  : __bfloat162float(static_cast<const __nv_bfloat16*>(src)[i]);
    float u = g;
    if constexpr (MUON) {
      // python/tikun/muon_nd.py:112-115 in f32: buf = mu*buf + om*g; u = mu*buf + om*g
      const float buf = __fadd_rn(__fmul_rn(a.mu, mom[i]), __fmul_rn(a.om, g));
      mom[i] = buf;
      u = a.nesterov ? __fadd_rn(__fmul_rn(a.mu, buf), __fmul_rn(a.om, g)) : buf;
    }
    s = fma((double)u, (double)u, s);
  }
  __shared__ double red[8];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_down_sync(0xffffffffu, s, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    partials[(int64_t)b * gridDim.x + blockIdx.x] = t;
  }
}

// Pass 2: normalise (tensor_engine.rs:37-44: x * 1/max(||U||, 1e-7) in f32),
// pre-scale by 2^k, round to the operand type and write X (m x n) and X^T
// (n x m) through a 32x32 shared-memory transpose.  grid (ceil(C/32),
// ceil(R/32), batch), block (32, 8).  With steps == 0 it writes the output
// (or applies the update) instead.
template <int SDT, bool MUON, int FMT>
__global__ void __launch_bounds__(256)
prep_write_kernel(const PrepArgs a, const double* __restrict__ partials, int nblk) {
  __shared__ float s_scale;
  __shared__ uint16_t tile[32][33];
  const int b = blockIdx.z;
  const int tid = threadIdx.y * 32 + threadIdx.x;
  {
    double s = 0.0;
    for (int i = tid; i < nblk; i += 256) s += partials[(int64_t)b * nblk + i];
    __shared__ double red[8];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_down_sync(0xffffffffu, s, off);
    if ((tid & 31) == 0) red[tid >> 5] = s;
    __syncthreads();
    if (tid == 0) {
      double t = 0.0;
      for (int w = 0; w < 8; ++w) t += red[w];
      const float nrm = __double2float_rn(sqrt(t));
      s_scale = __fdiv_rn(1.0f, fmaxf(nrm, 1e-7f));
    }
    __syncthreads();
  }
  const float inv = s_scale;
  const void* src = a.src[b];
  const float* mom = MUON ? a.mom[b] : nullptr;
  const int c = blockIdx.x * 32 + threadIdx.x;
  const bool tall = a.rows > a.cols;  // X = G^T
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = blockIdx.y * 32 + threadIdx.y + 8 * k;
    float x = 0.f;
    if (r < a.rows && c < a.cols) {
      const int64_t i = (int64_t)r * a.cols + c;
      const float g = SDT == TK_F32 ? static_cast<const float*>(src)[i]
                                    : __bfloat162float(static_cast<const __nv_bfloat16*>(src)[i]);
      float u = g;
      if constexpr (MUON) {
        const float buf = mom[i];
        u = a.nesterov ? __fadd_rn(__fmul_rn(a.mu, buf), __fmul_rn(a.om, g)) : buf;
      }
      x = __fmul_rn(u, inv);
      if (a.steps == 0) {
        void* dst = a.dst[b];
        if (a.dst_dtype == TK_F32) {
          float* p = static_cast<float*>(dst) + i;
          *p = a.update ? __fadd_rn(*p, __fmul_rn(a.upd_scale, x)) : x;
        } else {
          __nv_bfloat16* p = static_cast<__nv_bfloat16*>(dst) + i;
          *p = __float2bfloat16_rn(a.update ? __fadd_rn(__bfloat162float(*p), __fmul_rn(a.upd_scale, x)) : x);
        }
        continue;
      }
      // same-layout target: X (wide) or X^T (tall); row length of G is cols
      uint16_t* same = tall ? a.xt + (int64_t)b * a.xt_bs : a.x + (int64_t)b * a.x_bs;
      const int64_t same_ld = tall ? a.xt_ld : a.x_ld;
      const uint16_t h = to_half_bits<FMT>(__fmul_rn(x, a.prescale));
      same[(int64_t)r * same_ld + c] = h;
      tile[threadIdx.y + 8 * k][threadIdx.x] = h;
    }
  }
  if (a.steps == 0) return;
  __syncthreads();
  // transposed target: element (r, c) of G goes to row c, column r
  uint16_t* other = tall ? a.x + (int64_t)b * a.x_bs : a.xt + (int64_t)b * a.xt_bs;
  const int64_t other_ld = tall ? a.x_ld : a.xt_ld;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int cc = blockIdx.x * 32 + threadIdx.y + 8 * k;  // row of the target
    const int rr = blockIdx.y * 32 + threadIdx.x;           // column of the target
    if (cc < a.cols && rr < a.rows) other[(int64_t)cc * other_ld + rr] = tile[threadIdx.x][threadIdx.y + 8 * k];
  }
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static int get_encode(EncodeTiledFn* out) {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  static cudaError_t status = cudaSuccess;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    status = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                              cudaEnableDefault, &q);
    if (status == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = (EncodeTiledFn)p;
  });
  if (fn == nullptr)
    return set_error(TK_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  *out = fn;
  return TK_OK;
}

// 3-D map over [batch][rows][ld] half-precision elements, logical inner extent
// `inner`, box 64 x box_rows x 1, 128-byte swizzle, zero fill out of bounds.
static int make_map(CUtensorMap* map, const void* base, int fmt, int64_t inner, int64_t rows,
                    int64_t ld, int64_t batch, int box_rows) {
  EncodeTiledFn enc;
  TK_TRY(get_encode(&enc));
  const cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, (cuuint64_t)batch};
  const cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), (cuuint64_t)(rows * ld * 2)};
  const cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, fmt == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                   3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(TK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for a %lld x %lld x %lld map",
                     (int)r, (long long)batch, (long long)rows, (long long)inner);
  return TK_OK;
}

template <int EPI, int FMT>
static int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& g,
                       cudaStream_t s) {
  static bool attr_set[64] = {};
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(TK_ERR_CUDA, "device index %d out of range", dev);
  if (!attr_set[dev]) {
    TK_CUDA_TRY(cudaFuncSetAttribute(gemm_tn_kernel<EPI, FMT>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    attr_set[dev] = true;
  }
  int sms = 0;
  TK_TRY(sm_count(&sms));
  const int n_tiles = g.batch * g.tiles_per_mat;
  if (n_tiles == 0) return TK_OK;
  const int grid = std::min(n_tiles, sms);
  gemm_tn_kernel<EPI, FMT><<<grid, THREADS, SMEM_BYTES, s>>>(ma, mb, g);
  TK_CUDA_TRY(cudaGetLastError());
  return TK_OK;
}

template <int EPI>
static int launch_gemm_fmt(int fmt, const CUtensorMap& ma, const CUtensorMap& mb,
                           const GemmArgs& g, cudaStream_t s) {
  return fmt == 0 ? launch_gemm<EPI, 0>(ma, mb, g, s) : launch_gemm<EPI, 1>(ma, mb, g, s);
}

static int launch_gemm_epi(int epi, int fmt, const CUtensorMap& ma, const CUtensorMap& mb,
                           const GemmArgs& g, cudaStream_t s) {
  switch (epi) {
    case EPI_PLAIN: return launch_gemm_fmt<EPI_PLAIN>(fmt, ma, mb, g, s);
    case EPI_GRAM: return launch_gemm_fmt<EPI_GRAM>(fmt, ma, mb, g, s);
    case EPI_POLY: return launch_gemm_fmt<EPI_POLY>(fmt, ma, mb, g, s);
    case EPI_XUPD: return launch_gemm_fmt<EPI_XUPD>(fmt, ma, mb, g, s);
    case EPI_FINAL: return launch_gemm_fmt<EPI_FINAL>(fmt, ma, mb, g, s);
  }
  return set_error(TK_ERR_INVALID, "bad epilogue %d", epi);
}

static int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

static size_t align256(size_t x) { return (x + 255) / 256 * 256; }

GroupLayout group_layout(int64_t rows, int64_t cols, int64_t batch) {
  GroupLayout L;
  L.R = rows;
  L.C = cols;
  L.tall = rows > cols;
  L.m = std::min(rows, cols);
  L.n = std::max(rows, cols);
  L.batch = batch;
  L.ldx = round_up(L.n, 64);
  L.ldm = round_up(L.m, 64);
  L.x_bytes = align256((size_t)(batch * L.m * L.ldx * 2));
  L.xt_bytes = align256((size_t)(batch * L.n * L.ldm * 2));
  L.a_bytes = align256((size_t)(batch * L.m * L.ldm * 2));
  L.nblk = (int)std::max<int64_t>(1, std::min<int64_t>(64, (rows * cols + 65535) / 65536));
  L.scratch_bytes = L.x_bytes + 2 * L.xt_bytes + 2 * L.a_bytes +
                    align256(sizeof(double) * batch * L.nblk) +
                    align256(sizeof(void*) * batch * 3) + 256;
  return L;
}

// Power-of-two pre-scale of the first iterate in f16 mode: RMS of the
// normalised matrix is 1/sqrt(m n); lift it to about 2^-4.
static int prescale_exp(int fmt, int64_t m, int64_t n) {
  if (fmt != 0) return 0;
  const double r = std::sqrt((double)m * (double)n) / 16.0;
  int k = (int)std::floor(std::log2(std::max(r, 1.0)));
  return std::max(0, std::min(k, 60));
}

int run_group(const GroupLayout& L, const GroupIO& io, int steps, int fmt, void* scratch,
              int* err_dev, cudaStream_t s) {
  if (L.batch == 0 || L.m == 0) return TK_OK;
  char* cur = static_cast<char*>(scratch);
  uint16_t* X = reinterpret_cast<uint16_t*>(cur);
  cur += L.x_bytes;
  uint16_t* XT[2] = {reinterpret_cast<uint16_t*>(cur),
                     reinterpret_cast<uint16_t*>(cur + L.xt_bytes)};
  cur += 2 * L.xt_bytes;
  uint16_t* Am = reinterpret_cast<uint16_t*>(cur);
  cur += L.a_bytes;
  uint16_t* Bm = reinterpret_cast<uint16_t*>(cur);
  cur += L.a_bytes;
  double* partials = reinterpret_cast<double*>(cur);
  cur += align256(sizeof(double) * L.batch * L.nblk);
  void** ptrs = reinterpret_cast<void**>(cur);  // src[batch], dst[batch], mom[batch]

  std::vector<void*> host_ptrs(3 * L.batch);
  for (int64_t i = 0; i < L.batch; ++i) {
    host_ptrs[i] = const_cast<void*>(io.src[i]);
    host_ptrs[L.batch + i] = io.dst[i];
    host_ptrs[2 * L.batch + i] = io.mom ? io.mom[i] : nullptr;
  }
  TK_CUDA_TRY(cudaMemcpyAsync(ptrs, host_ptrs.data(), sizeof(void*) * host_ptrs.size(),
                              cudaMemcpyHostToDevice, s));

  const int k = prescale_exp(fmt, L.m, L.n);
  PrepArgs pa;
  std::memset(&pa, 0, sizeof(pa));
  pa.src = reinterpret_cast<const void* const*>(ptrs);
  pa.dst = ptrs + L.batch;
  pa.mom = reinterpret_cast<float* const*>(ptrs + 2 * L.batch);
  pa.rows = L.R;
  pa.cols = L.C;
  pa.mu = io.mu;
  pa.om = io.om;
  pa.nesterov = io.nesterov;
  pa.x = X;
  pa.x_ld = L.ldx;
  pa.x_bs = L.m * L.ldx;
  pa.xt = XT[0];
  pa.xt_ld = L.ldm;
  pa.xt_bs = L.n * L.ldm;
  pa.prescale = std::ldexp(1.0f, k);
  pa.steps = steps;
  pa.dst_dtype = io.dst_dtype;
  pa.update = io.update;
  pa.upd_scale = io.upd_scale;

  const bool muon = io.mom != nullptr;
  {
    dim3 g1(L.nblk, (unsigned)L.batch);
    if (io.src_dtype == TK_F32) {
      if (muon) prep_stats_kernel<TK_F32, true><<<g1, 256, 0, s>>>(pa, partials);
      else prep_stats_kernel<TK_F32, false><<<g1, 256, 0, s>>>(pa, partials);
    } else {
      if (muon) prep_stats_kernel<TK_BF16, true><<<g1, 256, 0, s>>>(pa, partials);
      else prep_stats_kernel<TK_BF16, false><<<g1, 256, 0, s>>>(pa, partials);
    }
    TK_CUDA_TRY(cudaGetLastError());
    dim3 g2((unsigned)((L.C + 31) / 32), (unsigned)((L.R + 31) / 32), (unsigned)L.batch);
    dim3 b2(32, 8);
#define TK_PREP_WRITE(SDT, MU, F) prep_write_kernel<SDT, MU, F><<<g2, b2, 0, s>>>(pa, partials, L.nblk)
    if (io.src_dtype == TK_F32) {
      if (muon) { if (fmt == 0) TK_PREP_WRITE(TK_F32, true, 0); else TK_PREP_WRITE(TK_F32, true, 1); }
      else { if (fmt == 0) TK_PREP_WRITE(TK_F32, false, 0); else TK_PREP_WRITE(TK_F32, false, 1); }
    } else {
      if (muon) { if (fmt == 0) TK_PREP_WRITE(TK_BF16, true, 0); else TK_PREP_WRITE(TK_BF16, true, 1); }
      else { if (fmt == 0) TK_PREP_WRITE(TK_BF16, false, 0); else TK_PREP_WRITE(TK_BF16, false, 1); }
    }
#undef TK_PREP_WRITE
    TK_CUDA_TRY(cudaGetLastError());
  }
  if (steps == 0) return TK_OK;

  CUtensorMap mX128, mX256, mA128, mA256, mB256, mXT128[2];
  TK_TRY(make_map(&mX128, X, fmt, L.n, L.m, L.ldx, L.batch, 128));
  TK_TRY(make_map(&mX256, X, fmt, L.n, L.m, L.ldx, L.batch, 256));
  TK_TRY(make_map(&mA128, Am, fmt, L.m, L.m, L.ldm, L.batch, 128));
  TK_TRY(make_map(&mA256, Am, fmt, L.m, L.m, L.ldm, L.batch, 256));
  TK_TRY(make_map(&mB256, Bm, fmt, L.m, L.m, L.ldm, L.batch, 256));
  TK_TRY(make_map(&mXT128[0], XT[0], fmt, L.m, L.n, L.ldm, L.batch, 128));
  TK_TRY(make_map(&mXT128[1], XT[1], fmt, L.m, L.n, L.ldm, L.batch, 128));

  const int tm_sq = (int)((L.m + BM - 1) / BM), tn_sq = (int)((L.m + BN - 1) / BN);
  const int tm_x = (int)((L.n + BM - 1) / BM);
  const float inv_pre = std::ldexp(1.0f, -k), inv_pre2 = std::ldexp(1.0f, -2 * k);
  int cur_xt = 0;
  for (int it = 0; it < steps; ++it) {
    GemmArgs g;
    std::memset(&g, 0, sizeof(g));
    g.batch = (int)L.batch;
    g.err = err_dev;
    // GEMM1: A = X X^T
    g.M = g.N = (int)L.m;
    g.K = (int)L.n;
    g.tiles_m = tm_sq;
    g.tiles_n = tn_sq;
    g.tiles_per_mat = sym_tiles(tm_sq, tn_sq);
    g.symmetric = 1;
    g.alpha = it == 0 ? inv_pre2 : 1.0f;
    g.out = Am;
    g.out_ld = L.ldm;
    g.out_bs = L.m * L.ldm;
    TK_TRY(launch_gemm_epi(EPI_GRAM, fmt, mX128, mX256, g, s));
    // GEMM2: B = b A + c A A
    g.K = (int)L.m;
    g.alpha = NS_C;
    g.beta = NS_B;
    g.aux = Am;
    g.aux_ld = L.ldm;
    g.aux_bs = L.m * L.ldm;
    g.out = Bm;
    TK_TRY(launch_gemm_epi(EPI_POLY, fmt, mA128, mA256, g, s));
    // GEMM3: X_new^T = post (a X^T + X^T B)
    GemmArgs h;
    std::memset(&h, 0, sizeof(h));
    h.batch = (int)L.batch;
    h.err = err_dev;
    h.M = (int)L.n;
    h.N = (int)L.m;
    h.K = (int)L.m;
    h.tiles_m = tm_x;
    h.tiles_n = tn_sq;
    h.tiles_per_mat = tm_x * tn_sq;
    h.symmetric = 0;
    const float post = it == 0 ? inv_pre : 1.0f;
    h.alpha = post;
    h.beta = NS_A * post;
    h.aux = XT[cur_xt];
    h.aux_ld = L.ldm;
    h.aux_bs = L.n * L.ldm;
    if (it + 1 < steps) {
      h.out = XT[cur_xt ^ 1];
      h.out_ld = L.ldm;
      h.out_bs = L.n * L.ldm;
      h.out2 = X;
      h.out2_ld = L.ldx;
      h.out2_bs = L.m * L.ldx;
      TK_TRY(launch_gemm_epi(EPI_XUPD, fmt, mXT128[cur_xt], mB256, h, s));
      cur_xt ^= 1;
    } else {
      h.fin_ptrs = ptrs + L.batch;
      h.fin_dtype = io.dst_dtype;
      h.fin_update = io.update;
      h.fin_scale = io.upd_scale;
      // D[r][c] = X_final^T[r][c]; a wide input's output is X_final: O[c][r]
      h.fin_transposed = L.tall ? 0 : 1;
      h.fin_ld = L.C;
      TK_TRY(launch_gemm_epi(EPI_FINAL, fmt, mXT128[cur_xt], mB256, h, s));
    }
  }
  return TK_OK;
}

// ------------------------------------------------------------------ test hook
// Plain batched TN GEMM D = alpha * P Q^T on half-precision operands, for the
// kernel's own tests.
int plain_gemm(const uint16_t* P, const uint16_t* Q, uint16_t* D, int batch, int M, int N, int K,
               int64_t ldp, int64_t ldq, int64_t ldd, float alpha, int fmt, int* err_dev,
               cudaStream_t s) {
  CUtensorMap ma, mb;
  TK_TRY(make_map(&ma, P, fmt, K, M, ldp, batch, 128));
  TK_TRY(make_map(&mb, Q, fmt, K, N, ldq, batch, 256));
  GemmArgs g;
  std::memset(&g, 0, sizeof(g));
  g.M = M;
  g.N = N;
  g.K = K;
  g.batch = batch;
  g.tiles_m = (M + BM - 1) / BM;
  g.tiles_n = (N + BN - 1) / BN;
  g.tiles_per_mat = g.tiles_m * g.tiles_n;
  g.alpha = alpha;
  g.out = D;
  g.out_ld = ldd;
  g.out_bs = (int64_t)M * ldd;
  g.err = err_dev;
  return launch_gemm_epi(EPI_PLAIN, fmt, ma, mb, g, s);
}

}  // namespace ns
}  // namespace tk
