// Muon Newton-Schulz on sm_100a: tcgen05 tensor-core GEMMs fed by TMA, with the
// momentum / Nesterov prologue, the Frobenius normalisation and the scaled
// parameter update fused around them.
//
// The quintic iteration of crates/tikun-cpu/src/tensor_engine.rs:12-77,
//     A = X X^T;  B = b A + c A A;  X <- a X + B X       (a, b, c) = (3.4445, -4.7750, 2.0315)
// on X (m x n, m <= n; a tall input is transposed first, :18-34) runs as three
// "TN" GEMMs, D[M x N] = P[M x K] * Q[N x K]^T, whose operands are all K-major
// row-major arrays in HBM.  With f16 operands and m >= 256 the polynomial is
// folded so that no epilogue reads a second matrix:
//   GEMM1  A = X X^T and A' = c A + b I   P = Q = X (read from X^T, MN-major)
//   GEMM2  B' = A A' + a I                P = A, Q = A' (A' symmetric)
//   GEMM3  X_new^T = X^T B'               P = X^T, Q = B' (B' symmetric)
// Below 256 rows (and with bf16 operands) GEMM2 forms B = c A A + b A and
// GEMM3 X_new^T = X^T B + a X^T, the b A and a X^T terms added in f32 by the
// epilogues.  GEMM3 produces X_new^T directly and stores only that; GEMM1
// reads X^T as both of its operands in the MN-major layout (64 x 64 TMA boxes
// of X^T, K along its rows), so no m x n copy of X is ever written.  Symmetric
// tiles store each element above the diagonal twice (at (r, c) and (c, r)),
// which keeps A and B exactly symmetric in storage.
//
// Kernel: persistent, one CTA per SM, 320 threads.  Warp 0 issues TMA loads of
// 128x64 and 256x64 operand tiles (128-byte swizzle, no multicast) into a
// 4-stage ring; warp 1 allocates 512 TMEM columns (two 128x256 f32
// accumulators) and one thread issues tcgen05.mma (M=128, N=256, K=16); eight
// epilogue warps (2..9, two per TMEM lane quadrant, each taking half of the
// columns) drain one accumulator with tcgen05.ld while the next tile
// accumulates into the other one.  Every mbarrier wait is bounded (4 s of
// %globaltimer); a wait that gives up raises a CTA abort flag and records a
// code in a device status word.
//
// Matrices of TK_NS_PAIR_MIN_M rows and more run the same GEMMs on a CTA-pair
// kernel: clusters of two CTAs share one tcgen05.mma.cta_group::2 (M = 256,
// N = 256), each CTA loading half of A's and half of B's rows, so an SM draws
// a third less operand data per MMA and holds six ring stages instead of four.
//
// Operands are f16 (default), bf16, f16 pairs throughout (format 2) or f16
// pairs for X only (format 3), accumulation f32.  In f16 mode the first
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
#include <atomic>
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
// per epilogue warp: a 32 x 33-word tile for transposing a 32 x 32 block
constexpr int TRANS_WORDS = 32 * 33;
constexpr int EPI_WARPS = 8;
constexpr int TRANS_BYTES = EPI_WARPS * TRANS_WORDS * 4;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 256 + TRANS_BYTES + 1024;
constexpr int THREADS = 64 + 32 * 8;  // producer, MMA issuer, 8 epilogue warps
constexpr uint32_t TMEM_COLS = 512;
// CTA-pair kernel: 256 x 256 tiles over two CTAs, each loading 128 rows of A
// and of B per K block into a 6-stage ring of 32 KB stages.
constexpr int P_BM = 256, P_BN = 256, P_HALF = 128, P_STAGES = 6;
constexpr int P_A_BYTES = P_HALF * BK * 2;
constexpr int P_STAGE_BYTES = 2 * P_A_BYTES;
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 256 + TRANS_BYTES + 1024;
static_assert(P_SMEM_BYTES <= 232448, "pair kernel shared memory above the 227 KB limit");
static_assert(SMEM_BYTES <= 232448, "kernel shared memory above the 227 KB limit");

constexpr float NS_A = 3.4445f, NS_B = -4.7750f, NS_C = 2.0315f;

// The symmetric products X X^T (GEMM1, over K = n) and A A' (GEMM2, over
// K = m) compute only the tiles on or above the diagonal and mirror them, or
// -- up to these K -- every tile, stored once with no mirror stores or
// transposes.  At short K the epilogues set the pace and the full grid, 1.5x
// the MMA work, is faster (measured on B200: 48 x 768^2 +9 %, 24 x 1024^2
// +20 %, 96 x 512^2 +25 %; GEMM2 at K = 768-1024 gained nothing).
#ifndef TK_NS_FULL_K1
#define TK_NS_FULL_K1 1024
#endif
#ifndef TK_NS_FULL_K2
#define TK_NS_FULL_K2 512
#endif
// Matrices with at least this many rows (m, after the transpose of a tall
// one) run on the CTA-pair kernel; smaller ones on the single-CTA kernel.
// Measured on B200 over whole Newton-Schulz calls (pair against single):
// 8 x 4096^2 +8 %, 6 x 2048 x 8192 +5 %, 16 x 4096 x 1024 +5 %, 24 x 1024^2
// +3 %; 48 x 768^2 -1 %, 12 x 768 x 3072 -2 %, 96 x 512^2 -9 %.
#ifndef TK_NS_PAIR_MIN_M
#define TK_NS_PAIR_MIN_M 1024
#endif

// Epilogues, each on v = alpha*acc (+ gamma*aux when aux is set: a second
// matrix of the output's shape, read in the epilogue).  SYM: a symmetric
// product (upper tiles only, mirrored), stored as v + beta*I and, when out2 is
// set, also as alpha2*acc + beta2*I.  XUPD: v stored row-wise to out and
// transposed to out2.  FINAL: v applied to the Newton-Schulz output or the
// parameter.
enum Epi { EPI_PLAIN = 0, EPI_SYM = 1, EPI_XUPD = 3, EPI_FINAL = 4 };

struct GemmArgs {
  int M, N, K;
  int batch;
  int tiles_m, tiles_n, tiles_per_mat;
  int symmetric;  // enumerate only the tiles on or above the diagonal
  int mirror;     // SYM epilogue: store each entry above the diagonal twice
  float alpha, beta;    // SYM: out = alpha*acc + beta*I; XUPD/FINAL: alpha*acc
  float alpha2, beta2;  // SYM with out2: out2 = alpha2*acc + beta2*I
  float gamma;          // weight of aux
  const uint16_t* aux;  // optional; same layout as the output
  int64_t aux_ld, aux_bs;
  uint16_t* out;  // GEMM1: A; GEMM2: B'; GEMM3: X^T (next)
  int64_t out_ld, out_bs;
  uint16_t* out2;  // GEMM1: A' = c A + b I; GEMM3: X (transposed store)
  int64_t out2_ld, out2_bs;
  int64_t lo_off, lo_off2;  // format 2: lo values of out / out2, in elements after the hi
  int* err;
  // final iteration: per-matrix destination (NS output or parameter).  A tall
  // matrix's output is X_final^T = D itself (O[r][c], row length N); a wide
  // one's is X_final (O[c][r], row length M).
  int fin_dtype;   // TK_F32 / TK_BF16
  int fin_update;  // 0: store O; 1: p = p + scale * O
  float fin_scale_wide, fin_scale_tall;
  uint64_t fin_tall[kMaxBatch / 64];
  void* fin_ptrs[kMaxBatch];
  // the final parameters also go to these byte offsets from each local
  // address: the same parameter in other GPUs' arenas (peer memory)
  int fin_npeers;
  int64_t fin_peer_delta[kMaxPeers];
};

__device__ __forceinline__ bool bit_of(const uint64_t* mask, int b) {
  return (mask[b >> 6] >> (b & 63)) & 1ull;
}

// ------------------------------------------------------------------ helpers
// bf16 <-> f32 by bit manipulation: a raw 16-bit load followed by a shift keeps
// independent loads free to overlap (no conversion intrinsic in between).
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);  // quiet NaN
  u += 0x7fffu + ((u >> 16) & 1u);                                           // nearest even
  return (uint16_t)(u >> 16);
}

// Operand formats: 0 = f16, 1 = bf16, 2 = f16 pairs (every operand value v
// stored as hi = f16(v) and lo = f16(v - hi), lo_off elements after hi in the
// same row, and each GEMM accumulating hi*hi + hi*lo + lo*hi), 3 = f16 pairs
// for X^T only (GEMM1 and GEMM2 run in format 0; GEMM3 accumulates
// X^T hi * B' + X^T lo * B' and stores X_new^T as pairs).
template <int FMT>
__device__ __forceinline__ uint16_t to_half_bits(float x) {
  if constexpr (FMT != 1) return __half_as_ushort(__float2half_rn(x));
  else return f32_to_bf16_bits(x);
}

template <int FMT>
__device__ __forceinline__ float from_half_bits(uint16_t h) {
  if constexpr (FMT != 1) return __half2float(__ushort_as_half(h));
  else return bf16_bits_to_f32(h);
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
// The epilogue runs on 8 warps, two per TMEM lane quadrant (32 accumulator
// rows each), each converting half of the tile's 256 columns in chunks of 32.
// Within a chunk lane l holds row r0 + l, columns c0 .. c0 + 31.

// Two f32 values -> one word of two 16-bit values (lo in the low half).
template <int FMT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (FMT != 1) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

// 32 f32 values -> their f16 pairs: hi[k] packs f16(v[2k]), f16(v[2k+1]) and
// lo[k] the f16 roundings of what those leave (v - hi is exact in f32).
__device__ __forceinline__ void pack_split(const float (&v)[32], uint32_t (&hi)[16],
                                           uint32_t (&lo)[16]) {
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const __half2 h = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(v[2 * k] - hf.x, v[2 * k + 1] - hf.y);
    hi[k] = *reinterpret_cast<const uint32_t*>(&h);
    lo[k] = *reinterpret_cast<const uint32_t*>(&l);
  }
}

__device__ __forceinline__ uint16_t half_at(const uint32_t (&w)[16], int j) {
  return (uint16_t)(w[j >> 1] >> ((j & 1) * 16));
}

// 32 16-bit values (16 words) -> four 16-byte stores; dst 16-byte aligned.
__device__ __forceinline__ void store_words16(uint16_t* dst, const uint32_t (&w)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q)
    reinterpret_cast<uint4*>(dst)[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
}

// Transposes the warp's 32 x 32 block of 16-bit values held as pairs along
// the row (lane l: row l, w[k] = columns 2k, 2k+1) into pairs along the column
// (lane l: column l, w[k] = rows 2k, 2k+1) through shared memory.  Row stride
// 17 words: the stores are free of bank conflicts, and each load touches 16
// words with two lanes per word.
__device__ __forceinline__ void warp_transpose16(uint32_t* sm, uint32_t (&w)[16]) {
  const int lane = threadIdx.x & 31;
  __syncwarp();
#pragma unroll
  for (int k = 0; k < 16; ++k) sm[lane * 17 + k] = w[k];
  __syncwarp();
  const uint32_t sel = (lane & 1) ? 0x7632u : 0x5410u;  // high or low halves
#pragma unroll
  for (int k = 0; k < 16; ++k)
    w[k] = __byte_perm(sm[(2 * k) * 17 + (lane >> 1)], sm[(2 * k + 1) * 17 + (lane >> 1)], sel);
  __syncwarp();
}

// Stores the warp's 32 x 32 block of 16-bit values (lane l: row l, 16 words)
// to dst + row*ld (rows r0 .. r0+31, columns c0 .. c0+31 of the output) with
// each store instruction covering 8 rows x 64 contiguous bytes, instead of 32
// rows x 16 bytes: the block passes through shared memory (64-byte rows, the
// 16-byte granules of row i rotated by (i/2)%4, so both phases are free of
// bank conflicts).  Rows from `rows` on are not written; the block must be 32
// columns wide.  dst + row*ld + c0 must be 16-byte aligned.
__device__ __forceinline__ void store_block16(uint16_t* dst, int64_t ld, int r0, int c0, int rows,
                                              const uint32_t (&w)[16], uint32_t* sm) {
  const int lane = threadIdx.x & 31;
  uint4* buf = reinterpret_cast<uint4*>(sm);  // 32 rows x 4 granules
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 4; ++q)
    buf[lane * 4 + (q ^ ((lane >> 1) & 3))] =
        make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  __syncwarp();
  const int j = lane & 3;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int i = 8 * q + (lane >> 2);
    const uint4 val = buf[i * 4 + (j ^ ((i >> 1) & 3))];
    if (i < rows) reinterpret_cast<uint4*>(dst + (int64_t)(r0 + i) * ld + c0)[j] = val;
  }
  __syncwarp();
}

// The same for 32-bit values (row stride 33 words).
__device__ __forceinline__ void warp_transpose32(uint32_t* sm, uint32_t (&x)[32]) {
  const int lane = threadIdx.x & 31;
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 32; ++j) sm[lane * 33 + j] = x[j];
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 32; ++i) x[i] = sm[i * 33 + lane];
  __syncwarp();
}

// acc[j] = alpha*acc[j] (+ gamma*aux[r][c0+j] when aux is set).
template <int FMT>
__device__ __forceinline__ void scale_add_aux(const GemmArgs& a, int b, int r, int c0, bool full,
                                              float (&acc)[32]) {
  if (a.aux == nullptr) {
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[j] = a.alpha * acc[j];
    return;
  }
  const uint16_t* src = a.aux + (int64_t)b * a.aux_bs + (int64_t)r * a.aux_ld + c0;
  if (full) {
    uint4 raw[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) raw[q] = reinterpret_cast<const uint4*>(src)[q];
    const uint16_t* h = reinterpret_cast<const uint16_t*>(raw);
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[j] = a.alpha * acc[j] + a.gamma * from_half_bits<FMT>(h[j]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      acc[j] = a.alpha * acc[j] + (c0 + j < a.N ? a.gamma * from_half_bits<FMT>(src[j]) : 0.f);
  }
}

// A chunk of a symmetric product: the row part on or above the diagonal, and
// its mirror (c, r) for c > r -- transposed through shared memory when the
// whole 32 x 32 block lies above the diagonal.  w is consumed.
__device__ __forceinline__ void sym_store(const GemmArgs& a, uint16_t* base, int64_t ld,
                                          uint32_t (&w)[16], int r, int r0, int c0, bool full,
                                          bool wfull, uint32_t* tsm) {
  if (wfull && c0 >= r0 + 32) {  // the block lies above the diagonal
    store_block16(base, ld, r0, c0, 32, w, tsm);
    warp_transpose16(tsm, w);
    store_block16(base, ld, c0, r0, 32, w, tsm);
    return;
  }
  if (full && c0 >= r) {
    store_words16(base + (int64_t)r * ld + c0, w);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (r < a.M && c0 + j < a.N && c0 + j >= r) base[(int64_t)r * ld + c0 + j] = half_at(w, j);
  }
  if (!(wfull && c0 + 32 <= r0)) {  // consecutive lanes write consecutive r
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (r < a.M && c0 + j < a.N && c0 + j > r) base[(int64_t)(c0 + j) * ld + r] = half_at(w, j);
  }
}

// A chunk of a symmetric product computed over every tile (no mirror): the
// row part as it is.
__device__ __forceinline__ void row_store(const GemmArgs& a, uint16_t* base, int64_t ld,
                                          uint32_t (&w)[16], int r, int r0, int c0, bool full,
                                          bool wfull, uint32_t* tsm) {
  if (wfull) {
    store_block16(base, ld, r0, c0, 32, w, tsm);
    return;
  }
  if (r >= a.M) return;
  if (full) {
    store_words16(base + (int64_t)r * ld + c0, w);
    return;
  }
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (c0 + j < a.N) base[(int64_t)r * ld + c0 + j] = half_at(w, j);
}

__device__ __forceinline__ void sym_out(const GemmArgs& a, uint16_t* base, int64_t ld,
                                        uint32_t (&w)[16], int r, int r0, int c0, bool full,
                                        bool wfull, uint32_t* tsm) {
  if (a.mirror) sym_store(a, base, ld, w, r, r0, c0, full, wfull, tsm);
  else row_store(a, base, ld, w, r, r0, c0, full, wfull, tsm);
}

// The final parameter update of a 32 x 32 block whose lane l holds the
// Newton-Schulz output for parameter row row0 + l, columns col0 .. col0+31:
// p = p + scale * o (or p = o), in the parameter's dtype, locally and into
// the peers' copies.  The block passes through shared memory (128-byte rows,
// 16-byte granules of row i rotated by i % 8) so that each access instruction
// covers 4 rows x 128 bytes (f32) or 8 rows x 64 bytes (bf16).
__device__ __forceinline__ void final_block(const GemmArgs& a, void* dst, int64_t ld, int row0,
                                            int col0, const float (&o)[32], float scale,
                                            uint32_t* sm) {
  const int lane = threadIdx.x & 31;
  float4* buf = reinterpret_cast<float4*>(sm);  // 32 rows x 8 granules
  __syncwarp();
#pragma unroll
  for (int g = 0; g < 8; ++g)
    buf[lane * 8 + (g ^ (lane & 7))] = make_float4(o[4 * g], o[4 * g + 1], o[4 * g + 2], o[4 * g + 3]);
  __syncwarp();
  if (a.fin_dtype == TK_F32) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int i = 4 * q + (lane >> 3), g = lane & 7;
      const float4 ov = buf[i * 8 + (g ^ (i & 7))];
      float4* pp = reinterpret_cast<float4*>(static_cast<float*>(dst) + (int64_t)(row0 + i) * ld + col0) + g;
      float4 pv = ov;
      if (a.fin_update) {
        pv = *pp;
        pv.x = __fadd_rn(pv.x, __fmul_rn(scale, ov.x));
        pv.y = __fadd_rn(pv.y, __fmul_rn(scale, ov.y));
        pv.z = __fadd_rn(pv.z, __fmul_rn(scale, ov.z));
        pv.w = __fadd_rn(pv.w, __fmul_rn(scale, ov.w));
      }
      *pp = pv;
      for (int k = 0; k < a.fin_npeers; ++k)
        *reinterpret_cast<float4*>(reinterpret_cast<char*>(pp) + a.fin_peer_delta[k]) = pv;
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int i = 8 * q + (lane >> 2), g = lane & 3;  // 8 bf16 = granules 2g, 2g+1 of o
      const float4 o0 = buf[i * 8 + ((2 * g) ^ (i & 7))];
      const float4 o1 = buf[i * 8 + ((2 * g + 1) ^ (i & 7))];
      const float ov[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
      uint4* pp = reinterpret_cast<uint4*>(static_cast<uint16_t*>(dst) + (int64_t)(row0 + i) * ld + col0) + g;
      uint4 in = make_uint4(0u, 0u, 0u, 0u);
      if (a.fin_update) in = *pp;
      const uint32_t iw[4] = {in.x, in.y, in.z, in.w};
      uint32_t ow[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        float lo = ov[2 * h], hi = ov[2 * h + 1];
        if (a.fin_update) {
          lo = __fadd_rn(bf16_bits_to_f32(iw[h] & 0xffffu), __fmul_rn(scale, lo));
          hi = __fadd_rn(bf16_bits_to_f32(iw[h] >> 16), __fmul_rn(scale, hi));
        }
        ow[h] = (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
      }
      const uint4 out = make_uint4(ow[0], ow[1], ow[2], ow[3]);
      *pp = out;
      for (int k = 0; k < a.fin_npeers; ++k)
        *reinterpret_cast<uint4*>(reinterpret_cast<char*>(pp) + a.fin_peer_delta[k]) = out;
    }
  }
  __syncwarp();
}

// Prefetches into L2 the parameter lines of the 32 x 128 region (accumulator
// rows r0 .., columns c0 ..) that a final-epilogue warp will update, while
// the tile's MMAs run.  In-range addresses only.
__device__ __forceinline__ void prefetch_final(const GemmArgs& a, int b, int r0, int c0) {
  if (!a.fin_update) return;
  const int lane = threadIdx.x & 31;
  const bool tall = bit_of(a.fin_tall, b);
  const int esz = a.fin_dtype == TK_F32 ? 4 : 2;
  const char* p = static_cast<const char*>(a.fin_ptrs[b]);
  if (tall) {  // parameter row r, columns c0 .. c0+127: one lane per row
    const int r = r0 + lane;
    if (r >= a.M || c0 >= a.N) return;
    const int c1 = min(c0 + 128, a.N);
    const char* lo = p + ((int64_t)r * a.N + c0) * esz;
    const char* hi = p + ((int64_t)r * a.N + c1) * esz;
    for (const char* x = lo; x < hi; x += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(x));
  } else {  // parameter rows c0 .. c0+127, columns r0 .. r0+31: four rows per lane
    if (r0 >= a.M) return;
    const int r1 = min(r0 + 32, a.M);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = c0 + lane + 32 * k;
      if (c >= a.N) break;
      const char* lo = p + ((int64_t)c * a.M + r0) * esz;
      const char* hi = p + ((int64_t)c * a.M + r1) * esz;
      for (const char* x = lo; x < hi; x += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(x));
    }
  }
}

// One 32-column chunk.  Stores that run along columns (the mirror of a
// symmetric product, X = (X^T)^T, a wide matrix's parameter) go through a warp
// transpose when the whole 32 x 32 block is in range, so that each lane writes
// 64 contiguous bytes.
template <int EPI, int FMT>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& a, int b, int r, int c0,
                                               const uint32_t (&v)[32], uint32_t* tsm) {
  const int lane = threadIdx.x & 31;
  const int r0 = r - lane;
  const bool full = c0 + 32 <= a.N;
  const bool wfull = full && r0 + 32 <= a.M;  // warp-uniform
  if (!wfull && r >= a.M) return;
  float acc[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) acc[j] = __uint_as_float(v[j]);

  if constexpr (EPI == EPI_PLAIN) {
    uint16_t* base = a.out + (int64_t)b * a.out_bs;
    if (wfull && (a.out_ld & 7) == 0 && (a.out_bs & 7) == 0 &&
        (reinterpret_cast<uintptr_t>(a.out) & 15) == 0) {
      uint32_t w[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) w[k] = pack2<FMT>(a.alpha * acc[2 * k], a.alpha * acc[2 * k + 1]);
      store_block16(base, a.out_ld, r0, c0, 32, w, tsm);
      return;
    }
    uint16_t* dst = base + (int64_t)r * a.out_ld + c0;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (full || c0 + j < a.N) dst[j] = to_half_bits<FMT>(a.alpha * acc[j]);
    return;
  }

  if constexpr (EPI == EPI_SYM) {
    {  // out = alpha*acc (+ gamma*aux) + beta*I
      float o[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) o[j] = acc[j];
      scale_add_aux<FMT>(a, b, r, c0, full, o);
#pragma unroll
      for (int j = 0; j < 32; ++j) o[j] += (c0 + j == r ? a.beta : 0.f);
      uint16_t* base = a.out + (int64_t)b * a.out_bs;
      if constexpr (FMT == 2) {
        uint32_t w[16], wl[16];
        pack_split(o, w, wl);
        sym_out(a, base, a.out_ld, w, r, r0, c0, full, wfull, tsm);
        sym_out(a, base + a.lo_off, a.out_ld, wl, r, r0, c0, full, wfull, tsm);
      } else {
        uint32_t w[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) w[k] = pack2<FMT>(o[2 * k], o[2 * k + 1]);
        sym_out(a, base, a.out_ld, w, r, r0, c0, full, wfull, tsm);
      }
    }
    if (a.out2 != nullptr) {  // out2 = alpha2*acc + beta2*I
      float o[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) o[j] = a.alpha2 * acc[j] + (c0 + j == r ? a.beta2 : 0.f);
      uint16_t* base = a.out2 + (int64_t)b * a.out2_bs;
      if constexpr (FMT == 2) {
        uint32_t w[16], wl[16];
        pack_split(o, w, wl);
        sym_out(a, base, a.out2_ld, w, r, r0, c0, full, wfull, tsm);
        sym_out(a, base + a.lo_off2, a.out2_ld, wl, r, r0, c0, full, wfull, tsm);
      } else {
        uint32_t w[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) w[k] = pack2<FMT>(o[2 * k], o[2 * k + 1]);
        sym_out(a, base, a.out2_ld, w, r, r0, c0, full, wfull, tsm);
      }
    }
    return;
  }

  if constexpr (EPI == EPI_XUPD || EPI == EPI_FINAL) {
    float o[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) o[j] = acc[j];
    scale_add_aux<FMT>(a, b, r, c0, full, o);
    if constexpr (EPI == EPI_XUPD) {
      uint32_t w[16], wl[16];
      if constexpr (FMT >= 2) {  // X^T kept as f16 pairs (formats 2 and 3)
        pack_split(o, w, wl);
      } else {
#pragma unroll
        for (int k = 0; k < 16; ++k) w[k] = pack2<FMT>(o[2 * k], o[2 * k + 1]);
      }
      // formats 2 and 3 store the lo halves as a second pass over the same code
      constexpr int kParts = FMT >= 2 ? 2 : 1;
#pragma unroll
      for (int part = 0; part < kParts; ++part) {
        uint32_t (&ww)[16] = part == 0 ? w : wl;
        uint16_t* d1base = a.out + (int64_t)b * a.out_bs + (part == 0 ? 0 : a.lo_off);
        uint16_t* d1 = d1base + (int64_t)r * a.out_ld + c0;
        if (wfull) {
          store_block16(d1base, a.out_ld, r0, c0, 32, ww, tsm);
        } else if (full) {
          store_words16(d1, ww);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (c0 + j < a.N) d1[j] = half_at(ww, j);
        }
        if (a.out2 == nullptr) continue;  // no transposed copy wanted
        uint16_t* d2 = a.out2 + (int64_t)b * a.out2_bs + (part == 0 ? 0 : a.lo_off2);
        if (wfull) {
          warp_transpose16(tsm, ww);
          store_block16(d2, a.out2_ld, c0, r0, 32, ww, tsm);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (c0 + j < a.N) d2[(int64_t)(c0 + j) * a.out2_ld + r] = half_at(ww, j);
        }
      }
    } else {
      void* dst = a.fin_ptrs[b];
      const bool tall = bit_of(a.fin_tall, b);
      const float scale = tall ? a.fin_scale_tall : a.fin_scale_wide;
      // Blocks fully in range with 16-byte aligned parameter rows: the
      // parameter's rows are the block's rows (tall) or, after a warp
      // transpose, its columns (wide); final_block updates them with
      // coalesced accesses.
      const size_t esz = a.fin_dtype == TK_F32 ? 4 : 2;
      const int64_t prow = tall ? a.N : a.M;  // parameter row length
      if (wfull && ((size_t)prow * esz) % 16 == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        if (!tall) {
          uint32_t t[32];
#pragma unroll
          for (int k = 0; k < 32; ++k) t[k] = __float_as_uint(o[k]);
          warp_transpose32(tsm, t);
#pragma unroll
          for (int k = 0; k < 32; ++k) o[k] = __uint_as_float(t[k]);
        }
        final_block(a, dst, prow, tall ? r0 : c0, tall ? c0 : r0, o, scale, tsm);
        return;
      }
      // edges and unaligned parameters: element by element; element j is at
      // i0 + j * stride.  Both loops are unrolled so that o stays in
      // registers (indexed at run time it would live in local memory, and
      // the block path above would read it from there too).
      const int64_t i0 = tall ? (int64_t)r * a.N + c0 : (int64_t)c0 * a.M + r;
      const int64_t stride = tall ? 1 : a.M;
      if (a.fin_dtype == TK_F32) {
        float* p = static_cast<float*>(dst);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < a.N) {
            float* pj = p + i0 + j * stride;
            const float val = a.fin_update ? __fadd_rn(*pj, __fmul_rn(scale, o[j])) : o[j];
            *pj = val;
            for (int q = 0; q < a.fin_npeers; ++q)
              *reinterpret_cast<float*>(reinterpret_cast<char*>(pj) + a.fin_peer_delta[q]) = val;
          }
      } else {
        uint16_t* p = static_cast<uint16_t*>(dst);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < a.N) {
            uint16_t* pj = p + i0 + j * stride;
            const uint16_t val = f32_to_bf16_bits(
                a.fin_update ? __fadd_rn(bf16_bits_to_f32(*pj), __fmul_rn(scale, o[j])) : o[j]);
            *pj = val;
            for (int q = 0; q < a.fin_npeers; ++q)
              *reinterpret_cast<uint16_t*>(reinterpret_cast<char*>(pj) + a.fin_peer_delta[q]) = val;
          }
      }
    }
  }
}

// ------------------------------------------------------------------ GEMM kernel
template <int EPI, int FMT, bool MN>
__global__ void __launch_bounds__(THREADS, 1)
gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmA_lo, const __grid_constant__ CUtensorMap tmB_lo,
               const __grid_constant__ GemmArgs args) {
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
      mbar_init(&tempty[s], EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if constexpr (FMT >= 2) {
      tma_prefetch_desc(&tmA_lo);
      tma_prefetch_desc(&tmB_lo);
    }
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
  // format 2: three passes over K into one accumulator -- (A hi, B hi),
  // (A hi, B lo), (A lo, B hi); format 3 (GEMM3 only, A = X^T held as f16
  // pairs, B in f16): two -- (A hi, B), (A lo, B)
  constexpr int kSegments = FMT == 2 ? 3 : FMT == 3 ? 2 : 1;
  const int total_kb = num_kb * kSegments;

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
        for (int kt = 0; kt < total_kb; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, args.err, 1)) {
            ok = false;
            break;
          }
          const int seg = kt / num_kb, kb = kt - seg * num_kb;
          const CUtensorMap* ma = seg == (FMT == 3 ? 1 : 2) ? &tmA_lo : &tmA;
          const CUtensorMap* mb = (FMT == 2 && seg == 1) ? &tmB_lo : &tmB;
          uint8_t* st = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          if constexpr (MN) {
            // operands stored K x MN (rows along K): 64-element MN atoms of
            // 64 K rows, 8 KB each -- 2 for A, 4 for B
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_3d(st + j * 8192, ma, &full[stage], tm * BM + 64 * j, kb * BK, b);
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_3d(st + A_TILE_BYTES + j * 8192, mb, &full[stage], tn * BN + 64 * j,
                          kb * BK, b);
          } else {
            tma_load_3d(st, ma, &full[stage], kb * BK, tm * BM, b);
            tma_load_3d(st + A_TILE_BYTES, mb, &full[stage], kb * BK, tn * BN, b);
          }
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
      constexpr uint32_t IDESC =
          MN ? idesc_f16_mn(FMT == 1 ? 1 : 0, BM, BN) : idesc_f16(FMT == 1 ? 1 : 0, BM, BN);
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
        for (int kb = 0; kb < total_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, args.err, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          if constexpr (MN) {
            // a K step of 16 rows is 2048 bytes (two 8-row groups)
            const uint64_t da = smem_desc_mn_sw128(sa, 8192);
            const uint64_t db = smem_desc_mn_sw128(sa + A_TILE_BYTES, 8192);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              umma_f16(d, da + 128 * k, db + 128 * k, IDESC, (kb | k) != 0 ? 1u : 0u);
          } else {
            const uint64_t da = smem_desc_k_sw128(sa);
            const uint64_t db = smem_desc_k_sw128(sa + A_TILE_BYTES);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              umma_f16(d, da + 2 * k, db + 2 * k, IDESC, (kb | k) != 0 ? 1u : 0u);
          }
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
    // ---------------- epilogue: warps 2..9, one accumulator row per thread;
    // warp w reads TMEM lanes 32*(w%4) .. +31 and half of the columns
    const int q = warp & 3;
    const int col0 = ((warp - 2) >> 2) * (BN / 2);
    const int row_in_tile = q * 32 + lane;
    uint32_t* tsm = reinterpret_cast<uint32_t*>(smem + STAGES * STAGE_BYTES + 256) +
                    (warp - 2) * TRANS_WORDS;
    int it = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t use = static_cast<uint32_t>(it >> 1);
      int b, tm, tn;
      decode_tile(args, t, b, tm, tn);
      if constexpr (EPI == EPI_FINAL)  // the parameters this warp will update, into L2
        prefetch_final(args, b, tm * BM + q * 32, tn * BN + col0);
      if (!mbar_wait(&tfull[acc], use & 1, abort_flag, args.err, 5)) break;
      tc_fence_after();
      const int r = tm * BM + row_in_tile;
      const int c_base = tn * BN;
      const uint32_t taddr = tmem_base + static_cast<uint32_t>(acc * BN) +
                             (static_cast<uint32_t>(q * 32) << 16);
      for (int cc = col0; cc < col0 + BN / 2; cc += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(cc), v);
        tmem_ld_wait();
        if (c_base + cc < args.N) epilogue_chunk<EPI, FMT>(args, b, r, c_base + cc, v, tsm);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }
  if constexpr (EPI == EPI_FINAL) {
    if (args.fin_npeers) __threadfence_system();  // peer stores visible before the kernel ends
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ CTA-pair GEMM kernel
// The same GEMMs on 256 x 256 tiles computed by a cluster of two CTAs with
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16).  Each CTA loads 128
// rows of A and 128 rows of B per K block -- 32 KB instead of the 48 KB a
// single CTA needs for its 128 x 256 tile -- so the same tensor work draws a
// third less operand traffic into each SM, and six stages fit in the ring.
// The leader (even CTA) issues every MMA and commits each stage to both CTAs'
// "empty" barriers; both CTAs' TMA bytes count on the leader's "full"
// barrier; each CTA's epilogue drains its own 128 accumulator rows and
// arrives on the leader's "tmem empty" barrier.
__device__ __forceinline__ void decode_tile_pair(const GemmArgs& a, int t, int& b, int& tm,
                                                 int& tn) {
  b = t / a.tiles_per_mat;
  int r = t - b * a.tiles_per_mat;
  if (!a.symmetric) {
    tm = r / a.tiles_n;
    tn = r - tm * a.tiles_n;
    return;
  }
  // square tiles: row block i holds column blocks i .. tiles_n-1
  for (int i = 0; i < a.tiles_m; ++i) {
    const int cnt = a.tiles_n - i;
    if (r < cnt) {
      tm = i;
      tn = i + r;
      return;
    }
    r -= cnt;
  }
  tm = a.tiles_m;  // unreachable for a valid tile index
  tn = 0;
}

__host__ __device__ inline int sym_tiles_pair(int tiles_m, int tiles_n) {
  int s = 0;
  for (int i = 0; i < tiles_m; ++i) s += tiles_n - i;
  return s;
}

template <int EPI, int FMT, bool MN>
__global__ void __launch_bounds__(THREADS, 1)
gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmA_lo,
                 const __grid_constant__ CUtensorMap tmB_lo, const __grid_constant__ GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + P_STAGES * P_STAGE_BYTES);
  uint64_t* empty = full + P_STAGES;
  uint64_t* tfull = empty + P_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);  // the leader's producer; both CTAs' bytes
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], 2 * EPI_WARPS);  // both CTAs' epilogue warps
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if constexpr (FMT >= 2) {
      tma_prefetch_desc(&tmA_lo);
      tma_prefetch_desc(&tmB_lo);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers initialised in both CTAs before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_tiles = args.batch * args.tiles_per_mat;
  const int cl = static_cast<int>(cluster_id_x()), ncl = static_cast<int>(cluster_count_x());
  const int num_kb = (args.K + BK - 1) / BK;
  constexpr int kSegments = FMT == 2 ? 3 : FMT == 3 ? 2 : 1;
  const int total_kb = num_kb * kSegments;
  const int row_half = static_cast<int>(rank) * P_HALF;  // this CTA's rows of A and of B

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs)
      const uint32_t full_leader = mapa_shared(smem_u32(full), 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued = 0, issued_parity = 0;
      for (int t = cl; ok && t < n_tiles; t += ncl) {
        int b, tm, tn;
        decode_tile_pair(args, t, b, tm, tn);
        for (int kt = 0; kt < total_kb; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, args.err, 1)) {
            ok = false;
            break;
          }
          const int seg = kt / num_kb, kb = kt - seg * num_kb;
          const CUtensorMap* ma = seg == (FMT == 3 ? 1 : 2) ? &tmA_lo : &tmA;
          const CUtensorMap* mb = (FMT == 2 && seg == 1) ? &tmB_lo : &tmB;
          uint8_t* st = smem + stage * P_STAGE_BYTES;
          const uint32_t bar = full_leader + static_cast<uint32_t>(stage * 8);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * P_STAGE_BYTES);
          const int ra = tm * P_BM + row_half, rb = tn * P_BN + row_half;
          if constexpr (MN) {
#pragma unroll
            for (int j = 0; j < P_HALF / 64; ++j)
              tma_load_3d_pair(st + j * 8192, ma, bar, ra + 64 * j, kb * BK, b);
#pragma unroll
            for (int j = 0; j < P_HALF / 64; ++j)
              tma_load_3d_pair(st + P_A_BYTES + j * 8192, mb, bar, rb + 64 * j, kb * BK, b);
          } else {
            tma_load_3d_pair(st, ma, bar, kb * BK, ra, b);
            tma_load_3d_pair(st + P_A_BYTES, mb, bar, kb * BK, rb, b);
          }
          issued |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // give up: let the copies already issued land before shared memory
        // is released.  The leader sees them on its own barriers; the other
        // CTA's bytes also count there, so it waits out a fixed 2 ms instead.
        if (leader) {
          for (int st = 0; st < P_STAGES; ++st)
            if (issued & (1u << st)) wait_no_abort(&full[st], (issued_parity >> st) & 1u);
        } else {
          const unsigned long long t0 = globaltimer();
          while (globaltimer() - t0 < 2000000ull) __nanosleep(100000);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (the leader only)
      constexpr uint32_t IDESC = MN ? idesc_f16_mn(FMT == 1 ? 1 : 0, P_BM, P_BN)
                                    : idesc_f16(FMT == 1 ? 1 : 0, P_BM, P_BN);
      const uint32_t empty0 = mapa_shared(smem_u32(empty), 0), empty1 = mapa_shared(smem_u32(empty), 1);
      const uint32_t tfull0 = mapa_shared(smem_u32(tfull), 0), tfull1 = mapa_shared(smem_u32(tfull), 1);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it = 0;
      for (int t = cl; ok && t < n_tiles; t += ncl, ++it) {
        const int acc = it & 1;
        const uint32_t use = static_cast<uint32_t>(it >> 1);
        if (!mbar_wait(&tempty[acc], (use & 1) ^ 1, abort_flag, args.err, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * P_BN);
        for (int kb = 0; kb < total_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, args.err, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * P_STAGE_BYTES);
          if constexpr (MN) {
            const uint64_t da = smem_desc_mn_sw128(sa, 8192);
            const uint64_t db = smem_desc_mn_sw128(sa + P_A_BYTES, 8192);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              umma_f16_pair(d, da + 128 * k, db + 128 * k, IDESC, (kb | k) != 0 ? 1u : 0u);
          } else {
            const uint64_t da = smem_desc_k_sw128(sa);
            const uint64_t db = smem_desc_k_sw128(sa + P_A_BYTES);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              umma_f16_pair(d, da + 2 * k, db + 2 * k, IDESC, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(empty0 + static_cast<uint32_t>(stage * 8));
          umma_commit_pair(empty1 + static_cast<uint32_t>(stage * 8));
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) {
          umma_commit_pair(tfull0 + static_cast<uint32_t>(acc * 8));
          umma_commit_pair(tfull1 + static_cast<uint32_t>(acc * 8));
        }
      }
      // every issued MMA has finished before TMEM is released
      umma_commit_pair(mapa_shared(smem_u32(drain), 0));
      if (!wait_no_abort(drain, 0) && args.err) atomicCAS(args.err, 0, 4);
    }
  } else {
    // ---------------- epilogue: warps 2..9 of both CTAs, one accumulator row
    // per thread; warp w reads TMEM lanes 32*(w%4) .. +31 and half of the columns
    const int q = warp & 3;
    const int col0 = ((warp - 2) >> 2) * (P_BN / 2);
    const int row_in_tile = q * 32 + lane;
    const uint32_t tempty_leader = mapa_shared(smem_u32(tempty), 0);
    uint32_t* tsm = reinterpret_cast<uint32_t*>(smem + P_STAGES * P_STAGE_BYTES + 256) +
                    (warp - 2) * TRANS_WORDS;
    int it = 0;
    for (int t = cl; t < n_tiles; t += ncl, ++it) {
      const int acc = it & 1;
      const uint32_t use = static_cast<uint32_t>(it >> 1);
      int b, tm, tn;
      decode_tile_pair(args, t, b, tm, tn);
      if constexpr (EPI == EPI_FINAL)
        prefetch_final(args, b, tm * P_BM + row_half + q * 32, tn * P_BN + col0);
      if (!mbar_wait(&tfull[acc], use & 1, abort_flag, args.err, 5)) break;
      tc_fence_after();
      const int r = tm * P_BM + row_half + row_in_tile;
      const int c_base = tn * P_BN;
      const uint32_t taddr = tmem_base + static_cast<uint32_t>(acc * P_BN) +
                             (static_cast<uint32_t>(q * 32) << 16);
      for (int cc = col0; cc < col0 + P_BN / 2; cc += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(cc), v);
        tmem_ld_wait();
        if (c_base + cc < args.N) epilogue_chunk<EPI, FMT>(args, b, r, c_base + cc, v, tsm);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader + static_cast<uint32_t>(acc * 8));
    }
  }
  if constexpr (EPI == EPI_FINAL) {
    if (args.fin_npeers) __threadfence_system();  // peer stores visible before the kernel ends
  }
  tc_fence_before();
  cluster_sync();  // both CTAs done with the pair's MMAs, TMEM and shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
  cluster_sync();
}

// ------------------------------------------------------------------ prologue
template <int SDT>
__device__ __forceinline__ float load_src1(const void* src, int64_t i) {
  if constexpr (SDT == TK_F32) return static_cast<const float*>(src)[i];
  else return bf16_bits_to_f32(static_cast<const uint16_t*>(src)[i]);
}

template <int SDT>
__device__ __forceinline__ void load_src4(const void* src, int64_t i, float (&g)[4]) {
  if constexpr (SDT == TK_F32) {
    const float4 v = *reinterpret_cast<const float4*>(static_cast<const float*>(src) + i);
    g[0] = v.x; g[1] = v.y; g[2] = v.z; g[3] = v.w;
  } else {
    const uint2 v = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(src) + i);
    g[0] = bf16_bits_to_f32(v.x & 0xffffu); g[1] = bf16_bits_to_f32(v.x >> 16);
    g[2] = bf16_bits_to_f32(v.y & 0xffffu); g[3] = bf16_bits_to_f32(v.y >> 16);
  }
}

// python/tikun/muon_nd.py:112-115 in f32: buf = mu*buf + om*g; u = mu*buf + om*g
__device__ __forceinline__ float muon_u(const PrepArgs& a, float& buf, float g) {
  buf = __fadd_rn(__fmul_rn(a.mu, buf), __fmul_rn(a.om, g));
  return a.nesterov ? __fadd_rn(__fmul_rn(a.mu, buf), __fmul_rn(a.om, g)) : buf;
}

// Pass 1: per matrix, optional Muon momentum update, f64 sum of squares of the
// matrix handed to Newton-Schulz.  grid (nblk, batch); each block takes an
// equal range of 4-element groups (128-bit momentum accesses).
template <int SDT, bool MUON>
__global__ void __launch_bounds__(256)
prep_stats_kernel(const __grid_constant__ PrepArgs a, double* __restrict__ partials) {
  const int b = blockIdx.y;
  const int64_t total = a.m * a.n;
  const void* src = a.src[b];
  float* mom = MUON ? a.mom[b] : nullptr;
  const bool vec = ((uintptr_t)src % (SDT == TK_F32 ? 16 : 8)) == 0 &&
                   (!MUON || ((uintptr_t)mom % 16) == 0);
  const int64_t groups = vec ? total / 4 : 0;
  const int64_t g0 = groups * blockIdx.x / gridDim.x, g1 = groups * (blockIdx.x + 1) / gridDim.x;
  double s = 0.0;
  for (int64_t q = g0 + threadIdx.x; q < g1; q += blockDim.x) {
    float g[4];
    load_src4<SDT>(src, q * 4, g);
    float u[4];
    if constexpr (MUON) {
      float4 m4 = *reinterpret_cast<float4*>(mom + q * 4);
      float bb[4] = {m4.x, m4.y, m4.z, m4.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) u[j] = muon_u(a, bb[j], g[j]);
      *reinterpret_cast<float4*>(mom + q * 4) = make_float4(bb[0], bb[1], bb[2], bb[3]);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) u[j] = g[j];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) s = fma((double)u[j], (double)u[j], s);
  }
  // elements past the last whole group (or all of them when unaligned),
  // split over the blocks the same way
  const int64_t rest0 = groups * 4, rest = total - rest0;
  const int64_t e0 = rest0 + rest * blockIdx.x / gridDim.x;
  const int64_t e1 = rest0 + rest * (blockIdx.x + 1) / gridDim.x;
  for (int64_t i = e0 + threadIdx.x; i < e1; i += blockDim.x) {
    const float g = load_src1<SDT>(src, i);
    float u = g;
    if constexpr (MUON) {
      float bb = mom[i];
      u = muon_u(a, bb, g);
      mom[i] = bb;
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

// Per matrix: 1 / max(||U||_F, 1e-7) in f32 (tensor_engine.rs:37-41) from the
// f64 partial sums, in a fixed order.  grid (batch), block 32.
__global__ void __launch_bounds__(32)
prep_scale_kernel(const double* __restrict__ partials, int nblk, float* __restrict__ scales) {
  double s = 0.0;
  for (int i = threadIdx.x; i < nblk; i += 32) s += partials[(int64_t)blockIdx.x * nblk + i];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_down_sync(0xffffffffu, s, off);
  if (threadIdx.x == 0) {
    const float nrm = __double2float_rn(sqrt(s));
    scales[blockIdx.x] = __fdiv_rn(1.0f, fmaxf(nrm, 1e-7f));
  }
}

// Normalised Newton-Schulz input u * 1/max(||U||, 1e-7) in f32
// (tensor_engine.rs:42-44) of element i, u = the Nesterov/momentum value
// (python/tikun/muon_nd.py:112-115) or the input itself.
template <int SDT, bool MUON>
__device__ __forceinline__ float prep_value(const PrepArgs& a, const void* src, const float* mom,
                                            int64_t i, float inv) {
  const float g = load_src1<SDT>(src, i);
  float u = g;
  if constexpr (MUON) {
    const float buf = mom[i];
    u = a.nesterov ? __fadd_rn(__fmul_rn(a.mu, buf), __fmul_rn(a.om, g)) : buf;
  }
  return __fmul_rn(u, inv);
}

// Pass 2 with zero iterations: the normalised matrix is the output (or the
// update) itself.  Grid (ceil(m/32) * ceil(n/32), 1, batch) over the input's
// 32x32 tiles, block (32, 8).
template <int SDT, bool MUON>
__global__ void __launch_bounds__(256)
prep_output_kernel(const __grid_constant__ PrepArgs a, const float* __restrict__ scales) {
  const int b = blockIdx.z;
  const float inv = __ldg(scales + b);
  const bool tall = (a.tall[b >> 6] >> (b & 63)) & 1ull;
  const int64_t rows = tall ? a.n : a.m, cols = tall ? a.m : a.n;
  const int64_t tiles_c = (cols + 31) / 32;
  const int64_t tr = blockIdx.x / tiles_c, tc = blockIdx.x - tr * tiles_c;
  const void* src = a.src[b];
  const float* mom = MUON ? a.mom[b] : nullptr;
  const int64_t c = tc * 32 + threadIdx.x;
  void* dst = a.dst[b];
  const float sc = tall ? a.upd_scale_tall : a.upd_scale_wide;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int64_t r = tr * 32 + threadIdx.y + 8 * k;
    if (r >= rows || c >= cols) continue;
    const int64_t i = r * cols + c;
    const float x = prep_value<SDT, MUON>(a, src, mom, i, inv);
    if (a.dst_dtype == TK_F32) {
      float* p = static_cast<float*>(dst) + i;
      *p = a.update ? __fadd_rn(*p, __fmul_rn(sc, x)) : x;
    } else {
      uint16_t* p = static_cast<uint16_t*>(dst) + i;
      *p = f32_to_bf16_bits(a.update ? __fadd_rn(bf16_bits_to_f32(*p), __fmul_rn(sc, x)) : x);
    }
  }
}

// Pass 2: normalise, pre-scale by 2^k, round to the operand type and write
// X^T (n x m).  The input G is R x C (m x n for a wide matrix, n x m for a
// tall one).  Grid (ceil(m/64) * ceil(n/64), 1, batch) over G's
// 64x64 tiles, 256 threads: thread (q, y) = (tid % 16, tid / 16) takes
// columns 4q .. 4q+3 of tile rows y, y+16, y+32, y+48 -- a 16-byte momentum
// load, an 8-byte (bf16) or 16-byte (f32) input load and an 8-byte store
// into the same-layout target per row when the four are in range and
// aligned -- and, after a shared-memory transpose, rows 4q .. 4q+3 of tile
// columns y, y+16, y+32, y+48 into the transposed target, again 8 bytes per
// store.  Rows of 65 halves keep the transposed reads to two-way bank
// conflicts.
template <int SDT, bool MUON, int FMT>
__global__ void __launch_bounds__(256)
prep_write_kernel(const __grid_constant__ PrepArgs a, const float* __restrict__ scales) {
  constexpr int T = 64, S = T + 1;
  __shared__ uint16_t tile[T][S];
  __shared__ uint16_t tile_lo[FMT == 2 ? T : 1][S];  // format 2: the lo halves
  const int b = blockIdx.z;
  const float inv = __ldg(scales + b);
  const bool tall = (a.tall[b >> 6] >> (b & 63)) & 1ull;  // G = X^T
  const int64_t rows = tall ? a.n : a.m, cols = tall ? a.m : a.n;
  const int64_t tiles_c = (cols + T - 1) / T;
  const int64_t r0 = (blockIdx.x / tiles_c) * T, c0 = (blockIdx.x % tiles_c) * T;
  const void* src = a.src[b];
  const float* mom = MUON ? a.mom[b] : nullptr;
  const int q = threadIdx.x & 15, y = threadIdx.x >> 4;
  // 4-element vector accesses of a row need every row start aligned
  const bool vec = (cols & 3) == 0 &&
                   (reinterpret_cast<uintptr_t>(src) & (SDT == TK_F32 ? 15 : 7)) == 0 &&
                   (!MUON || (reinterpret_cast<uintptr_t>(mom) & 15) == 0);
  // The target is X^T, the only copy of the iterate the GEMMs read: a tall
  // input already has its layout (stored as it is); a wide one is stored
  // through the shared-memory transpose.  X^T rows are 64-element padded, so
  // the 4-element stores are 8-byte aligned.
  uint16_t* xt = a.xt + (int64_t)b * a.xt_bs;
  const bool want_same = tall, want_other = !tall;
  uint16_t* same = xt;
  const int64_t same_ld = a.xt_ld, same_lo = a.xt_lo;
  const int64_t c = c0 + 4 * q;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int ty = y + 16 * k;
    const int64_t r = r0 + ty;
    float x[4] = {0.f, 0.f, 0.f, 0.f};
    const bool whole = r < rows && c + 3 < cols;
    if (whole && vec) {
      const int64_t i = r * cols + c;
      float g[4], buf[4] = {0.f, 0.f, 0.f, 0.f};
      load_src4<SDT>(src, i, g);
      if constexpr (MUON) {
        const float4 m4 = *reinterpret_cast<const float4*>(mom + i);
        buf[0] = m4.x; buf[1] = m4.y; buf[2] = m4.z; buf[3] = m4.w;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float u = g[j];
        if constexpr (MUON)
          u = a.nesterov ? __fadd_rn(__fmul_rn(a.mu, buf[j]), __fmul_rn(a.om, g[j])) : buf[j];
        x[j] = __fmul_rn(u, inv);
      }
    } else if (r < rows) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (c + j < cols) x[j] = prep_value<SDT, MUON>(a, src, mom, r * cols + c + j, inv);
    }
    uint16_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float v = __fmul_rn(x[j], a.prescale);
      h[j] = to_half_bits<FMT>(v);
      l[j] = 0;
      if constexpr (FMT == 2) l[j] = to_half_bits<FMT>(v - from_half_bits<FMT>(h[j]));
      tile[ty][4 * q + j] = h[j];
      if constexpr (FMT == 2) tile_lo[ty][4 * q + j] = l[j];
    }
    if (!want_same) {
    } else if (whole) {
      *reinterpret_cast<uint2*>(same + r * same_ld + c) =
          make_uint2(h[0] | ((uint32_t)h[1] << 16), h[2] | ((uint32_t)h[3] << 16));
      if constexpr (FMT == 2)
        *reinterpret_cast<uint2*>(same + r * same_ld + same_lo + c) =
            make_uint2(l[0] | ((uint32_t)l[1] << 16), l[2] | ((uint32_t)l[3] << 16));
    } else if (r < rows) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (c + j < cols) {
          same[r * same_ld + c + j] = h[j];
          if constexpr (FMT == 2) same[r * same_ld + same_lo + c + j] = l[j];
        }
    }
  }
  __syncthreads();
  if (!want_other) return;
  // transposed target: element (r, c) of G goes to row c, column r
  uint16_t* other = xt;
  const int64_t other_ld = a.xt_ld, other_lo = a.xt_lo;
  const int64_t rr = r0 + 4 * q;  // columns of the target
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int tx = y + 16 * k;
    const int64_t cc = c0 + tx;  // row of the target
    if (cc >= cols) continue;
    uint16_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      h[j] = tile[4 * q + j][tx];
      l[j] = 0;
      if constexpr (FMT == 2) l[j] = tile_lo[4 * q + j][tx];
    }
    uint16_t* d = other + cc * other_ld + rr;
    if (rr + 3 < rows) {
      *reinterpret_cast<uint2*>(d) =
          make_uint2(h[0] | ((uint32_t)h[1] << 16), h[2] | ((uint32_t)h[3] << 16));
      if constexpr (FMT == 2)
        *reinterpret_cast<uint2*>(d + other_lo) =
            make_uint2(l[0] | ((uint32_t)l[1] << 16), l[2] | ((uint32_t)l[3] << 16));
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (rr + j < rows) {
          d[j] = h[j];
          if constexpr (FMT == 2) d[other_lo + j] = l[j];
        }
    }
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

static thread_local int g_gemm_reserved_sms = 0;

void set_gemm_reserved_sms(int n) { g_gemm_reserved_sms = n < 0 ? 0 : n; }

// ma_lo / mb_lo: the lo halves' maps in format 2 (the same maps otherwise).
template <int EPI, int FMT, bool MN = false>
static int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& ma_lo,
                       const CUtensorMap& mb_lo, const GemmArgs& g, cudaStream_t s) {
  // per device, set once; threads that race here set the same attribute
  static std::atomic<bool> attr_set[64] = {};
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(TK_ERR_CUDA, "device index %d out of range", dev);
  if (!attr_set[dev].load(std::memory_order_acquire)) {
    TK_CUDA_TRY(cudaFuncSetAttribute(gemm_tn_kernel<EPI, FMT, MN>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    attr_set[dev].store(true, std::memory_order_release);
  }
  int sms = 0;
  TK_TRY(sm_count(&sms));
  const int n_tiles = g.batch * g.tiles_per_mat;
  if (n_tiles == 0) return TK_OK;
  const int grid = std::min(n_tiles, std::max(1, sms - g_gemm_reserved_sms));
  gemm_tn_kernel<EPI, FMT, MN><<<grid, THREADS, SMEM_BYTES, s>>>(ma, mb, ma_lo, mb_lo, g);
  TK_CUDA_TRY(cudaGetLastError());
  return TK_OK;
}

// An operand: the map of its (hi) values and, in format 2, of its lo halves.
struct Operand {
  CUtensorMap hi, lo;
};

template <int EPI, bool MN = false>
static int launch_gemm_fmt(int fmt, const Operand& a, const Operand& b, const GemmArgs& g,
                           cudaStream_t s) {
  if (fmt == 2) return launch_gemm<EPI, 2, MN>(a.hi, b.hi, a.lo, b.lo, g, s);
  if constexpr (EPI == EPI_XUPD || EPI == EPI_FINAL) {
    if (fmt == 3) return launch_gemm<EPI, 3, MN>(a.hi, b.hi, a.lo, b.hi, g, s);
  }
  if (fmt != 0 && fmt != 1) return set_error(TK_ERR_INVALID, "operand format %d for this GEMM", fmt);
  return fmt == 0 ? launch_gemm<EPI, 0, MN>(a.hi, b.hi, a.hi, b.hi, g, s)
                  : launch_gemm<EPI, 1, MN>(a.hi, b.hi, a.hi, b.hi, g, s);
}

// CTA-pair launch: clusters of 2, as many as fit at once (at most one pair
// per two SMs outside the reserved ones), each looping over 256 x 256 tiles.
template <int EPI, int FMT, bool MN = false>
static int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& ma_lo,
                       const CUtensorMap& mb_lo, const GemmArgs& g, cudaStream_t s) {
  // per device, computed once; threads that race here compute the same value
  static std::atomic<int> max_clusters[64] = {};
  int dev = 0;
  TK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(TK_ERR_CUDA, "device index %d out of range", dev);
  auto* kern = gemm_pair_kernel<EPI, FMT, MN>;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = P_SMEM_BYTES;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int sms = 0;
  TK_TRY(sm_count(&sms));
  int ncl = max_clusters[dev].load(std::memory_order_acquire);
  if (ncl == 0) {
    TK_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     P_SMEM_BYTES));
    cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
    int n = 0;
    TK_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
    if (n < 1) return set_error(TK_ERR_CUDA, "no CTA pair of the GEMM kernel fits on an SM pair");
    ncl = n;
    max_clusters[dev].store(n, std::memory_order_release);
  }
  const int n_tiles = g.batch * g.tiles_per_mat;
  if (n_tiles == 0) return TK_OK;
  const int usable = std::max(1, std::min(ncl, (sms - g_gemm_reserved_sms) / 2));
  cfg.gridDim = dim3(2 * std::min(n_tiles, usable), 1, 1);
  TK_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, ma, mb, ma_lo, mb_lo, g));
  return TK_OK;
}

template <int EPI, bool MN = false>
static int launch_pair_fmt(int fmt, const Operand& a, const Operand& b, const GemmArgs& g,
                           cudaStream_t s) {
  if (fmt == 2) return launch_pair<EPI, 2, MN>(a.hi, b.hi, a.lo, b.lo, g, s);
  if constexpr (EPI == EPI_XUPD || EPI == EPI_FINAL) {
    if (fmt == 3) return launch_pair<EPI, 3, MN>(a.hi, b.hi, a.lo, b.hi, g, s);
  }
  if (fmt != 0 && fmt != 1) return set_error(TK_ERR_INVALID, "operand format %d for this GEMM", fmt);
  return fmt == 0 ? launch_pair<EPI, 0, MN>(a.hi, b.hi, a.hi, b.hi, g, s)
                  : launch_pair<EPI, 1, MN>(a.hi, b.hi, a.hi, b.hi, g, s);
}

template <int EPI, bool MN = false>
static int launch_any(bool pair, int fmt, const Operand& a, const Operand& b, const GemmArgs& g,
                      cudaStream_t s) {
  return pair ? launch_pair_fmt<EPI, MN>(fmt, a, b, g, s) : launch_gemm_fmt<EPI, MN>(fmt, a, b, g, s);
}

// The hi (and, in format 2, lo) maps of an operand stored with row stride
// `rs` elements, the lo values lo_off elements after the hi ones.
static int make_operand(Operand* op, const uint16_t* base, int fmt, int64_t inner, int64_t rows,
                        int64_t rs, int64_t lo_off, int64_t batch, int box_rows) {
  TK_TRY(make_map(&op->hi, base, fmt == 1 ? 1 : 0, inner, rows, rs, batch, box_rows));
  if (fmt == 2) TK_TRY(make_map(&op->lo, base + lo_off, 0, inner, rows, rs, batch, box_rows));
  else op->lo = op->hi;
  return TK_OK;
}

static int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

static size_t align256(size_t x) { return (x + 255) / 256 * 256; }

GroupLayout group_layout(int64_t m, int64_t n, int64_t batch, bool split) {
  GroupLayout L;
  L.m = m;
  L.n = n;
  L.batch = batch;
  L.split = split;
  L.ldm = round_up(L.m, 64);
  // format 2: each row holds the hi values, then the lo values
  L.rsm = split ? 2 * L.ldm : L.ldm;
  L.xt_bytes = align256((size_t)(batch * L.n * L.rsm * 2));
  L.a_bytes = align256((size_t)(batch * L.m * L.rsm * 2));
  L.nblk = (int)std::max<int64_t>(1, std::min<int64_t>(256, (m * n + 16383) / 16384));
  L.scratch_bytes = 2 * L.xt_bytes + 3 * L.a_bytes +
                    align256(sizeof(double) * batch * L.nblk) + align256(sizeof(float) * batch) +
                    256;
  return L;
}

// Power-of-two pre-scale of the first iterate in f16 mode: RMS of the
// normalised matrix is 1/sqrt(m n); lift it to about 2^-4.
static int prescale_exp(int fmt, int64_t m, int64_t n) {
  if (fmt == 1) return 0;
  const double r = std::sqrt((double)m * (double)n) / 16.0;
  int k = (int)std::floor(std::log2(std::max(r, 1.0)));
  return std::max(0, std::min(k, 60));
}

int run_group(const GroupLayout& L, const GroupIO& io, int steps, int fmt, void* scratch,
              int* err_dev, cudaStream_t s) {
  if (L.batch == 0 || L.m == 0) return TK_OK;
  if (L.batch > kMaxBatch) return set_error(TK_ERR_INVALID, "batch of %lld > %d", (long long)L.batch, kMaxBatch);
  // format 3 keeps X as f16 pairs and A, A', B' in f16, which needs the
  // folded polynomial; below 256 rows the full pairs (format 2) run instead,
  // on the same scratch layout
  if (fmt == 3 && L.m < 256) fmt = 2;
  if (L.split != (fmt >= 2))
    return set_error(TK_ERR_INVALID, "scratch layout does not match operand format %d", fmt);
  char* cur = static_cast<char*>(scratch);
  uint16_t* XT[2] = {reinterpret_cast<uint16_t*>(cur),
                     reinterpret_cast<uint16_t*>(cur + L.xt_bytes)};
  cur += 2 * L.xt_bytes;
  uint16_t* Am = reinterpret_cast<uint16_t*>(cur);
  cur += L.a_bytes;
  uint16_t* Bm = reinterpret_cast<uint16_t*>(cur);
  cur += L.a_bytes;
  uint16_t* Ap = reinterpret_cast<uint16_t*>(cur);
  cur += L.a_bytes;
  double* partials = reinterpret_cast<double*>(cur);
  cur += align256(sizeof(double) * L.batch * L.nblk);
  float* scales = reinterpret_cast<float*>(cur);

  const int k = prescale_exp(fmt, L.m, L.n);
  // kernel parameters carry the per-matrix pointers and orientation bits
  static thread_local PrepArgs pa;
  std::memset(&pa, 0, sizeof(pa));
  for (int64_t i = 0; i < L.batch; ++i) {
    pa.src[i] = io.src[i];
    pa.dst[i] = io.dst[i];
    pa.mom[i] = io.mom ? io.mom[i] : nullptr;
    if (io.tall[i]) pa.tall[i >> 6] |= 1ull << (i & 63);
  }
  pa.m = L.m;
  pa.n = L.n;
  pa.mu = io.mu;
  pa.om = io.om;
  pa.nesterov = io.nesterov;
  pa.xt = XT[0];
  pa.xt_ld = L.rsm;
  pa.xt_bs = L.n * L.rsm;
  pa.xt_lo = L.ldm;
  pa.prescale = std::ldexp(1.0f, k);
  pa.steps = steps;
  pa.dst_dtype = io.dst_dtype;
  pa.update = io.update;
  pa.upd_scale_wide = io.upd_scale_wide;
  pa.upd_scale_tall = io.upd_scale_tall;

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
    prep_scale_kernel<<<(unsigned)L.batch, 32, 0, s>>>(partials, L.nblk, scales);
    TK_CUDA_TRY(cudaGetLastError());
    if (steps == 0) {  // the normalised matrix is the result
      dim3 g0((unsigned)(((L.m + 31) / 32) * ((L.n + 31) / 32)), 1, (unsigned)L.batch);
      dim3 b0(32, 8);
      if (io.src_dtype == TK_F32) {
        if (muon) prep_output_kernel<TK_F32, true><<<g0, b0, 0, s>>>(pa, scales);
        else prep_output_kernel<TK_F32, false><<<g0, b0, 0, s>>>(pa, scales);
      } else {
        if (muon) prep_output_kernel<TK_BF16, true><<<g0, b0, 0, s>>>(pa, scales);
        else prep_output_kernel<TK_BF16, false><<<g0, b0, 0, s>>>(pa, scales);
      }
      TK_CUDA_TRY(cudaGetLastError());
      return TK_OK;
    }
    dim3 g2((unsigned)(((L.m + 63) / 64) * ((L.n + 63) / 64)), 1, (unsigned)L.batch);
    dim3 b2(256);
#define TK_PREP_WRITE(SDT, MU, F) prep_write_kernel<SDT, MU, F><<<g2, b2, 0, s>>>(pa, scales)
#define TK_PREP_WRITE_FMT(SDT, MU)                   \
  do {                                               \
    if (fmt == 0) TK_PREP_WRITE(SDT, MU, 0);         \
    else if (fmt == 1) TK_PREP_WRITE(SDT, MU, 1);    \
    else TK_PREP_WRITE(SDT, MU, 2);                  \
  } while (0)
    if (io.src_dtype == TK_F32) {
      if (muon) TK_PREP_WRITE_FMT(TK_F32, true);
      else TK_PREP_WRITE_FMT(TK_F32, false);
    } else {
      if (muon) TK_PREP_WRITE_FMT(TK_BF16, true);
      else TK_PREP_WRITE_FMT(TK_BF16, false);
    }
#undef TK_PREP_WRITE_FMT
#undef TK_PREP_WRITE
    TK_CUDA_TRY(cudaGetLastError());
  }
  if (steps == 0) return TK_OK;

  // One iteration with f16 operands, with A' = c A + b I and
  // B' = a I + b A + c A^2 = A A' + a I:
  //   GEMM1  A = X X^T, A' = c A + b I   (one product, two symmetric stores)
  //   GEMM2  B' = A A' + a I             (A' is symmetric, so A A'^T = A A')
  //   GEMM3  X_new^T = X^T B'            (B' is symmetric: X_new = B' X)
  // No epilogue reads a second matrix, so none waits on memory.  Rounding
  // a + B_ii and c A_ij + b to 16 bits costs accuracy: with bf16 operands
  // about 0.5 % more Newton-Schulz error, and with f16 operands on matrices
  // under 256 rows a parameter drift over 10 Muon steps close to 1e-3 (it is
  // below 3e-4 from 256 rows up).  There the epilogues add b A and a X^T in
  // f32 instead: GEMM2 B = c A A + b A, GEMM3 X_new^T = X^T B + a X^T.
  // Split operands (format 2) keep every stored value to about 22 bits, so
  // the folded form's roundings cost nothing there and it is used at all sizes.
  const bool fold = fmt >= 2 || (fmt == 0 && L.m >= 256);
  // format 3: A, A' and B' and the GEMMs that make them are f16; X^T and
  // GEMM3 (two passes over X^T's hi and lo values) keep the pairs
  const int fmt_mm = fmt == 3 ? 0 : fmt, fmt_x = fmt == 3 ? 2 : fmt;
  // GEMM1 (X X^T) reads X^T as both operands, MN-major: 64 x 64 boxes of
  // X^T's rows (K = n) and columns (M, N = m), so that no m x n copy of X is
  // ever written -- GEMM3 stores only X_new^T.
  // B operands are 256-row boxes for the single-CTA kernel and 128-row
  // halves for the CTA pair
  const bool pair = L.m >= TK_NS_PAIR_MIN_M;
  const int kBRows = pair ? P_HALF : BN;
  Operand mA128, mA256, mAp256, mB256, mXT128[2], mXTmn[2];
  TK_TRY(make_operand(&mA128, Am, fmt_mm, L.m, L.m, L.rsm, L.ldm, L.batch, 128));
  TK_TRY(make_operand(&mA256, Am, fmt_mm, L.m, L.m, L.rsm, L.ldm, L.batch, kBRows));
  TK_TRY(make_operand(&mAp256, Ap, fmt_mm, L.m, L.m, L.rsm, L.ldm, L.batch, kBRows));
  TK_TRY(make_operand(&mB256, Bm, fmt_mm, L.m, L.m, L.rsm, L.ldm, L.batch, kBRows));
  for (int q = 0; q < 2; ++q) {
    TK_TRY(make_operand(&mXT128[q], XT[q], fmt_x, L.m, L.n, L.rsm, L.ldm, L.batch, 128));
    TK_TRY(make_operand(&mXTmn[q], XT[q], fmt_x, L.m, L.n, L.rsm, L.ldm, L.batch, 64));
  }

  const int kTM = pair ? P_BM : BM, kTN = pair ? P_BN : BN;
  const int tm_sq = (int)((L.m + kTM - 1) / kTM), tn_sq = (int)((L.m + kTN - 1) / kTN);
  const bool mirror1 = L.n > TK_NS_FULL_K1, mirror2 = L.m > TK_NS_FULL_K2;
  const int tm_x = (int)((L.n + kTM - 1) / kTM);
  auto n_sym = [pair](int a, int b) { return pair ? sym_tiles_pair(a, b) : sym_tiles(a, b); };
  const float inv_pre = std::ldexp(1.0f, -k), inv_pre2 = std::ldexp(1.0f, -2 * k);
  int cur_xt = 0;
  static thread_local GemmArgs g, h;
  NvtxRange range("tikun/ns_iterations");
  for (int it = 0; it < steps; ++it) {
    std::memset(&g, 0, sizeof(g));
    g.batch = (int)L.batch;
    g.err = err_dev;
    // GEMM1: A = X X^T and A' = c A + b I
    g.M = g.N = (int)L.m;
    g.K = (int)L.n;
    g.tiles_m = tm_sq;
    g.tiles_n = tn_sq;
    g.symmetric = g.mirror = mirror1 ? 1 : 0;
    g.tiles_per_mat = mirror1 ? n_sym(tm_sq, tn_sq) : tm_sq * tn_sq;
    g.alpha = it == 0 ? inv_pre2 : 1.0f;
    g.beta = 0.0f;
    g.out = Am;
    g.out_ld = L.rsm;
    g.out_bs = L.m * L.rsm;
    g.lo_off = g.lo_off2 = L.ldm;
    if (fold) {
      g.alpha2 = NS_C * g.alpha;
      g.beta2 = NS_B;
      g.out2 = Ap;
      g.out2_ld = L.rsm;
      g.out2_bs = L.m * L.rsm;
    }
    TK_TRY((launch_any<EPI_SYM, true>(pair, fmt_mm, mXTmn[cur_xt], mXTmn[cur_xt], g, s)));
    // GEMM2: B' = A A' + a I  (bf16: B = c A A + b A)
    g.K = (int)L.m;
    g.symmetric = g.mirror = mirror2 ? 1 : 0;
    g.tiles_per_mat = mirror2 ? n_sym(tm_sq, tn_sq) : tm_sq * tn_sq;
    g.out = Bm;
    g.out2 = nullptr;
    if (fold) {
      g.alpha = 1.0f;
      g.beta = NS_A;
      TK_TRY(launch_any<EPI_SYM>(pair, fmt_mm, mA128, mAp256, g, s));
    } else {
      g.alpha = NS_C;
      g.gamma = NS_B;
      g.aux = Am;
      g.aux_ld = L.rsm;
      g.aux_bs = L.m * L.rsm;
      TK_TRY(launch_any<EPI_SYM>(pair, fmt_mm, mA128, mA256, g, s));
    }
    // GEMM3: X_new^T = post * X^T B' (post undoes the first iterate's pre-scale)
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
    h.alpha = it == 0 ? inv_pre : 1.0f;
    h.lo_off = L.ldm;   // X^T rows
    if (!fold) {  // + a X^T
      h.gamma = NS_A * h.alpha;
      h.aux = XT[cur_xt];
      h.aux_ld = L.rsm;
      h.aux_bs = L.n * L.rsm;
    }
    if (it + 1 < steps) {
      h.out = XT[cur_xt ^ 1];
      h.out_ld = L.rsm;
      h.out_bs = L.n * L.rsm;
      h.out2 = nullptr;  // GEMM1 reads X^T directly
      TK_TRY(launch_any<EPI_XUPD>(pair, fmt, mXT128[cur_xt], mB256, h, s));
      cur_xt ^= 1;
    } else {
      h.fin_dtype = io.dst_dtype;
      h.fin_update = io.update;
      h.fin_scale_wide = io.upd_scale_wide;
      h.fin_scale_tall = io.upd_scale_tall;
      for (int64_t i = 0; i < L.batch; ++i) {
        h.fin_ptrs[i] = io.dst[i];
        h.fin_tall[i >> 6] = pa.tall[i >> 6];
      }
      if (io.peers != nullptr) {
        h.fin_npeers = io.peers->n;
        for (int q = 0; q < io.peers->n; ++q) h.fin_peer_delta[q] = io.peers->delta[q];
      }
      TK_TRY(launch_any<EPI_FINAL>(pair, fmt, mXT128[cur_xt], mB256, h, s));
    }
  }
  return TK_OK;
}

// ------------------------------------------------------------------ peer copies
constexpr int kCopyThreads = 512;
constexpr int kCopyUnroll = 4;

__global__ void __launch_bounds__(kCopyThreads)
peer_copy_kernel(const __grid_constant__ PeerCopyList list, const __grid_constant__ PeerSet peers) {
  const uint64_t total = list.unit0[list.n];
  const uint64_t per = (total + gridDim.x - 1) / gridDim.x;
  const uint64_t u0 = (uint64_t)blockIdx.x * per;
  const uint64_t u1 = u0 + per < total ? u0 + per : total;
  int e = 0;
  for (uint64_t base = u0; base < u1; base += (uint64_t)kCopyThreads * kCopyUnroll) {
    uint4 v[kCopyUnroll];
    const uint8_t* src[kCopyUnroll];
    uint32_t len[kCopyUnroll];  // bytes of the unit (16 but at an entry's end)
#pragma unroll
    for (int k = 0; k < kCopyUnroll; ++k) {
      const uint64_t u = base + (uint64_t)k * kCopyThreads + threadIdx.x;
      len[k] = 0;
      src[k] = nullptr;
      if (u >= u1) continue;
      while (e + 1 < list.n && list.unit0[e + 1] <= u) ++e;
      const uint64_t off = (u - list.unit0[e]) * 16;
      const uint64_t rem = list.bytes[e] - off;
      src[k] = list.src[e] + off;
      len[k] = rem >= 16 ? 16u : (uint32_t)rem;
      if (len[k] == 16) v[k] = *reinterpret_cast<const uint4*>(src[k]);
    }
#pragma unroll
    for (int k = 0; k < kCopyUnroll; ++k) {
      if (len[k] == 0) continue;
      for (int q = 0; q < peers.n; ++q) {
        uint8_t* dst = const_cast<uint8_t*>(src[k]) + peers.delta[q];
        if (len[k] == 16) *reinterpret_cast<uint4*>(dst) = v[k];
        else
          for (uint32_t b = 0; b < len[k]; ++b) dst[b] = src[k][b];
      }
    }
  }
  __threadfence_system();  // peer stores visible before the kernel ends
}

int launch_peer_copy(const PeerCopyList& list, const PeerSet& peers, int blocks, cudaStream_t s) {
  if (list.n <= 0 || peers.n <= 0 || list.unit0[list.n] == 0) return TK_OK;
  if (list.n > kMaxBatch || peers.n > kMaxPeers)
    return set_error(TK_ERR_INVALID, "peer copy list of %d entries to %d peers", list.n, peers.n);
  for (int i = 0; i < list.n; ++i)
    if ((reinterpret_cast<uintptr_t>(list.src[i]) & 15) != 0)
      return set_error(TK_ERR_INVALID, "peer copy source %p is not 16-byte aligned", list.src[i]);
  for (int q = 0; q < peers.n; ++q)
    if (peers.delta[q] % 16 != 0)
      return set_error(TK_ERR_INVALID, "peer delta %lld is not a multiple of 16",
                       (long long)peers.delta[q]);
  peer_copy_kernel<<<std::max(1, blocks), kCopyThreads, 0, s>>>(list, peers);
  TK_CUDA_TRY(cudaGetLastError());
  return TK_OK;
}

// ------------------------------------------------------------------ test hooks
// A wait that cannot complete: one thread waits on a fresh mbarrier that no
// one arrives on, with the given bound.  It must give up, record code 9 in the
// status word and return, leaving the context usable.
__global__ void bounded_wait_probe_kernel(int* err, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, err, 9, limit_ns);
}

int bounded_wait_probe(int* err_dev, int limit_ms, cudaStream_t s) {
  if (limit_ms < 1 || limit_ms > 2000) return set_error(TK_ERR_INVALID, "limit %d ms outside 1..2000", limit_ms);
  bounded_wait_probe_kernel<<<1, 32, 0, s>>>(err_dev, (unsigned long long)limit_ms * 1000000ull);
  TK_CUDA_TRY(cudaGetLastError());
  return TK_OK;
}


// Plain batched TN GEMM D = alpha * P Q^T on half-precision operands, for the
// kernel's own tests.
int plain_gemm(const uint16_t* P, const uint16_t* Q, uint16_t* D, int batch, int M, int N, int K,
               int64_t ldp, int64_t ldq, int64_t ldd, float alpha, int fmt, int* err_dev,
               cudaStream_t s) {
  if (fmt != 0 && fmt != 1) return set_error(TK_ERR_INVALID, "plain GEMM format %d", fmt);
  CUtensorMap ma, mb;
  TK_TRY(make_map(&ma, P, fmt, K, M, ldp, batch, 128));
  TK_TRY(make_map(&mb, Q, fmt, K, N, ldq, batch, 256));
  static thread_local GemmArgs g;
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
  return fmt == 0 ? launch_gemm<EPI_PLAIN, 0>(ma, mb, ma, mb, g, s)
                  : launch_gemm<EPI_PLAIN, 1>(ma, mb, ma, mb, g, s);
}

}  // namespace ns
}  // namespace tk
