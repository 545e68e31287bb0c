// aux_kernels.cuh - HBM-bound helper kernels of the checksum library.
//
//   encode_weight_kernel   per-tile plain and column-index-weighted row
//                          checksums of B[N, K] (the "Be" of checkers.py:119),
//                          split into bf16 terms for the check MMA
//   encode_f16_cluster_kernel  the same block for fp16 B, each checksum of a
//                          tile scaled by a power of two (one launch, an
//                          8-CTA cluster per tile); encode_f16_few_rows_kernel
//                          for tiles of at most 32 rows (decode tokens);
//                          encode_f16_sums_kernel + encode_f16_finish_kernel
//                          for large weights
//   transpose_encode_kernel  K-major copy of an N-major right operand
//                          B[K, N] (torch.bmm's mat2), with the same
//                          checksum block computed on the way
//   colsum_partial_kernel  column sums of a row-major [R, C] matrix (bf16, fp16
//                          or fp32) over
//                          blocks of rows (optionally row-weighted, with |x| max)
//   reduce_partials_kernel sum (and max) of those partials in fixed order
//   rowdot_kernel          per-row sum or dot with a vector (warp per row)
//   ref_finalize_kernel    corner = dot(u, v) + M*sum(bias), sum_c, ok flag
//                          (pytorch/abft/checkers.py:96-126)
//   locate_finalize_kernel global row/column mismatch search and pairing
//
// Every sum runs in a fixed order, so results are bit-reproducible run to
// run (the reference's fp32 atomics, abft_fused.cu:45-46 and :71-88, are
// not); the only atomics here take maxima, which do not depend on order.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../include/abft_b200.h"
#include "ptx.cuh"

namespace abft {

__device__ __forceinline__ void unpack8(const uint4 w, float (&x)[8]) {
  x[0] = __uint_as_float(w.x << 16);
  x[1] = __uint_as_float(w.x & 0xFFFF0000u);
  x[2] = __uint_as_float(w.y << 16);
  x[3] = __uint_as_float(w.y & 0xFFFF0000u);
  x[4] = __uint_as_float(w.z << 16);
  x[5] = __uint_as_float(w.z & 0xFFFF0000u);
  x[6] = __uint_as_float(w.w << 16);
  x[7] = __uint_as_float(w.w & 0xFFFF0000u);
}

// Eight consecutive elements of a row as fp32 (16- or 32-byte aligned),
// for the element types of the post-hoc check: bf16, fp16 or fp32.
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&x)[8]) {
  unpack8(__ldg(reinterpret_cast<const uint4*>(p)), x);
}
__device__ __forceinline__ void load8(const __half* p, float (&x)[8]) {
  const uint4 q = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const float* p, float (&x)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(float v) { return v; }

// Round an fp32 value to the element type T (and back): the rounding of a
// torch reduction whose result has type T (fp32 accumulation inside).
template <typename T>
__device__ __forceinline__ float round_to(float x);
template <>
__device__ __forceinline__ float round_to<__nv_bfloat16>(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
template <>
__device__ __forceinline__ float round_to<__half>(float x) { return __half2float(__float2half_rn(x)); }
template <>
__device__ __forceinline__ float round_to<float>(float x) { return x; }

// Split v into three bf16 terms whose sum carries 24 significant bits:
// hi = rn(v), mid = rn(v - hi), lo = rn(v - hi - mid); both differences are
// exact in fp32.
__device__ __forceinline__ void split3_bf16(float v, __nv_bfloat16& hi, __nv_bfloat16& mid, __nv_bfloat16& lo) {
  hi = __float2bfloat16_rn(v);
  const float r1 = v - __bfloat162float(hi);
  mid = __float2bfloat16_rn(r1);
  const float r2 = r1 - __bfloat162float(mid);
  lo = __float2bfloat16_rn(r2);
}

// Sign of local column j in the third checksum: +1 when j has an even number
// of set bits, -1 otherwise (the Thue-Morse sequence; no three consecutive
// columns share a sign).
__host__ __device__ __forceinline__ float col_sign(int j) { return (__builtin_popcount(j) & 1) ? -1.f : 1.f; }

// Per-tile checksum block of B[N, K]: the 8 rows the fused GEMM appends to
// each B-operand tile of bd data rows.
// out is [tiles_n * 8, K] row-major in B's element type; rows of tile t:
//   8t+0..2 = split3(v1), 8t+3..5 = split3(v2), 8t+6..7 = split2(v3), with
//   v1[k] = sum_j B[t*bd + j, k],  v2[k] = sum_j (j+1) B[t*bd + j, k],
//   v3[k] = sum_j col_sign(j) B[t*bd + j, k]
// (j over the tile's valid rows; fp32 sums in a fixed order).
// bf16 has fp32's exponent range, so the terms are the sums themselves.
// fp16 does not (largest finite 65504): each of v1, v2, v3 of a tile is
// scaled by 2^-e, e chosen so that its largest |value| over k lands in
// [2^14, 2^15), before the split; the scale table after the rows holds
// 8 floats per tile, [0..2] the largest |v1|, |v2|, |v3| (NaN sums are
// passed over, as fmaxf does) and [4..6] the factors 2^e. Multiplying by a
// power of two is exact, so the check MMA's sums times 2^e equal the
// unscaled ones.
// grid (ceil(K/64), tiles_n, batch), 256 threads. K % 8 == 0. Batch z reads
// B + z * b_stride, writes out + z * out_stride and table + z * table_stride.
__device__ __forceinline__ void write_checksum_rows(float a1, float a2, float a3, __nv_bfloat16* o, int K) {
  __nv_bfloat16 h[8];
  split3_bf16(a1, h[0], h[1], h[2]);
  split3_bf16(a2, h[3], h[4], h[5]);
  h[6] = __float2bfloat16_rn(a3);
  h[7] = __float2bfloat16_rn(a3 - __bfloat162float(h[6]));
#pragma unroll
  for (int q = 0; q < 8; ++q) o[static_cast<int64_t>(q) * K] = h[q];
}

// fp16 terms: hi = rn(x), mid = rn(x - hi), lo = rn(x - hi - mid); with
// |x| < 2^15 no term overflows and both differences are exact in fp32.
__device__ __forceinline__ void split3_f16(float x, __half& hi, __half& mid, __half& lo) {
  hi = __float2half_rn(x);
  const float r1 = x - __half2float(hi);
  mid = __float2half_rn(r1);
  lo = __float2half_rn(r1 - __half2float(mid));
}

__device__ __forceinline__ void write_checksum_rows_f16(float a1, float a2, float a3, __half* o, int K) {
  __half h[8];
  split3_f16(a1, h[0], h[1], h[2]);
  split3_f16(a2, h[3], h[4], h[5]);
  h[6] = __float2half_rn(a3);
  h[7] = __float2half_rn(a3 - __half2float(h[6]));
#pragma unroll
  for (int q = 0; q < 8; ++q) o[static_cast<int64_t>(q) * K] = h[q];
}

// The exponent e of an fp16 checksum scale for largest magnitude m: 2^-e m
// in [2^14, 2^15) for normal m; 0 for zero, subnormal or non-finite m;
// limited to [-100, 100] so that 2^e and 2^-e are normal floats.
__host__ __device__ __forceinline__ int f16_chk_exponent(uint32_t mbits) {
  const int be = static_cast<int>((mbits >> 23) & 0xFFu);
  if (be == 0 || be == 0xFF) return 0;
  const int e = (be - 127) - 14;
  return e < -100 ? -100 : (e > 100 ? 100 : e);
}
__host__ __device__ __forceinline__ float pow2f_exact(int e) {  // 2^e, e in [-126, 127]
  const uint32_t bits = static_cast<uint32_t>(e + 127) << 23;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

__device__ __forceinline__ void unpack8_as(const uint4 w, float (&x)[8], const __nv_bfloat16*) { unpack8(w, x); }
__device__ __forceinline__ void unpack8_as(const uint4 w, float (&x)[8], const __half*) {
  const uint32_t q[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&q[i]));
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

// Where the fp16 encode keeps sum q (0..2) of k column kb*64 + t until the
// tile's scale is known: inside the bytes that k-block's final rows occupy
// (8 rows x c columns x 2 bytes, c = its valid columns, a multiple of 8),
// read as 8 segments of 2c bytes; the 3c floats fill the first 12c of
// those 16c bytes. Only the CTA that handles the k-block touches them, so
// it may read them back and then overwrite them with the rows.
// rows_tile: the tile's first checksum row.
__device__ __forceinline__ float* f16_stage_slot(__half* rows_tile, int K, int kb, int c, int q, int t) {
  const int f = q * c + t;
  const int seg = (2 * f) / c;           // (4 f) / (2 c): row of the segment, < 6
  const int off = 4 * f - seg * 2 * c;   // byte offset inside it, a multiple of 4
  return reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(rows_tile + static_cast<int64_t>(seg) * K + kb * 64) +
                                  off);
}

// The three checksums of k columns [kb*64, kb*64 + 64) of tile nt, for
// thread t < 64 (column kb*64 + t; zero past K). 256 threads; starts with a
// block barrier, so that a caller may loop over k-blocks reusing `red`.
template <typename T>
__device__ __forceinline__ void kblock_checksums(const T* __restrict__ B, int64_t ldb, int N, int K, int bd, int nt,
                                                 int kb, float (&red)[3][32][65], float& a1, float& a2, float& a3) {
  const int t = threadIdx.x, c8 = t & 7, rg = t >> 3;
  const int k0 = kb * 64 + c8 * 8;
  float s1[8], s2[8], s3[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) s1[e] = s2[e] = s3[e] = 0.f;
  if (k0 < K) {
    // Rows rg, rg + 32, ... of the tile (at most 8: a tile has at most 256
    // rows), added in that order. Every load of the thread is issued before
    // the first is used, so the pass waits for one memory round trip rather
    // than one per row; the order of the sums is that of a row-at-a-time loop.
    const int nrows = min(bd, N - nt * bd);
    const T* base = B + static_cast<int64_t>(nt) * bd * ldb + k0;
    uint4 w[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = rg + 32 * u;
      w[u] = j < nrows ? __ldg(reinterpret_cast<const uint4*>(base + static_cast<int64_t>(j) * ldb))
                       : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = rg + 32 * u;
      if (j >= nrows) break;
      float x[8];
      unpack8_as(w[u], x, B);
      const float wt = static_cast<float>(j + 1);
      const float sg = col_sign(j);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        s1[e] += x[e];
        s2[e] = fmaf(wt, x[e], s2[e]);
        s3[e] = fmaf(sg, x[e], s3[e]);
      }
    }
  }
  __syncthreads();  // the previous k-block's reads of red are done
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    red[0][rg][c8 * 8 + e] = s1[e];
    red[1][rg][c8 * 8 + e] = s2[e];
    red[2][rg][c8 * 8 + e] = s3[e];
  }
  __syncthreads();
  a1 = a2 = a3 = 0.f;
  if (t < 64 && kb * 64 + t < K) {
    for (int g = 0; g < 32; ++g) {
      a1 += red[0][g][t];
      a2 += red[1][g][t];
      a3 += red[2][g][t];
    }
  }
}

// Under CUDA-graph capture, the fused GEMM's launch tag is frozen in its
// node, so every replay must start from cleared state: the report's
// launch_tag (when `tag` is set) and the `n` stream-K flags (when `flags`
// is set) are zeroed here, one graph node ahead of the GEMM.
__global__ void __launch_bounds__(256) clear_launch_state_kernel(unsigned long long* tag,
                                                                 unsigned long long* flags, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (flags != nullptr && i < n) flags[i] = 0ull;
  if (tag != nullptr && i == 0) *tag = 0ull;
}

// bf16 checksum block: one k-block of one tile per CTA.
__global__ void __launch_bounds__(256) encode_weight_kernel(const __nv_bfloat16* __restrict__ B, int64_t ldb, int N,
                                                            int K, int bd, __nv_bfloat16* __restrict__ out,
                                                            int64_t b_stride, int64_t out_stride) {
  __shared__ float red[3][32][65];
  B += static_cast<int64_t>(blockIdx.z) * b_stride;
  out += static_cast<int64_t>(blockIdx.z) * out_stride;
  const int kb = blockIdx.x, nt = blockIdx.y, t = threadIdx.x;
  float a1, a2, a3;
  kblock_checksums(B, ldb, N, K, bd, nt, kb, red, a1, a2, a3);
  const int col = kb * 64 + t;
  if (t < 64 && col < K) write_checksum_rows(a1, a2, a3, out + static_cast<int64_t>(nt) * 8 * K + col, K);
}

// fp16 checksum block of a large weight, in two launches after the table
// is zeroed: encode_f16_sums_kernel (one k-block of one tile per CTA) keeps
// the sums in the rows' own bytes and raises the tile's maxima with an
// atomic max on the bit patterns of non-negative floats (NaN sums passed
// over); encode_f16_finish_kernel writes the scaled rows and the factors.
__global__ void __launch_bounds__(256) encode_f16_sums_kernel(const __half* __restrict__ B, int64_t ldb, int N, int K,
                                                              int bd, __half* __restrict__ out, int64_t b_stride,
                                                              int64_t out_stride, float* __restrict__ table,
                                                              int64_t table_stride) {
  __shared__ float red[3][32][65];
  B += static_cast<int64_t>(blockIdx.z) * b_stride;
  out += static_cast<int64_t>(blockIdx.z) * out_stride;
  const int kb = blockIdx.x, nt = blockIdx.y, t = threadIdx.x;
  float a1, a2, a3;
  kblock_checksums(B, ldb, N, K, bd, nt, kb, red, a1, a2, a3);
  if (t >= 64) return;  // whole warps
  const int c = min(64, K - kb * 64);
  float m1 = 0.f, m2 = 0.f, m3 = 0.f;
  if (t < c) {
    __half* const rows_tile = out + static_cast<int64_t>(nt) * 8 * K;
    *f16_stage_slot(rows_tile, K, kb, c, 0, t) = a1;
    *f16_stage_slot(rows_tile, K, kb, c, 1, t) = a2;
    *f16_stage_slot(rows_tile, K, kb, c, 2, t) = a3;
    m1 = fmaxf(m1, fabsf(a1));
    m2 = fmaxf(m2, fabsf(a2));
    m3 = fmaxf(m3, fabsf(a3));
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, d));
    m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, d));
    m3 = fmaxf(m3, __shfl_xor_sync(0xffffffffu, m3, d));
  }
  if ((t & 31) == 0) {
    float* const tb = table + static_cast<int64_t>(blockIdx.z) * table_stride + static_cast<int64_t>(nt) * 8;
    atomicMax(reinterpret_cast<unsigned int*>(tb + 0), __float_as_uint(m1));
    atomicMax(reinterpret_cast<unsigned int*>(tb + 1), __float_as_uint(m2));
    atomicMax(reinterpret_cast<unsigned int*>(tb + 2), __float_as_uint(m3));
  }
}

// Per (k-block, tile, batch), 64 threads: read the k-block's staged sums,
// then write the scaled fp16 rows over them; the first k-block also writes
// the tile's factors 2^e into the table.
__global__ void __launch_bounds__(64) encode_f16_finish_kernel(__half* __restrict__ out, int K, int64_t out_stride,
                                                              float* __restrict__ table, int64_t table_stride) {
  const int kb = blockIdx.x, nt = blockIdx.y, t = threadIdx.x;
  out += static_cast<int64_t>(blockIdx.z) * out_stride;
  float* const tb = table + static_cast<int64_t>(blockIdx.z) * table_stride + static_cast<int64_t>(nt) * 8;
  __half* const rows_tile = out + static_cast<int64_t>(nt) * 8 * K;
  const int c = min(64, K - kb * 64);
  float a1 = 0.f, a2 = 0.f, a3 = 0.f;
  if (t < c) {
    a1 = *f16_stage_slot(rows_tile, K, kb, c, 0, t);
    a2 = *f16_stage_slot(rows_tile, K, kb, c, 1, t);
    a3 = *f16_stage_slot(rows_tile, K, kb, c, 2, t);
  }
  __syncthreads();  // every staged sum read before any row overwrites it
  const int e1 = f16_chk_exponent(__float_as_uint(tb[0]));
  const int e2 = f16_chk_exponent(__float_as_uint(tb[1]));
  const int e3 = f16_chk_exponent(__float_as_uint(tb[2]));
  if (kb == 0 && t == 0) {
    tb[4] = pow2f_exact(e1);
    tb[5] = pow2f_exact(e2);
    tb[6] = pow2f_exact(e3);
  }
  if (t < c)
    write_checksum_rows_f16(a1 * pow2f_exact(-e1), a2 * pow2f_exact(-e2), a3 * pow2f_exact(-e3),
                            rows_tile + kb * 64 + t, K);
}

// fp16 checksum block in one launch (small encodes, e.g. the tokens of a
// decode step, where launches and host calls cost more than the bytes):
// the kEncCluster CTAs of a cluster
// share one tile of one batch (grid (tiles * kEncCluster, batch)). CTA r
// forms the sums of k-blocks r, r + kEncCluster, ... and keeps them in the
// rows' own bytes (f16_stage_slot) with their largest magnitudes; the
// cluster then combines those maxima through distributed shared memory,
// and each CTA writes the scaled rows of its k-blocks. CTA 0 writes the
// tile's table entries. Both cluster barriers are reached by every thread.
constexpr int kEncCluster = 8;

__global__ void __launch_bounds__(256) encode_f16_cluster_kernel(const __half* __restrict__ B, int64_t ldb, int N,
                                                                 int K, int bd, __half* __restrict__ out,
                                                                 int64_t b_stride, int64_t out_stride,
                                                                 float* __restrict__ table, int64_t table_stride) {
  __shared__ float red[3][32][65];
  __shared__ float wmax[2][3];
  __shared__ float cmax[3];
  const int rank = static_cast<int>(cluster_ctarank());
  const int nt = static_cast<int>(blockIdx.x) / kEncCluster;
  B += static_cast<int64_t>(blockIdx.y) * b_stride;
  out += static_cast<int64_t>(blockIdx.y) * out_stride;
  const int t = threadIdx.x;
  const int num_kb = (K + 63) / 64;
  __half* const rows_tile = out + static_cast<int64_t>(nt) * 8 * K;
  float m1 = 0.f, m2 = 0.f, m3 = 0.f;
  for (int kb = rank; kb < num_kb; kb += kEncCluster) {
    float a1, a2, a3;
    kblock_checksums(B, ldb, N, K, bd, nt, kb, red, a1, a2, a3);
    const int c = min(64, K - kb * 64);
    if (t < c) {
      *f16_stage_slot(rows_tile, K, kb, c, 0, t) = a1;
      *f16_stage_slot(rows_tile, K, kb, c, 1, t) = a2;
      *f16_stage_slot(rows_tile, K, kb, c, 2, t) = a3;
      m1 = fmaxf(m1, fabsf(a1));
      m2 = fmaxf(m2, fabsf(a2));
      m3 = fmaxf(m3, fabsf(a3));
    }
  }
  if (t < 64) {
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
      m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, d));
      m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, d));
      m3 = fmaxf(m3, __shfl_xor_sync(0xffffffffu, m3, d));
    }
    if ((t & 31) == 0) {
      wmax[t >> 5][0] = m1;
      wmax[t >> 5][1] = m2;
      wmax[t >> 5][2] = m3;
    }
  }
  __syncthreads();
  if (t < 3) cmax[t] = fmaxf(wmax[0][t], wmax[1][t]);
  cluster_sync_all();  // every CTA's maxima are in its shared memory
  float g[3] = {0.f, 0.f, 0.f};
#pragma unroll
  for (int q = 0; q < 3; ++q)
    for (int r = 0; r < kEncCluster; ++r)
      g[q] = fmaxf(g[q], ld_shared_cluster_f32(mapa_shared(smem_u32(&cmax[q]), static_cast<uint32_t>(r))));
  cluster_sync_all();  // no CTA leaves while another still reads its maxima
  const int e1 = f16_chk_exponent(__float_as_uint(g[0]));
  const int e2 = f16_chk_exponent(__float_as_uint(g[1]));
  const int e3 = f16_chk_exponent(__float_as_uint(g[2]));
  if (rank == 0 && t < 8) {
    float* const tb = table + static_cast<int64_t>(blockIdx.y) * table_stride + static_cast<int64_t>(nt) * 8;
    const float v[8] = {g[0], g[1], g[2], 0.f, pow2f_exact(e1), pow2f_exact(e2), pow2f_exact(e3), 0.f};
    float x = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) x = (i == t) ? v[i] : x;
    tb[t] = x;
  }
  const float f1 = pow2f_exact(-e1), f2 = pow2f_exact(-e2), f3 = pow2f_exact(-e3);
  for (int kb = rank; kb < num_kb; kb += kEncCluster) {
    const int c = min(64, K - kb * 64);
    float a1 = 0.f, a2 = 0.f, a3 = 0.f;
    if (t < c) {
      a1 = *f16_stage_slot(rows_tile, K, kb, c, 0, t);
      a2 = *f16_stage_slot(rows_tile, K, kb, c, 1, t);
      a3 = *f16_stage_slot(rows_tile, K, kb, c, 2, t);
    }
    __syncthreads();  // every staged sum of this k-block read before any row overwrites it
    if (t < c) write_checksum_rows_f16(a1 * f1, a2 * f2, a3 * f3, rows_tile + kb * 64 + t, K);
  }
}

// fp16 checksum block of a tile of at most 32 rows (the tokens of a decode
// step), in one launch: a cluster of kEncCluster CTAs per tile and batch,
// thread t of CTA r owning the 8-column chunks r * 256 + t + i * 2048
// (i < kFewRowsChunks). A thread adds its chunk's rows in order, from +0,
// with all of their loads in flight, and keeps the sums in registers while
// the cluster agrees on the tile's scales. With 32 rows or fewer every row
// is its own group in kblock_checksums' order and the groups past the last
// row add +0 to a sum that cannot be -0, so the sums are bit-identical.
// Requires N - nt * bd <= 32 for every tile and K <= kFewRowsMaxK.
constexpr int kFewRowsChunks = 2;
constexpr int kFewRowsMaxK = kEncCluster * 256 * 8 * kFewRowsChunks;

__global__ void __launch_bounds__(256) encode_f16_few_rows_kernel(const __half* __restrict__ B, int64_t ldb, int N,
                                                                  int K, int bd, __half* __restrict__ out,
                                                                  int64_t b_stride, int64_t out_stride,
                                                                  float* __restrict__ table, int64_t table_stride) {
  __shared__ float wmax[8][3];
  __shared__ float cmax[3];
  const int rank = static_cast<int>(cluster_ctarank());
  const int nt = static_cast<int>(blockIdx.x) / kEncCluster;
  B += static_cast<int64_t>(blockIdx.y) * b_stride + static_cast<int64_t>(nt) * bd * ldb;
  out += static_cast<int64_t>(blockIdx.y) * out_stride;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int nrows = min(bd, N - nt * bd);
  const int nchunks = K / 8;
  float a1[kFewRowsChunks][8], a2[kFewRowsChunks][8], a3[kFewRowsChunks][8];
  float m1 = 0.f, m2 = 0.f, m3 = 0.f;
#pragma unroll
  for (int i = 0; i < kFewRowsChunks; ++i) {
#pragma unroll
    for (int e = 0; e < 8; ++e) a1[i][e] = a2[i][e] = a3[i][e] = 0.f;
    const int c = rank * 256 + t + i * kEncCluster * 256;
    if (c < nchunks) {
      const __half* col = B + static_cast<int64_t>(c) * 8;
      for (int j0 = 0; j0 < nrows; j0 += 8) {
        uint4 w[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          w[u] = j0 + u < nrows ? __ldg(reinterpret_cast<const uint4*>(col + static_cast<int64_t>(j0 + u) * ldb))
                                : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int j = j0 + u;
          if (j >= nrows) break;
          float x[8];
          unpack8_as(w[u], x, B);
          const float wt = static_cast<float>(j + 1);
          const float sg = col_sign(j);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            a1[i][e] += x[e];
            a2[i][e] = fmaf(wt, x[e], a2[i][e]);
            a3[i][e] = fmaf(sg, x[e], a3[i][e]);
          }
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        m1 = fmaxf(m1, fabsf(a1[i][e]));
        m2 = fmaxf(m2, fabsf(a2[i][e]));
        m3 = fmaxf(m3, fabsf(a3[i][e]));
      }
    }
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, d));
    m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, d));
    m3 = fmaxf(m3, __shfl_xor_sync(0xffffffffu, m3, d));
  }
  if (lane == 0) {
    wmax[warp][0] = m1;
    wmax[warp][1] = m2;
    wmax[warp][2] = m3;
  }
  __syncthreads();
  if (t < 3) {
    float m = 0.f;
    for (int w8 = 0; w8 < 8; ++w8) m = fmaxf(m, wmax[w8][t]);
    cmax[t] = m;
  }
  cluster_sync_all();  // every CTA's maxima are in its shared memory
  float g[3] = {0.f, 0.f, 0.f};
#pragma unroll
  for (int q = 0; q < 3; ++q)
    for (int r = 0; r < kEncCluster; ++r)
      g[q] = fmaxf(g[q], ld_shared_cluster_f32(mapa_shared(smem_u32(&cmax[q]), static_cast<uint32_t>(r))));
  cluster_sync_all();  // no CTA leaves while another still reads its maxima
  const int e1 = f16_chk_exponent(__float_as_uint(g[0]));
  const int e2 = f16_chk_exponent(__float_as_uint(g[1]));
  const int e3 = f16_chk_exponent(__float_as_uint(g[2]));
  if (rank == 0 && t < 8) {
    float* const tb = table + static_cast<int64_t>(blockIdx.y) * table_stride + static_cast<int64_t>(nt) * 8;
    const float v[8] = {g[0], g[1], g[2], 0.f, pow2f_exact(e1), pow2f_exact(e2), pow2f_exact(e3), 0.f};
    float x = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) x = (i == t) ? v[i] : x;
    tb[t] = x;
  }
  const float f1 = pow2f_exact(-e1), f2 = pow2f_exact(-e2), f3 = pow2f_exact(-e3);
  __half* const rows_tile = out + static_cast<int64_t>(nt) * 8 * K;
#pragma unroll
  for (int i = 0; i < kFewRowsChunks; ++i) {
    const int c = rank * 256 + t + i * kEncCluster * 256;
    if (c >= nchunks) continue;
    __half h[8][8];  // [checksum row][column]
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      split3_f16(a1[i][e] * f1, h[0][e], h[1][e], h[2][e]);
      split3_f16(a2[i][e] * f2, h[3][e], h[4][e], h[5][e]);
      const float x3 = a3[i][e] * f3;
      h[6][e] = __float2half_rn(x3);
      h[7][e] = __float2half_rn(x3 - __half2float(h[6][e]));
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      uint32_t wd[4];
#pragma unroll
      for (int p2 = 0; p2 < 4; ++p2)
        wd[p2] = static_cast<uint32_t>(__half_as_ushort(h[q][2 * p2])) |
                 (static_cast<uint32_t>(__half_as_ushort(h[q][2 * p2 + 1])) << 16);
      *reinterpret_cast<uint4*>(rows_tile + static_cast<int64_t>(q) * K + static_cast<int64_t>(c) * 8) =
          make_uint4(wd[0], wd[1], wd[2], wd[3]);
    }
  }
}

// K-major copy of an N-major right operand plus (out != nullptr) its
// checksum block: per batch z, Bkn[k * ldb + n] (K rows of N columns) is
// written to Bt[n * K + k] (N rows of K, at z * N * K) and the checksum rows
// of tile nt (columns [nt*bd, nt*bd + bd) of Bkn, the same sums as
// encode_weight_kernel over the copy) to out + z * out_stride.
// One block moves a 64 (k) x bd (n) slab through shared memory: coalesced
// 16-byte reads along n, coalesced 128-byte row pieces along k on the way
// out. The slab is stored as 16-byte chunks, chunk c of k row kk at
// position c ^ tr_swz(kk), so that the column reads (8 k rows, one n) and
// the checksum row reads (8 k rows, one chunk) each hit 8 distinct chunks.
// grid (ceil(K/64), ceil(N/bd), batch), 256 threads; N % 8 == 0,
// K % 8 == 0, ldb % 8 == 0, bd <= 256 and a multiple of 8.
__device__ __forceinline__ int tr_swz(int kk) { return (kk ^ (kk >> 3)) & 7; }
__device__ __forceinline__ int tr_off(int kk, int c) { return kk * 256 + ((c ^ tr_swz(kk)) << 3); }

__global__ void __launch_bounds__(256) transpose_encode_kernel(const __nv_bfloat16* __restrict__ Bkn, int64_t ldb,
                                                               int64_t b_stride, int N, int K, int bd,
                                                               __nv_bfloat16* __restrict__ Bt,
                                                               __nv_bfloat16* __restrict__ out, int64_t out_stride) {
  __shared__ __align__(16) __nv_bfloat16 tile[64 * 256];
  __shared__ float red[3][4][64];
  const int z = blockIdx.z;
  Bkn += static_cast<int64_t>(z) * b_stride;
  Bt += static_cast<int64_t>(z) * N * K;
  const int k0 = blockIdx.x * 64, n0 = blockIdx.y * bd;
  const int nv = min(bd, N - n0);  // valid columns of the slab, a multiple of 8
  const int nc8 = bd / 8;
  const int t = threadIdx.x;
  for (int i = t; i < 64 * nc8; i += 256) {
    const int kk = i / nc8, c = i - kk * nc8;
    uint4 w = make_uint4(0u, 0u, 0u, 0u);
    if (k0 + kk < K && c * 8 < nv)
      w = __ldg(reinterpret_cast<const uint4*>(Bkn + static_cast<int64_t>(k0 + kk) * ldb + n0 + c * 8));
    *reinterpret_cast<uint4*>(tile + tr_off(kk, c)) = w;
  }
  __syncthreads();
  // rows n of the copy: 8 consecutive k per thread, one 16-byte store
  for (int i = t; i < nv * 8; i += 256) {
    const int n = i >> 3, kc = (i & 7) * 8;
    if (k0 + kc >= K) continue;
    uint32_t wd[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t lo = __bfloat16_as_ushort(tile[tr_off(kc + 2 * e, n >> 3) + (n & 7)]);
      const uint32_t hi = __bfloat16_as_ushort(tile[tr_off(kc + 2 * e + 1, n >> 3) + (n & 7)]);
      wd[e] = lo | (hi << 16);
    }
    *reinterpret_cast<uint4*>(Bt + static_cast<int64_t>(n0 + n) * K + k0 + kc) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
  }
  if (out == nullptr) return;
  // checksums: thread (k row kk, group g) sums the chunks c = g, g+4, ...
  // (columns j ascending within each), then the 4 groups are added in order
  const int kk = t & 63, g = t >> 6;
  float s1 = 0.f, s2 = 0.f, s3 = 0.f;
  for (int c = g; c * 8 < nv; c += 4) {
    float x[8];
    unpack8(*reinterpret_cast<const uint4*>(tile + tr_off(kk, c)), x);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int j = c * 8 + e;
      s1 += x[e];
      s2 = fmaf(static_cast<float>(j + 1), x[e], s2);
      s3 = fmaf(col_sign(j), x[e], s3);
    }
  }
  red[0][g][kk] = s1;
  red[1][g][kk] = s2;
  red[2][g][kk] = s3;
  __syncthreads();
  if (t < 64 && k0 + t < K) {
    const float a1 = (red[0][0][t] + red[0][1][t]) + (red[0][2][t] + red[0][3][t]);
    const float a2 = (red[1][0][t] + red[1][1][t]) + (red[1][2][t] + red[1][3][t]);
    const float a3 = (red[2][0][t] + red[2][1][t]) + (red[2][2][t] + red[2][3][t]);
    write_checksum_rows(a1, a2, a3,
                        out + static_cast<int64_t>(z) * out_stride + static_cast<int64_t>(blockIdx.y) * 8 * K + k0 + t,
                        K);
  }
}

// grid (ceil(Cc/64), nrb), 256 threads. Cc % 8 == 0.
// out_sum[rb*Cc + c] = sum_{r in block rb} w[r] * X[r, c]   (w == nullptr: 1)
// with stats (out_stat != nullptr): out_stat[rb*Cc + c] = max |X[r, c]| and
// out_stat[(nrb + rb)*Cc + c] = sum |X[r, c]|.
template <typename T>
__global__ void __launch_bounds__(256) colsum_partial_kernel(const T* __restrict__ X, int64_t ld, int R,
                                                             int Cc, int rows_per_block, const float* __restrict__ w,
                                                             float* __restrict__ out_sum, float* __restrict__ out_stat) {
  __shared__ float red[3][32][65];
  const int cb = blockIdx.x, rb = blockIdx.y, nrb = gridDim.y;
  const int t = threadIdx.x, c8 = t & 7, rg = t >> 3;
  const int col0 = cb * 64 + c8 * 8;
  const int r0 = rb * rows_per_block;
  const int r1 = min(R, r0 + rows_per_block);
  float s[8], m[8], a[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) s[e] = m[e] = a[e] = 0.f;
  if (col0 < Cc) {
    for (int r = r0 + rg; r < r1; r += 32) {
      float x[8];
      load8(X + static_cast<int64_t>(r) * ld + col0, x);
      const float wr = (w != nullptr) ? __ldg(w + r) : 1.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        s[e] = fmaf(wr, x[e], s[e]);
        m[e] = fmaxf(m[e], fabsf(x[e]));
        a[e] += fabsf(x[e]);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    red[0][rg][c8 * 8 + e] = s[e];
    red[1][rg][c8 * 8 + e] = m[e];
    red[2][rg][c8 * 8 + e] = a[e];
  }
  __syncthreads();
  if (t < 64) {
    const int col = cb * 64 + t;
    if (col < Cc) {
      float acc = 0.f, mx = 0.f, ab = 0.f;
      for (int g = 0; g < 32; ++g) {
        acc += red[0][g][t];
        mx = fmaxf(mx, red[1][g][t]);
        ab += red[2][g][t];
      }
      out_sum[static_cast<int64_t>(rb) * Cc + col] = acc;
      if (out_stat != nullptr) {
        out_stat[static_cast<int64_t>(rb) * Cc + col] = mx;
        out_stat[static_cast<int64_t>(nrb + rb) * Cc + col] = ab;
      }
    }
  }
}

// out[c] = sum_rb in[rb*n + c]; with stats also out_max[c] = max_rb and
// out_abs[c] = sum_rb of the two stat planes that follow in[] (see above).
__global__ void __launch_bounds__(256) reduce_partials_kernel(const float* __restrict__ in, const float* __restrict__ in_stat,
                                                              int nrb, int n, float* __restrict__ out,
                                                              float* __restrict__ out_max, float* __restrict__ out_abs) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n) return;
  float acc = 0.f, mx = 0.f, ab = 0.f;
  for (int rb = 0; rb < nrb; ++rb) {
    acc += in[static_cast<int64_t>(rb) * n + c];
    if (in_stat != nullptr) {
      mx = fmaxf(mx, in_stat[static_cast<int64_t>(rb) * n + c]);
      ab += in_stat[static_cast<int64_t>(nrb + rb) * n + c];
    }
  }
  out[c] = acc;
  if (in_stat != nullptr) {
    out_max[c] = mx;
    out_abs[c] = ab;
  }
}

// Warp per row: out[r] = sum_c X[r,c] * (vec ? vec[c] : 1); with stats
// out_max[r] = max_c |X[r,c]| and out_abs[r] = sum_c |X[r,c]|.
// 256 threads (8 rows) per block. Cc % 8 == 0, vec 16-byte aligned.
template <typename T>
__global__ void __launch_bounds__(256) rowdot_kernel(const T* __restrict__ X, int64_t ld, int R, int Cc,
                                                     const float* __restrict__ vec, float* __restrict__ out,
                                                     float* __restrict__ out_max, float* __restrict__ out_abs) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + warp;
  if (r >= R) return;
  const T* row = X + static_cast<int64_t>(r) * ld;
  float acc = 0.f, mx = 0.f, ab = 0.f;
  for (int c = lane * 8; c < Cc; c += 256) {
    float x[8];
    load8(row + c, x);
    if (vec != nullptr) {
      const float4 va = __ldg(reinterpret_cast<const float4*>(vec + c));
      const float4 vb = __ldg(reinterpret_cast<const float4*>(vec + c + 4));
      acc = fmaf(x[0], va.x, acc);
      acc = fmaf(x[1], va.y, acc);
      acc = fmaf(x[2], va.z, acc);
      acc = fmaf(x[3], va.w, acc);
      acc = fmaf(x[4], vb.x, acc);
      acc = fmaf(x[5], vb.y, acc);
      acc = fmaf(x[6], vb.z, acc);
      acc = fmaf(x[7], vb.w, acc);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) acc += x[e];
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      mx = fmaxf(mx, fabsf(x[e]));
      ab += fabsf(x[e]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
    mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    ab += __shfl_xor_sync(0xFFFFFFFFu, ab, o);
  }
  if (lane == 0) {
    out[r] = acc;
    if (out_max != nullptr) out_max[r] = mx;
    if (out_abs != nullptr) out_abs[r] = ab;
  }
}

// Fixed-order block sum over 1024 threads.
__device__ __forceinline__ float block_sum_1024(float v, float* scratch /*32*/) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float r = 0.f;
  if (warp == 0) {
    r = scratch[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xFFFFFFFFu, r, o);
  }
  __syncthreads();
  if (threadIdx.x == 0) scratch[0] = r;
  __syncthreads();
  return scratch[0];
}

// One block of 1024 threads. Follows pytorch/abft/checkers.py:112-126
// (corner = dot(s_a, s_b) + m * sum(bias), sum_c = sum(C)) and :96-110
// (diff, rel = diff / max(|sum_c|, 1), ok = diff <= tol_abs or rel <= tol_rel).
// With native_sums every intermediate is rounded to the operands' type T,
// as the python backend's tensors of that type are (s_a, s_b, dot, bias
// sum, m * bias sum, corner, sum_c, diff, rel), and the tolerances are
// compared as values of type T (for fp32 operands nothing changes).
template <typename T>
__global__ void __launch_bounds__(1024) ref_finalize_kernel(const float* __restrict__ u, const float* __restrict__ v,
                                                            int K, const T* __restrict__ bias, int N,
                                                            int M, const float* __restrict__ parts, int n_parts,
                                                            float tol_abs, float tol_rel, int native_sums,
                                                            abft_report* rep, int capacity, int tile_m, int tile_n) {
  __shared__ float scratch[32];
  auto rn = [&](float x) { return native_sums ? round_to<T>(x) : x; };
  float c = 0.f;
  for (int k = threadIdx.x; k < K; k += 1024) c = fmaf(rn(u[k]), rn(v[k]), c);
  float corner = rn(block_sum_1024(c, scratch));
  if (bias != nullptr) {
    float b = 0.f;
    for (int j = threadIdx.x; j < N; j += 1024) b += to_f32(bias[j]);
    const float bs = rn(block_sum_1024(b, scratch));
    if (native_sums)
      corner = rn(corner + rn(static_cast<float>(M) * bs));
    else
      corner += static_cast<float>(M) * bs;
  }
  float s = 0.f;
  for (int i = threadIdx.x; i < n_parts; i += 1024) s += parts[i];
  const float sum_c = rn(block_sum_1024(s, scratch));
  if (threadIdx.x == 0) {
    float diff = fabsf(corner - sum_c);
    float rel = diff / fmaxf(fabsf(sum_c), 1.f);
    float ta = tol_abs, tr = tol_rel;
    if (native_sums) {
      diff = rn(diff);
      rel = rn(diff / fmaxf(fabsf(sum_c), 1.f));
      ta = rn(tol_abs);
      tr = rn(tol_rel);
    }
    const bool ok = (diff <= ta) || (rel <= tr);
    rep->corner = corner;
    rep->sum_c = sum_c;
    rep->abs_err = diff;
    rep->rel_err = rel;
    rep->ref_ok = ok ? 1 : 0;
    rep->capacity = static_cast<uint32_t>(capacity);
    rep->tile_m = static_cast<uint32_t>(tile_m);
    rep->tile_n = static_cast<uint32_t>(tile_n);
    if (!ok) atomicOr(&rep->status, ABFT_STATUS_REF_FAIL);
  }
}

// One block of 1024 threads: global row and column mismatch search of a
// post-hoc check, then pairing of mismatching rows with mismatching columns
// of matching residual (a single fault at (i, j) shifts row sum i and column
// sum j by the same delta). The stored C is rounded to its output dtype, so
// each bound adds the worst-case rounding of the summed elements:
//   row i:  thr = thr_k * max_j |C[i,j]| + unit_out * sum_j |C[i,j]|
//   col j:  thr = thr_k * max_i |C[i,j]| + unit_out * sum_i |C[i,j]|
// with thr_k = tau * sqrt(K) and unit_out the relative rounding bound of
// the type (2^-9 bf16, 2^-12 fp16, 2^-25 fp32).
constexpr int kLocateMax = 256;
template <typename T>
__global__ void __launch_bounds__(1024) locate_finalize_kernel(
    const float* __restrict__ row_sum, const float* __restrict__ row_max, const float* __restrict__ row_abs,
    const float* __restrict__ row_exp, int M, const float* __restrict__ col_sum, const float* __restrict__ col_max,
    const float* __restrict__ col_abs, const float* __restrict__ col_exp, int N, const T* __restrict__ bias,
    float thr_k, float unit_out, abft_report* rep, int capacity) {
  __shared__ int rows[kLocateMax], cols[kLocateMax];
  __shared__ float rres[kLocateMax], cres[kLocateMax], rthr[kLocateMax], cthr[kLocateMax];
  __shared__ float scratch[32];
  __shared__ int nr, nc, dropped;
  // bias enters every row sum once and every column sum M times (checkers.py:120-124)
  float bsum = 0.f;
  if (bias != nullptr) {
    float b = 0.f;
    for (int j = threadIdx.x; j < N; j += 1024) b += to_f32(bias[j]);
    bsum = block_sum_1024(b, scratch);
  }
  if (threadIdx.x == 0) nr = nc = dropped = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < M; i += 1024) {
    const float res = row_sum[i] - (row_exp[i] + bsum);
    const float thr = fmaf(thr_k, row_max[i], unit_out * row_abs[i]);
    if (fabsf(res) > thr) {
      const int s = atomicAdd(&nr, 1);
      if (s < kLocateMax) {
        rows[s] = i;
        rres[s] = res;
        rthr[s] = thr;
      } else {
        atomicAdd(&dropped, 1);
      }
    }
  }
  for (int j = threadIdx.x; j < N; j += 1024) {
    const float bj = bias != nullptr ? static_cast<float>(M) * to_f32(bias[j]) : 0.f;
    const float res = col_sum[j] - (col_exp[j] + bj);
    const float thr = fmaf(thr_k, col_max[j], unit_out * col_abs[j]);
    if (fabsf(res) > thr) {
      const int s = atomicAdd(&nc, 1);
      if (s < kLocateMax) {
        cols[s] = j;
        cres[s] = res;
        cthr[s] = thr;
      } else {
        atomicAdd(&dropped, 1);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  const int n_r = min(nr, kLocateMax), n_c = min(nc, kLocateMax);
  // Deterministic order: insertion sort by index.
  for (int a = 1; a < n_r; ++a)
    for (int b = a; b > 0 && rows[b] < rows[b - 1]; --b) {
      int ti = rows[b]; rows[b] = rows[b - 1]; rows[b - 1] = ti;
      float tf = rres[b]; rres[b] = rres[b - 1]; rres[b - 1] = tf;
      tf = rthr[b]; rthr[b] = rthr[b - 1]; rthr[b - 1] = tf;
    }
  for (int a = 1; a < n_c; ++a)
    for (int b = a; b > 0 && cols[b] < cols[b - 1]; --b) {
      int ti = cols[b]; cols[b] = cols[b - 1]; cols[b - 1] = ti;
      float tf = cres[b]; cres[b] = cres[b - 1]; cres[b - 1] = tf;
      tf = cthr[b]; cthr[b] = cthr[b - 1]; cthr[b - 1] = tf;
    }
  uint32_t used_c[kLocateMax / 32];
  for (int w = 0; w < kLocateMax / 32; ++w) used_c[w] = 0u;
  abft_fault_record* recs = reinterpret_cast<abft_fault_record*>(rep + 1);
  uint32_t n_out = 0, n_loc = 0, status = 0;
  auto emit = [&](int row, int col, float res, float resw, float thr, uint32_t flags) {
    if (n_out < static_cast<uint32_t>(capacity)) {
      recs[n_out].row = row;
      recs[n_out].col = col;
      recs[n_out].residual = res;
      recs[n_out].residual_w = resw;
      recs[n_out].threshold = thr;
      recs[n_out].flags = flags;
    } else {
      status |= ABFT_STATUS_OVERFLOW;
      rep->overflow += 1u;
    }
    ++n_out;
  };
  for (int a = 0; a < n_r; ++a) {
    // the unique unused column whose residual matches within both thresholds
    int match = -1, count = 0;
    for (int b = 0; b < n_c; ++b) {
      if (used_c[b >> 5] & (1u << (b & 31))) continue;
      if (fabsf(rres[a] - cres[b]) <= rthr[a] + cthr[b]) {
        if (count == 0) match = b;
        ++count;
      }
    }
    if (count == 1) {
      used_c[match >> 5] |= 1u << (match & 31);
      emit(rows[a], cols[match], rres[a], cres[match], rthr[a], ABFT_REC_DETECTED | ABFT_REC_LOCATED);
      ++n_loc;
    } else {
      emit(rows[a], -1, rres[a], 0.f, rthr[a], ABFT_REC_DETECTED);
      status |= ABFT_STATUS_UNLOCATED;
    }
  }
  for (int b = 0; b < n_c; ++b) {
    if (used_c[b >> 5] & (1u << (b & 31))) continue;
    emit(-1, cols[b], cres[b], 0.f, cthr[b], ABFT_REC_DETECTED);
    status |= ABFT_STATUS_UNLOCATED;
  }
  if (dropped > 0) status |= ABFT_STATUS_OVERFLOW | ABFT_STATUS_UNLOCATED;
  if (n_out > 0 || dropped > 0) status |= ABFT_STATUS_FAULT;
  rep->n_faults = n_out + static_cast<uint32_t>(dropped);
  rep->n_located = n_loc;
  rep->overflow += static_cast<uint32_t>(dropped);
  rep->status |= status;
}

}  // namespace abft
