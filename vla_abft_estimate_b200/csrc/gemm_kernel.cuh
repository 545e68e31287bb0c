// gemm_kernel.cuh - fused checksum-protected bf16 / fp16 GEMM for sm_100a.
//
//   C[M, N] = A[M, K] * B[N, K]^T (+ bias)      (B = nn.Linear weight layout)
//
// or a batch of such products C[b] = A[b] B[b]^T in one launch (torch.bmm):
// every tensor map has the batch as its outermost coordinate and the tiles
// of all batches form one schedule.
//
// One persistent CTA per SM walks output tiles. Warp roles:
//   warp 0      TMA producer: per 64-wide k-block the A tile (128 rows) and
//               the B-operand tile (BN rows) into a STAGES-deep shared-memory
//               ring. With checks on, the B-operand tile is B's rows
//               [t*BD, t*BD + BD) (BD = BN - 8 data columns per tile) followed
//               by the tile's 8-row checksum block: B augmented with its row
//               checksums, one TMA box each.
//   warp 1      TMEM allocator and single-thread tcgen05.mma issuer: one
//               M=128 N=BN MMA per 16-wide k step. With checks on its last 8
//               accumulator columns are the expected checksums, formed by the
//               same instruction that forms the output (no second pass over
//               the A tile). Two BN-column accumulators: the epilogue of tile
//               t overlaps the main loop of tile t+1.
//   warps 14-15 with swapped operands, checks on and at most 64 tokens: per
//               k-block, the 8 token checksum rows of the B-operand tile,
//               summed in shared memory from the token rows the TMA just
//               loaded (no encode launch, no checksum copy).
//   warps 2-13  epilogue: warp w owns TMEM lane quadrant (w % 4), i.e. 32
//               output rows, and every third 32-column chunk of the tile
//               (from chunk (w - 2) / 4). Each thread streams its chunks from
//               TMEM once: row checksums, bias, rounding to the element
//               type and the store;
//               the three partial checksums of a row are then combined, the
//               row checked and a located fault corrected.
//
// Checksum algebra (extends the scalar corner check of
// pytorch/abft/checkers.py:112-126, dot(sum_rows(A), sum_cols(B)) vs sum(C),
// to one pair of checks per output row and tile): for row i of tile (mt, nt),
// j over the tile's valid data columns (local index),
//   expected  e1 = A[i,:] . v1,   v1[k] = sum_j        B[j,k]
//             e2 = A[i,:] . v2,   v2[k] = sum_j (j+1)  B[j,k]
//   actual    s1 = sum_j C[i,j],  s2 = sum_j (j+1) C[i,j]       (fp32 accumulator)
// and a third pair with column signs sg(j) = +-1 (Thue-Morse parity of j):
//   e3 = A[i,:] . v3,   v3[k] = sum_j sg(j) B[j,k];   s3 = sum_j sg(j) C[i,j]
// The checksum block holds v1 and v2 each split into three terms of the
// operands' type (hi + mid + lo: 24 significant bits in bf16; in fp16, whose
// range is narrow, each checksum of a tile is first scaled by a power of
// two that the epilogue multiplies back) and v3 in two. A single corrupted
// C[i,j*] (+delta) gives s1 - e1 = delta, s2 - e2 = (j*+1) delta and
// s3 - e3 = sg(j*) delta: the ratio of the first two pins the column, the
// third must agree with it (several faults in one row segment whose
// weighted mean column is an integer are rejected this way), and delta is
// subtracted before the store.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../include/abft_b200.h"
#include "aux_kernels.cuh"
#include "ptx.cuh"

namespace abft {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kEpiWarp0 = 2;  // warps 0 and 1: TMA producer, MMA issuer
// Epilogue: kEpiSplit warps per TMEM lane quadrant, so three per scheduler;
// warp (quadrant q, share t) owns the tile's 32-column chunks t, t + 3, ...
constexpr int kEpiSplit = 3;
constexpr int kEpiWarps = 4 * kEpiSplit;
constexpr int kEpiThreads = 32 * kEpiWarps;
// With swapped operands and checks on: the two warps that form each
// stage's token checksum rows in shared memory (idle otherwise).
constexpr int kBuildWarp = kEpiWarp0 + kEpiWarps;
constexpr int kBuildWarps = 2;
constexpr int kThreads = 32 * (kBuildWarp + kBuildWarps);
constexpr int kChkRows = 8;  // rows of the per-tile checksum block

// PAIR: a 2-CTA cluster shares one 256 x BN output tile. Each CTA holds 128
// rows of A and BN/2 rows of the B-operand tile per stage; one pair MMA
// (M = 256) issued by the even CTA reads both CTAs' halves and accumulates
// each CTA's 128 rows into that CTA's own TMEM.
template <int BN, bool CHECK, bool PAIR = false>
struct GemmCfg {
  static_assert(BN == 128 || BN == 256, "tile widths");
  // Stage = 16 KB of A + this CTA's B rows: 32 KB (pair of 256-wide tiles,
  // single 128-wide), 48 KB (single 256-wide), 24 KB (pair of 128-wide).
  static constexpr int kStages = PAIR ? ((BN == 256) ? 6 : 8) : ((BN == 256) ? 4 : 6);
  static constexpr int kBD = CHECK ? BN - kChkRows : BN;  // data columns per tile
  static constexpr int kTileM = PAIR ? 2 * kBM : kBM;    // output rows per tile
  static constexpr int kBRows = PAIR ? BN / 2 : BN;      // B-operand rows this CTA stages
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = kBRows * kBK * 2;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + kStages * kABytes;
  static constexpr int kOffX = kOffB + kStages * kBBytes;  // row-partial exchange
  static constexpr int kXBytes = kEpiSplit * kBM * 16;     // [share][row] float4, one tile at a time
  // Per epilogue warp, one 32-row x 32-column bf16 block of the output on
  // its way to global memory (rows transposed across lanes so that a warp
  // store covers 8 rows x 64 contiguous bytes).
  static constexpr int kStageBytes = 32 * 32 * 2;
  static constexpr int kOffStage = kOffX + (CHECK ? kXBytes : 0);
  static constexpr int kOffBar = kOffStage + kEpiWarps * kStageBytes;
  static constexpr int kNumBars = 3 * kStages + 2 * 2 + 3;  // full, empty, ready, tfull, tempty, xbar, xfree, drain
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 64 + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  // Row of the staged B-operand tile where the checksum block starts: after
  // all BD data rows, or, in a pair, after the odd CTA's BD - 128.
  static constexpr int kChkRow0 = PAIR ? kBD - kBRows : kBD;
  static_assert((kChkRow0 * 128) % 1024 == 0, "checksum rows must start on a swizzle atom");
};

// Division by a launch-constant d > 0 as a multiply and a shift, exact for
// every numerator below 2^31: m = floor(2^(32+l) / d) + 1 with 2^l >= d, so
// n * m / 2^(32+l) exceeds n / d by less than 1 / (2d) (Granlund-Montgomery).
struct FastDiv {
  uint64_t m;
  int s;  // 32 + l
};
__host__ __device__ __forceinline__ int fast_div(int n, const FastDiv& d) {
  return static_cast<int>((static_cast<uint64_t>(static_cast<uint32_t>(n)) * d.m) >> d.s);
}
inline FastDiv make_fast_div(int64_t d) {
  if (d < 1) d = 1;  // a divisor the kernel never uses (no tiles of that kind)
  int l = 0;
  while ((int64_t{1} << l) < d) ++l;
  FastDiv f;
  f.m = static_cast<uint64_t>((static_cast<unsigned __int128>(1) << (32 + l)) / static_cast<uint64_t>(d)) + 1;
  f.s = 32 + l;
  return f;
}

struct GemmParams {
  void* C;            // bf16 or fp16, the kernel instance's element type
  int64_t ldc;
  const void* bias;   // same type
  int M, N, K;
  int num_kb, tiles_m, tiles_n, num_tiles, group_m;
  uint32_t mode;
  float thr_k;  // thr_scale * sqrt(K)
  float thr_abs;
  const int* inj_rows;
  const int* inj_cols;
  const float* inj_deltas;
  int n_inj;
  abft_report* report;
  int capacity;
  float* tile_sumc;  // ABFT_MODE_REF: [num_tiles][kEpiWarps] partial sums of the stored outputs
  // Tile order: the full tiles [0, full_tiles) in grouped raster order over
  // tiles_n_full columns, then the tail column's tiles (one per tile row).
  int full_tiles, tiles_n_full;
  // Hybrid schedule: tiles [0, dp_tiles) are data-parallel (whole tiles,
  // unit + j*units); with sk != 0 the remaining tiles are stream-K: unit
  // c < G owns k-block iterations [c*W/G, (c+1)*W/G) of the W = sk_iters
  // that follow, G = sk_ctas <= units (fewer units, fewer pieces per tile).
  int dp_tiles;
  int sk;
  int sk_ctas;  // stream-K units: CTAs, or CTA pairs
  int64_t sk_iters;
  float* partials;  // [G][BN/4][128][4] fp32: a CTA's share of a tile it does not finish
  unsigned long long* flags;  // [G][kEpiWarps]: per epilogue warp, set to `nonce` once its share of the partial is visible
  uint64_t nonce;   // unique to this launch: stream-K flags and report->launch_tag carry it
  // Last tile column when it holds fewer than BD data columns (tail_n != 0):
  // its B-operand tile is compact (data rows, then with checks the 8
  // checksum rows) and one MMA of N = tail_n (a multiple of 16) covers it.
  int tail_n;
  int tail_box;      // rows the tail box copies into this CTA (checks: data rows, odd CTA of a pair; no checks, single CTA: tail_n), 0 = none
  uint32_t tail_tx;  // bytes one stage of a tail tile delivers (both CTAs of a pair)
  // Swapped operands (few output rows): the kernel computes C^T = W X^T, so
  // its rows are C's columns and its columns are C's rows. The output is
  // stored transposed (C[col * ldc + row]), the bias is indexed by the
  // kernel row, and fault records carry C's coordinates.
  int swap;
  // Swapped operands with checks and one compact token tile: the token
  // checksum rows of each stage are formed in shared memory by the build
  // warp (nothing is loaded for them); the MMA waits for that (ready
  // barriers) instead of for the copies alone.
  int build_chk;
  // Batched launch: `batch` products, C[b] at row b * c_rows of C (a batch
  // stride that is a whole number of ldc rows keeps the address arithmetic
  // in one 32-bit row index). Tile order:
  // the full tiles of batch 0, 1, ..., then the tail-column tiles batch by
  // batch. Fault records and injected faults use rows flattened over the
  // batch (C's row b * rows + i); bcounts ([batch][4] after the report's
  // records, or null) counts each batch's faults, located and corrected.
  int batch;
  int c_rows;
  uint32_t* bcounts;
  // fp16 checksum blocks carry a power-of-two scale per (tile, checksum):
  // float [tiles_n][8] whose entries 4..6 multiply the expected sums of v1,
  // v2, v3 (batch b at chk_scale + b * chk_scale_bstride); null for bf16.
  const float* chk_scale;
  int64_t chk_scale_bstride;
  // Divisors of tile_coords (every warp maps every tile it meets): tile
  // rows, full tiles per batch, tiles per raster group, and the height of
  // a raster group (the last group may be shorter).
  FastDiv fd_tiles_m, fd_full, fd_group, fd_gm, fd_gm_last;
};

// Walks the (tile, k-block range) segments one CTA owns. Data-parallel:
// whole tiles blockIdx.x, +gridDim.x, ...; stream-K: consecutive slices of
// the CTA's iteration range, cut at tile boundaries.
// A unit is one CTA, or one CTA pair (both CTAs walk the same segments).
struct SegmentIter {
  int64_t it, end;
  int tile_dp, stride;
  __device__ __forceinline__ SegmentIter(const GemmParams& p, int unit, int nunits) {
    tile_dp = unit;
    stride = nunits;
    const int64_t base = static_cast<int64_t>(p.dp_tiles) * p.num_kb;
    it = base + sk_begin(p, unit);
    end = base + sk_begin(p, unit + 1);
  }
  // First stream-K iteration of unit c, relative to the stream-K region
  // (units from sk_ctas on own none). Every range is non-empty: the host
  // keeps sk_ctas <= sk_iters.
  __device__ __forceinline__ static int64_t sk_begin(const GemmParams& p, int c) {
    if (c >= p.sk_ctas) return p.sk_iters;
    return (static_cast<int64_t>(c) * p.sk_iters) / p.sk_ctas;
  }
  __device__ __forceinline__ bool next(const GemmParams& p, int& tile, int& kb0, int& kb1) {
    if (tile_dp < p.dp_tiles) {
      tile = tile_dp;
      kb0 = 0;
      kb1 = p.num_kb;
      tile_dp += stride;
      return true;
    }
    if (!p.sk || it >= end) return false;
    tile = static_cast<int>(it / p.num_kb);
    kb0 = static_cast<int>(it - static_cast<int64_t>(tile) * p.num_kb);
    const int64_t left = end - it;
    kb1 = left < static_cast<int64_t>(p.num_kb - kb0) ? kb0 + static_cast<int>(left) : p.num_kb;
    it += kb1 - kb0;
    return true;
  }
};

__device__ __forceinline__ uint64_t ld_acquire_u64(const unsigned long long* f) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(f) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u64(unsigned long long* f, uint64_t v) {
  asm volatile("st.release.gpu.global.b64 [%0], %1;" ::"l"(f), "l"(v) : "memory");
}

// Bounded wait for another CTA's flag (stream-K partials) to hold this
// launch's nonce, warp-collective: lane 0 polls with back-off so that a
// waiting CTA puts a handful of requests on L2 rather than one per thread,
// then every lane re-reads the flag with acquire semantics before it
// touches the partial. All CTAs of the persistent grid are resident, and a
// CTA only waits for the first segment of higher-index CTAs, which is
// stored before they wait for anything. Flags left by earlier launches
// hold other nonces, so the workspace needs no clearing.
__device__ __forceinline__ bool wait_flag(const unsigned long long* f, uint64_t nonce, volatile int* abort_flag) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) {
    const uint64_t t0 = global_timer_ns();
    uint32_t backoff = 32;
    while (ld_acquire_u64(f) != nonce) {
      if (*abort_flag || global_timer_ns() - t0 > kWaitTimeoutNs) {
        *abort_flag = 1;
        ok = 0;
        break;
      }
      __nanosleep(backoff);
      if (backoff < 128) backoff <<= 1;
    }
  }
  ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
  if (ok) (void)ld_acquire_u64(f);
  return ok != 0;
}

// A flag no code path writes: the target of the bounded-wait self-test.
__device__ unsigned long long g_wait_selftest_flag = 0ull;

// Self-test of the bounded device waits every fused launch relies on: one
// warp waits through wait_flag (the stream-K hand-off) for a value the
// flag above never takes, then one thread through mbar_wait (the pipeline's
// barriers) for a phase of a fresh mbarrier that nothing arrives on. Each
// gives up after kWaitTimeoutNs and raises the abort flag instead of
// spinning on; the kernel then records ABFT_STATUS_DEVICE_TIMEOUT and, in
// n_faults, how many waits gave up (2 expected), and returns normally.
// One CTA of 32 threads; the host zeroes the report header first.
__global__ void __launch_bounds__(32) wait_selftest_kernel(abft_report* rep) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  const int lane = threadIdx.x;
  if (lane == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    abort_flag = 0;
  }
  __syncwarp();
  const bool flag_ok = wait_flag(&g_wait_selftest_flag, 1ull, &abort_flag);
  __syncwarp();
  if (lane == 0) {
    abort_flag = 0;  // let the second wait run to its own limit
    const bool bar_ok = mbar_wait(&bar, 0u, &abort_flag);
    const uint32_t gave_up = (flag_ok ? 0u : 1u) + (bar_ok ? 0u : 1u);
    rep->n_faults = gave_up;
    rep->status = gave_up ? ABFT_STATUS_DEVICE_TIMEOUT : 0u;
  }
}

// Bounded wait (one thread) until CTA 0 has reset the report header of this
// launch; every atomic on the report comes after it.
__device__ __forceinline__ bool report_ready(const GemmParams& p, volatile int* abort_flag) {
  const uint64_t t0 = global_timer_ns();
  while (ld_acquire_u64(reinterpret_cast<const unsigned long long*>(&p.report->launch_tag)) != p.nonce) {
    if (global_timer_ns() - t0 > kWaitTimeoutNs) {
      *abort_flag = 1;
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

__device__ __forceinline__ void tile_coords(int tile, const GemmParams& p, int& b, int& mt, int& nt) {
  const int all_full = p.batch * p.full_tiles;
  if (tile >= all_full) {
    const int t = tile - all_full;
    b = fast_div(t, p.fd_tiles_m);
    mt = t - b * p.tiles_m;
    nt = p.tiles_n - 1;
    return;
  }
  b = fast_div(tile, p.fd_full);
  tile -= b * p.full_tiles;
  const int group = p.group_m * p.tiles_n_full;
  const int g = fast_div(tile, p.fd_group);
  const int first_m = g * p.group_m;
  const bool last = first_m + p.group_m > p.tiles_m;  // the last raster group may be shorter
  const int gm = last ? p.tiles_m - first_m : p.group_m;
  const int w = tile - g * group;
  nt = fast_div(w, last ? p.fd_gm_last : p.fd_gm);
  mt = first_m + (w - nt * gm);
}

// Bounded wait that ignores the abort flag (used only while unwinding).
__device__ __forceinline__ void mbar_wait_unwind(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > 100000000ull) break;
  }
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Row checksums of the first NV (even) columns of a 32-column chunk whose
// first local column is base (a multiple of 32): s1 += sum x, s2 +=
// sum (base + e + 1) x[e], s3 += sum sg(base + e) x[e], amax = max |x|.
// The Thue-Morse sign of base + e is sg(base) * sg(e) (base has its low 5
// bits clear), and columns e, e + 1 (e even) always have opposite signs, so
// each pair goes with one packed add into the accumulator of its sign
// (sg(e) = +1: pp, -1: pn); the plain and the signed sums both follow from
// those two, and one packed FMA forms the weighted sum: three checksums for
// about one instruction per element.
template <int NV>
__device__ __forceinline__ void chunk_checksums(const float (&x)[32], int base, float& s1, float& s2, float& s3,
                                                float& amax) {
  static_assert(NV % 2 == 0 && NV <= 32, "pairs of columns");
  float2 pp = make_float2(0.f, 0.f), pn = make_float2(0.f, 0.f), pw = make_float2(0.f, 0.f);
  float m0 = 0.f, m1 = 0.f;
#pragma unroll
  for (int e = 0; e < NV; e += 2) {
    const float2 xx = make_float2(x[e], x[e + 1]);
    if (__builtin_popcount(e) & 1)
      pn = __fadd2_rn(pn, xx);
    else
      pp = __fadd2_rn(pp, xx);
    pw = __ffma2_rn(make_float2(static_cast<float>(e), static_cast<float>(e + 1)), xx, pw);
    m0 = fmaxf(m0, fabsf(xx.x));
    m1 = fmaxf(m1, fabsf(xx.y));
  }
  const float a = (pp.x + pp.y) + (pn.x + pn.y);
  const float t = (pp.x - pp.y) - (pn.x - pn.y);
  amax = fmaxf(amax, fmaxf(m0, m1));
  s1 += a;
  s2 += fmaf(static_cast<float>(base + 1), a, pw.x + pw.y);
  s3 += (__popc(base) & 1) ? -t : t;
}

// The operand / output element type of a kernel instance: bf16 (F16 =
// false) or fp16. Both use kind::f16 MMAs with fp32 accumulation; one MMA
// takes one type for A and B, so the checksum rows have the operands' type.
template <bool F16>
struct Elem;
template <>
struct Elem<false> {
  using T = __nv_bfloat16;
  static constexpr uint32_t kFmt = 1u;  // instruction-descriptor format
  static __device__ __forceinline__ float lo(uint32_t w) { return bf16_lo(w); }
  static __device__ __forceinline__ float hi(uint32_t w) { return bf16_hi(w); }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ T from_f(float x) { return __float2bfloat16_rn(x); }
  static __device__ __forceinline__ float to_f(T x) { return __bfloat162float(x); }
};
template <>
struct Elem<true> {
  using T = __half;
  static constexpr uint32_t kFmt = 0u;
  static __device__ __forceinline__ float lo(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu)));
  }
  static __device__ __forceinline__ float hi(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
  }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ T from_f(float x) { return __float2half_rn(x); }
  static __device__ __forceinline__ float to_f(T x) { return __half2float(x); }
};

// Token checksum rows of one stage of the swapped B-operand tile, formed by
// two warps, warp wb for k columns [32 wb, 32 wb + 32) of the 64-wide
// k-block. sb: the stage's tile, 128-byte rows with the 128-byte swizzle
// (row j's 16-byte chunk c at chunk c ^ (j & 7)); r0: the first checksum
// row, a multiple of 8; NG * 8 token rows are read (rows past the tokens
// hold zeros). Writes the warp's half of rows r0 .. r0+7 in
// encode_weight_kernel's format: split3(v1), split3(v2), split2(v3) of
//   v1[k] = sum_j x_j[k], v2[k] = sum_j (j+1) x_j[k], v3[k] = sum_j sg(j) x_j[k].
// Lane (hs, cw, e) = (lane >> 4, (lane >> 2) & 3, lane & 3) reads the two
// k values 8c + 2e, 8c + 2e + 1 (c = 4 wb + cw) of rows j = i + 4 hs,
// i = 8g + r (r < 4) known at compile time. The two halves of the warp
// read chunk groups c ^ r and c ^ r ^ 4, so every load hits 32 distinct
// banks. As i and 4 hs have disjoint bits, sg(j) = sg(i) sg(4 hs) and
// j + 1 = (i + 1) + 4 hs: a lane keeps P = sum over sg(i) = +1,
// Q = sum over sg(i) = -1 (one packed add) and W = sum (i + 1) x_j, forms
//   v1 = P + Q, v3 = sg(4 hs) (P - Q), v2 = W + 4 hs v1,
// and one exchange with lane ^ 16 gives both halves the totals.
template <int NG>
__device__ __forceinline__ void build_token_checksums(uint8_t* sb, int r0, int lane, int wb) {
  const int hs = lane >> 4;
  const int c = 4 * wb + ((lane >> 2) & 3);
  const int wofs = (lane & 3) * 4;
  const uint8_t* base[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) base[r] = sb + hs * 512 + ((c ^ (r + 4 * hs)) << 4) + wofs;
  float2 P = make_float2(0.f, 0.f), Q = make_float2(0.f, 0.f);
  float Wa = 0.f, Wb = 0.f;
#pragma unroll
  for (int g = 0; g < NG; ++g) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = 8 * g + r;
      const uint32_t w = *reinterpret_cast<const uint32_t*>(base[r] + i * 128);
      const float2 x = make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
      if (__builtin_popcount(i) & 1)
        Q = __fadd2_rn(Q, x);
      else
        P = __fadd2_rn(P, x);
      Wa = fmaf(static_cast<float>(i + 1), x.x, Wa);
      Wb = fmaf(static_cast<float>(i + 1), x.y, Wb);
    }
  }
  const float sh = hs ? -1.f : 1.f, w4 = 4.f * static_cast<float>(hs);
  float v1a = P.x + Q.x, v1b = P.y + Q.y;
  float v3a = sh * (P.x - Q.x), v3b = sh * (P.y - Q.y);
  float v2a = fmaf(w4, v1a, Wa), v2b = fmaf(w4, v1b, Wb);
  v1a += __shfl_xor_sync(0xffffffffu, v1a, 16);
  v1b += __shfl_xor_sync(0xffffffffu, v1b, 16);
  v2a += __shfl_xor_sync(0xffffffffu, v2a, 16);
  v2b += __shfl_xor_sync(0xffffffffu, v2b, 16);
  v3a += __shfl_xor_sync(0xffffffffu, v3a, 16);
  v3b += __shfl_xor_sync(0xffffffffu, v3b, 16);
  // Half 0 writes rows 0-2 (v1) and 6-7 (v3), half 1 rows 3-5 (v2).
  const float ua = hs ? v2a : v1a, ub = hs ? v2b : v1b;
  const int q0 = 3 * hs;
  __nv_bfloat16 ha[3], hb[3];
  split3_bf16(ua, ha[0], ha[1], ha[2]);
  split3_bf16(ub, hb[0], hb[1], hb[2]);
#pragma unroll
  for (int q = 0; q < 3; ++q)
    *reinterpret_cast<uint32_t*>(sb + (r0 + q0 + q) * 128 + ((c ^ (q0 + q)) << 4) + wofs) =
        static_cast<uint32_t>(__bfloat16_as_ushort(ha[q])) | (static_cast<uint32_t>(__bfloat16_as_ushort(hb[q])) << 16);
  if (!hs) {
    const __nv_bfloat16 a6 = __float2bfloat16_rn(v3a), b6 = __float2bfloat16_rn(v3b);
    const __nv_bfloat16 a7 = __float2bfloat16_rn(v3a - __bfloat162float(a6));
    const __nv_bfloat16 b7 = __float2bfloat16_rn(v3b - __bfloat162float(b6));
    *reinterpret_cast<uint32_t*>(sb + (r0 + 6) * 128 + ((c ^ 6) << 4) + wofs) =
        static_cast<uint32_t>(__bfloat16_as_ushort(a6)) | (static_cast<uint32_t>(__bfloat16_as_ushort(b6)) << 16);
    *reinterpret_cast<uint32_t*>(sb + (r0 + 7) * 128 + ((c ^ 7) << 4) + wofs) =
        static_cast<uint32_t>(__bfloat16_as_ushort(a7)) | (static_cast<uint32_t>(__bfloat16_as_ushort(b7)) << 16);
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// The k loop of one output tile: per 64-wide k-block wait for the stage, issue
// four K=16 MMAs of width NM and release the stage when they complete. NM is
// a template argument so that every instruction descriptor is a compile-time
// constant (a runtime descriptor slowed the issue loop down severalfold).
template <int BN, bool CHECK, bool PAIR, bool F16, int NM>
__device__ __forceinline__ bool mma_mainloop(uint8_t* smem, uint64_t* full, uint64_t* empty, int& stage,
                                             uint32_t& phase, int kb0, int kb1, uint32_t d,
                                             volatile int* abort_flag) {
  using Cfg = GemmCfg<BN, CHECK, PAIR>;
  constexpr int S = Cfg::kStages;
  constexpr int G = PAIR ? 2 : 1;
  constexpr uint32_t idesc = umma_idesc(Cfg::kTileM, NM, Elem<F16>::kFmt);
  static_assert(NM % 16 == 0 && NM >= 16 && NM <= BN, "MMA width");
  for (int kb = kb0; kb < kb1; ++kb) {
    if (!mbar_wait(&full[stage], phase, abort_flag)) return false;
    tc_fence_after();
    const uint32_t a_addr = smem_u32(smem + Cfg::kOffA + stage * Cfg::kABytes);
    const uint32_t b_addr = smem_u32(smem + Cfg::kOffB + stage * Cfg::kBBytes);
#pragma unroll
    for (int k = 0; k < kBK / 16; ++k) {
      const uint64_t adesc = sw128_kmajor_desc(a_addr + k * 32);
      const uint32_t accum = ((kb - kb0) | k) != 0 ? 1u : 0u;
      umma_bf16_ss_g<G>(d, adesc, sw128_kmajor_desc(b_addr + k * 32), idesc, accum);
    }
    // The stage is free in both CTAs of a pair once these MMAs have read it.
    if constexpr (PAIR)
      umma_commit_pair_both(&empty[stage], 0x3);
    else
      umma_commit(&empty[stage]);
    if (++stage == S) {
      stage = 0;
      phase ^= 1u;
    }
  }
  return true;
}

// mma_mainloop for a runtime width n (a multiple of 16 in [16, BN]): one
// compile-time instance per width.
template <int BN, bool CHECK, bool PAIR, bool F16, int NM = 16>
__device__ __forceinline__ bool mma_mainloop_n(int n, uint8_t* smem, uint64_t* full, uint64_t* empty, int& stage,
                                               uint32_t& phase, int kb0, int kb1, uint32_t d,
                                               volatile int* abort_flag) {
  if constexpr (NM <= BN) {
    if (n == NM)
      return mma_mainloop<BN, CHECK, PAIR, F16, NM>(smem, full, empty, stage, phase, kb0, kb1, d, abort_flag);
    return mma_mainloop_n<BN, CHECK, PAIR, F16, NM + 16>(n, smem, full, empty, stage, phase, kb0, kb1, d, abort_flag);
  } else {
    return false;
  }
}

// tmB2 (pairs with checks only): B rows for the odd CTA, whose share of a
// tile's data rows is BD - 128 rather than 128. tmBt: the rows of the tail
// tile column that the compact tail tile needs in this CTA (box
// p.tail_box rows): with checks its data rows; without checks (single CTA)
// all tail_n rows the narrow MMA reads. tmC: the output [batch][M][N] in
// 32 x 32 boxes with 64-byte swizzle, the layout of an epilogue warp's
// staging block (unused with swapped operands).
template <int BN, bool CHECK, bool PAIR, bool F16>
__global__ void __launch_bounds__(kThreads, 1)
    abft_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmB2, const __grid_constant__ CUtensorMap tmV,
                     const __grid_constant__ CUtensorMap tmBt, const __grid_constant__ CUtensorMap tmC,
                     const GemmParams p) {
  using Cfg = GemmCfg<BN, CHECK, PAIR>;
  using E = Elem<F16>;
  using T = typename E::T;
  constexpr int S = Cfg::kStages;
  constexpr int BD = Cfg::kBD;
  constexpr int G = PAIR ? 2 : 1;
  T* const Cout = static_cast<T*>(p.C);
  const T* const biasp = static_cast<const T*>(p.bias);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* ready = bars + 2 * S;  // [S] stage complete for the MMA (build_chk)
  uint64_t* tfull = bars + 3 * S;  // [2]
  uint64_t* tempty = tfull + 2;    // [2]
  uint64_t* xbar = tempty + 2;     // row partials written
  uint64_t* xfree = xbar + 1;      // row partials read (the buffer may be rewritten)
  uint64_t* drain = xfree + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kOffMisc + 4);
  // Mismatching rows of the tile slab in the epilogue, one counter per
  // parity of the row-partial exchange (two tiles in flight at most).
  uint32_t* ndet = reinterpret_cast<uint32_t*>(smem + Cfg::kOffMisc + 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;  // 0 = the pair's MMA issuer
  const int unit = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int nunits = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&ready[s], kBuildWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      // Pairs: one arrival per epilogue warp of either CTA, on the even CTA's barrier.
      mbar_init(&tempty[b], PAIR ? 2 * kEpiWarps : kEpiThreads);
    }
    mbar_init(xbar, kEpiThreads);
    mbar_init(xfree, kEpiThreads);
    mbar_init(drain, 1);
    *abort_flag = 0;
    ndet[0] = 0u;
    ndet[1] = 0u;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (PAIR && CHECK) tma_prefetch_desc(&tmB2);
    if (CHECK) tma_prefetch_desc(&tmV);
    if (p.tail_box > 0) tma_prefetch_desc(&tmBt);
    if (!p.swap) tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc_g<G>(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish_g<G>();
  }
  tc_fence_before();
  // Pairs: the barriers and TMEM of both CTAs exist before either CTA's
  // TMA, MMA or remote arrive can touch them.
  if constexpr (PAIR)
    cluster_sync_all();
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Everything above touches only shared memory, TMEM and the tensor maps
  // in parameter space, so it may overlap the previous kernel on the stream
  // (the launch allows programmatic serialization). Global memory is read
  // and written only after this wait.
  griddep_wait();
  if (blockIdx.x == 0 && p.bcounts != nullptr) {
    // Per-batch counters, zeroed before CTA 0 publishes the report header
    // (other CTAs touch them only after report_ready).
    for (int i = threadIdx.x; i < 4 * p.batch; i += kThreads) p.bcounts[i] = 0u;
    __threadfence();
    __syncthreads();  // CTA 0 only (a uniform branch), before its header thread publishes the tag
  }
  if (blockIdx.x == 0 && threadIdx.x == 32 * (kEpiWarp0 + kEpiWarps - 1) && p.report != nullptr) {
    // Reset the header, then publish this launch's tag: every other write to
    // the report waits for the tag (report_ready). An epilogue thread does
    // it (idle until the first accumulator), so that the producer's first
    // copy does not wait behind the fence.
    abft_report* r = p.report;
    r->status = 0;
    r->n_faults = 0;
    r->n_located = 0;
    r->n_corrected = 0;
    r->overflow = 0;
    r->capacity = static_cast<uint32_t>(p.capacity);
    r->tile_m = Cfg::kTileM;
    r->tile_n = BD;
    r->corner = 0.f;
    r->sum_c = 0.f;
    r->abs_err = 0.f;
    r->rel_err = 0.f;
    r->ref_ok = -1;
    r->batch = p.bcounts != nullptr ? static_cast<uint32_t>(p.batch) : 0u;
    __threadfence();
    st_release_u64(reinterpret_cast<unsigned long long*>(&r->launch_tag), p.nonce);
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_phase = 0;
      bool ok = true;
      // Pairs: both CTAs' copies complete on the even CTA's full barrier,
      // which expects the bytes of both.
      constexpr uint32_t kTx = G * (Cfg::kABytes + Cfg::kBBytes);
      const uint64_t pol_first = l2_policy_evict_first(), pol_last = l2_policy_evict_last();
      SegmentIter seg(p, unit, nunits);
      int tile, kb0, kb1;
      while (ok && seg.next(p, tile, kb0, kb1)) {
        int bz, mt, nt;
        tile_coords(tile, p, bz, mt, nt);
        const int arow = mt * Cfg::kTileM + static_cast<int>(rank) * kBM;
        // Compact tail tile: this CTA's data rows come from the tail box (and
        // the checksum rows follow them); in a pair the odd CTA's rows start
        // at tail_n / 2 within the tile.
        const bool tail = p.tail_n != 0 && nt == p.tiles_n - 1;
        const uint32_t tx = tail ? p.tail_tx : kTx;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + Cfg::kOffA + stage * Cfg::kABytes;
          uint8_t* sb = smem + Cfg::kOffB + stage * Cfg::kBBytes;
          const int kx = kb * kBK;
          if constexpr (PAIR) {
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], tx);
            tma_load_3d_pair(sa, &tmA, fb, kx, arow, bz);
            if (!CHECK) {
              const int half = tail ? p.tail_n / 2 : Cfg::kBRows;
              tma_load_3d_pair(sb, &tmB, fb, kx, nt * BN + static_cast<int>(rank) * half, bz);
            } else if (rank == 0) {
              tma_load_3d_pair(sb, &tmB, fb, kx, nt * BD, bz);
            } else if (!tail) {
              tma_load_3d_pair(sb, &tmB2, fb, kx, nt * BD + Cfg::kBRows, bz);
              tma_load_3d_pair(sb + Cfg::kChkRow0 * 128, &tmV, fb, kx, nt * kChkRows, bz);
            } else {
              if (p.tail_box > 0) tma_load_3d_pair(sb, &tmBt, fb, kx, nt * BD + p.tail_n / 2, bz);
              tma_load_3d_pair(sb + p.tail_box * 128, &tmV, fb, kx, nt * kChkRows, bz);
            }
          } else if (p.swap) {
            // Swapped operands (few tokens): the weight, this kernel's A,
            // streams through once while the token tile and its checksum
            // rows are read for every weight tile. Hinting the weight
            // evict-first and the tokens evict-last cut a one-token
            // 37888 x 3584 GEMM from 68.5 to 58.2 us; unswapped shapes, whose
            // B panels feed many tile rows, lose with the same hints.
            mbar_arrive_expect_tx(&full[stage], tx);
            tma_load_3d_hint(sa, &tmA, &full[stage], kx, arow, bz, pol_first);
            if (!tail) {
              tma_load_3d_hint(sb, &tmB, &full[stage], kx, nt * BD, bz, pol_last);
              if (CHECK) tma_load_3d_hint(sb + BD * 128, &tmV, &full[stage], kx, nt * kChkRows, bz, pol_last);
            } else if (!CHECK) {
              tma_load_3d_hint(sb, &tmBt, &full[stage], kx, nt * BD, bz, pol_last);
            } else {
              if (p.tail_box > 0) tma_load_3d_hint(sb, &tmBt, &full[stage], kx, nt * BD, bz, pol_last);
              if (!p.build_chk)
                tma_load_3d_hint(sb + p.tail_box * 128, &tmV, &full[stage], kx, nt * kChkRows, bz, pol_last);
            }
          } else {
            mbar_arrive_expect_tx(&full[stage], tx);
            tma_load_3d(sa, &tmA, &full[stage], kx, arow, bz);
            if (!tail) {
              tma_load_3d(sb, &tmB, &full[stage], kx, nt * BD, bz);
              if (CHECK) tma_load_3d(sb + BD * 128, &tmV, &full[stage], kx, nt * kChkRows, bz);
            } else if (!CHECK) {
              // compact tail: the tail_n rows the narrow MMA reads (rows past N read as zeros)
              tma_load_3d(sb, &tmBt, &full[stage], kx, nt * BD, bz);
            } else {
              if (p.tail_box > 0) tma_load_3d(sb, &tmBt, &full[stage], kx, nt * BD, bz);
              if (!p.build_chk) tma_load_3d(sb + p.tail_box * 128, &tmV, &full[stage], kx, nt * kChkRows, bz);
            }
          }
          issued_mask |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Unwinding: let every issued copy land before the CTA can exit.
        if constexpr (PAIR) {
          // The copies complete on the even CTA's barriers: give them a
          // fixed, generous time instead.
          const uint64_t t0 = global_timer_ns();
          while (issued_mask && global_timer_ns() - t0 < 200000ull) {
          }
        } else {
          for (int s = 0; s < S; ++s)
            if (issued_mask & (1u << s)) mbar_wait_unwind(&full[s], (issued_phase >> s) & 1u);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      SegmentIter seg(p, unit, nunits);
      int tile, kb0, kb1;
      while (ok && seg.next(p, tile, kb0, kb1)) {
        int bz, mt, nt;
        tile_coords(tile, p, bz, mt, nt);
        (void)bz;
        (void)mt;
        const bool tail = p.tail_n != 0 && nt == p.tiles_n - 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        uint64_t* avail = p.build_chk ? ready : full;
        if (!tail)
          ok = mma_mainloop<BN, CHECK, PAIR, F16, BN>(smem, avail, empty, stage, phase, kb0, kb1, d, abort_flag);
        else
          ok = mma_mainloop_n<BN, CHECK, PAIR, F16>(p.tail_n, smem, avail, empty, stage, phase, kb0, kb1, d,
                                                    abort_flag);
        if (!ok) break;
        if constexpr (PAIR)
          umma_commit_pair_both(&tfull[acc], 0x3);
        else
          umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Every MMA this thread issued must finish before TMEM is released.
      umma_commit_g<G>(drain);
      mbar_wait_unwind(drain, 0);
    }
    __syncwarp();
  } else if (warp >= kBuildWarp) {
    // ------------------------------------------------------------ token checksums
    // Swapped operands: the B-operand tile is the compact tile of the
    // p.N (<= 64) token rows, tail_box = round8(p.N) rows (the copy fills
    // the rows past p.N with zeros), then its 8 checksum rows. Per stage the
    // two warps (one half of the 64-wide k-block each) sum the token rows in
    // shared memory and write the checksum rows, which the MMA reads after
    // both have arrived on the ready barrier.
    // fp16 instances never build: their token checksums need a scale taken
    // over all of K, which the host's encode pass supplies instead.
    if (CHECK && !PAIR && !F16 && p.build_chk) {
      const int wb = warp - kBuildWarp;
      int stage = 0;
      uint32_t phase = 0;
      SegmentIter seg(p, unit, nunits);
      int tile, kb0, kb1;
      bool ok = true;
      while (ok && seg.next(p, tile, kb0, kb1)) {
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sb = smem + Cfg::kOffB + stage * Cfg::kBBytes;
          switch (p.tail_box >> 3) {
            case 1: build_token_checksums<1>(sb, p.tail_box, lane, wb); break;
            case 2: build_token_checksums<2>(sb, p.tail_box, lane, wb); break;
            case 3: build_token_checksums<3>(sb, p.tail_box, lane, wb); break;
            case 4: build_token_checksums<4>(sb, p.tail_box, lane, wb); break;
            case 5: build_token_checksums<5>(sb, p.tail_box, lane, wb); break;
            case 6: build_token_checksums<6>(sb, p.tail_box, lane, wb); break;
            case 7: build_token_checksums<7>(sb, p.tail_box, lane, wb); break;
            default: build_token_checksums<8>(sb, p.tail_box, lane, wb); break;
          }
          // the MMA reads the rows through the async proxy
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&ready[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // Each thread owns one output row (TMEM lane) and every kEpiSplit-th
    // 32-column chunk of the tile, and streams them from TMEM once; the
    // accumulator is released after the row checks (the MMA meanwhile fills
    // the other buffer).
    const int q = warp & 3;              // TMEM lane quadrant this warp may access
    const int ep = warp - kEpiWarp0;     // 0 .. kEpiWarps - 1
    const int t = ep >> 2;               // column share: chunks t, t + kEpiSplit, ...
    const int r = q * 32 + lane;         // row within the tile
    constexpr int NCT = BN / 32;         // 32-column chunks per tile
    float4* xchg = reinterpret_cast<float4*>(smem + Cfg::kOffX);
    // This warp's staging block: 32 rows of 64 bytes, the four 16-byte
    // pieces of row y permuted by XOR with (y >> 1) & 3 so that both the
    // row-per-lane writes and the 8-rows-per-instruction reads are free of
    // bank conflicts.
    uint8_t* stg = smem + Cfg::kOffStage + ep * Cfg::kStageBytes;
    const int rd_row = lane >> 2;  // read side: row (within 8) and piece of this lane
    const int rd_piece = lane & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    int xuse = 0;  // uses of the row-partial exchange buffer
    // This warp's staging block is the source of a bulk store that may not
    // have read it yet (lane 0 issued it; warp-uniform).
    bool stg_busy = false;
    // Hand the accumulator back to the MMA issuer (in a pair, the even CTA:
    // one arrival per warp after all its lanes' TMEM reads). The reads have
    // completed (tcgen05.wait::ld) and the fence orders them before the
    // arrival; the MMA that overwrites the accumulator reads nothing this
    // thread wrote, so the arrival need not wait for the output stores.
    auto release_acc = [&](int a) {
      tc_fence_before();
      if constexpr (PAIR) {
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&tempty[a]), 0));
      } else {
        mbar_arrive_relaxed(&tempty[a]);
      }
    };
    SegmentIter seg(p, unit, nunits);
    int tile, kb0, kb1;
    while (seg.next(p, tile, kb0, kb1)) {
      int bz, mt, nt;
      tile_coords(tile, p, bz, mt, nt);
      // Warp-uniform outcome: the tcgen05.ld below are warp-collective.
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&tfull[acc], acc_phase, abort_flag))) break;
      tc_fence_after();
      const uint32_t tacc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      // Accumulator columns the MMA wrote: BN, or the compact tail tile's
      // width; stream-K partials carry only those.
      const int acc_w = (p.tail_n != 0 && nt == p.tiles_n - 1) ? p.tail_n : BN;

      if (kb0 != 0) {
        // Stream-K contributor: the tile's first k-blocks belong to a lower
        // CTA, which finishes the tile. Hand it the fp32 partial (every
        // column the MMA wrote, checksum columns included), column-major so that each
        // warp store is 32 consecutive words. A segment that starts inside
        // a tile is the first segment of this CTA, so it is stored before
        // this CTA waits for anything: the wait chain is one link long.
        // Layout [cta][column group of 4][row][4]: a warp's float4 store
        // covers 32 consecutive rows, 512 contiguous bytes.
        float4* dst = reinterpret_cast<float4*>(p.partials) + static_cast<size_t>(blockIdx.x) * (BN / 4) * kBM + r;
#pragma unroll 1
        for (int c = t; c < NCT; c += kEpiSplit) {
          if (c * 32 >= acc_w) break;  // warp-uniform
          uint32_t v[32];
          __syncwarp();
          tmem_ld_32x32b_x32(tacc + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int g = 0; g < 8; ++g)
            __stcg(dst + (c * 8 + g) * kBM, make_float4(__uint_as_float(v[4 * g]), __uint_as_float(v[4 * g + 1]),
                                                        __uint_as_float(v[4 * g + 2]), __uint_as_float(v[4 * g + 3])));
        }
        release_acc(acc);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
        // Each warp publishes its own share (32 rows x its chunks):
        // every lane makes its stores visible device-wide, then lane 0
        // releases the warp's flag. A finisher warp waits only for the
        // warps whose rows and columns it reads; no CTA-wide hand-off.
        __threadfence();
        __syncwarp();
        if (lane == 0) st_release_u64(&p.flags[blockIdx.x * kEpiWarps + ep], p.nonce);
        continue;
      }

      // Accumulator column of the expected checksums: BD, or right after the
      // data rows of a compact tail tile (its data columns rounded up to 8).
      const int chk_col = (p.tail_n != 0 && nt == p.tiles_n - 1) ? ((p.N - nt * BD + 7) & ~7) : BD;
      // The expected checksums seed share 0's sums; the other shares need
      // neither them nor their stream-K partials.
      uint32_t chk[kChkRows];
      if (CHECK && t == 0) {
        __syncwarp();
        tmem_ld_32x32b_x8(tacc + static_cast<uint32_t>(chk_col), chk);
        tmem_ld_wait();
      }
      if (kb1 != p.num_kb) {
        // Stream-K finisher (this unit owns the tile's first k-blocks): fold
        // in the partials of the units that own its later k-blocks (units
        // unit+1, ..., ulast; in a pair, their CTAs of the same rank). Every
        // element gets acc + p[unit+1] + p[unit+2] + ... in that order (a
        // fixed summation order). Once every contributor's flag holds this
        // launch's nonce, the fold runs chunk by chunk with the loads of two
        // contributors in flight at a time, one TMEM read and write per chunk.
        const int64_t tile_end = static_cast<int64_t>(tile - p.dp_tiles + 1) * p.num_kb;
        int ulast = unit;
        while (ulast + 1 < p.sk_ctas && SegmentIter::sk_begin(p, ulast + 1) < tile_end) ++ulast;
        // this warp's rows and chunks; for share 0 with checks also the warp
        // of the same rows that stored the chunk holding the checksum columns
        const int chk_ep = (ep & 3) + 4 * ((chk_col >> 5) % kEpiSplit);
        bool okp = true;
#pragma unroll 1
        for (int u = unit + 1; u <= ulast; ++u) {
          const int cc = u * G + static_cast<int>(rank);
          if (!wait_flag(&p.flags[cc * kEpiWarps + ep], p.nonce, abort_flag) ||
              (CHECK && t == 0 && chk_ep != ep && !wait_flag(&p.flags[cc * kEpiWarps + chk_ep], p.nonce, abort_flag))) {
            okp = false;
            break;
          }
        }
        if (!__all_sync(0xFFFFFFFFu, okp)) break;
        const float4* part = reinterpret_cast<const float4*>(p.partials) + r;
        constexpr size_t kPartF4 = static_cast<size_t>(BN / 4) * kBM;  // float4 of one CTA's partial
#pragma unroll 1
        for (int c = t; c < NCT; c += kEpiSplit) {
          if (c * 32 >= acc_w) break;  // warp-uniform: nothing stored from here on
          uint32_t v[32];
          __syncwarp();
          tmem_ld_32x32b_x32(tacc + c * 32, v);
          tmem_ld_wait();
          const size_t coff = static_cast<size_t>(c * 8) * kBM;
          int u = unit + 1;
#pragma unroll 1
          for (; u < ulast; u += 2) {
            const float4* sa = part + static_cast<size_t>(u * G + static_cast<int>(rank)) * kPartF4 + coff;
            const float4* sb = part + static_cast<size_t>((u + 1) * G + static_cast<int>(rank)) * kPartF4 + coff;
            float4 qa[8], qb[8];
#pragma unroll
            for (int g = 0; g < 8; ++g) qa[g] = __ldcg(sa + g * kBM);
#pragma unroll
            for (int g = 0; g < 8; ++g) qb[g] = __ldcg(sb + g * kBM);
#pragma unroll
            for (int g = 0; g < 8; ++g) {
              v[4 * g] = __float_as_uint((__uint_as_float(v[4 * g]) + qa[g].x) + qb[g].x);
              v[4 * g + 1] = __float_as_uint((__uint_as_float(v[4 * g + 1]) + qa[g].y) + qb[g].y);
              v[4 * g + 2] = __float_as_uint((__uint_as_float(v[4 * g + 2]) + qa[g].z) + qb[g].z);
              v[4 * g + 3] = __float_as_uint((__uint_as_float(v[4 * g + 3]) + qa[g].w) + qb[g].w);
            }
          }
          if (u == ulast) {
            const float4* sa = part + static_cast<size_t>(u * G + static_cast<int>(rank)) * kPartF4 + coff;
            float4 qa[8];
#pragma unroll
            for (int g = 0; g < 8; ++g) qa[g] = __ldcg(sa + g * kBM);
#pragma unroll
            for (int g = 0; g < 8; ++g) {
              v[4 * g] = __float_as_uint(__uint_as_float(v[4 * g]) + qa[g].x);
              v[4 * g + 1] = __float_as_uint(__uint_as_float(v[4 * g + 1]) + qa[g].y);
              v[4 * g + 2] = __float_as_uint(__uint_as_float(v[4 * g + 2]) + qa[g].z);
              v[4 * g + 3] = __float_as_uint(__uint_as_float(v[4 * g + 3]) + qa[g].w);
            }
          }
          __syncwarp();
          tmem_st_32x32b_x32(tacc + c * 32, v);
        }
        tmem_st_wait();
        if (CHECK && t == 0) {
#pragma unroll 1
          for (int u = unit + 1; u <= ulast; ++u) {
            const float4* src = part + static_cast<size_t>(u * G + static_cast<int>(rank)) * kPartF4;
            const float4 c0 = __ldcg(src + (chk_col / 4) * kBM);
            const float4 c1 = __ldcg(src + (chk_col / 4 + 1) * kBM);
            const float add[kChkRows] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
            for (int e = 0; e < kChkRows; ++e) chk[e] = __float_as_uint(__uint_as_float(chk[e]) + add[e]);
          }
        }
      }

      const int row0 = mt * Cfg::kTileM + static_cast<int>(rank) * kBM;  // first row of this CTA's slab
      const int grow = row0 + r;
      const int col0 = nt * BD;
      const int ncols = min(BD, p.N - col0);
      const bool row_ok = grow < p.M;

      // Debug faults added to the fp32 accumulator: does this row (in this
      // thread's chunks) hold any? The rare rows that do scan the list again
      // per chunk (inj_add) rather than keep it in registers. Batch offsets
      // of the flattened fault coordinates: C's rows are the kernel's rows,
      // or its columns with swapped operands.
      const int inj_row = p.swap ? grow : bz * p.M + grow;
      const int inj_cbase = (p.swap ? bz * p.N : 0) + col0;  // list column of the tile's local column 0
      bool n_my = false;
      if (p.n_inj > 0 && row_ok) {
        for (int i = 0; i < p.n_inj; ++i) {
          const int ic = p.inj_cols[i] - inj_cbase;
          n_my |= p.inj_rows[i] == inj_row && ic >= 0 && ic < ncols && ((ic >> 5) % kEpiSplit) == t;
        }
      }
      // Sum of the injected deltas at local column lc of the tile.
      auto inj_add = [&](int lc) {
        float d = 0.f;
        for (int i = 0; i < p.n_inj; ++i)
          if (p.inj_rows[i] == inj_row && p.inj_cols[i] - inj_cbase == lc) d += p.inj_deltas[i];
        return d;
      };

      // One pass over the accumulator in 32-column chunks: each chunk feeds
      // the row checksums (with checks on) and is rounded, staged and stored
      // at once (swapped operands: straight to C's transposed position).
      // Share 0 starts its sums from the negated expected checksums (split
      // checksum columns added up), so the shares' partials add up to the
      // residuals.
      float s1 = 0.f, s2 = 0.f, s3 = 0.f, amax = 0.f;
      if (CHECK && t == 0) {
        s1 = -((__uint_as_float(chk[0]) + __uint_as_float(chk[1])) + __uint_as_float(chk[2]));
        s2 = -((__uint_as_float(chk[3]) + __uint_as_float(chk[4])) + __uint_as_float(chk[5]));
        s3 = -(__uint_as_float(chk[6]) + __uint_as_float(chk[7]));
        if constexpr (F16) {
          // fp16 checksum rows hold v * 2^-e (each checksum's largest value
          // scaled below 2^15): the expected sums are 2^e times the MMA's,
          // exact powers of two.
          const float* sc = p.chk_scale + bz * p.chk_scale_bstride + nt * 8;
          s1 *= __ldg(sc + 4);
          s2 *= __ldg(sc + 5);
          s3 *= __ldg(sc + 6);
        }
      }
      float row_out_sum = 0.f;
      const uint4* bp = reinterpret_cast<const uint4*>(biasp + col0);
      const int rd_grow = row0 + q * 32 + rd_row;  // global row of this lane's first read-side row
      const float row_bias = (p.swap && p.bias != nullptr && row_ok) ? E::to_f(biasp[grow]) : 0.f;
      const int crow0 = bz * p.c_rows;  // this batch's first row of C
#pragma unroll 1
      for (int c = t; c < NCT; c += kEpiSplit) {
        const int base = c * 32;  // first local column of the chunk
        if (base >= ncols) break;  // warp-uniform: nothing valid from here on
        uint32_t v[32];
        __syncwarp();
        tmem_ld_32x32b_x32(tacc + base, v);
        tmem_ld_wait();
        float x[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) x[e] = __uint_as_float(v[e]);
        if (n_my) {
#pragma unroll
          for (int e = 0; e < 32; ++e) x[e] += inj_add(base + e);
        }
        if constexpr (CHECK) {
          if (base + 32 <= ncols)
            chunk_checksums<32>(x, base, s1, s2, s3, amax);
          else if (base + 24 == ncols)  // the chunk of a full tile that holds its 8 checksum columns
            chunk_checksums<24>(x, base, s1, s2, s3, amax);
          else {
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int col = base + e;
              if (col < ncols) {
                s1 += x[e];
                s2 = fmaf(static_cast<float>(col + 1), x[e], s2);
                s3 += (__popc(col) & 1) ? -x[e] : x[e];
                amax = fmaxf(amax, fabsf(x[e]));
              }
            }
          }
        }
        if (p.swap) {
          // Lane l holds kernel row row0 + q*32 + l = C column: for each of
          // this chunk's C rows a warp writes 32 consecutive columns.
          if (row_ok) {
            T* cc = Cout + static_cast<int64_t>(crow0 + col0 + base) * p.ldc + grow;
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              if (base + e < ncols) {
                const T o = E::from_f(x[e] + row_bias);
                cc[static_cast<int64_t>(e) * p.ldc] = o;
                if (p.mode & ABFT_MODE_REF) row_out_sum += E::to_f(o);
              }
            }
          }
          continue;
        }
        if (stg_busy) {
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
          stg_busy = false;
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const bool gvalid = row_ok && (base + g * 8 < ncols);
          if (p.bias != nullptr && gvalid) {
            const uint4 bw = __ldg(bp + c * 4 + g);
            x[g * 8 + 0] += E::lo(bw.x);
            x[g * 8 + 1] += E::hi(bw.x);
            x[g * 8 + 2] += E::lo(bw.y);
            x[g * 8 + 3] += E::hi(bw.y);
            x[g * 8 + 4] += E::lo(bw.z);
            x[g * 8 + 5] += E::hi(bw.z);
            x[g * 8 + 6] += E::lo(bw.w);
            x[g * 8 + 7] += E::hi(bw.w);
          }
          const uint4 packed =
              make_uint4(E::pack2(x[g * 8 + 0], x[g * 8 + 1]), E::pack2(x[g * 8 + 2], x[g * 8 + 3]),
                         E::pack2(x[g * 8 + 4], x[g * 8 + 5]), E::pack2(x[g * 8 + 6], x[g * 8 + 7]));
          *reinterpret_cast<uint4*>(stg + lane * 64 + ((g ^ ((lane >> 1) & 3)) << 4)) = packed;
          if ((p.mode & ABFT_MODE_REF) && gvalid) {
            row_out_sum += ((E::lo(packed.x) + E::hi(packed.x)) + (E::lo(packed.y) + E::hi(packed.y))) +
                           ((E::lo(packed.z) + E::hi(packed.z)) + (E::lo(packed.w) + E::hi(packed.w)));
          }
        }
        if (base + 32 <= ncols) {
          // A whole 32 x 32 block: one bulk tensor store (rows past M are
          // clipped by the map); the next write of the block waits for it
          // to have been read.
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tmC, stg, col0 + base, row0 + q * 32, bz);
            bulk_commit_group();
          }
          stg_busy = true;
          continue;
        }
        __syncwarp();
        // Partial block (next to the checksum columns, or the last tile
        // column): plain stores. Instruction i covers rows 8i..8i+7 of the
        // block, four lanes per row, each lane one 16-byte piece (8 columns).
        const int lcol = base + rd_piece * 8;  // local column of this lane's piece
        const bool col_ok = lcol < ncols;
        T* cbase = Cout + static_cast<int64_t>(crow0 + rd_grow) * p.ldc + col0 + lcol;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int y = i * 8 + rd_row;
          const uint4 val = *reinterpret_cast<const uint4*>(stg + y * 64 + ((rd_piece ^ ((y >> 1) & 3)) << 4));
          if (col_ok && rd_grow + i * 8 < p.M) *reinterpret_cast<uint4*>(cbase + static_cast<int64_t>(i * 8) * p.ldc) = val;
        }
      }

      bool aborted = false;
      if constexpr (CHECK) {
        // Exchange the row partials of the kEpiSplit shares through shared
        // memory; amax >= 0 and s3 rides in .w. One buffer: before writing
        // it a thread waits until every thread has read the previous tile's
        // partials (xfree). The xbar barrier (release/acquire) also orders
        // every chunk store of the row before a rewrite.
        int fix_col = -1;  // local column to correct, if any
        float fix_delta = 0.f;
        const uint32_t xph = static_cast<uint32_t>(xuse & 1);
        if (xuse > 0 && !mbar_wait(xfree, xph ^ 1u, abort_flag)) aborted = true;
        ++xuse;
        if (!aborted) {
          xchg[t * kBM + r] = make_float4(s1, s2, amax, s3);
          mbar_arrive(xbar);
          if (!mbar_wait(xbar, xph, abort_flag)) aborted = true;
          // Everyone has finished the previous tile, whose slab counter (the
          // other parity) is free again: clear it for the tile after this one.
          if (!aborted && ep == 0 && lane == 0) ndet[xph ^ 1u] = 0u;
        }
        if (!aborted) {
          float res1 = 0.f, res2 = 0.f, res3 = 0.f, tmax = 0.f;
#pragma unroll
          for (int j = 0; j < kEpiSplit; ++j) {
            const float4 pj = xchg[j * kBM + r];
            res1 += pj.x;
            res2 += pj.y;
            res3 += pj.w;
            tmax = fmaxf(tmax, pj.z);
          }
          const float thr = fmaf(p.thr_k, tmax, p.thr_abs);
          const bool det = row_ok && (fabsf(res1) > thr || fabsf(res2) > thr * static_cast<float>(ncols));
          // Count the slab's mismatching rows (one share per row) before
          // releasing the exchange buffer: once every thread has arrived on
          // xfree the count is complete.
          if (det && t == 0) atomicAdd(&ndet[xph], 1u);
          mbar_arrive(xfree);
          if (det) {
            uint32_t flags = ABFT_REC_DETECTED;
            uint32_t st_extra = 0u;
            int col = -1;
            if (fabsf(res1) > thr) {
              const float pos = res2 / res1;
              const float pr = rintf(pos);
              if (fabsf(pos - pr) <= 0.1f && pr >= 1.f && pr <= static_cast<float>(ncols)) {
                const int cpos = static_cast<int>(pr) - 1;
                const float sg = (__popc(cpos) & 1) ? -1.f : 1.f;
                if (fabsf(res3 - sg * res1) <= 0.5f * fabsf(res1)) {
                  col = cpos;
                  flags |= ABFT_REC_LOCATED;
                }
              }
            }
            if (col >= 0 && (p.mode & ABFT_MODE_CORRECT)) {
              // A single upset touches a few rows; a mismatch in most rows of
              // the slab means stale checksums or a bad operand, where a
              // "correction" would corrupt a right output: leave it as is.
              uint32_t nd = ~0u;
              if (mbar_wait(xfree, xph, abort_flag)) nd = ndet[xph];
              const uint32_t valid = static_cast<uint32_t>(min(kBM, p.M - row0));
              if (nd > static_cast<uint32_t>(ABFT_SUSPECT_ROWS) || (nd >= 4u && 2u * nd > valid)) {
                flags |= ABFT_REC_SUPPRESSED;
                st_extra = ABFT_STATUS_SUSPECT;
              } else {
                fix_col = col;
                fix_delta = res1;
                flags |= ABFT_REC_CORRECTED;
              }
            }
            if (t == 0 && report_ready(p, abort_flag)) {
              abft_report* rep = p.report;
              const uint32_t slot = atomicAdd(&rep->n_faults, 1u);
              if (flags & ABFT_REC_LOCATED) atomicAdd(&rep->n_located, 1u);
              if (flags & ABFT_REC_CORRECTED) atomicAdd(&rep->n_corrected, 1u);
              uint32_t st = ABFT_STATUS_FAULT | st_extra | ((flags & ABFT_REC_LOCATED) ? 0u : ABFT_STATUS_UNLOCATED);
              if (slot < static_cast<uint32_t>(p.capacity)) {
                abft_fault_record* rec = reinterpret_cast<abft_fault_record*>(rep + 1) + slot;
                if (!p.swap) {
                  rec->row = bz * p.M + grow;
                  rec->col = col >= 0 ? col0 + col : -1;
                } else {
                  rec->row = col >= 0 ? bz * p.N + col0 + col : -1;
                  rec->col = grow;
                }
                rec->residual = res1;
                rec->residual_w = res2;
                rec->threshold = thr;
                rec->flags = flags;
              } else {
                atomicAdd(&rep->overflow, 1u);
                st |= ABFT_STATUS_OVERFLOW;
              }
              atomicOr(&rep->status, st);
              if (p.bcounts != nullptr) {
                uint32_t* bc = p.bcounts + 4 * bz;
                atomicAdd(bc, 1u);
                if (flags & ABFT_REC_LOCATED) atomicAdd(bc + 1, 1u);
                if (flags & ABFT_REC_CORRECTED) atomicAdd(bc + 2, 1u);
              }
            }
          }
        }
        // Correction: the owner of the located column's chunk reads the fp32
        // accumulator of that element again -- the chunk, warp-collectively
        // -- and stores accumulator - residual (+ bias) over the value stored
        // above, in the same arithmetic order as the chunk pass (injected
        // delta, correction, bias).
        const int fix_chunk = fix_col >> 5;
        const bool mine = fix_col >= 0 && (fix_chunk % kEpiSplit) == t;
        uint32_t need = __ballot_sync(0xFFFFFFFFu, mine);
        if (need != 0u && stg_busy) {
          // The element was written by this warp's bulk stores: let them
          // complete before the rewrite.
          if (lane == 0) {
            bulk_wait_all();
            fence_proxy_async_global();
          }
          __syncwarp();
          stg_busy = false;
        }
        while (need != 0u) {
          const int cfix = __shfl_sync(0xFFFFFFFFu, fix_chunk, __ffs(need) - 1);
          uint32_t v[32];
          __syncwarp();
          tmem_ld_32x32b_x32(tacc + cfix * 32, v);
          tmem_ld_wait();
          const bool here = mine && fix_chunk == cfix;
          if (here) {
            const int e0 = fix_col & 31;
            float val = 0.f;
#pragma unroll
            for (int e = 0; e < 32; ++e) val = (e == e0) ? __uint_as_float(v[e]) : val;
            if (n_my) val += inj_add(fix_col);
            const float bcol = p.swap ? row_bias : (p.bias != nullptr ? E::to_f(biasp[col0 + fix_col]) : 0.f);
            const T o_old = E::from_f(val + bcol);
            const T o_new = E::from_f((val - fix_delta) + bcol);
            const int64_t off = p.swap ? static_cast<int64_t>(crow0 + col0 + fix_col) * p.ldc + grow
                                       : static_cast<int64_t>(crow0 + grow) * p.ldc + col0 + fix_col;
            Cout[off] = o_new;
            if (p.mode & ABFT_MODE_REF) row_out_sum += E::to_f(o_new) - E::to_f(o_old);
          }
          need &= ~__ballot_sync(0xFFFFFFFFu, here);
        }
      }
      release_acc(acc);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
      if (p.mode & ABFT_MODE_REF) {
        // Deterministic per-tile partial sums of the stored outputs: a fixed
        // warp tree per epilogue warp; the 8 partials of a tile are added in
        // warp order by the finishing kernel.
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) row_out_sum += __shfl_xor_sync(0xFFFFFFFFu, row_out_sum, o);
        if (lane == 0) p.tile_sumc[(tile * G + static_cast<int>(rank)) * kEpiWarps + ep] = row_out_sum;
      }
      // Leave the tile loop together: the TMEM loads above are warp-collective.
      if (__any_sync(0xFFFFFFFFu, aborted)) break;
    }
    // Bulk stores still in flight read this CTA's shared memory.
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  // Pairs: the even CTA's MMAs (which write both CTAs' TMEM and read both
  // CTAs' shared memory) and the odd CTA's remote arrivals are all done
  // before either CTA frees TMEM or exits.
  if constexpr (PAIR)
    cluster_sync_all();
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_g<G>(tmem_base, Cfg::kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag && p.report != nullptr) {
    // Bounded: report_ready gives up if CTA 0 never published the header;
    // the status is then lost with the header.
    if (report_ready(p, abort_flag)) atomicOr(&p.report->status, ABFT_STATUS_DEVICE_TIMEOUT);
  }
}

}  // namespace abft
