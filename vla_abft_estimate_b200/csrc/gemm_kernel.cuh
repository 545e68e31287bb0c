// gemm_kernel.cuh - fused checksum-protected bf16 GEMM for sm_100a.
//
//   C[M, N] = A[M, K] * B[N, K]^T (+ bias)      (B = nn.Linear weight layout)
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
//   warps 2-9   epilogue: warp w owns TMEM lane quadrant (w % 4), i.e. 32
//               output rows, and column half (w - 2) / 4 of the tile. Each
//               thread copies its BN/2 accumulator columns to registers and
//               releases the accumulator, then reduces, checks, corrects,
//               adds bias, rounds to bf16 and stores.
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
// The checksum block holds v1 and v2 each split into three bf16 terms
// (hi + mid + lo, 24 significant bits) and v3 in two. A single corrupted
// C[i,j*] (+delta) gives s1 - e1 = delta, s2 - e2 = (j*+1) delta and
// s3 - e3 = sg(j*) delta: the ratio of the first two pins the column, the
// third must agree with it (several faults in one row segment whose
// weighted mean column is an integer are rejected this way), and delta is
// subtracted before the bf16 store.
#pragma once

#include <cuda_bf16.h>

#include "../../include/abft_b200.h"
#include "ptx.cuh"

namespace abft {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 320;
constexpr int kEpiWarp0 = 2;
constexpr int kEpiThreads = 256;
constexpr int kChkRows = 8;  // rows of the per-tile checksum block

template <int BN, bool CHECK>
struct GemmCfg {
  static constexpr int kStages = (BN == 256) ? 4 : 6;
  static constexpr int kBD = CHECK ? BN - kChkRows : BN;  // data columns per tile
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + kStages * kABytes;
  static constexpr int kOffX = kOffB + kStages * kBBytes;  // row-half partial exchange
  static constexpr int kXBytes = 2 * 2 * kBM * 16;         // [tile parity][half][row] float4
  static constexpr int kOffBar = kOffX + (CHECK ? kXBytes : 0);
  static constexpr int kNumBars = 2 * kStages + 2 * 3 + 2;  // full, empty, tfull, tempty, xbar, drain, pbar
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 64 + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert((kBD * 128) % 1024 == 0, "checksum rows must start on a swizzle atom");
};

struct GemmParams {
  __nv_bfloat16* C;
  int64_t ldc;
  const __nv_bfloat16* bias;
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
  float* tile_sumc;  // ABFT_MODE_REF: [num_tiles][8] partial sums of the stored outputs
  // Hybrid schedule: tiles [0, dp_tiles) are data-parallel (whole tiles,
  // blockIdx.x + j*gridDim.x); with sk != 0 the remaining tiles are
  // stream-K: CTA c owns k-block iterations [c*W/G, (c+1)*W/G) of the
  // W = sk_iters = (num_tiles - dp_tiles) * num_kb that follow, G = gridDim.x.
  int dp_tiles;
  int sk;
  int64_t sk_iters;
  float* partials;  // [G][128][BN] fp32: a CTA's share of a tile it does not finish
  int* flags;       // [G]: set to 1 once that CTA's partial is visible
};

// Walks the (tile, k-block range) segments one CTA owns. Data-parallel:
// whole tiles blockIdx.x, +gridDim.x, ...; stream-K: consecutive slices of
// the CTA's iteration range, cut at tile boundaries.
struct SegmentIter {
  int64_t it, end;
  int tile_dp;
  __device__ __forceinline__ explicit SegmentIter(const GemmParams& p) {
    tile_dp = blockIdx.x;
    const int64_t base = static_cast<int64_t>(p.dp_tiles) * p.num_kb;
    it = base + sk_begin(p, blockIdx.x);
    end = base + sk_begin(p, blockIdx.x + 1);
  }
  // First stream-K iteration of CTA c, relative to the stream-K region.
  __device__ __forceinline__ static int64_t sk_begin(const GemmParams& p, int c) {
    return (static_cast<int64_t>(c) * p.sk_iters) / gridDim.x;
  }
  __device__ __forceinline__ bool next(const GemmParams& p, int& tile, int& kb0, int& kb1) {
    if (tile_dp < p.dp_tiles) {
      tile = tile_dp;
      kb0 = 0;
      kb1 = p.num_kb;
      tile_dp += gridDim.x;
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

__device__ __forceinline__ int ld_acquire_flag(const int* f) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}

// Bounded wait for another CTA's flag (stream-K partials), warp-collective:
// lane 0 polls with back-off so that a waiting CTA puts a handful of
// requests on L2 rather than one per thread, then every lane re-reads the
// flag with acquire semantics before it touches the partial. All CTAs of
// the persistent grid are resident, and a CTA only waits for the first
// segment of higher-index CTAs, which is stored before they wait for
// anything.
__device__ __forceinline__ bool wait_flag(const int* f, volatile int* abort_flag) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) {
    const uint64_t t0 = global_timer_ns();
    uint32_t backoff = 32;
    while (ld_acquire_flag(f) == 0) {
      if (*abort_flag || global_timer_ns() - t0 > kWaitTimeoutNs) {
        *abort_flag = 1;
        ok = 0;
        break;
      }
      __nanosleep(backoff);
      if (backoff < 512) backoff <<= 1;
    }
  }
  ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
  if (ok) (void)ld_acquire_flag(f);
  return ok != 0;
}

__device__ __forceinline__ void tile_coords(int tile, const GemmParams& p, int& mt, int& nt) {
  const int group = p.group_m * p.tiles_n;
  const int g = tile / group;
  const int first_m = g * p.group_m;
  const int gm = min(p.tiles_m - first_m, p.group_m);
  const int w = tile - g * group;
  mt = first_m + w % gm;
  nt = w / gm;
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

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

// The k loop of one output tile: per 64-wide k-block wait for the stage, issue
// four K=16 MMAs and release the stage when they complete. With SPLIT (a
// checked tail tile of fewer than BD data columns) each step issues the data
// MMA with the runtime descriptor `idesc` and a separate N=8 MMA of the
// checksum rows into accumulator columns [BD, BN).
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

template <int BN, bool CHECK, bool SPLIT>
__device__ __forceinline__ bool mma_mainloop(uint8_t* smem, uint64_t* full, uint64_t* empty, int& stage,
                                             uint32_t& phase, int kb0, int kb1, uint32_t d, uint32_t idesc,
                                             volatile int* abort_flag) {
  using Cfg = GemmCfg<BN, CHECK>;
  constexpr int S = Cfg::kStages;
  constexpr int BD = Cfg::kBD;
  constexpr uint32_t idesc_full = umma_idesc_bf16(kBM, BN);
  constexpr uint32_t idesc_chk = umma_idesc_bf16(kBM, kChkRows);
  for (int kb = kb0; kb < kb1; ++kb) {
    if (!mbar_wait(&full[stage], phase, abort_flag)) return false;
    tc_fence_after();
    const uint32_t a_addr = smem_u32(smem + Cfg::kOffA + stage * Cfg::kABytes);
    const uint32_t b_addr = smem_u32(smem + Cfg::kOffB + stage * Cfg::kBBytes);
#pragma unroll
    for (int k = 0; k < kBK / 16; ++k) {
      const uint64_t adesc = sw128_kmajor_desc(a_addr + k * 32);
      const uint32_t accum = ((kb - kb0) | k) != 0 ? 1u : 0u;
      if (!SPLIT) {
        umma_bf16_ss(d, adesc, sw128_kmajor_desc(b_addr + k * 32), idesc_full, accum);
      } else {
        umma_bf16_ss(d, adesc, sw128_kmajor_desc(b_addr + k * 32), idesc, accum);
        umma_bf16_ss(d + BD, adesc, sw128_kmajor_desc(b_addr + BD * 128 + k * 32), idesc_chk, accum);
      }
    }
    umma_commit(&empty[stage]);
    if (++stage == S) {
      stage = 0;
      phase ^= 1u;
    }
  }
  return true;
}

template <int BN, bool CHECK>
__global__ void __launch_bounds__(kThreads, 1)
    abft_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmV, const GemmParams p) {
  using Cfg = GemmCfg<BN, CHECK>;
  constexpr int S = Cfg::kStages;
  constexpr int BD = Cfg::kBD;
  constexpr int NV = BN / 2;  // accumulator columns per epilogue thread
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* tfull = bars + 2 * S;  // [2]
  uint64_t* tempty = tfull + 2;    // [2]
  uint64_t* xbar = tempty + 2;     // [2] row-half partials exchanged
  uint64_t* drain = xbar + 2;
  uint64_t* pbar = drain + 1;  // epilogue threads stored their stream-K partial
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Cfg::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiThreads);
      mbar_init(&xbar[b], kEpiThreads);
    }
    mbar_init(drain, 1);
    mbar_init(pbar, kEpiThreads);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (CHECK) tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (blockIdx.x == 0 && threadIdx.x == 0 && p.report != nullptr) {
    p.report->capacity = static_cast<uint32_t>(p.capacity);
    p.report->tile_m = kBM;
    p.report->tile_n = BD;
    if (!(p.mode & ABFT_MODE_REF)) p.report->ref_ok = -1;
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_phase = 0;
      bool ok = true;
      constexpr uint32_t kTx = Cfg::kABytes + Cfg::kBBytes;
      SegmentIter seg(p);
      int tile, kb0, kb1;
      while (ok && seg.next(p, tile, kb0, kb1)) {
        int mt, nt;
        tile_coords(tile, p, mt, nt);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sb = smem + Cfg::kOffB + stage * Cfg::kBBytes;
          mbar_arrive_expect_tx(&full[stage], kTx);
          tma_load_2d(smem + Cfg::kOffA + stage * Cfg::kABytes, &tmA, &full[stage], kb * kBK, mt * kBM);
          tma_load_2d(sb, &tmB, &full[stage], kb * kBK, nt * BD);
          if (CHECK) tma_load_2d(sb + BD * 128, &tmV, &full[stage], kb * kBK, nt * kChkRows);
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
        for (int s = 0; s < S; ++s)
          if (issued_mask & (1u << s)) mbar_wait_unwind(&full[s], (issued_phase >> s) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_full = umma_idesc_bf16(kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      SegmentIter seg(p);
      int tile, kb0, kb1;
      while (ok && seg.next(p, tile, kb0, kb1)) {
        int mt, nt;
        tile_coords(tile, p, mt, nt);
        // A checked tail tile narrower than BD multiplies only its valid data
        // rows, then the checksum rows separately into columns [BD, BN).
        const int ncols = min(BD, p.N - nt * BD);
        const bool split = CHECK && ncols < BD;
        const uint32_t idesc_data = split ? umma_idesc_bf16(kBM, ncols) : idesc_full;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        // Full tiles keep every instruction descriptor a compile-time
        // constant; only a checked tail tile takes the runtime-N path.
        if (!split)
          ok = mma_mainloop<BN, CHECK, false>(smem, full, empty, stage, phase, kb0, kb1, d, idesc_full, abort_flag);
        else
          ok = mma_mainloop<BN, CHECK, true>(smem, full, empty, stage, phase, kb0, kb1, d, idesc_data, abort_flag);
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Every MMA this thread issued must finish before TMEM is released.
      umma_commit(drain);
      mbar_wait_unwind(drain, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // Each thread owns one output row (TMEM lane) and one column half of the
    // tile and streams it from TMEM in 32-column chunks: with checks, pass 1
    // reduces the row's checksums and pass 2 writes the corrected output;
    // the accumulator is released after pass 2 (the MMA meanwhile fills the
    // other buffer).
    const int q = warp & 3;                 // TMEM lane quadrant this warp may access
    const int h = (warp - kEpiWarp0) >> 2;  // column half of the tile
    const int r = q * 32 + lane;            // row within the tile
    const int ep = warp - kEpiWarp0;        // 0..7
    constexpr int NCH = NV / 32;            // 32-column chunks per thread
    float4* xchg = reinterpret_cast<float4*>(smem + Cfg::kOffX);
    int acc = 0;
    uint32_t acc_phase = 0;
    int xuse = 0;  // uses of the row-half exchange buffers
    SegmentIter seg(p);
    int tile, kb0, kb1;
    while (seg.next(p, tile, kb0, kb1)) {
      int mt, nt;
      tile_coords(tile, p, mt, nt);
      // Warp-uniform outcome: the tcgen05.ld below are warp-collective.
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&tfull[acc], acc_phase, abort_flag))) break;
      tc_fence_after();
      const uint32_t tacc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      const uint32_t tcol = tacc + static_cast<uint32_t>(h * NV);  // this thread's first column

      if (kb0 != 0) {
        // Stream-K contributor: the tile's first k-blocks belong to a lower
        // CTA, which finishes the tile. Hand it the fp32 partial (all BN
        // columns, checksum columns included). A segment that starts inside
        // a tile is the first segment of this CTA, so it is stored before
        // this CTA waits for anything: the wait chain is one link long.
        float4* dst = reinterpret_cast<float4*>(p.partials + (static_cast<size_t>(blockIdx.x) * kBM + r) * BN + h * NV);
#pragma unroll 1
        for (int c = 0; c < NCH; ++c) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld_32x32b_x32(tcol + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int g = 0; g < 8; ++g)
            dst[c * 8 + g] = make_float4(__uint_as_float(v[4 * g]), __uint_as_float(v[4 * g + 1]),
                                         __uint_as_float(v[4 * g + 2]), __uint_as_float(v[4 * g + 3]));
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
        __threadfence();
        mbar_arrive(pbar);
        if (ep == 0 && lane == 0 && mbar_wait(pbar, 0, abort_flag)) atomicExch(&p.flags[blockIdx.x], 1);
        continue;
      }

      uint32_t chk[kChkRows];
      if (CHECK) {
        __syncwarp();
        tmem_ld_32x32b_x8(tacc + BD, chk);
        tmem_ld_wait();
      }
      if (kb1 != p.num_kb) {
        // Stream-K finisher (this CTA owns the tile's first k-blocks): fold
        // in the partials of the CTAs that own its later k-blocks (CTAs
        // blockIdx.x+1, +2, ..., cmax), in that order, writing the sums back
        // to TMEM chunk by chunk.
        const int64_t tile_end = static_cast<int64_t>(tile - p.dp_tiles + 1) * p.num_kb;
        int cmax = static_cast<int>(blockIdx.x);
        bool okp = true;
        for (int c = static_cast<int>(blockIdx.x) + 1; c < static_cast<int>(gridDim.x); ++c) {
          if (SegmentIter::sk_begin(p, c) >= tile_end) break;
          if (!wait_flag(&p.flags[c], abort_flag)) {
            okp = false;
            break;
          }
          cmax = c;
        }
        if (!__all_sync(0xFFFFFFFFu, okp)) break;
#pragma unroll 1
        for (int c = 0; c < NCH; ++c) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld_32x32b_x32(tcol + c * 32, v);
          tmem_ld_wait();
          for (int cc = static_cast<int>(blockIdx.x) + 1; cc <= cmax; ++cc) {
            const float4* src =
                reinterpret_cast<const float4*>(p.partials + (static_cast<size_t>(cc) * kBM + r) * BN + h * NV) + c * 8;
#pragma unroll
            for (int g = 0; g < 8; ++g) {
              const float4 q4 = src[g];
              v[4 * g] = __float_as_uint(__uint_as_float(v[4 * g]) + q4.x);
              v[4 * g + 1] = __float_as_uint(__uint_as_float(v[4 * g + 1]) + q4.y);
              v[4 * g + 2] = __float_as_uint(__uint_as_float(v[4 * g + 2]) + q4.z);
              v[4 * g + 3] = __float_as_uint(__uint_as_float(v[4 * g + 3]) + q4.w);
            }
          }
          __syncwarp();
          tmem_st_32x32b_x32(tcol + c * 32, v);
        }
        tmem_st_wait();
        if (CHECK) {
          for (int cc = static_cast<int>(blockIdx.x) + 1; cc <= cmax; ++cc) {
            const float* row = p.partials + (static_cast<size_t>(cc) * kBM + r) * BN + BD;
#pragma unroll
            for (int e = 0; e < kChkRows; ++e) chk[e] = __float_as_uint(__uint_as_float(chk[e]) + row[e]);
          }
        }
      }

      const int grow = mt * kBM + r;
      const int col0 = nt * BD;
      const int ncols = min(BD, p.N - col0);
      const int hcol0 = h * NV;  // first local column of this thread
      const bool row_ok = grow < p.M;

      // Debug faults added to the fp32 accumulator (same values in both passes).
      constexpr int kMaxInj = 4;
      int inj_c[kMaxInj];
      float inj_d[kMaxInj];
      int n_my = 0;
#pragma unroll
      for (int i = 0; i < kMaxInj; ++i) {
        inj_c[i] = -1;
        inj_d[i] = 0.f;
      }
      if (p.n_inj > 0 && row_ok) {
        for (int i = 0; i < p.n_inj; ++i) {
          const int ic = p.inj_cols[i] - col0 - hcol0;
          if (p.inj_rows[i] == grow && ic >= 0 && ic < NV && hcol0 + ic < ncols && n_my < kMaxInj) {
#pragma unroll
            for (int j = 0; j < kMaxInj; ++j)
              if (j == n_my) {
                inj_c[j] = ic;
                inj_d[j] = p.inj_deltas[i];
              }
            ++n_my;
          }
        }
      }

      int fix_col = -1;  // local column to correct, if any
      float fix_delta = 0.f;
      bool aborted = false;
      if (CHECK) {
        float s1 = 0.f, s2 = 0.f, s3 = 0.f, amax = 0.f;
#pragma unroll 1
        for (int c = 0; c < NCH; ++c) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld_32x32b_x32(tcol + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            float x = __uint_as_float(v[e]);
            const int lc = c * 32 + e;  // column within this thread's half
            if (n_my) {
#pragma unroll
              for (int i = 0; i < kMaxInj; ++i) x += (inj_c[i] == lc) ? inj_d[i] : 0.f;
            }
            const int col = hcol0 + lc;
            if (col < ncols) {
              s1 += x;
              s2 = fmaf(static_cast<float>(col + 1), x, s2);
              s3 += (__popc(col) & 1) ? -x : x;
              amax = fmaxf(amax, fabsf(x));
            }
          }
        }
        // Exchange the half-row partials with the partner thread (other half);
        // amax >= 0 and s3 rides in .w.
        const int xb = xuse & 1;
        const uint32_t xphase = (xuse >> 1) & 1u;
        ++xuse;
        xchg[(xb * 2 + h) * kBM + r] = make_float4(s1, s2, amax, s3);
        mbar_arrive(&xbar[xb]);
        if (!mbar_wait(&xbar[xb], xphase, abort_flag)) {
          aborted = true;
        } else {
          const float4 p0 = xchg[(xb * 2 + 0) * kBM + r];
          const float4 p1 = xchg[(xb * 2 + 1) * kBM + r];
          const float t1 = p0.x + p1.x;
          const float t2 = p0.y + p1.y;
          const float t3 = p0.w + p1.w;
          const float tmax = fmaxf(p0.z, p1.z);
          const float e1 = (__uint_as_float(chk[0]) + __uint_as_float(chk[1])) + __uint_as_float(chk[2]);
          const float e2 = (__uint_as_float(chk[3]) + __uint_as_float(chk[4])) + __uint_as_float(chk[5]);
          const float e3 = __uint_as_float(chk[6]) + __uint_as_float(chk[7]);
          const float res1 = t1 - e1;
          const float res2 = t2 - e2;
          const float res3 = t3 - e3;
          const float thr = fmaf(p.thr_k, tmax, p.thr_abs);
          const bool det = row_ok && (fabsf(res1) > thr || fabsf(res2) > thr * static_cast<float>(ncols));
          if (det) {
            uint32_t flags = ABFT_REC_DETECTED;
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
              fix_col = col;
              fix_delta = res1;
              flags |= ABFT_REC_CORRECTED;
            }
            if (h == 0) {
              abft_report* rep = p.report;
              const uint32_t slot = atomicAdd(&rep->n_faults, 1u);
              if (flags & ABFT_REC_LOCATED) atomicAdd(&rep->n_located, 1u);
              if (flags & ABFT_REC_CORRECTED) atomicAdd(&rep->n_corrected, 1u);
              uint32_t st = ABFT_STATUS_FAULT | ((flags & ABFT_REC_LOCATED) ? 0u : ABFT_STATUS_UNLOCATED);
              if (slot < static_cast<uint32_t>(p.capacity)) {
                abft_fault_record* rec = reinterpret_cast<abft_fault_record*>(rep + 1) + slot;
                rec->row = grow;
                rec->col = col >= 0 ? col0 + col : -1;
                rec->residual = res1;
                rec->residual_w = res2;
                rec->threshold = thr;
                rec->flags = flags;
              } else {
                atomicAdd(&rep->overflow, 1u);
                st |= ABFT_STATUS_OVERFLOW;
              }
              atomicOr(&rep->status, st);
            }
          }
        }
      }

      // Pass 2: final values -> bf16 -> global.
      const int fix_local = fix_col - hcol0;  // column within this thread's half, or out of range
      float row_out_sum = 0.f;
      __nv_bfloat16* crow = p.C + static_cast<int64_t>(grow) * p.ldc + col0 + hcol0;
      const uint4* bp = reinterpret_cast<const uint4*>(p.bias + col0 + hcol0);
#pragma unroll 1
      for (int c = 0; c < NCH; ++c) {
        uint32_t v[32];
        __syncwarp();
        tmem_ld_32x32b_x32(tcol + c * 32, v);
        tmem_ld_wait();
        float x[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          x[e] = __uint_as_float(v[e]);
          const int lc = c * 32 + e;
          if (n_my) {
#pragma unroll
            for (int i = 0; i < kMaxInj; ++i) x[e] += (inj_c[i] == lc) ? inj_d[i] : 0.f;
          }
          if (fix_col >= 0) x[e] -= (fix_local == lc) ? fix_delta : 0.f;
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int gcol = c * 32 + g * 8;  // first column of this 8-column group within the half
          const bool gvalid = row_ok && (hcol0 + gcol < ncols);
          if (p.bias != nullptr && gvalid) {
            const uint4 bw = __ldg(bp + (gcol >> 3));
            x[g * 8 + 0] += bf16_lo(bw.x);
            x[g * 8 + 1] += bf16_hi(bw.x);
            x[g * 8 + 2] += bf16_lo(bw.y);
            x[g * 8 + 3] += bf16_hi(bw.y);
            x[g * 8 + 4] += bf16_lo(bw.z);
            x[g * 8 + 5] += bf16_hi(bw.z);
            x[g * 8 + 6] += bf16_lo(bw.w);
            x[g * 8 + 7] += bf16_hi(bw.w);
          }
          const uint4 packed =
              make_uint4(pack_bf16x2(x[g * 8 + 0], x[g * 8 + 1]), pack_bf16x2(x[g * 8 + 2], x[g * 8 + 3]),
                         pack_bf16x2(x[g * 8 + 4], x[g * 8 + 5]), pack_bf16x2(x[g * 8 + 6], x[g * 8 + 7]));
          if (gvalid) {
            reinterpret_cast<uint4*>(crow)[gcol >> 3] = packed;
            if (p.mode & ABFT_MODE_REF) {
              row_out_sum += ((bf16_lo(packed.x) + bf16_hi(packed.x)) + (bf16_lo(packed.y) + bf16_hi(packed.y))) +
                             ((bf16_lo(packed.z) + bf16_hi(packed.z)) + (bf16_lo(packed.w) + bf16_hi(packed.w)));
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
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
        if (lane == 0) p.tile_sumc[tile * 8 + ep] = row_out_sum;
      }
      if (aborted) break;
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag && p.report != nullptr) atomicOr(&p.report->status, ABFT_STATUS_DEVICE_TIMEOUT);
}

}  // namespace abft
