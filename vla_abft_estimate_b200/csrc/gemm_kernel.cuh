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
// The checksum block holds v1 and v2 each split into three bf16 terms
// (hi + mid + lo, 24 significant bits) plus two zero rows. A single corrupted
// C[i,j*] (+delta) gives s1 - e1 = delta and s2 - e2 = (j*+1) delta: the
// ratio pins the column, and delta is subtracted before the bf16 store.
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
  static constexpr int kNumBars = 2 * kStages + 2 * 3 + 1;  // full, empty, tfull, tempty, xbar, drain
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
};

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
template <int BN, bool CHECK, bool SPLIT>
__device__ __forceinline__ bool mma_mainloop(uint8_t* smem, uint64_t* full, uint64_t* empty, int& stage,
                                             uint32_t& phase, int num_kb, uint32_t d, uint32_t idesc,
                                             volatile int* abort_flag) {
  using Cfg = GemmCfg<BN, CHECK>;
  constexpr int S = Cfg::kStages;
  constexpr int BD = Cfg::kBD;
  constexpr uint32_t idesc_full = umma_idesc_bf16(kBM, BN);
  constexpr uint32_t idesc_chk = umma_idesc_bf16(kBM, kChkRows);
  for (int kb = 0; kb < num_kb; ++kb) {
    if (!mbar_wait(&full[stage], phase, abort_flag)) return false;
    tc_fence_after();
    const uint32_t a_addr = smem_u32(smem + Cfg::kOffA + stage * Cfg::kABytes);
    const uint32_t b_addr = smem_u32(smem + Cfg::kOffB + stage * Cfg::kBBytes);
#pragma unroll
    for (int k = 0; k < kBK / 16; ++k) {
      const uint64_t adesc = sw128_kmajor_desc(a_addr + k * 32);
      const uint32_t accum = (kb | k) != 0 ? 1u : 0u;
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
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        int mt, nt;
        tile_coords(tile, p, mt, nt);
        for (int kb = 0; kb < p.num_kb; ++kb) {
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
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
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
          ok = mma_mainloop<BN, CHECK, false>(smem, full, empty, stage, phase, p.num_kb, d, idesc_full, abort_flag);
        else
          ok = mma_mainloop<BN, CHECK, true>(smem, full, empty, stage, phase, p.num_kb, d, idesc_data, abort_flag);
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
    const int q = warp & 3;                 // TMEM lane quadrant this warp may access
    const int h = (warp - kEpiWarp0) >> 2;  // column half of the tile
    const int r = q * 32 + lane;            // row within the tile
    const int ep = warp - kEpiWarp0;        // 0..7
    float4* xchg = reinterpret_cast<float4*>(smem + Cfg::kOffX);
    int acc = 0;
    uint32_t acc_phase = 0;
    int local_tile = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++local_tile) {
      int mt, nt;
      tile_coords(tile, p, mt, nt);
      // Warp-uniform outcome: the tcgen05.ld below are warp-collective.
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&tfull[acc], acc_phase, abort_flag))) break;
      tc_fence_after();
      const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
      const uint32_t tacc = tmem_base + lane_base + static_cast<uint32_t>(acc * BN);
      uint32_t v[NV];
#pragma unroll
      for (int c = 0; c < NV / 32; ++c)
        tmem_ld_32x32b_x32(tacc + h * NV + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
      uint32_t chk[kChkRows];
      if (CHECK) tmem_ld_32x32b_x8(tacc + BD, chk);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }

      const int grow = mt * kBM + r;
      const int col0 = nt * BD;
      const int ncols = min(BD, p.N - col0);
      const int hcol0 = h * NV;  // first local column of this thread
      const bool row_ok = grow < p.M;

      // Debug fault injection into the fp32 accumulator.
      if (p.n_inj > 0 && row_ok) {
        for (int i = 0; i < p.n_inj; ++i) {
          const int ic = p.inj_cols[i] - col0 - hcol0;
          if (p.inj_rows[i] == grow && ic >= 0 && ic < NV && hcol0 + ic < ncols) {
            const float dlt = p.inj_deltas[i];
#pragma unroll
            for (int e = 0; e < NV; ++e)
              if (e == ic) v[e] = __float_as_uint(__uint_as_float(v[e]) + dlt);
          }
        }
      }

      int fix_col = -1;  // local column to correct, if any
      float fix_delta = 0.f;
      bool aborted = false;
      if (CHECK) {
        float s1 = 0.f, s2 = 0.f, amax = 0.f;
#pragma unroll
        for (int e = 0; e < NV; ++e) {
          const float x = __uint_as_float(v[e]);
          const int col = hcol0 + e;
          if (col < ncols) {
            s1 += x;
            s2 = fmaf(static_cast<float>(col + 1), x, s2);
            amax = fmaxf(amax, fabsf(x));
          }
        }
        // Exchange the half-row partials with the partner thread (other half).
        const int xb = local_tile & 1;
        xchg[(xb * 2 + h) * kBM + r] = make_float4(s1, s2, amax, 0.f);
        mbar_arrive(&xbar[xb]);
        if (!mbar_wait(&xbar[xb], (local_tile >> 1) & 1u, abort_flag)) {
          aborted = true;
        } else {
          const float4 p0 = xchg[(xb * 2 + 0) * kBM + r];
          const float4 p1 = xchg[(xb * 2 + 1) * kBM + r];
          const float t1 = p0.x + p1.x;
          const float t2 = p0.y + p1.y;
          const float tmax = fmaxf(p0.z, p1.z);
          const float e1 = (__uint_as_float(chk[0]) + __uint_as_float(chk[1])) + __uint_as_float(chk[2]);
          const float e2 = (__uint_as_float(chk[3]) + __uint_as_float(chk[4])) + __uint_as_float(chk[5]);
          const float res1 = t1 - e1;
          const float res2 = t2 - e2;
          const float thr = fmaf(p.thr_k, tmax, p.thr_abs);
          const bool det = row_ok && (fabsf(res1) > thr || fabsf(res2) > thr * static_cast<float>(ncols));
          if (det) {
            uint32_t flags = ABFT_REC_DETECTED;
            int col = -1;
            if (fabsf(res1) > thr) {
              const float pos = res2 / res1;
              const float pr = rintf(pos);
              if (fabsf(pos - pr) <= 0.1f && pr >= 1.f && pr <= static_cast<float>(ncols)) {
                col = static_cast<int>(pr) - 1;
                flags |= ABFT_REC_LOCATED;
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

      // Final values -> bf16 -> global.
      const int fix_local = fix_col - hcol0;
      if (fix_col >= 0 && fix_local >= 0 && fix_local < NV) {
#pragma unroll
        for (int e = 0; e < NV; ++e)
          if (e == fix_local) v[e] = __float_as_uint(__uint_as_float(v[e]) - fix_delta);
      }
      float row_out_sum = 0.f;
      __nv_bfloat16* crow = p.C + static_cast<int64_t>(grow) * p.ldc + col0 + hcol0;
      const uint4* bp = reinterpret_cast<const uint4*>(p.bias + col0 + hcol0);
#pragma unroll
      for (int g = 0; g < NV / 8; ++g) {
        const bool gvalid = row_ok && (hcol0 + g * 8 < ncols);
        float x[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = __uint_as_float(v[g * 8 + e]);
        if (p.bias != nullptr && gvalid) {
          const uint4 bw = __ldg(bp + g);
          x[0] += bf16_lo(bw.x);
          x[1] += bf16_hi(bw.x);
          x[2] += bf16_lo(bw.y);
          x[3] += bf16_hi(bw.y);
          x[4] += bf16_lo(bw.z);
          x[5] += bf16_hi(bw.z);
          x[6] += bf16_lo(bw.w);
          x[7] += bf16_hi(bw.w);
        }
        const uint4 packed = make_uint4(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]), pack_bf16x2(x[4], x[5]),
                                        pack_bf16x2(x[6], x[7]));
        if (gvalid) {
          reinterpret_cast<uint4*>(crow)[g] = packed;
          if (p.mode & ABFT_MODE_REF) {
            row_out_sum += ((bf16_lo(packed.x) + bf16_hi(packed.x)) + (bf16_lo(packed.y) + bf16_hi(packed.y))) +
                           ((bf16_lo(packed.z) + bf16_hi(packed.z)) + (bf16_lo(packed.w) + bf16_hi(packed.w)));
          }
        }
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
