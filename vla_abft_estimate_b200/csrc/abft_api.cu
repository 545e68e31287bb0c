// abft_api.cu - the extern "C" entry points of libabft_b200.so.
//
// Host side of the library: argument validation, TMA tensor-map encoding,
// workspace layout and the launch sequence of each call. Declarations and the
// reference interface each entry replaces are in include/abft_b200.h.
#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>

#include <string.h>

#include <atomic>
#include <mutex>
#include <random>

#include "aux_kernels.cuh"
#include "gemm_kernel.cuh"

using namespace abft;

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

constexpr int kMaxDevices = 64;
struct DeviceInfo {
  bool init;
  bool ok;
  int sms;
  bool attr_set[16];  // slots 8..15: the fp16 instances of slots 0..7
  int pair_clusters[2][2];  // co-resident 2-CTA clusters of the pair kernels [bn == 256][check], 0 = not asked yet
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_mu;

int current_device(int* dev_out, DeviceInfo* info) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return ABFT_ERR_NO_DEVICE;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.init) {
    int major = 0, minor = 0, sms = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaGetLastError();
    d.ok = (major == 10 && minor == 0);
    d.sms = sms;
    d.init = true;
  }
  if (!d.ok) return ABFT_ERR_NO_DEVICE;
  *dev_out = dev;
  *info = d;
  return ABFT_OK;
}

template <int BN, bool CHECK, bool PAIR, bool F16 = false>
int ensure_smem_attr_locked(int dev, int slot) {
  if (F16) slot += 8;
  if (g_dev[dev].attr_set[slot]) return ABFT_OK;
  if (cudaFuncSetAttribute(abft_gemm_kernel<BN, CHECK, PAIR, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           GemmCfg<BN, CHECK, PAIR>::kSmemBytes) != cudaSuccess) {
    cudaGetLastError();
    return ABFT_ERR_CUDA;
  }
  g_dev[dev].attr_set[slot] = true;
  return ABFT_OK;
}

template <int BN, bool CHECK, bool PAIR, bool F16>
int ensure_smem_attr(int dev, int slot) {
  std::lock_guard<std::mutex> lk(g_mu);
  return ensure_smem_attr_locked<BN, CHECK, PAIR, F16>(dev, slot);
}

// attr_set slots of the pair kernels [bn == 256][check]
constexpr int kPairSlot[2][2] = {{7, 6}, {5, 4}};

cudaLaunchAttribute pair_cluster_attr() {
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeClusterDimension;
  at.val.clusterDim.x = 2;
  at.val.clusterDim.y = 1;
  at.val.clusterDim.z = 1;
  return at;
}

// How many 2-CTA clusters of the pair kernel can be resident at once on
// device `dev` (every unit of a persistent launch must be resident: stream-K
// finishers wait for later units). Falls back to sms / 2 if the query fails.
// The bf16 instance answers for both element types: the fp16 one has the
// same block, shared-memory footprint and register bound (128 per thread).
template <int BN, bool CHECK>
int pair_units_on(int dev, int sms) {
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceInfo& d = g_dev[dev];
  int& cached = d.pair_clusters[BN == 256][CHECK];
  if (cached == 0) {
    int n = 0;
    if (ensure_smem_attr_locked<BN, CHECK, true>(dev, kPairSlot[BN == 256][CHECK]) == ABFT_OK) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * static_cast<unsigned>(sms / 2));
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = GemmCfg<BN, CHECK, true>::kSmemBytes;
      cudaLaunchAttribute at = pair_cluster_attr();
      cfg.attrs = &at;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, abft_gemm_kernel<BN, CHECK, true, false>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
    }
    cached = n > 0 ? n : sms / 2;
  }
  return cached < sms / 2 ? cached : sms / 2;
}

// Encoded tensor maps are a pure function of (kind, address, extents,
// strides, box): a small per-thread direct-mapped cache skips the encoder
// for operands seen before (weights every call; activation and output
// buffers whenever the caller's allocator hands back the same block).
struct TmapKey {
  const void* ptr;
  int64_t inner, outer, ld, batch, bstride;
  int box, kind;  // kind: 0 operand, 1 output; + 2 for fp16 elements
  bool operator==(const TmapKey& o) const {
    return ptr == o.ptr && inner == o.inner && outer == o.outer && ld == o.ld && batch == o.batch &&
           bstride == o.bstride && box == o.box && kind == o.kind;
  }
};
struct TmapEntry {
  TmapKey key;
  CUtensorMap map;
  bool valid;
};
constexpr int kTmapCacheSize = 64;
thread_local TmapEntry t_tmaps[kTmapCacheSize];

TmapEntry& tmap_slot(const TmapKey& k) {
  uint64_t h = reinterpret_cast<uintptr_t>(k.ptr) >> 4;
  h ^= static_cast<uint64_t>(k.outer) * 0x9E3779B97F4A7C15ull;
  h ^= static_cast<uint64_t>(k.box * 8 + k.kind) * 0xC2B2AE3D27D4EB4Full;
  h ^= h >> 29;
  return t_tmaps[h % kTmapCacheSize];
}

inline CUtensorMapDataType tmap_type(int dtype) {
  return dtype == ABFT_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// A 3-D map over `batch` row-major [outer, ld] matrices of 16-bit elements
// (bf16 or fp16, `dtype`), matrix b at ptr + b * bstride elements (bstride
// ignored for batch <= 1), read in boxes of 64 (inner) x box_outer rows x 1
// matrix with 128-byte swizzle.
int make_tmap_kmajor(CUtensorMap* m, const void* ptr, int64_t inner, int64_t outer, int64_t ld, int box_outer,
                     int64_t batch = 1, int64_t bstride = 0, int dtype = ABFT_DTYPE_BF16) {
  if (batch <= 1) {
    batch = 1;
    bstride = ld * outer;
  }
  const TmapKey key{ptr, inner, outer, ld, batch, bstride, box_outer, dtype == ABFT_DTYPE_F16 ? 2 : 0};
  TmapEntry& e = tmap_slot(key);
  if (e.valid && e.key == key) {
    *m = e.map;
    return ABFT_OK;
  }
  EncodeTiledFn enc = get_encoder();
  if (enc == nullptr) return ABFT_ERR_DRIVER;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer), static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 2, static_cast<cuuint64_t>(bstride) * 2};
  cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(box_outer), 1u};
  cuuint32_t es[3] = {1u, 1u, 1u};
  CUresult r = enc(m, tmap_type(dtype), 3, const_cast<void*>(ptr), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return ABFT_ERR_ALIGNMENT;
  e.key = key;
  e.map = *m;
  e.valid = true;
  return ABFT_OK;
}

// The output map: `batch` row-major [rows, ld] bf16 or fp16 matrices
// (matrix b at ptr + b * bstride elements), stored in 32 x 32 boxes whose
// shared-memory source uses the 64-byte swizzle (an epilogue warp's staging
// block).
int make_tmap_store(CUtensorMap* m, void* ptr, int64_t cols, int64_t rows, int64_t ld, int64_t batch,
                    int64_t bstride, int dtype) {
  if (batch <= 1) {
    batch = 1;
    bstride = ld * rows;
  }
  const TmapKey key{ptr, cols, rows, ld, batch, bstride, 32, dtype == ABFT_DTYPE_F16 ? 3 : 1};
  TmapEntry& e = tmap_slot(key);
  if (e.valid && e.key == key) {
    *m = e.map;
    return ABFT_OK;
  }
  EncodeTiledFn enc = get_encoder();
  if (enc == nullptr) return ABFT_ERR_DRIVER;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 2, static_cast<cuuint64_t>(bstride) * 2};
  cuuint32_t box[3] = {32u, 32u, 1u};
  cuuint32_t es[3] = {1u, 1u, 1u};
  CUresult r = enc(m, tmap_type(dtype), 3, ptr, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return ABFT_ERR_ALIGNMENT;
  e.key = key;
  e.map = *m;
  e.valid = true;
  return ABFT_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// A value unique to one fused launch: stream-K flags and report->launch_tag
// carry it, so neither needs clearing before the launch (a stale value from
// another launch differs). Distinct for 2^64 calls in a process (an odd
// multiplier makes the counter map one-to-one); the random salt separates
// processes; never 0, the content of zeroed memory.
uint64_t next_launch_nonce() {
  static std::atomic<uint64_t> counter{0};
  static const uint64_t salt = [] {
    std::random_device rd;
    return (static_cast<uint64_t>(rd()) << 32) ^ static_cast<uint64_t>(rd());
  }();
  const uint64_t n = salt + (counter.fetch_add(1, std::memory_order_relaxed) + 1) * 0x9E3779B97F4A7C15ull;
  return n != 0 ? n : 1;
}

int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ABFT_OK : ABFT_ERR_CUDA;
}

// Rows per block of a column-sum pass: enough row blocks that the grid has
// at least two blocks per SM.
int rows_per_block(int64_t R, int64_t C, int sms) {
  const int64_t col_blocks = cdiv(C, 64);
  const int64_t want_rb = cdiv(2 * static_cast<int64_t>(sms), col_blocks);
  int64_t rpb = cdiv(R, want_rb < 1 ? 1 : want_rb);
  rpb = cdiv(rpb, 32) * 32;
  if (rpb < 32) rpb = 32;
  return static_cast<int>(rpb);
}

// Column sums of a row-major [R, C] matrix of element type `dtype` into
// out[C] (with stats also out_max[C] and out_abs[C]), through partials in
// `partial` ([nrb][C], and 2 * [nrb][C] more with stats).
int colsum(const void* X, int64_t ld, int64_t R, int64_t C, const float* w, float* partial, float* out,
           float* out_max, float* out_abs, int sms, cudaStream_t s, int dtype = ABFT_DTYPE_BF16) {
  const int rpb = rows_per_block(R, C, sms);
  const int nrb = static_cast<int>(cdiv(R, rpb));
  float* pstat = out_max != nullptr ? partial + static_cast<int64_t>(nrb) * C : nullptr;
  dim3 g(static_cast<unsigned>(cdiv(C, 64)), static_cast<unsigned>(nrb));
  const int r = static_cast<int>(R), c = static_cast<int>(C);
  if (dtype == ABFT_DTYPE_F16)
    colsum_partial_kernel<<<g, 256, 0, s>>>(static_cast<const __half*>(X), ld, r, c, rpb, w, partial, pstat);
  else if (dtype == ABFT_DTYPE_F32)
    colsum_partial_kernel<<<g, 256, 0, s>>>(static_cast<const float*>(X), ld, r, c, rpb, w, partial, pstat);
  else
    colsum_partial_kernel<<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(X), ld, r, c, rpb, w, partial, pstat);
  reduce_partials_kernel<<<static_cast<unsigned>(cdiv(C, 256)), 256, 0, s>>>(partial, pstat, nrb, c, out, out_max,
                                                                             out_abs);
  return launch_status();
}

size_t colsum_partial_floats(int64_t R, int64_t C, int sms, bool with_stats) {
  const int rpb = rows_per_block(R, C, sms);
  return static_cast<size_t>(cdiv(R, rpb)) * C * (with_stats ? 3 : 1);
}

int rowdot(const void* X, int64_t ld, int64_t R, int64_t C, const float* vec, float* out, float* out_max,
           float* out_abs, cudaStream_t s, int dtype = ABFT_DTYPE_BF16) {
  const unsigned g = static_cast<unsigned>(cdiv(R, 8));
  const int r = static_cast<int>(R), c = static_cast<int>(C);
  if (dtype == ABFT_DTYPE_F16)
    rowdot_kernel<<<g, 256, 0, s>>>(static_cast<const __half*>(X), ld, r, c, vec, out, out_max, out_abs);
  else if (dtype == ABFT_DTYPE_F32)
    rowdot_kernel<<<g, 256, 0, s>>>(static_cast<const float*>(X), ld, r, c, vec, out, out_max, out_abs);
  else
    rowdot_kernel<<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(X), ld, r, c, vec, out, out_max, out_abs);
  return launch_status();
}

// ref_finalize_kernel / locate_finalize_kernel with the bias (and the
// rounding of native sums) of element type `dtype`.
void ref_finalize(int dtype, const float* u, const float* v, int K, const void* bias, int N, int M, const float* parts,
                  int n_parts, float tol_abs, float tol_rel, int native_sums, abft_report* rep, int capacity,
                  int tile_m, int tile_n, cudaStream_t s) {
  if (dtype == ABFT_DTYPE_F16)
    ref_finalize_kernel<<<1, 1024, 0, s>>>(u, v, K, static_cast<const __half*>(bias), N, M, parts, n_parts, tol_abs,
                                           tol_rel, native_sums, rep, capacity, tile_m, tile_n);
  else if (dtype == ABFT_DTYPE_F32)
    ref_finalize_kernel<<<1, 1024, 0, s>>>(u, v, K, static_cast<const float*>(bias), N, M, parts, n_parts, tol_abs,
                                           tol_rel, native_sums, rep, capacity, tile_m, tile_n);
  else
    ref_finalize_kernel<<<1, 1024, 0, s>>>(u, v, K, static_cast<const __nv_bfloat16*>(bias), N, M, parts, n_parts,
                                           tol_abs, tol_rel, native_sums, rep, capacity, tile_m, tile_n);
}

// Rounding bound of a stored element relative to its magnitude, 2^-(p+1)
// for p significand bits (the convention the bf16 bound 2^-9 set).
float unit_roundoff(int dtype) {
  return dtype == ABFT_DTYPE_F32 ? 1.0f / 33554432.0f : (dtype == ABFT_DTYPE_F16 ? 1.0f / 4096.0f : 1.0f / 512.0f);
}

// Tile schedule of one launch. Whole-tile (data-parallel) waves first; when
// the last wave would leave units idle, its tiles may instead run stream-K
// over the first sk_ctas units: each gets an equal share of those tiles'
// k-block iterations, and partial tiles meet in the workspace. More units
// shorten the tail but cut each tile into more pieces, and every extra piece
// costs the finisher one partial fold. Estimated times, in k-block steps of
// one unit:
//   data-parallel tail   (waves + 1) * num_kb
//   stream-K over G      waves * num_kb + ceil(W / G) + store + fold * (pieces - 1)
// with W = rem * num_kb and pieces the most unit ranges one tile can meet.
// A compact tail tile counts as a full one: its narrow MMA is cheap, but it
// streams the same A slices through the load pipeline.
// store: a contributor writes its partial tile and publishes the flag, and
// the finisher sees it; fold: the finisher adds one partial into TMEM.
// Measured in microseconds; one k-block step of a 256-wide tile takes about
// kKbUs256 (kKbFrac128 of that for a 128-wide tile). The constants rank the
// candidate schedules; they do not predict absolute times (the epilogue of
// the last wave and the launch are left out). Fitted to bench.py
// --tile-grid (all four tile shapes interleaved, 14 GEMM shapes, checks off
// and on): the pick is the fastest tile shape or within 3.2% of it (one
// timer step) on every shape.
constexpr double kSkStoreUs = 3.0;
constexpr double kSkFoldUs = 1.0;
constexpr double kKbUs256 = 0.33;
// A 128-wide tile's k-block takes this fraction of a 256-wide one: half the
// MMA work, but the same A slice streams from shared memory.
constexpr double kKbFrac128 = 0.7;

double kb_us(int bn) { return bn == 256 ? kKbUs256 : kKbUs256 * kKbFrac128; }

struct Schedule {
  int grid;  // units
  int dp_tiles;
  int sk;
  int sk_ctas;
  int64_t sk_iters;
  double est;  // estimated duration in k-block steps
};

// Rows of the last tile column's data box: its data columns rounded up to 8,
// so that the checksum rows after them start on a 1024-byte swizzle atom
// (the rows past N are zero-filled by the copy).
int tail_rows(int64_t N, int bd) {
  const int64_t tiles_n = cdiv(N, bd);
  return (static_cast<int>(N - (tiles_n - 1) * bd) + 7) / 8 * 8;
}

// MMA width of the last tile column's compact tile (its data rows, then with
// checks the 8 checksum rows), or 0 when that column needs no narrower MMA.
int tail_width(int64_t N, int bd, int bn, bool check) {
  const int rows = tail_rows(N, bd);
  const int tn = (rows + (check ? kChkRows : 0) + 15) / 16 * 16;
  return (rows < bd && tn < bn) ? tn : 0;
}

Schedule make_schedule(int64_t tiles, int num_kb, int units, int bn) {
  const double store = kSkStoreUs / kb_us(bn), fold = kSkFoldUs / kb_us(bn);
  Schedule s;
  s.sk = 0;
  s.sk_ctas = 0;
  s.sk_iters = 0;
  s.dp_tiles = static_cast<int>(tiles);
  s.grid = static_cast<int>(tiles < units ? tiles : units);
  s.est = static_cast<double>(cdiv(tiles, units)) * num_kb;
  const int64_t waves = tiles / units, rem = tiles % units;
  if (rem == 0 || num_kb < 2) return s;
  const int64_t w = rem * num_kb;
  int64_t best_g = 0;
  for (int64_t g = rem + 1; g <= units && g <= w; ++g) {
    const int64_t lmin = w / g;  // shortest unit range
    const int64_t pieces = cdiv(num_kb - 1, lmin) + 1;
    const double t = static_cast<double>(waves * num_kb + cdiv(w, g)) + store + fold * (pieces - 1);
    if (t < s.est) {
      s.est = t;
      best_g = g;
    }
  }
  if (best_g == 0) return s;
  s.sk = 1;
  s.sk_ctas = static_cast<int>(best_g);
  s.sk_iters = w;
  s.dp_tiles = static_cast<int>(waves * units);
  s.grid = waves > 0 ? units : static_cast<int>(best_g);
  return s;
}

// Schedule of `batch` M x N x K products with tile_m x bn tiles (bd data
// columns) over `units` units.
Schedule schedule_for(int64_t M, int64_t N, int64_t K, int tile_m, int bn, int bd, int units, int64_t batch = 1) {
  return make_schedule(batch * cdiv(M, tile_m) * cdiv(N, bd), static_cast<int>(cdiv(K, kBK)), units, bn);
}

// A CTA pair runs a 128 x 256 share of a tile per SM about this much faster
// than a single CTA (each CTA stages half the B-operand tile per k-block).
// Pairs of 128-wide tiles run a k-block no faster than single 128 x 128
// CTAs (0.32 against 0.31 us, bench.py --tile-grid) and leave half the
// units: they are available on request (tile_m 256, tile_n 128) but never
// picked.
constexpr double kPairSpeedup = 1.15;

// Estimated time (microseconds) of an M x N x K launch with tile_m x bn
// tiles (tile_m 256: CTA pairs over `units` pairs).
double est_time(int64_t M, int64_t N, int64_t K, int bn, bool check, int tile_m, int units, int64_t batch = 1) {
  const int bd = check ? bn - kChkRows : bn;
  const double t = schedule_for(M, N, K, tile_m, bn, bd, units, batch).est * kb_us(bn);
  return tile_m == 256 ? t / kPairSpeedup : t;
}

int pick_tile_m(int64_t M, int64_t N, int64_t K, int sms, uint32_t mode, int bn, int64_t batch = 1) {
  if (bn != 256 || sms < 2 || M <= 0 || N <= 0 || K <= 0) return 128;
  const bool check = (mode & (ABFT_MODE_DETECT | ABFT_MODE_CORRECT)) != 0;
  return est_time(M, N, K, bn, check, 256, sms / 2, batch) < est_time(M, N, K, bn, check, 128, sms, batch) ? 256
                                                                                                           : 128;
}

// abft_pick_tile_n for `batch` products.
int pick_tile_n(int64_t M, int64_t N, int64_t K, int sms, uint32_t mode, int64_t batch) {
  if (sms <= 0) sms = 148;
  if (M <= 0 || N <= 0 || K <= 0) return 256;
  const bool check = (mode & (ABFT_MODE_DETECT | ABFT_MODE_CORRECT)) != 0;
  double best_cost = 0.0;
  int best = 256;
  for (int bn : {256, 128}) {
    double cost = est_time(M, N, K, bn, check, 128, sms, batch);
    if (bn == 256 && sms >= 2) {
      const double tp = est_time(M, N, K, bn, check, 256, sms / 2, batch);
      if (tp < cost) cost = tp;
    }
    if (bn == 256 || cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

inline int64_t batch_of(const abft_gemm_args* a) { return a->batch > 1 ? a->batch : 1; }

// Swapped operands: with few output rows the weight goes on the MMA's
// 128-row side and the rows of A form one narrow tile, C^T = B A^T.
bool use_swap(const abft_gemm_args* a) {
  if (a->swap_ab == 1) return false;
  if (a->swap_ab == 2) return true;
  // automatic only when the caller left the tile height to the library
  return a->tile_m == 0 && a->M <= 64 && a->N >= 2 * a->M;
}

// The arguments in the swapped frame: A' = B (the weight, [N, K]), B' = A
// ([M, K]); C, ldc and the bias keep their memory meaning (the kernel stores
// transposed and indexes the bias by its row); checksums of A' are made per
// call; injected faults keep their C coordinates by exchanging the arrays.
abft_gemm_args swapped_args(const abft_gemm_args* a) {
  abft_gemm_args s = *a;
  s.A = a->B;
  s.B = a->A;
  s.M = a->N;
  s.N = a->M;
  s.lda = a->ldb;
  s.ldb = a->lda;
  s.stride_a = a->stride_b;
  s.stride_b = a->stride_a;
  s.checksums = nullptr;
  s.tile_n = 128;
  s.tile_m = 128;
  s.inject_rows = a->inject_cols;
  s.inject_cols = a->inject_rows;
  return s;
}

// Everything about a launch that depends only on the arguments and the
// device: tile shape, unit count, schedule and workspace layout.
struct Plan {
  bool check, pair;
  int bn, bd, tile_m, units, grid, num_kb;
  int64_t tiles;
  Schedule sch;
  size_t v_off, pa_off, u_off, pb_off, vf_off, parts_off, sk_part_off, sk_flag_off, total;
};

// dev < 0: no device to ask (co-resident pairs assumed sms / 2).
int make_plan_uncached(const abft_gemm_args* a, int dev, int sms, Plan* pl);

// Plans depend on the shape, mode, tile requests, batch and device only: a
// per-thread direct-mapped cache keeps the tile search off repeated calls.
struct PlanKey {
  int64_t M, N, K, batch;
  uint32_t mode;
  int tile_n, tile_m, has_cks, dev, sms, dtype;
  bool operator==(const PlanKey& o) const {
    return M == o.M && N == o.N && K == o.K && batch == o.batch && mode == o.mode && tile_n == o.tile_n &&
           tile_m == o.tile_m && has_cks == o.has_cks && dev == o.dev && sms == o.sms && dtype == o.dtype;
  }
};
struct PlanEntry {
  PlanKey key;
  Plan plan;
  bool valid;
};
constexpr int kPlanCacheSize = 32;
thread_local PlanEntry t_plans[kPlanCacheSize];

int make_plan(const abft_gemm_args* a, int dev, int sms, Plan* pl) {
  const PlanKey key{a->M, a->N, a->K, batch_of(a), a->mode, a->tile_n, a->tile_m, a->checksums != nullptr ? 1 : 0,
                    dev, sms, a->dtype};
  uint64_t h = static_cast<uint64_t>(a->M) * 0x9E3779B97F4A7C15ull ^ static_cast<uint64_t>(a->N) * 0xC2B2AE3D27D4EB4Full ^
               static_cast<uint64_t>(a->K) * 0x165667B19E3779F9ull ^ (static_cast<uint64_t>(key.batch) << 7) ^
               (static_cast<uint64_t>(a->mode) << 3) ^ static_cast<uint64_t>(a->tile_n + a->tile_m + key.has_cks);
  h ^= h >> 31;
  PlanEntry& e = t_plans[h % kPlanCacheSize];
  if (e.valid && e.key == key) {
    *pl = e.plan;
    return ABFT_OK;
  }
  const int rc = make_plan_uncached(a, dev, sms, pl);
  if (rc == ABFT_OK) {
    e.key = key;
    e.plan = *pl;
    e.valid = true;
  }
  return rc;
}

int make_plan_uncached(const abft_gemm_args* a, int dev, int sms, Plan* pl) {
  const int64_t nb = batch_of(a);
  pl->check = (a->mode & (ABFT_MODE_DETECT | ABFT_MODE_CORRECT)) != 0;
  pl->bn = a->tile_n ? a->tile_n : pick_tile_n(a->M, a->N, a->K, sms, a->mode, nb);
  pl->tile_m = a->tile_m ? a->tile_m : pick_tile_m(a->M, a->N, a->K, sms, a->mode, pl->bn, nb);
  if (pl->tile_m != 128 && pl->tile_m != 256) return ABFT_ERR_UNSUPPORTED;
  if (pl->tile_m == 256 && sms < 2) return ABFT_ERR_UNSUPPORTED;
  pl->pair = pl->tile_m == 256;
  pl->bd = pl->check ? pl->bn - kChkRows : pl->bn;
  pl->num_kb = static_cast<int>(cdiv(a->K, kBK));
  pl->tiles = nb * cdiv(a->M, pl->tile_m) * cdiv(a->N, pl->bd);
  if (pl->tiles >= (1ll << 31)) return ABFT_ERR_UNSUPPORTED;
  if (!pl->pair)
    pl->units = sms;
  else if (dev < 0)
    pl->units = sms / 2;
  else
    pl->units = pl->bn == 256 ? (pl->check ? pair_units_on<256, true>(dev, sms) : pair_units_on<256, false>(dev, sms))
                              : (pl->check ? pair_units_on<128, true>(dev, sms) : pair_units_on<128, false>(dev, sms));
  pl->sch = schedule_for(a->M, a->N, a->K, pl->tile_m, pl->bn, pl->bd, pl->units, nb);
  pl->grid = pl->sch.grid * (pl->pair ? 2 : 1);

  size_t off = 0;
  pl->v_off = pl->pa_off = pl->u_off = pl->pb_off = pl->vf_off = pl->parts_off = pl->sk_part_off = pl->sk_flag_off = 0;
  if (pl->check && a->checksums == nullptr) {
    pl->v_off = off;
    off = align256(off + static_cast<size_t>(nb) * abft_checksum_bytes_typed(a->N, a->K, pl->bn, a->dtype));
  }
  if (a->mode & ABFT_MODE_REF) {
    pl->pa_off = off;
    off = align256(off + 4 * colsum_partial_floats(a->M, a->K, sms, false));
    pl->u_off = off;
    off = align256(off + 4 * static_cast<size_t>(a->K));
    pl->pb_off = off;
    off = align256(off + 4 * colsum_partial_floats(a->N, a->K, sms, false));
    pl->vf_off = off;
    off = align256(off + 4 * static_cast<size_t>(a->K));
    pl->parts_off = off;  // a partial sum per epilogue warp and 128-row slab of a tile
    off = align256(off + 4 * kEpiWarps * static_cast<size_t>(pl->tiles) * (pl->pair ? 2 : 1));
  }
  if (pl->sch.sk) {
    pl->sk_part_off = off;
    off = align256(off + static_cast<size_t>(pl->grid) * kBM * pl->bn * sizeof(float));
    pl->sk_flag_off = off;
    off = align256(off + static_cast<size_t>(pl->grid) * kEpiWarps * sizeof(unsigned long long));  // a flag per epilogue warp
  }
  pl->total = off;
  return ABFT_OK;
}

int validate_gemm(const abft_gemm_args* a) {
  if (a == nullptr || a->A == nullptr || a->B == nullptr || a->C == nullptr) return ABFT_ERR_INVALID_ARG;
  if (a->M < 0 || a->N < 0 || a->K < 0 || a->batch < 0) return ABFT_ERR_INVALID_ARG;
  if (a->M > (1ll << 30) || a->N > (1ll << 30) || a->K > (1ll << 30)) return ABFT_ERR_UNSUPPORTED;
  if (a->b_kn != 0 && a->b_kn != 1) return ABFT_ERR_INVALID_ARG;
  if (a->dtype != ABFT_DTYPE_BF16 && a->dtype != ABFT_DTYPE_F16) return a->dtype == ABFT_DTYPE_F32 ? ABFT_ERR_UNSUPPORTED : ABFT_ERR_INVALID_ARG;
  if (a->lda < a->K || a->ldb < (a->b_kn ? a->N : a->K) || a->ldc < a->N) return ABFT_ERR_INVALID_ARG;
  if (a->b_kn && a->checksums != nullptr) return ABFT_ERR_INVALID_ARG;
  if (a->batch > 1) {
    // flattened rows (batch * M, batch * N) are 32-bit in the kernel
    if (a->M * a->batch >= (1ll << 31) || a->N * a->batch >= (1ll << 31)) return ABFT_ERR_UNSUPPORTED;
    if (a->stride_a < 0 || a->stride_b < 0 || a->stride_c < 0) return ABFT_ERR_INVALID_ARG;
    if ((a->stride_a % 8) || (a->stride_b % 8) || (a->stride_c % 8)) return ABFT_ERR_ALIGNMENT;
    // C's batches are whole groups of ldc rows, disjoint: row b * (stride_c / ldc) starts batch b
    if (a->stride_c % a->ldc || a->stride_c / a->ldc < a->M) return ABFT_ERR_INVALID_ARG;
    if ((a->stride_c / a->ldc) * a->batch >= (1ll << 31)) return ABFT_ERR_UNSUPPORTED;
    if (a->mode & ABFT_MODE_REF) return ABFT_ERR_UNSUPPORTED;
  }
  if ((a->K % 8) || (a->N % 8) || (a->lda % 8) || (a->ldb % 8) || (a->ldc % 8)) return ABFT_ERR_ALIGNMENT;
  if (!aligned16(a->A) || !aligned16(a->B) || !aligned16(a->C)) return ABFT_ERR_ALIGNMENT;
  if (a->bias != nullptr && !aligned16(a->bias)) return ABFT_ERR_ALIGNMENT;
  if (a->mode & ~(ABFT_MODE_DETECT | ABFT_MODE_CORRECT | ABFT_MODE_REF | ABFT_MODE_REF_BF16)) return ABFT_ERR_INVALID_ARG;
  if (a->tile_n != 0 && a->tile_n != 128 && a->tile_n != 256) return ABFT_ERR_UNSUPPORTED;
  if (a->tile_m != 0 && a->tile_m != 128 && a->tile_m != 256) return ABFT_ERR_UNSUPPORTED;
  if (a->swap_ab < 0 || a->swap_ab > 2) return ABFT_ERR_INVALID_ARG;
  if (a->mode != ABFT_MODE_OFF && (a->report == nullptr || a->report_capacity < 0)) return ABFT_ERR_INVALID_ARG;
  if (a->report != nullptr && !aligned16(a->report)) return ABFT_ERR_ALIGNMENT;
  if (a->batch > 65535) return ABFT_ERR_UNSUPPORTED;  // grid z of the encode passes
  if (a->n_inject < 0 || a->n_inject > ABFT_MAX_INJECT) return ABFT_ERR_INVALID_ARG;
  if (a->n_inject > 0 && (a->inject_rows == nullptr || a->inject_cols == nullptr || a->inject_deltas == nullptr))
    return ABFT_ERR_INVALID_ARG;
  if (a->checksums != nullptr && !aligned16(a->checksums)) return ABFT_ERR_ALIGNMENT;
  if (!(a->thr_scale >= 0.f) || !(a->thr_abs >= 0.f)) return ABFT_ERR_INVALID_ARG;
  return ABFT_OK;
}

// The frames of a call: `r` has B K-major (an N-major B replaced by its
// copy at the start of the workspace, `copy`; any aligned placeholder while
// only sizes are wanted), `k` is the frame the kernel runs in (r, or r with
// swapped operands for few-row products).
struct Frames {
  abft_gemm_args r, k;
  bool kn, swap;
  size_t copy_bytes;
};

void make_frames(const abft_gemm_args* a, void* copy, Frames* f) {
  f->kn = a->b_kn == 1;
  f->r = *a;
  f->copy_bytes = 0;
  if (f->kn) {
    f->copy_bytes = align256(static_cast<size_t>(batch_of(a)) * a->N * a->K * 2);
    f->r.b_kn = 0;
    f->r.B = copy;
    f->r.ldb = a->K;
    f->r.stride_b = a->N * a->K;
  }
  f->swap = use_swap(&f->r);
  f->k = f->swap ? swapped_args(&f->r) : f->r;
}

template <int BN, bool CHECK, bool PAIR, bool F16>
int launch_gemm(int dev, int slot, const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmB2,
                const CUtensorMap& tmV, const CUtensorMap& tmBt, const CUtensorMap& tmC, const GemmParams& p, int grid,
                cudaStream_t s) {
  int rc = ensure_smem_attr<BN, CHECK, PAIR, F16>(dev, slot);
  if (rc != ABFT_OK) return rc;
  constexpr size_t smem = GemmCfg<BN, CHECK, PAIR>::kSmemBytes;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  // Programmatic serialization: the kernel's prologue (barriers, TMEM,
  // tensor-map prefetch) may start before the previous kernel on the stream
  // has finished; it waits (griddepcontrol.wait) before any global access.
  // The kernel never signals its own dependents early, so the next kernel
  // starts only once every CTA of this one has exited.
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if constexpr (PAIR) {
    at[1] = pair_cluster_attr();
    cfg.numAttrs = 2;
  }
  if (cudaLaunchKernelEx(&cfg, abft_gemm_kernel<BN, CHECK, PAIR, F16>, tmA, tmB, tmB2, tmV, tmBt, tmC, p) !=
      cudaSuccess)
    return launch_status(), ABFT_ERR_CUDA;
  return launch_status();
}

template <bool F16>
int launch_gemm_typed(const Plan& ws, bool check, int dev, const CUtensorMap& tmA, const CUtensorMap& tmB,
                      const CUtensorMap& tmB2, const CUtensorMap& tmV, const CUtensorMap& tmBt, const CUtensorMap& tmC,
                      const GemmParams& p, cudaStream_t s) {
  const int grid = ws.grid;
  if (ws.pair && ws.bn == 256)
    return check ? launch_gemm<256, true, true, F16>(dev, kPairSlot[1][1], tmA, tmB, tmB2, tmV, tmBt, tmC, p, grid, s)
                 : launch_gemm<256, false, true, F16>(dev, kPairSlot[1][0], tmA, tmB, tmB2, tmV, tmBt, tmC, p, grid, s);
  if (ws.pair)
    return check ? launch_gemm<128, true, true, F16>(dev, kPairSlot[0][1], tmA, tmB, tmB2, tmV, tmBt, tmC, p, grid, s)
                 : launch_gemm<128, false, true, F16>(dev, kPairSlot[0][0], tmA, tmB, tmB2, tmV, tmBt, tmC, p, grid, s);
  if (ws.bn == 256)
    return check ? launch_gemm<256, true, false, F16>(dev, 0, tmA, tmB, tmB2, tmV, tmBt, tmC, p, grid, s)
                 : launch_gemm<256, false, false, F16>(dev, 1, tmA, tmB, tmB2, tmV, tmBt, tmC, p, grid, s);
  return check ? launch_gemm<128, true, false, F16>(dev, 2, tmA, tmB, tmB2, tmV, tmBt, tmC, p, grid, s)
               : launch_gemm<128, false, false, F16>(dev, 3, tmA, tmB, tmB2, tmV, tmBt, tmC, p, grid, s);
}

// fp16 encodes with at most this many (k-block, tile, batch) triples run as
// one cluster launch; larger ones as memset + two launches of a CTA each
// (the cluster kernel's CTAs walk kEncCluster times fewer k-blocks in
// parallel: 132 against 59 us for an 8192^2 weight).
constexpr int64_t kEncOneLaunchCtas = 1024;

// Rows part of one batch's checksum block, then (fp16) its scale table of
// 8 floats per tile.
size_t checksum_rows_bytes(int64_t N, int64_t K, int32_t tile_n) {
  return static_cast<size_t>(cdiv(N, tile_n - kChkRows)) * kChkRows * static_cast<size_t>(K) * 2;
}

}  // namespace

extern "C" {

int abft_version(void) { return ABFT_B200_VERSION; }

const char* abft_status_string(int status) {
  switch (status) {
    case ABFT_OK: return "ok";
    case ABFT_ERR_INVALID_ARG: return "invalid argument";
    case ABFT_ERR_ALIGNMENT: return "alignment: pointers must be 16-byte aligned, K, N and leading dimensions multiples of 8";
    case ABFT_ERR_UNSUPPORTED: return "unsupported shape or tile width";
    case ABFT_ERR_WORKSPACE: return "workspace missing or too small";
    case ABFT_ERR_CUDA: return "CUDA runtime error";
    case ABFT_ERR_NO_DEVICE: return "no sm_100 (B200) device is current";
    case ABFT_ERR_DRIVER: return "cuTensorMapEncodeTiled unavailable from the driver";
    default: return "unknown status";
  }
}

size_t abft_report_bytes(int32_t capacity) {
  if (capacity < 0) capacity = 0;
  return sizeof(abft_report) + static_cast<size_t>(capacity) * sizeof(abft_fault_record);
}

size_t abft_report_bytes_batched(int32_t capacity, int32_t batch) {
  return abft_report_bytes(capacity) + (batch > 1 ? static_cast<size_t>(batch) * 4 * sizeof(uint32_t) : 0);
}

int32_t abft_pick_tile_n(int64_t M, int64_t N, int64_t K, int32_t num_sms, uint32_t mode) {
  return pick_tile_n(M, N, K, num_sms, mode, 1);
}

size_t abft_checksum_bytes(int64_t N, int64_t K, int32_t tile_n) {
  if (tile_n != 128 && tile_n != 256) return 0;
  return checksum_rows_bytes(N, K, tile_n);
}

size_t abft_checksum_bytes_typed(int64_t N, int64_t K, int32_t tile_n, int32_t dtype) {
  if (tile_n != 128 && tile_n != 256) return 0;
  if (dtype == ABFT_DTYPE_BF16) return checksum_rows_bytes(N, K, tile_n);
  if (dtype != ABFT_DTYPE_F16) return 0;
  return checksum_rows_bytes(N, K, tile_n) + static_cast<size_t>(cdiv(N, tile_n - kChkRows)) * 8 * sizeof(float);
}

int abft_encode_weight_typed(const void* B, int64_t N, int64_t K, int64_t ldb, int64_t stride_b, int32_t batch,
                             int32_t tile_n, int32_t dtype, void* out, void* stream) {
  if (B == nullptr || out == nullptr || N <= 0 || K <= 0 || ldb < K || batch < 1 || stride_b < 0)
    return ABFT_ERR_INVALID_ARG;
  if (dtype != ABFT_DTYPE_BF16 && dtype != ABFT_DTYPE_F16)
    return dtype == ABFT_DTYPE_F32 ? ABFT_ERR_UNSUPPORTED : ABFT_ERR_INVALID_ARG;
  if ((K % 8) || (ldb % 8) || (stride_b % 8) || !aligned16(B) || !aligned16(out)) return ABFT_ERR_ALIGNMENT;
  if (tile_n != 128 && tile_n != 256) return ABFT_ERR_UNSUPPORTED;
  if (N > (1ll << 30) || K > (1ll << 30) || batch > 65535) return ABFT_ERR_UNSUPPORTED;
  int dev;
  DeviceInfo info;
  int rc = current_device(&dev, &info);
  if (rc != ABFT_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int bd = tile_n - kChkRows;
  const int num_kb = static_cast<int>(cdiv(K, kBK));
  const int64_t tiles = cdiv(N, bd);
  const size_t bytes = abft_checksum_bytes_typed(N, K, tile_n, dtype);  // one batch's block
  if (dtype == ABFT_DTYPE_BF16) {
    dim3 g(static_cast<unsigned>(num_kb), static_cast<unsigned>(tiles), static_cast<unsigned>(batch));
    encode_weight_kernel<<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(B), ldb, static_cast<int>(N),
                                           static_cast<int>(K), bd, static_cast<__nv_bfloat16*>(out), stride_b,
                                           static_cast<int64_t>(bytes / 2));
    return launch_status();
  }
  float* table = reinterpret_cast<float*>(static_cast<uint8_t*>(out) + checksum_rows_bytes(N, K, tile_n));
  const __half* Bh = static_cast<const __half*>(B);
  __half* oh = static_cast<__half*>(out);
  if (static_cast<int64_t>(num_kb) * tiles * batch > kEncOneLaunchCtas) {
    // Large: a CTA per k-block of each tile; the tables are zeroed first
    // (one row of tiles * 8 floats per batch).
    if (cudaMemset2DAsync(table, bytes, 0, static_cast<size_t>(tiles) * 8 * sizeof(float),
                          static_cast<size_t>(batch), s) != cudaSuccess)
      return launch_status(), ABFT_ERR_CUDA;
    dim3 g(static_cast<unsigned>(num_kb), static_cast<unsigned>(tiles), static_cast<unsigned>(batch));
    encode_f16_sums_kernel<<<g, 256, 0, s>>>(Bh, ldb, static_cast<int>(N), static_cast<int>(K), bd, oh, stride_b,
                                             static_cast<int64_t>(bytes / 2), table, static_cast<int64_t>(bytes / 4));
    rc = launch_status();
    if (rc != ABFT_OK) return rc;
    encode_f16_finish_kernel<<<g, 64, 0, s>>>(oh, static_cast<int>(K), static_cast<int64_t>(bytes / 2), table,
                                               static_cast<int64_t>(bytes / 4));
    return launch_status();
  }
  // Small: one cluster of kEncCluster CTAs per tile and batch forms the
  // sums, agrees on the tile's scales and writes the rows and the table
  // (column-parallel for at most 32 rows: a decode step's tokens).
  const bool few_rows = N <= 32 && K <= kFewRowsMaxK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(tiles * kEncCluster), static_cast<unsigned>(batch));
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute at;
  at.id = cudaLaunchAttributeClusterDimension;
  at.val.clusterDim.x = kEncCluster;
  at.val.clusterDim.y = 1;
  at.val.clusterDim.z = 1;
  cfg.attrs = &at;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, few_rows ? encode_f16_few_rows_kernel : encode_f16_cluster_kernel, Bh, ldb,
                         static_cast<int>(N), static_cast<int>(K), bd, oh, stride_b, static_cast<int64_t>(bytes / 2),
                         table, static_cast<int64_t>(bytes / 4)) != cudaSuccess)
    return launch_status(), ABFT_ERR_CUDA;
  return launch_status();
}

int abft_encode_weight_batched(const void* B, int64_t N, int64_t K, int64_t ldb, int64_t stride_b, int32_t batch,
                               int32_t tile_n, void* out, void* stream) {
  return abft_encode_weight_typed(B, N, K, ldb, stride_b, batch, tile_n, ABFT_DTYPE_BF16, out, stream);
}

int abft_encode_weight(const void* B, int64_t N, int64_t K, int64_t ldb, int32_t tile_n, void* out, void* stream) {
  return abft_encode_weight_typed(B, N, K, ldb, 0, 1, tile_n, ABFT_DTYPE_BF16, out, stream);
}

size_t abft_gemm_workspace_bytes(const abft_gemm_args* args) {
  if (args == nullptr) return 0;
  int dev;
  DeviceInfo info;
  int sms = 148;
  const bool have_dev = current_device(&dev, &info) == ABFT_OK;
  if (have_dev) sms = info.sms;
  if (args->num_sms > 0 && args->num_sms < sms) sms = args->num_sms;
  Plan pl;
  Frames f;
  make_frames(args, args->workspace, &f);
  if (make_plan(&f.k, have_dev ? dev : -1, sms, &pl) != ABFT_OK) return 0;
  return f.copy_bytes + pl.total;
}

int32_t abft_pick_tile_m(int64_t M, int64_t N, int64_t K, int32_t num_sms, uint32_t mode, int32_t tile_n) {
  if (num_sms <= 0) num_sms = 148;
  return pick_tile_m(M, N, K, num_sms, mode, tile_n);
}

int abft_wait_selftest(void* report, void* stream) {
  if (report == nullptr) return ABFT_ERR_INVALID_ARG;
  if (!aligned16(report)) return ABFT_ERR_ALIGNMENT;
  int dev;
  DeviceInfo info;
  const int rc = current_device(&dev, &info);
  if (rc != ABFT_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(report, 0, sizeof(abft_report), s) != cudaSuccess) return launch_status(), ABFT_ERR_CUDA;
  wait_selftest_kernel<<<1, 32, 0, s>>>(static_cast<abft_report*>(report));
  return launch_status();
}

int abft_gemm(const abft_gemm_args* args, void* stream) { return abft_gemm_bf16(args, stream); }

int abft_gemm_plan(const abft_gemm_args* args, abft_plan_info* info) {
  if (info == nullptr) return ABFT_ERR_INVALID_ARG;
  int rc = validate_gemm(args);
  if (rc != ABFT_OK) return rc;
  int dev;
  DeviceInfo dinfo;
  rc = current_device(&dev, &dinfo);
  if (rc != ABFT_OK) return rc;
  memset(info, 0, sizeof(*info));
  if (args->M == 0 || args->N == 0) return ABFT_OK;  // abft_gemm launches nothing
  if (args->K == 0) return ABFT_ERR_UNSUPPORTED;
  int sms = dinfo.sms;
  if (args->num_sms > 0 && args->num_sms < sms) sms = args->num_sms;
  Frames fr;
  make_frames(args, args->workspace, &fr);
  Plan pl;
  rc = make_plan(&fr.k, dev, sms, &pl);
  if (rc != ABFT_OK) return rc;
  const int64_t cols = cdiv(fr.k.N, pl.bd);
  info->tile_n = pl.bn;
  info->tile_m = pl.tile_m;
  info->data_cols = pl.bd;
  info->tiles_n = static_cast<int32_t>(cols);
  info->last_cols = static_cast<int32_t>(fr.k.N - (cols - 1) * pl.bd);
  info->swapped = fr.swap ? 1 : 0;
  info->units = pl.units;
  info->grid = pl.grid;
  info->dp_tiles = pl.sch.dp_tiles;
  info->sk_units = pl.sch.sk ? pl.sch.sk_ctas : 0;
  info->tiles = pl.tiles;
  info->workspace_bytes = fr.copy_bytes + pl.total;
  return ABFT_OK;
}

int abft_gemm_bf16(const abft_gemm_args* args, void* stream) {
  int rc = validate_gemm(args);
  if (rc != ABFT_OK) return rc;
  int dev;
  DeviceInfo info;
  rc = current_device(&dev, &info);
  if (rc != ABFT_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t nb = batch_of(args);
  if (args->M == 0 || args->N == 0) {
    // No kernel runs: reset the report here (the kernel resets it otherwise;
    // batch 0 in the header: no per-batch counters follow).
    if (args->report != nullptr && cudaMemsetAsync(args->report, 0, sizeof(abft_report), s) != cudaSuccess)
      return launch_status(), ABFT_ERR_CUDA;
    return ABFT_OK;
  }
  if (args->K == 0) return ABFT_ERR_UNSUPPORTED;

  int sms = info.sms;
  if (args->num_sms > 0 && args->num_sms < sms) sms = args->num_sms;
  Frames fr;
  make_frames(args, args->workspace, &fr);
  abft_gemm_args* a = &fr.k;
  const bool swap = fr.swap;
  Plan ws;
  rc = make_plan(a, dev, sms, &ws);
  if (rc != ABFT_OK) return rc;
  const int bn = ws.bn;
  const bool check = ws.check;
  const size_t need = fr.copy_bytes + ws.total;
  if (need > 0 && (args->workspace == nullptr || args->workspace_bytes < need || !aligned16(args->workspace)))
    return ABFT_ERR_WORKSPACE;
  // the K-major copy of an N-major B first, then the plan's regions
  uint8_t* wsb = static_cast<uint8_t*>(args->workspace) + fr.copy_bytes;
  const int bd = ws.bd;  // data columns per output tile

  // Every tensor map is encoded before the first launch of the call, so a
  // layout the encoder rejects returns an error with no device work queued.
  // An N-major B is copied K-major by a pre-pass that, unless the operands
  // are swapped (the copy is then the kernel's A and the checksums come
  // from the rows of A), also forms the checksum block.
  const bool f16 = a->dtype == ABFT_DTYPE_F16;
  // fp16 checksum rows are scaled per tile from the largest sum over all of
  // K, which neither the transposing pre-pass nor the in-kernel token
  // builder sees: they use the two-pass encode (after the copy, if any).
  const bool enc_kn = fr.kn && check && !swap && !f16;
  // Swapped operands with at most 64 tokens (one compact tail tile): the
  // kernel's build warp forms the token checksum rows of every stage in
  // shared memory; nothing is encoded or loaded for them. More tokens (a
  // forced swap) keep the encode pre-pass.
  const bool build =
      check && swap && !f16 && !ws.pair && a->N <= 64 && a->N < bd && tail_width(a->N, bd, bn, check) != 0;
  const bool enc_plain = check && a->checksums == nullptr && !enc_kn && !build;
  const void* V = check ? (a->checksums != nullptr ? a->checksums : wsb + ws.v_off) : nullptr;

  // B-operand boxes: the whole data width of a tile, or in a pair the even
  // CTA's 128 rows (tmB) and the odd CTA's remaining data rows (tmB2).
  CUtensorMap tmA, tmB, tmB2;
  const int dt = a->dtype;
  rc = make_tmap_kmajor(&tmA, a->A, a->K, a->M, a->lda, kBM, nb, a->stride_a, dt);
  if (rc != ABFT_OK) return rc;
  rc = make_tmap_kmajor(&tmB, a->B, a->K, a->N, a->ldb, ws.pair ? bn / 2 : bd, nb, a->stride_b, dt);
  if (rc != ABFT_OK) return rc;
  tmB2 = tmB;
  if (ws.pair && check) {
    rc = make_tmap_kmajor(&tmB2, a->B, a->K, a->N, a->ldb, bd - bn / 2, nb, a->stride_b, dt);
    if (rc != ABFT_OK) return rc;
  }
  // A batch's checksum block: its rows, then (fp16) its scale table.
  const size_t chk_bytes = check ? abft_checksum_bytes_typed(a->N, a->K, bn, dt) : 0;
  CUtensorMap tmV = tmA;  // placeholder when checks are off or built in the kernel
  if (check && !build) {
    const int64_t vrows = cdiv(a->N, bd) * kChkRows;
    rc = make_tmap_kmajor(&tmV, V, a->K, vrows, a->K, kChkRows, nb, static_cast<int64_t>(chk_bytes / 2), dt);
    if (rc != ABFT_OK) return rc;
  }
  CUtensorMap tmC = tmA;  // placeholder with swapped operands (transposed plain stores)
  if (!swap) {
    rc = make_tmap_store(&tmC, a->C, a->N, a->M, a->ldc, nb, nb > 1 ? (a->stride_c / a->ldc) * a->ldc : 0, dt);
    if (rc != ABFT_OK) return rc;
  }

  GemmParams p;
  p.C = a->C;
  p.ldc = a->ldc;
  p.bias = a->bias;
  p.chk_scale = nullptr;
  p.chk_scale_bstride = 0;
  if (check && f16) {
    p.chk_scale = reinterpret_cast<const float*>(static_cast<const uint8_t*>(V) + checksum_rows_bytes(a->N, a->K, bn));
    p.chk_scale_bstride = static_cast<int64_t>(chk_bytes / 4);
  }
  p.M = static_cast<int>(a->M);
  p.N = static_cast<int>(a->N);
  p.K = static_cast<int>(a->K);
  p.num_kb = static_cast<int>(cdiv(a->K, kBK));
  p.tiles_m = static_cast<int>(cdiv(a->M, ws.tile_m));
  p.tiles_n = static_cast<int>(cdiv(a->N, bd));
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.group_m = 16;
  p.mode = a->mode;
  if (p.mode & ABFT_MODE_CORRECT) p.mode |= ABFT_MODE_DETECT;
  p.thr_k = static_cast<float>(static_cast<double>(a->thr_scale) * sqrt(static_cast<double>(a->K)));
  p.thr_abs = a->thr_abs;
  p.inj_rows = a->inject_rows;
  p.inj_cols = a->inject_cols;
  p.inj_deltas = a->inject_deltas;
  p.n_inj = a->n_inject;
  p.report = static_cast<abft_report*>(a->report);
  p.capacity = a->report_capacity;
  p.tile_sumc = (a->mode & ABFT_MODE_REF) ? reinterpret_cast<float*>(wsb + ws.parts_off) : nullptr;
  p.swap = swap ? 1 : 0;
  p.build_chk = build ? 1 : 0;
  p.batch = static_cast<int>(nb);
  p.c_rows = nb > 1 ? static_cast<int>(a->stride_c / a->ldc) : 0;
  p.bcounts = (nb > 1 && a->report != nullptr)
                  ? reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(a->report) + abft_report_bytes(a->report_capacity))
                  : nullptr;

  // Compact tail tile: when the last tile column holds ncols < bd data
  // columns, its B-operand tile is those rows (then, with checks, the 8
  // checksum rows) and one MMA of N = round16(ncols [+ 8]) covers it.
  p.tail_n = 0;
  p.tail_box = 0;
  p.tail_tx = 0;
  CUtensorMap tmBt = tmA;  // placeholder unless a tail box is needed
  {
    const int ncols = tail_rows(a->N, bd);  // data rows of the tail box, a multiple of 8
    const int tn = tail_width(a->N, bd, bn, check);
    if (tn != 0) {
      const uint32_t a_bytes = static_cast<uint32_t>(kBM * kBK * 2);
      const uint32_t row_bytes = static_cast<uint32_t>(kBK * 2);  // one B row of one k-block
      p.tail_n = tn;
      if (!check && ws.pair) {
        p.tail_tx = 2 * (a_bytes + (bn / 2) * row_bytes);
      } else if (!check) {
        // The box of the tn rows the narrow MMA reads, not a whole tile:
        // with few rows (decode) the zero fill of a full box costs more
        // shared-memory bandwidth than the rows themselves.
        rc = make_tmap_kmajor(&tmBt, a->B, a->K, a->N, a->ldb, tn, nb, a->stride_b);
        if (rc != ABFT_OK) return rc;
        p.tail_box = tn;
        p.tail_tx = a_bytes + static_cast<uint32_t>(tn) * row_bytes;
      } else {
        // Data rows copied by the tail box into this CTA (a pair: the odd
        // CTA holds the rows from tn / 2 on; the even CTA keeps its usual box).
        const int box = ws.pair ? ncols - tn / 2 : ncols;
        if (box < 0 || box % 8) return ABFT_ERR_UNSUPPORTED;  // checksum rows must start on a swizzle atom
        p.tail_box = box;
        if (box > 0) {
          rc = make_tmap_kmajor(&tmBt, a->B, a->K, a->N, a->ldb, box, nb, a->stride_b);
          if (rc != ABFT_OK) return rc;
        }
        p.tail_tx = (ws.pair ? 2 * a_bytes + (bn / 2) * row_bytes : a_bytes) +
                    static_cast<uint32_t>(box + (build ? 0 : kChkRows)) * row_bytes;
      }
    }
  }

  // Tile order: full tiles first, then the tail column's (one per tile row).
  p.tiles_n_full = p.tiles_n - (p.tail_n ? 1 : 0);
  p.full_tiles = p.tiles_m * p.tiles_n_full;
  p.fd_tiles_m = make_fast_div(p.tiles_m);
  p.fd_full = make_fast_div(p.full_tiles);
  p.fd_group = make_fast_div(static_cast<int64_t>(p.group_m) * p.tiles_n_full);
  p.fd_gm = make_fast_div(p.group_m);
  p.fd_gm_last = make_fast_div(p.tiles_m - (cdiv(p.tiles_m, p.group_m) - 1) * p.group_m);

  const Schedule& sch = ws.sch;
  p.dp_tiles = sch.dp_tiles;
  p.sk = sch.sk;
  p.sk_ctas = sch.sk_ctas;
  p.sk_iters = sch.sk_iters;
  p.partials = nullptr;
  p.flags = nullptr;
  p.nonce = next_launch_nonce();
  if (sch.sk) {
    p.partials = reinterpret_cast<float*>(wsb + ws.sk_part_off);
    p.flags = reinterpret_cast<unsigned long long*>(wsb + ws.sk_flag_off);
  }
  if (fr.kn) {
    const int cbd = enc_kn ? bd : 256;  // copies 16-bit elements of either type
    dim3 g(static_cast<unsigned>(cdiv(args->K, kBK)), static_cast<unsigned>(cdiv(args->N, cbd)),
           static_cast<unsigned>(nb));
    transpose_encode_kernel<<<g, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(args->B), args->ldb, nb > 1 ? args->stride_b : 0, static_cast<int>(args->N),
        static_cast<int>(args->K), cbd, static_cast<__nv_bfloat16*>(args->workspace),
        enc_kn ? static_cast<__nv_bfloat16*>(const_cast<void*>(V)) : nullptr,
        enc_kn ? static_cast<int64_t>(chk_bytes / 2) : 0);
    rc = launch_status();
    if (rc != ABFT_OK) return rc;
  }
  if (enc_plain) {
    rc = abft_encode_weight_typed(a->B, a->N, a->K, a->ldb, nb > 1 ? a->stride_b : 0, static_cast<int32_t>(nb), bn, dt,
                                  const_cast<void*>(V), stream);
    if (rc != ABFT_OK) return rc;
  }
  // A CUDA graph replays this launch with the nonce frozen in its kernel
  // node, so the stream-K flags and the report tag that the previous replay
  // left would already match it: a finisher would fold a stale partial and
  // report atomics could run ahead of the header reset. Under stream capture
  // one small kernel clears both in the graph, ahead of the GEMM (a kernel,
  // not memset nodes: one node, and the GEMM's griddepcontrol.wait covers
  // it). An eager launch draws a fresh nonce and needs no clearing.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cap) != cudaSuccess) return launch_status(), ABFT_ERR_CUDA;
  if (cap != cudaStreamCaptureStatusNone && (p.report != nullptr || p.flags != nullptr)) {
    const int nflags = p.flags != nullptr ? ws.grid * kEpiWarps : 0;
    clear_launch_state_kernel<<<static_cast<unsigned>(cdiv(nflags > 0 ? nflags : 1, 256)), 256, 0, s>>>(
        p.report != nullptr ? reinterpret_cast<unsigned long long*>(&p.report->launch_tag) : nullptr, p.flags,
        nflags);
    rc = launch_status();
    if (rc != ABFT_OK) return rc;
  }
  rc = f16 ? launch_gemm_typed<true>(ws, check, dev, tmA, tmB, tmB2, tmV, tmBt, tmC, p, s)
           : launch_gemm_typed<false>(ws, check, dev, tmA, tmB, tmB2, tmV, tmBt, tmC, p, s);
  if (rc != ABFT_OK) return rc;

  if (a->mode & ABFT_MODE_REF) {
    float* pa = reinterpret_cast<float*>(wsb + ws.pa_off);
    float* u = reinterpret_cast<float*>(wsb + ws.u_off);
    float* pb = reinterpret_cast<float*>(wsb + ws.pb_off);
    float* vf = reinterpret_cast<float*>(wsb + ws.vf_off);
    rc = colsum(a->A, a->lda, a->M, a->K, nullptr, pa, u, nullptr, nullptr, sms, s, dt);
    if (rc != ABFT_OK) return rc;
    rc = colsum(a->B, a->ldb, a->N, a->K, nullptr, pb, vf, nullptr, nullptr, sms, s, dt);
    if (rc != ABFT_OK) return rc;
    // corner + (rows of C) * sum(bias): the bias runs along the kernel's
    // rows when the operands are swapped
    ref_finalize(dt, u, vf, p.K, p.bias, swap ? p.M : p.N, swap ? p.N : p.M, p.tile_sumc,
                 p.num_tiles * kEpiWarps * (ws.pair ? 2 : 1), a->tol_abs, a->tol_rel,
                 (a->mode & ABFT_MODE_REF_BF16) ? 1 : 0, p.report, p.capacity, ws.tile_m, bd, s);
    rc = launch_status();
  }
  return rc;
}

namespace {
struct CheckWs {
  float *pa, *u, *pb, *v, *rsum, *rmax, *rabs, *rexp, *pc, *csum, *cmax, *cabs, *cexp;
  size_t floats;
};
// Carves the check-only workspace; with base == nullptr only counts floats.
void check_ws_layout(float* base, int64_t M, int64_t N, int64_t K, int sms, CheckWs* w) {
  size_t off = 0;
  auto take = [&](size_t n) {
    float* p = base != nullptr ? base + off : nullptr;
    off += (n + 63) & ~size_t(63);
    return p;
  };
  const size_t pb_n = colsum_partial_floats(N, K, sms, false), pk_n = colsum_partial_floats(K, N, sms, false);
  const size_t pc_n = colsum_partial_floats(M, N, sms, true);
  w->pa = take(colsum_partial_floats(M, K, sms, false));
  w->u = take(K);
  w->pb = take(pb_n > pk_n ? pb_n : pk_n);
  w->v = take(K);
  w->rsum = take(M);
  w->rmax = take(M);
  w->rabs = take(M);
  w->rexp = take(M);
  w->pc = take(pc_n > pk_n ? pc_n : pk_n);
  w->csum = take(N);
  w->cmax = take(N);
  w->cabs = take(N);
  w->cexp = take(N);
  w->floats = off;
}
}  // namespace

size_t abft_check_workspace_bytes(const abft_check_args* c) {
  if (c == nullptr || c->M <= 0 || c->N <= 0 || c->K <= 0) return 0;
  int dev;
  DeviceInfo info;
  int sms = 148;
  if (current_device(&dev, &info) == ABFT_OK) sms = info.sms;
  CheckWs w;
  check_ws_layout(nullptr, c->M, c->N, c->K, sms, &w);
  return align256(w.floats * 4);
}

int abft_check_only(const abft_check_args* c, void* stream) {
  if (c == nullptr || c->A == nullptr || c->B == nullptr || c->C == nullptr || c->report == nullptr)
    return ABFT_ERR_INVALID_ARG;
  const int64_t M = c->M, N = c->N, K = c->K;
  if (M <= 0 || N <= 0 || K <= 0 || c->report_capacity < 0 || (c->b_kn != 0 && c->b_kn != 1))
    return ABFT_ERR_INVALID_ARG;
  if (c->flags & ~(ABFT_CHECK_LOCATE | ABFT_CHECK_NATIVE_SUMS)) return ABFT_ERR_INVALID_ARG;
  if (c->dtype != ABFT_DTYPE_BF16 && c->dtype != ABFT_DTYPE_F16 && c->dtype != ABFT_DTYPE_F32)
    return ABFT_ERR_INVALID_ARG;
  if (M > (1ll << 30) || N > (1ll << 30) || K > (1ll << 30)) return ABFT_ERR_UNSUPPORTED;
  if (c->lda < K || c->ldc < N || c->ldb < (c->b_kn ? N : K)) return ABFT_ERR_INVALID_ARG;
  // rows are read 8 elements at a time (16 or 32 bytes): every row start aligned
  if ((K % 8) || (N % 8) || (c->lda % 8) || (c->ldb % 8) || (c->ldc % 8)) return ABFT_ERR_ALIGNMENT;
  if (!aligned16(c->A) || !aligned16(c->B) || !aligned16(c->C) || !aligned16(c->report)) return ABFT_ERR_ALIGNMENT;
  if (c->bias != nullptr && !aligned16(c->bias)) return ABFT_ERR_ALIGNMENT;
  if (!(c->thr_scale >= 0.f)) return ABFT_ERR_INVALID_ARG;
  int dev;
  DeviceInfo info;
  int rc = current_device(&dev, &info);
  if (rc != ABFT_OK) return rc;
  const size_t need = abft_check_workspace_bytes(c);
  if (c->workspace == nullptr || c->workspace_bytes < need || !aligned16(c->workspace)) return ABFT_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int sms = info.sms;
  CheckWs w;
  check_ws_layout(static_cast<float*>(c->workspace), M, N, K, sms, &w);
  const int dt = c->dtype;

  if (cudaMemsetAsync(c->report, 0, sizeof(abft_report), s) != cudaSuccess) return launch_status(), ABFT_ERR_CUDA;
  abft_report* rep = static_cast<abft_report*>(c->report);

  // s_a = A.sum(0) and s_b = B.sum(1)   (pytorch/abft/checkers.py:117-118)
  rc = colsum(c->A, c->lda, M, K, nullptr, w.pa, w.u, nullptr, nullptr, sms, s, dt);
  if (rc != ABFT_OK) return rc;
  if (c->b_kn == 0)
    rc = colsum(c->B, c->ldb, N, K, nullptr, w.pb, w.v, nullptr, nullptr, sms, s, dt);
  else
    rc = rowdot(c->B, c->ldb, K, N, nullptr, w.v, nullptr, nullptr, s, dt);
  if (rc != ABFT_OK) return rc;
  // row sums of C (sum_c = sum of the row sums, fixed order)
  rc = rowdot(c->C, c->ldc, M, N, nullptr, w.rsum, w.rmax, w.rabs, s, dt);
  if (rc != ABFT_OK) return rc;
  ref_finalize(dt, w.u, w.v, static_cast<int>(K), c->bias, static_cast<int>(N), static_cast<int>(M), w.rsum,
               static_cast<int>(M), c->tol_abs, c->tol_rel, (c->flags & ABFT_CHECK_NATIVE_SUMS) ? 1 : 0, rep,
               c->report_capacity, 0, 0, s);
  rc = launch_status();
  if (rc != ABFT_OK || !(c->flags & ABFT_CHECK_LOCATE)) return rc;

  // Expected row sums A (B e), expected column sums (e^T A) B, actual column sums.
  rc = rowdot(c->A, c->lda, M, K, w.v, w.rexp, nullptr, nullptr, s, dt);
  if (rc != ABFT_OK) return rc;
  if (c->b_kn == 0)
    rc = rowdot(c->B, c->ldb, N, K, w.u, w.cexp, nullptr, nullptr, s, dt);
  else
    rc = colsum(c->B, c->ldb, K, N, w.u, w.pb, w.cexp, nullptr, nullptr, sms, s, dt);
  if (rc != ABFT_OK) return rc;
  rc = colsum(c->C, c->ldc, M, N, nullptr, w.pc, w.csum, w.cmax, w.cabs, sms, s, dt);
  if (rc != ABFT_OK) return rc;
  const float thr_k = static_cast<float>(static_cast<double>(c->thr_scale) * sqrt(static_cast<double>(K)));
  const float unit = unit_roundoff(dt);  // worst-case relative rounding of a stored element
  const int m32 = static_cast<int>(M), n32 = static_cast<int>(N);
  if (dt == ABFT_DTYPE_F16)
    locate_finalize_kernel<<<1, 1024, 0, s>>>(w.rsum, w.rmax, w.rabs, w.rexp, m32, w.csum, w.cmax, w.cabs, w.cexp, n32,
                                              static_cast<const __half*>(c->bias), thr_k, unit, rep, c->report_capacity);
  else if (dt == ABFT_DTYPE_F32)
    locate_finalize_kernel<<<1, 1024, 0, s>>>(w.rsum, w.rmax, w.rabs, w.rexp, m32, w.csum, w.cmax, w.cabs, w.cexp, n32,
                                              static_cast<const float*>(c->bias), thr_k, unit, rep, c->report_capacity);
  else
    locate_finalize_kernel<<<1, 1024, 0, s>>>(w.rsum, w.rmax, w.rabs, w.rexp, m32, w.csum, w.cmax, w.cabs, w.cexp, n32,
                                              static_cast<const __nv_bfloat16*>(c->bias), thr_k, unit, rep,
                                              c->report_capacity);
  return launch_status();
}

// ---- abft_check_only_noalloc -------------------------------------------------
// The fixed scratch of the no-allocation entry point (include/abft_b200.h).
// Host code must not use the array's name as an address: the device address
// comes from cudaGetSymbolAddress, once per device, with that device current.
static __device__ __align__(256) unsigned char g_noalloc_scratch[ABFT_NO_ALLOC_SCRATCH_BYTES];

namespace {
void* g_noalloc_ptr[kMaxDevices];  // per-device address of g_noalloc_scratch, guarded by g_mu
}  // namespace

int abft_check_only_noalloc(const abft_check_args* args, void* stream) {
  if (args == nullptr) return ABFT_ERR_INVALID_ARG;
  int dev;
  DeviceInfo info;
  int rc = current_device(&dev, &info);
  if (rc != ABFT_OK) return rc;
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
        cudaGetLastError();
        return ABFT_ERR_CUDA;
      }
      g_noalloc_ptr[dev] = p;
    }
    scratch = g_noalloc_ptr[dev];
  }
  if (abft_check_workspace_bytes(args) > ABFT_NO_ALLOC_SCRATCH_BYTES) return ABFT_ERR_WORKSPACE;
  abft_check_args c = *args;
  c.workspace = scratch;
  c.workspace_bytes = ABFT_NO_ALLOC_SCRATCH_BYTES;
  return abft_check_only(&c, stream);
}

}  // extern "C"
