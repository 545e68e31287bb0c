/*
 * abft_b200.h - C ABI of the B200 (sm_100a) checksum-protected GEMM library.
 *
 * The library replaces the native entry of the reference's `pytorch/abft`
 * fused checker and the GEMM that precedes every check:
 *
 *   reference                                          this library
 *   -------------------------------------------------  ---------------------------
 *   F.linear(x, W, b) then CheapSumChecker.check       abft_gemm_bf16 (GEMM, check,
 *     (pytorch/abft/injector.py:152-161,                 locate and correct in one
 *      pytorch/abft/checkers.py:55-126)                  kernel)
 *   abft_fused(a, b, c, bias) -> [corner, sum_c]       abft_check_only
 *     (pytorch/abft/kernels/abft_fused.cpp:11-31,
 *      pytorch/abft/kernels/abft_fused.cu:92-141)
 *   s_b = b.sum(dim=1) recomputed per call             abft_encode_weight (once per
 *     (pytorch/abft/checkers.py:119)                     weight, cacheable)
 *   torch.bmm(a, b) then a Python loop of per-batch    abft_gemm_bf16 with batch > 1
 *     2-D checks (pytorch/abft/injector.py:176-187)     (all batches in one launch,
 *                                                        per-batch fault counts)
 *
 * Conventions
 *   - Every pointer argument that names tensor data is a DEVICE pointer.
 *     Matrices are row-major bf16 (raw 16-bit storage) -- the fused GEMM also
 *     takes fp16 (abft_gemm_args.dtype) and the post-hoc check fp16 and fp32
 *     (abft_check_args.dtype); leading dimensions are in elements.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - The library allocates nothing per call.  Scratch space, when a call needs
 *     any, comes from the caller through `workspace`.
 *   - Every entry point returns an abft_status code (0 = ABFT_OK) and never
 *     throws.  abft_status_string() turns a code into text.
 *   - Calls are reentrant: distinct calls on distinct buffers may run
 *     concurrently on different streams.
 *   - The fused GEMM kernel is launched with programmatic stream
 *     serialization: its prologue may overlap the previous kernel on the
 *     stream, and it reads or writes global memory only after that kernel
 *     has completed (griddepcontrol.wait).
 *   - abft_gemm_bf16 / abft_gemm and abft_check_only may be captured in a
 *     CUDA graph. Under stream capture the fused GEMM adds one small kernel
 *     ahead of its own that clears the stream-K flags in the workspace and
 *     the report's launch_tag, because a replay reuses the launch tag frozen
 *     in the kernel node; every replay then writes a fresh report. The
 *     caller keeps the workspace, report and operands alive for as long as
 *     the graph may replay, and does not overlap replays with other calls
 *     that use the same workspace.
 */
#ifndef ABFT_B200_H_
#define ABFT_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ABFT_B200_VERSION 5

/* ---- return codes ------------------------------------------------------- */
enum abft_status {
  ABFT_OK = 0,
  ABFT_ERR_INVALID_ARG = -1,   /* null pointer, negative size, bad mode      */
  ABFT_ERR_ALIGNMENT = -2,     /* base or leading dimension breaks TMA rules */
  ABFT_ERR_UNSUPPORTED = -3,   /* shape / tile combination not built         */
  ABFT_ERR_WORKSPACE = -4,     /* workspace missing or too small             */
  ABFT_ERR_CUDA = -5,          /* CUDA runtime error (launch or attribute)   */
  ABFT_ERR_NO_DEVICE = -6,     /* no sm_100 device current                   */
  ABFT_ERR_DRIVER = -7         /* tensor-map encoder unavailable             */
};

/* ---- element types of the post-hoc check (abft_check_args.dtype) -------- */
#define ABFT_DTYPE_BF16 0      /* bfloat16 (raw 16-bit storage)                */
#define ABFT_DTYPE_F16  1      /* IEEE half                                    */
#define ABFT_DTYPE_F32  2      /* IEEE single                                  */

/* ---- mode bits for abft_gemm_bf16 -------------------------------------- */
#define ABFT_MODE_OFF      0u  /* plain GEMM (+bias); same kernel, checks compiled out */
#define ABFT_MODE_DETECT   1u  /* per-tile weighted row checksums: detect + locate     */
#define ABFT_MODE_CORRECT  2u  /* also correct located faults before the bf16 store    */
#define ABFT_MODE_REF      4u  /* scalar corner-vs-sum(C) check of checkers.py:112-126 */
#define ABFT_MODE_REF_BF16 8u  /* with MODE_REF: bf16-rounded sums (python backend)    */

/* ---- status bits in abft_report.status ---------------------------------- */
#define ABFT_STATUS_FAULT          1u  /* at least one checksum mismatch          */
#define ABFT_STATUS_UNLOCATED      2u  /* a mismatch could not be pinned to a column */
#define ABFT_STATUS_OVERFLOW       4u  /* more faults than record slots          */
#define ABFT_STATUS_DEVICE_TIMEOUT 8u  /* a bounded device wait gave up          */
#define ABFT_STATUS_REF_FAIL      16u  /* scalar reference-rule check failed     */
/* Mismatches in so many rows of one 128-row slab of a tile segment (more
 * than ABFT_SUSPECT_ROWS, or at least 4 and more than half of the slab's
 * rows) that the checksums or an operand, not single output elements, are
 * wrong -- e.g. a cached checksum block that no longer matches its weight.
 * Nothing in such a slab is corrected (its records carry
 * ABFT_REC_SUPPRESSED instead of ABFT_REC_CORRECTED), so the stored output
 * is the plain product; re-encode the weight's checksums. */
#define ABFT_STATUS_SUSPECT       32u
#define ABFT_SUSPECT_ROWS         16

/* ---- record flags ------------------------------------------------------- */
#define ABFT_REC_DETECTED   1u
#define ABFT_REC_LOCATED    2u
#define ABFT_REC_CORRECTED  4u
#define ABFT_REC_SUPPRESSED 8u  /* located, but left uncorrected (ABFT_STATUS_SUSPECT) */

/* One detected fault: the (row, tile-segment) whose checksums disagree.
 * `col` is the located global column, or -1 when the weighted residual did
 * not pin a single column. In a batched call `row` is flattened over the
 * batch: b * M + i for row i of batch b. `residual` is (actual - expected) row sum over the
 * tile segment (the fault magnitude for a single fault), `residual_w` the same
 * for the column-index-weighted sum, `threshold` the bound it was tested on. */
typedef struct abft_fault_record {
  int32_t row;
  int32_t col;
  float residual;
  float residual_w;
  float threshold;
  uint32_t flags;
} abft_fault_record;

/* Fault report, device-resident, caller-allocated with abft_report_bytes(),
 * 16-byte aligned. abft_gemm_bf16 / abft_check_only reset the header on the
 * call's stream (the fused kernel resets it itself and publishes launch_tag,
 * a value unique to the launch, once the header is valid), so the caller
 * need not zero it. */
typedef struct abft_report {
  uint32_t status;       /* ABFT_STATUS_* bits                               */
  uint32_t n_faults;     /* mismatching (row, tile) segments, all of them     */
  uint32_t n_located;    /* of those, pinned to one column                    */
  uint32_t n_corrected;  /* of those, corrected in the stored output          */
  uint32_t overflow;     /* records dropped for lack of capacity              */
  uint32_t capacity;     /* record slots after this header                    */
  uint32_t tile_m;       /* output tile the checksums were defined on         */
  uint32_t tile_n;       /* data columns per tile (tile width - 8 with checks) */
  float corner;          /* ABFT_MODE_REF: dot(sum_rows(A), sum_cols(B)) + M*sum(bias) */
  float sum_c;           /* ABFT_MODE_REF: sum of the stored output            */
  float abs_err;         /* ABFT_MODE_REF: |corner - sum_c|                    */
  float rel_err;         /* ABFT_MODE_REF: abs_err / max(|sum_c|, 1)           */
  int32_t ref_ok;        /* ABFT_MODE_REF: 1 pass, 0 fail; -1 not evaluated     */
  uint32_t batch;        /* per-batch counter entries after the records (0 = none) */
  uint64_t launch_tag;   /* fused GEMM: tag of the launch that wrote the header */
  /* abft_fault_record records[capacity] follows (64-byte header); a batched
   * fused call (batch > 1) then writes uint32_t counts[batch][4] = {faults,
   * located, corrected, 0} of each batch, complete even when records
   * overflowed. Size such a report with abft_report_bytes_batched(). */
} abft_report;

/* Arguments of the fused checksum-protected GEMM
 *   C[M, N] = A[M, K] * B[N, K]^T (+ bias[N])
 * B is stored like nn.Linear.weight: N rows of K contiguous elements.       */
typedef struct abft_gemm_args {
  const void* A;          /* [M, lda], element type `dtype` (bf16 or fp16)    */
  const void* B;          /* [N, ldb]                                         */
  void* C;                /* [M, ldc] output                                  */
  const void* bias;       /* [N] or NULL                                      */
  int64_t M, N, K;
  int64_t lda, ldb, ldc;
  uint32_t mode;          /* ABFT_MODE_* bits                                 */
  int32_t tile_n;         /* 0 = choose, else 128 or 256                      */
  float thr_scale;        /* tau in thr = tau * sqrt(K) * max|C_row_segment|  */
  float thr_abs;          /* absolute floor added to thr                      */
  float tol_abs, tol_rel; /* ABFT_MODE_REF tolerances (checkers.py:96-110)    */
  const void* checksums;  /* abft_encode_weight_typed(B, tile_n, dtype)      */
                          /* output, or NULL                                  */
  void* workspace;        /* device scratch, abft_gemm_workspace_bytes()      */
  size_t workspace_bytes;
  const int32_t* inject_rows;   /* debug: faults added to the fp32 accumulator */
  const int32_t* inject_cols;   /*        before the checksum epilogue, device */
  const float* inject_deltas;   /*        arrays of n_inject entries           */
  int32_t n_inject;             /*        (at most ABFT_MAX_INJECT)             */
  void* report;           /* abft_report + records, or NULL when mode == OFF  */
  int32_t report_capacity;
  int32_t num_sms;        /* 0 = all SMs of the current device                */
  int32_t tile_m;         /* 0 = choose; 128; or 256: each tile is shared by  */
                          /* a 2-CTA cluster (one pair MMA, M = 256), with     */
                          /* either tile_n                                    */
  int32_t swap_ab;        /* 0 = choose; 1 = never; 2 = always: compute C^T =  */
                          /* B A^T with the weight on the MMA's 128-row side   */
                          /* and the few rows of A as a narrow tile (chosen    */
                          /* for M <= 64 when tile_m is 0); checksums then     */
                          /* come from A, per                                  */
                          /* call, and `checksums` is not used                */
  /* Batched products (torch.bmm): C[b] = A[b] B[b]^T for b < batch, in one
   * launch. batch 0 or 1 is a single product and the strides are ignored.
   * With batch > 1, matrix b of each operand starts stride_* elements after
   * matrix b - 1 (multiples of 8; stride_c a multiple of ldc of at least
   * M * ldc: C's batches are disjoint row blocks), `checksums` (optional)
   * holds the blocks
   * of all batches back to back (abft_encode_weight_batched), inject_rows
   * and the records use rows flattened over the batch, the report needs
   * abft_report_bytes_batched(report_capacity, batch) bytes, and
   * ABFT_MODE_REF is not supported. */
  int32_t batch;
  /* Layout of B: 0 = [N, ldb] (K-major, nn.Linear.weight); 1 = [K, ldb]
   * with N columns (N-major, torch.bmm's mat2 as stored), copied K-major
   * into the workspace by the call (its checksums computed on the way;
   * `checksums` must then be NULL). */
  int32_t b_kn;
  int64_t stride_a, stride_b, stride_c;
  /* Element type of A, B, C and bias: ABFT_DTYPE_BF16 (0) or ABFT_DTYPE_F16;
   * fp32 operands return ABFT_ERR_UNSUPPORTED (check them post hoc). Both
   * types run the same kind::f16 MMAs with fp32 accumulation; fp16 checksum
   * rows carry a per-tile scale (abft_encode_weight_typed). */
  int32_t dtype;
} abft_gemm_args;

#define ABFT_MAX_INJECT 64

/* Library version (ABFT_B200_VERSION) and the human-readable text of a code. */
int abft_version(void);
const char* abft_status_string(int status);

/* Bytes of a report with `capacity` records. */
size_t abft_report_bytes(int32_t capacity);

/* Bytes of the report of a batched fused call: `capacity` records and the
 * per-batch counters (equal to abft_report_bytes(capacity) for batch <= 1). */
size_t abft_report_bytes_batched(int32_t capacity, int32_t batch);

/* Tile width (256 or 128) the library picks for an M x N x K GEMM in `mode`
 * when tile_n == 0: the shorter estimated time over num_sms (whole-tile
 * waves, with stream-K for a last wave that would leave SMs idle; a 128-wide
 * tile's k-block counted as 0.7 of a 256-wide one; for 256-wide tiles the
 * better of 128-row tiles and CTA pairs). */
int32_t abft_pick_tile_n(int64_t M, int64_t N, int64_t K, int32_t num_sms, uint32_t mode);

/* Tile height (128, or 256 = CTA pairs) the library picks when tile_m == 0,
 * for a given tile_n: the shorter estimated schedule, pairs over num_sms / 2
 * units at a per-SM speed-up of 1.15 (128 whenever tile_n != 256: pairs of
 * 128-wide tiles run only on request). */
int32_t abft_pick_tile_m(int64_t M, int64_t N, int64_t K, int32_t num_sms, uint32_t mode, int32_t tile_n);

/* Bytes of the per-tile checksum block of a [N, K] weight for tile_n. */
size_t abft_checksum_bytes(int64_t N, int64_t K, int32_t tile_n);

/* Per-tile weighted row checksums of B (the "Be" encoding of checkers.py:119,
 * restricted to each output tile and paired with a column-index-weighted
 * and a signed copy), as the 8 bf16 rows the fused GEMM appends to each
 * B-operand tile. With checks on, an output tile of width tile_n carries
 * D = tile_n - 8 data columns. out is bf16 [ceil(N/D) * 8, K] row-major; for
 * tile t, with j over the tile's valid rows and fp32 sums,
 *   v1[k] = sum_j B[t*D + j, k]
 *   v2[k] = sum_j (j+1) B[t*D + j, k]
 *   v3[k] = sum_j sg(j) B[t*D + j, k],  sg(j) = (-1)^popcount(j)
 *           (the Thue-Morse sign of the local column j)
 * Rows 8t+0..2 hold v1 split into three bf16 terms (hi = bf16(v1),
 * mid = bf16(v1 - hi), lo = bf16(v1 - hi - mid)), rows 8t+3..5 the same for
 * v2, rows 8t+6..7 v3 as two terms (hi, v3 - hi). All eight rows are read by
 * the fused check: a block built with any row left zero reports faults on
 * clean outputs. Cache it per weight. Replaces the per-call
 * `b_2d.sum(dim=1)` of checkers.py:119. */
int abft_encode_weight(const void* B, int64_t N, int64_t K, int64_t ldb,
                       int32_t tile_n, void* out, void* stream);

/* abft_encode_weight of `batch` matrices B + b * stride_b (stride_b a
 * multiple of 8 elements); block b lands at out + b * abft_checksum_bytes(N,
 * K, tile_n). */
int abft_encode_weight_batched(const void* B, int64_t N, int64_t K, int64_t ldb, int64_t stride_b,
                               int32_t batch, int32_t tile_n, void* out, void* stream);

/* Bytes of one batch's checksum block for element type `dtype`: for bf16
 * abft_checksum_bytes; for fp16 the same rows (fp16 terms) followed by a
 * scale table of 8 floats per tile; 0 for other types or tile widths. */
size_t abft_checksum_bytes_typed(int64_t N, int64_t K, int32_t tile_n, int32_t dtype);

/* abft_encode_weight_batched for B of element type `dtype`; block b lands
 * at out + b * abft_checksum_bytes_typed(N, K, tile_n, dtype).
 * fp16 has a narrow exponent range (largest finite 65504), so for each tile
 * and each of v1, v2, v3 an exponent e is chosen that puts the largest
 * |value| over k in [2^14, 2^15) (e = 0 when that value is 0 or not
 * finite; e within [-100, 100]); the rows hold the fp16 terms of v * 2^-e
 * (three for v1 and v2, two for v3, as above) and table entries 8t+4..6 the
 * factors 2^e, which the fused check multiplies back (exact). Entries
 * 8t+0..2 hold the largest |v1|, |v2|, |v3| (NaN sums passed over); 8t+3
 * and 8t+7 are 0. One launch (an 8-CTA cluster per tile and batch). */
int abft_encode_weight_typed(const void* B, int64_t N, int64_t K, int64_t ldb, int64_t stride_b,
                             int32_t batch, int32_t tile_n, int32_t dtype, void* out, void* stream);

/* Workspace the fused GEMM needs for these arguments (0 when none). */
size_t abft_gemm_workspace_bytes(const abft_gemm_args* args);

/* What abft_gemm launches for these arguments on the current device, in the
 * frame the kernel runs in (with swapped operands, few output rows: the
 * weight on the kernel's row side). No device work. */
typedef struct abft_plan_info {
  int32_t tile_n;         /* MMA tile width: 256 or 128                           */
  int32_t tile_m;         /* output rows per tile: 128, or 256 (CTA pairs)        */
  int32_t data_cols;      /* data columns per tile (tile_n - 8 with checks)       */
  int32_t tiles_n;        /* tile columns                                          */
  int32_t last_cols;      /* data columns of the last tile column (a compact tail
                             tile when fewer than data_cols)                       */
  int32_t swapped;        /* 1: operands swapped                                   */
  int32_t units;          /* CTAs, or CTA pairs, the schedule spreads tiles over   */
  int32_t grid;           /* CTAs launched                                         */
  int32_t dp_tiles;       /* tiles run whole (data-parallel waves)                 */
  int32_t sk_units;       /* units sharing the remaining tiles stream-K (0: none)  */
  int64_t tiles;          /* output tiles of the launch (all batches)              */
  uint64_t workspace_bytes;
} abft_plan_info;

/* Fills *info for the arguments abft_gemm would take (validated the same
 * way; only sizes are read, so placeholder addresses do). Returns ABFT_OK
 * (info all zero when M or N is 0: nothing launches) or the error abft_gemm
 * would return first. */
int abft_gemm_plan(const abft_gemm_args* args, abft_plan_info* info);

/* The fused checksum-protected GEMM. Replaces F.linear + CheapSumChecker.check
 * (pytorch/abft/injector.py:152-161 -> pytorch/abft/checkers.py:55-126). */
int abft_gemm_bf16(const abft_gemm_args* args, void* stream);

/* The same entry under a type-neutral name (args->dtype selects the type in
 * both). */
int abft_gemm(const abft_gemm_args* args, void* stream);

/* Self-test of the library's bounded device waits (failure detection
 * without a fault): one small launch waits for a device flag that nothing
 * sets and for an mbarrier phase that never completes, through the same
 * bounded waits the fused kernel uses. Each gives up after its limit (2 s)
 * instead of hanging; the report (abft_report_bytes(0) bytes, 16-byte
 * aligned, zeroed by the call) then holds ABFT_STATUS_DEVICE_TIMEOUT and
 * n_faults = 2 (the waits that gave up). The launch takes about 4 s; the
 * context stays usable. */
int abft_wait_selftest(void* report, void* stream);

/* Post-hoc check of an existing output C = A * B^T (+ bias), the drop-in for
 * the reference's abft_fused(a, b, c, bias) -> [corner, sum_c]
 * (pytorch/abft/kernels/abft_fused.cpp:11-31, abft_fused.cu:92-141) and the
 * "python" backend arithmetic (pytorch/abft/checkers.py:112-126):
 *   corner = dot(sum_i A[i,:], sum_j B[j,:]) + M * sum(bias)
 *   sum_c  = sum(C)
 *   ok     = |corner - sum_c| <= tol_abs  or  |corner - sum_c| / max(|sum_c|, 1) <= tol_rel
 * Results land in report->corner/sum_c/abs_err/rel_err/ref_ok.
 * A, B, C and bias all have the element type `dtype` (bf16, fp16 or fp32,
 * the types the reference's extension dispatches on, abft_fused.cu:116-118);
 * sums accumulate in fp32.
 * ABFT_CHECK_NATIVE_SUMS rounds every intermediate (both sum vectors, the
 * dot, the bias term, sum_c, the errors and the tolerances) to that element
 * type, as the reference's python backend does on tensors of that type (a
 * no-op for fp32); otherwise all sums are fp32 (the reference's
 * force_fp32_check intent, pytorch/abft/config.py:21). Its older name
 * ABFT_CHECK_BF16_SUMS is the same bit.
 * ABFT_CHECK_LOCATE also compares every row and column sum of C with
 * A (B e) and (e^T A) B and records mismatches: a row and a column whose
 * residuals agree are one located fault (row, col); an unpaired row is
 * recorded as (row, -1) and an unpaired column as (-1, col). */
#define ABFT_CHECK_LOCATE      1u
#define ABFT_CHECK_NATIVE_SUMS 2u
#define ABFT_CHECK_BF16_SUMS   ABFT_CHECK_NATIVE_SUMS

typedef struct abft_check_args {
  const void* A;          /* [M, lda] of `dtype`                              */
  const void* B;          /* [N, ldb] (b_kn == 0) or [K, ldb] (b_kn == 1)     */
  const void* C;          /* [M, ldc]                                         */
  const void* bias;       /* [N] or NULL                                      */
  int64_t M, N, K;
  int64_t lda, ldb, ldc;
  int32_t b_kn;           /* layout of B, see above                           */
  uint32_t flags;         /* ABFT_CHECK_* bits                                */
  float tol_abs, tol_rel; /* scalar rule tolerances (checkers.py:96-110)      */
  float thr_scale;        /* tau of the row/column bounds (ABFT_CHECK_LOCATE) */
  int32_t report_capacity;
  void* report;           /* abft_report + records                            */
  void* workspace;        /* device scratch, abft_check_workspace_bytes()     */
  size_t workspace_bytes;
  int32_t dtype;          /* ABFT_DTYPE_* of A, B, C and bias (0 = bf16)      */
} abft_check_args;

size_t abft_check_workspace_bytes(const abft_check_args* args);
int abft_check_only(const abft_check_args* args, void* stream);

/* abft_check_only without a caller-provided workspace; it allocates nothing.
 * No counterpart in the reference (its check allocates its outputs with
 * torch::zeros on every call, pytorch/abft/kernels/abft_fused.cu:98-99).
 *
 * For callers that cannot call cudaMalloc: a serving loop that may not
 * stall on the device synchronisation cudaMalloc implies, an engine whose
 * memory pool already reserves the device memory, or a binding from a
 * runtime with no device allocator of its own. They still pass A, B, C,
 * bias and the report; `workspace` and `workspace_bytes` are ignored.
 *
 * Scratch comes from one fixed device array of ABFT_NO_ALLOC_SCRATCH_BYTES
 * (4 MiB) inside the library, which every GPU that loads the library holds
 * until the process exits. A shape whose abft_check_workspace_bytes()
 * exceeds it is rejected with ABFT_ERR_WORKSPACE before any device work.
 * The need grows mostly with N: 4096^3 takes 0.55 MiB, 16384^3 1.25 MiB,
 * 65536^3 3.75 MiB, while M = K = 8192 with N = 131072 (4.3 MiB) is rejected.
 * The first call on each device looks up the array's device address once,
 * with that device current; make that first call before any stream capture.
 * All calls share the array and every call overwrites the part it uses
 * before reading it (nothing has to start at zero; the report header is
 * reset on the call's stream as in abft_check_only). Calls that overlap on
 * the GPU -- on different streams, or on different host threads for the
 * same device -- race on the array: serialise them. */
#define ABFT_NO_ALLOC_SCRATCH_BYTES (4u << 20)
int abft_check_only_noalloc(const abft_check_args* args, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* ABFT_B200_H_ */
