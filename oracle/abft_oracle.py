"""CPU oracle for the checksum-protected GEMM -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the arithmetic the CUDA library must
reproduce. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg import it, and only as the checker; the product path never calls it.

Parity status
  * The scalar corner check (``cheap_sum_check``) follows the reference's
    python backend, pytorch/abft/checkers.py:112-126 (sums), :96-110
    (tolerance rule), and is pinned against outputs of the reference itself
    (tests/golden/ref_checker_cases.*, written by tests/golden/make_golden.py).
  * The fault-injection index sequence (``InjectorRng``) follows
    pytorch/abft/injector.py:24, :53-56 and :58-75 and is pinned the same way.
  * The per-tile weighted row-checksum check (``rowcheck_gemm``) and the
    post-hoc row/column locate (``locate_post_hoc``) have no counterpart in
    the reference (it detects only; pytorch/abft/config.py:22 detect_only).
    They extend its checksum algebra and are pinned by the injected
    coordinates the reference's own injector RNG picks, plus seeded fixtures
    committed under tests/golden/.
"""
from __future__ import annotations

import math
import random
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

REC_DETECTED = 1
REC_LOCATED = 2
REC_CORRECTED = 4
REC_SUPPRESSED = 8

TILE_M = 128
# A slab of TILE_M rows in one tile column whose mismatching rows exceed
# this count (or number at least 4 and more than half of its valid rows)
# is left uncorrected: the checksums, not single elements, are wrong.
SUSPECT_ROWS = 16


# ---------------------------------------------------------------- bf16 helpers
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 storage -> float32 values."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 storage, round to nearest even (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if np.any(nan):
        out[nan] = np.uint16(0x7FC0)
    return out


def f16_round(x: np.ndarray) -> np.ndarray:
    """Round float values to the nearest IEEE half (ties to even; beyond
    65504 to infinity), returned as float32."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float values to the nearest bf16 value (returned as float32)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x, dtype=np.float32)))


# ------------------------------------------------- reference scalar corner check
@dataclass
class CheapSumResult:
    ok: bool
    abs_err: float
    rel_err: float
    abft_corner: float
    sum_c: float


def cheap_sum_check(
    a: np.ndarray,
    b_kn: np.ndarray,
    c: np.ndarray,
    bias: Optional[np.ndarray] = None,
    tol_abs: float = 1e-2,
    tol_rel: float = 1e-2,
    emulate_bf16: bool = False,
    emulate_f16: bool = False,
) -> CheapSumResult:
    """pytorch/abft/checkers.py:112-126 and :96-110.

    s_a = A.sum(0), s_b = B.sum(1), corner = dot(s_a, s_b) (+ m * sum(bias)),
    sum_c = C.sum(); ok = |corner - sum_c| <= tol_abs or
    |corner - sum_c| / max(|sum_c|, 1) <= tol_rel.

    With ``emulate_bf16`` (``emulate_f16``) every intermediate is rounded to
    bf16 (fp16) the way the reference's python backend does on tensors of
    that type (its results are tensors of the input type; the survey
    confirmed ``a.sum(0).dtype == bfloat16``). Otherwise the arithmetic is
    float64, the fp32-accumulating "triton" backend's intent
    (pytorch/abft/triton_backend.py:42-49) without its rounding.
    """
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b_kn, dtype=np.float64)
    c = np.asarray(c, dtype=np.float64)

    def r(x):
        x = np.asarray(x, dtype=np.float64)
        if emulate_bf16:
            return bf16_round(x).astype(np.float64)
        if emulate_f16:
            return x.astype(np.float32).astype(np.float16).astype(np.float64)
        return x

    def f(x) -> float:
        return float(np.asarray(x).reshape(-1)[0])

    s_a = r(a.sum(axis=0))
    s_b = r(b.sum(axis=1))
    corner = f(r(np.dot(s_a, s_b)))
    if bias is not None:
        m = a.shape[0]
        bsum = f(r(np.asarray(bias, np.float64).sum()))
        corner = f(r(corner + f(r(float(m) * bsum))))
    sum_c = f(r(c.sum()))
    diff = f(r(abs(corner - sum_c)))
    denom = max(abs(sum_c), 1.0)
    rel = f(r(diff / denom))
    if emulate_bf16 or emulate_f16:
        # torch compares a tensor of the input type with a Python float in that type
        tol_abs = f(r(np.float32(tol_abs)))
        tol_rel = f(r(np.float32(tol_rel)))
    ok = bool(diff <= tol_abs or rel <= tol_rel)
    return CheapSumResult(ok, float(diff), float(rel), float(corner), float(sum_c))


# ------------------------------------------------------ injector RNG restatement
class InjectorRng:
    """The random stream of pytorch/abft/injector.py.

    One ``random.Random(seed)`` per injector (:24). A call consumes
    ``rng.random()`` for the injection coin when injection is on and its
    probability is positive (:63-66), then ``rng.randrange(numel)`` for the
    index (:71); the check gate consumes ``rng.random()`` when
    sample_rate < 1 (:53-56), after the injection (wrapped() order, :154-159).
    """

    def __init__(self, seed: int):
        self.rng = random.Random(seed)

    def maybe_inject(self, numel: int, inject: bool, probability: float) -> Optional[int]:
        if not inject or probability <= 0.0:
            return None
        if self.rng.random() >= probability:
            return None
        if numel == 0:
            return None
        return self.rng.randrange(numel)

    def sample(self, sample_rate: float) -> bool:
        if sample_rate >= 1.0:
            return True
        return self.rng.random() < sample_rate


def seeded_fault_positions(m: int, n: int, count: int, seed: int) -> List[Tuple[int, int]]:
    """``count`` fault positions in distinct rows and columns.

    Positions come from ``random.Random(seed).randrange(m*n)`` (the index
    scheme of pytorch/abft/injector.py:71, row-major: row = idx // n,
    col = idx % n); draws that reuse a row or column are skipped.
    """
    rng = random.Random(seed)
    out: List[Tuple[int, int]] = []
    rows, cols = set(), set()
    while len(out) < count:
        idx = rng.randrange(m * n)
        r, c = divmod(idx, n)
        if r in rows or c in cols:
            continue
        rows.add(r)
        cols.add(c)
        out.append((r, c))
    return out


# ----------------------------------------------- per-tile weighted row checksums
def split3_bf16(v: np.ndarray) -> np.ndarray:
    """Three bf16 terms (hi, mid, lo) of float32 values, summing to 24 bits."""
    v = np.asarray(v, dtype=np.float32)
    hi = bf16_round(v)
    r1 = (v - hi).astype(np.float32)
    mid = bf16_round(r1)
    r2 = (r1 - mid).astype(np.float32)
    lo = bf16_round(r2)
    return np.stack([hi, mid, lo])


def col_signs(n: int) -> np.ndarray:
    """+1 / -1 by the parity of the set bits of 0..n-1 (Thue-Morse)."""
    j = np.arange(n)
    par = np.zeros(n, dtype=np.int64)
    x = j.copy()
    while np.any(x):
        par ^= x & 1
        x >>= 1
    return np.where(par == 1, -1.0, 1.0)


def encode_weight(w: np.ndarray, tile_n: int) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Per-tile checksums of a [N, K] weight (float64).

    v1[t, k] = sum_j w[t*tile_n + j, k];  v2[t, k] = sum_j (j+1) w[t*tile_n + j, k];
    v3[t, k] = sum_j sign(j) w[t*tile_n + j, k] (sign: Thue-Morse parity of j)
    over the tile's valid rows j. Row-checksum "Be" of checkers.py:119 per tile.
    """
    w = np.asarray(w, dtype=np.float64)
    n, k = w.shape
    tiles = -(-n // tile_n)
    v1 = np.zeros((tiles, k))
    v2 = np.zeros((tiles, k))
    v3 = np.zeros((tiles, k))
    for t in range(tiles):
        blk = w[t * tile_n:(t + 1) * tile_n]
        wt = np.arange(1, blk.shape[0] + 1, dtype=np.float64)
        v1[t] = blk.sum(axis=0)
        v2[t] = wt @ blk
        v3[t] = col_signs(blk.shape[0]) @ blk
    return v1, v2, v3


def encode_weight_f32_order(w: np.ndarray, tile_n: int) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """v1, v2, v3 of ``encode_weight`` as the library's encode pass forms them
    in fp32: within a tile, group g (0..31) adds rows g, g + 32, ... in that
    order, then the 32 group sums are added in order of g. The products
    (j+1) * w and +-w of 16-bit inputs are exact in fp32, so separate
    multiply and add round as the kernel's fused multiply-add does."""
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    tiles = -(-n // tile_n)
    out = np.zeros((3, tiles, k), dtype=np.float32)
    for t in range(tiles):
        blk = w[t * tile_n:(t + 1) * tile_n]
        nr = blk.shape[0]
        sg = col_signs(nr).astype(np.float32)
        acc = np.zeros((3, k), dtype=np.float32)
        for g in range(32):
            part = np.zeros((3, k), dtype=np.float32)
            for j in range(g, nr, 32):
                x = blk[j]
                part[0] = part[0] + x
                part[1] = part[1] + np.float32(j + 1) * x
                part[2] = part[2] + sg[j] * x
            acc = acc + part
        out[:, t] = acc
    return out[0], out[1], out[2]


def f16_checksum_exponent(m: float) -> int:
    """Exponent e of an fp16 checksum scale for largest magnitude m (a
    float32): 2^-e m in [2^14, 2^15) for normal m; 0 for zero, subnormal or
    non-finite m; limited to [-100, 100]."""
    bits = int(np.float32(m).view(np.uint32))
    be = (bits >> 23) & 0xFF
    if be == 0 or be == 0xFF:
        return 0
    return max(-100, min(100, be - 127 - 14))


def encode_weight_f16_block(w: np.ndarray, tile_n: int) -> bytes:
    """The bytes of the fp16 checksum block of a [N, K] fp16 weight for
    output tiles of ``tile_n`` data columns: per tile 8 rows of K halves
    (v1 and v2 each as three fp16 terms, v3 as two, each checksum scaled by
    2^-e), then a table of 8 float32 per tile: [max|v1|, max|v2|, max|v3|,
    0, 2^e1, 2^e2, 2^e3, 0] (maxima over the non-NaN sums)."""
    v = encode_weight_f32_order(w, tile_n)
    tiles, k = v[0].shape
    rows = np.zeros((tiles, 8, k), dtype=np.float16)
    table = np.zeros((tiles, 8), dtype=np.float32)
    for t in range(tiles):
        for q in range(3):
            mags = np.abs(v[q][t])
            mags = mags[~np.isnan(mags)]  # NaN sums are passed over, as fmaxf does
            m = np.float32(mags.max() if mags.size else 0.0)
            e = f16_checksum_exponent(m)
            x = (v[q][t] * np.float32(2.0 ** -e)).astype(np.float32)
            hi = x.astype(np.float16)
            r1 = (x - hi.astype(np.float32)).astype(np.float32)
            mid = r1.astype(np.float16)
            if q < 2:
                lo = (r1 - mid.astype(np.float32)).astype(np.float16)
                rows[t, 3 * q:3 * q + 3] = np.stack([hi, mid, lo])
            else:
                rows[t, 6:8] = np.stack([hi, mid])
            table[t, q] = m
            table[t, 4 + q] = np.float32(2.0 ** e)
    return rows.tobytes() + table.tobytes()


@dataclass
class RowcheckResult:
    records: List[Tuple[int, int, int]]  # (row, col or -1, flags), sorted
    residuals: Dict[Tuple[int, int], Tuple[float, float, float]]  # (row, tile) -> (res1, res2, thr)
    out: np.ndarray  # float32 values of the bf16 output
    acc: np.ndarray  # float64 accumulator incl. injected faults


def thr_k(thr_scale: float, k: int) -> float:
    """tau * sqrt(K), rounded to float32 as the library does on the host."""
    return float(np.float32(float(thr_scale) * math.sqrt(k)))


def rowcheck_gemm(
    a: np.ndarray,
    w: np.ndarray,
    bias: Optional[np.ndarray] = None,
    *,
    tile_n: int,
    thr_scale: float = 1e-3,
    thr_abs: float = 0.0,
    inject: Sequence[Tuple[int, int, float]] = (),
    correct: bool = True,
    checksum_weight: Optional[np.ndarray] = None,
    out_dtype: str = "bf16",
) -> RowcheckResult:
    """Restatement of the fused kernel's checksum epilogue.

    For each output tile (TILE_M x tile_n) and each valid row i in it, with j
    over the tile's valid columns (local index) and acc = A W^T + injected:
      s1 = sum_j acc[i,j]            e1 = A[i,:] . v1
      s2 = sum_j (j+1) acc[i,j]      e2 = A[i,:] . v2
      s3 = sum_j sg(j) acc[i,j]      e3 = A[i,:] . v3      (sg = Thue-Morse sign)
      res_q = s_q - e_q, thr = tau*sqrt(K) * max_j |acc[i,j]| + thr_abs
      detected: |res1| > thr or |res2| > thr * ncols
      located:  |res1| > thr, p = res2/res1 within 0.1 of an integer in [1, ncols]
                and |res3 - sg(p-1) res1| <= res1 / 2
                -> column p-1; corrected (if enabled) by acc[i, col] -= res1,
                unless the slab of TILE_M rows holding row i has more than
                SUSPECT_ROWS mismatching rows in this tile column (or at
                least 4 and more than half of its valid rows): then the
                record is flagged suppressed and nothing is changed.
    Output = bf16(acc (+ bias)), or fp16 with ``out_dtype="f16"``.
    ``checksum_weight`` (default ``w``) is the weight the checksums were
    encoded from: another one models a stale cached checksum block.
    """
    a = np.asarray(a, dtype=np.float64)
    w = np.asarray(w, dtype=np.float64)
    m, k = a.shape
    n = w.shape[0]
    acc = a @ w.T
    for (r, c, d) in inject:
        acc[r, c] += d
    fixed = acc.copy()
    tk = thr_k(thr_scale, k)
    v1, v2, v3 = encode_weight(w if checksum_weight is None else checksum_weight, tile_n)
    records: List[Tuple[int, int, int]] = []
    residuals: Dict[Tuple[int, int], Tuple[float, float, float]] = {}
    for t in range(v1.shape[0]):
        c0 = t * tile_n
        c1 = min(n, c0 + tile_n)
        nc = c1 - c0
        wt = np.arange(1, nc + 1, dtype=np.float64)
        sg = col_signs(nc)
        seg = acc[:, c0:c1]
        s1 = seg.sum(axis=1)
        s2 = seg @ wt
        s3 = seg @ sg
        e1 = a @ v1[t]
        e2 = a @ v2[t]
        e3 = a @ v3[t]
        amax = np.abs(seg).max(axis=1)
        res1 = s1 - e1
        res2 = s2 - e2
        res3 = s3 - e3
        thr = tk * amax + thr_abs
        det = (np.abs(res1) > thr) | (np.abs(res2) > thr * nc)
        for i in np.nonzero(det)[0]:
            flags = REC_DETECTED
            col = -1
            if abs(res1[i]) > thr[i]:
                pos = res2[i] / res1[i]
                pr = float(np.rint(pos))
                if abs(pos - pr) <= 0.1 and 1.0 <= pr <= nc:
                    c = int(pr) - 1
                    if abs(res3[i] - sg[c] * res1[i]) <= 0.5 * abs(res1[i]):
                        col = c
                        flags |= REC_LOCATED
            if col >= 0 and correct:
                s0 = (int(i) // TILE_M) * TILE_M
                nd = int(det[s0:s0 + TILE_M].sum())
                valid = min(TILE_M, m - s0)
                if nd > SUSPECT_ROWS or (nd >= 4 and 2 * nd > valid):
                    flags |= REC_SUPPRESSED
                else:
                    fixed[i, c0 + col] -= res1[i]
                    flags |= REC_CORRECTED
            records.append((int(i), c0 + col if col >= 0 else -1, flags))
            residuals[(int(i), t)] = (float(res1[i]), float(res2[i]), float(thr[i]))
    out = fixed if bias is None else fixed + np.asarray(bias, np.float64)[None, :]
    rnd = f16_round if out_dtype == "f16" else bf16_round
    return RowcheckResult(sorted(records), residuals, rnd(out.astype(np.float32)), acc)


# -------------------------------------------------- post-hoc row / column locate
def locate_post_hoc(
    a: np.ndarray,
    b_kn: np.ndarray,
    c: np.ndarray,
    bias: Optional[np.ndarray] = None,
    thr_scale: float = 1e-3,
    unit: float = 2.0 ** -9,
) -> List[Tuple[int, int]]:
    """Classic row/column checksum locate on an existing output C.

    Row i mismatches when |sum_j C[i,j] - (A (B e))_i - sum(bias)| >
    tau sqrt(K) max_j |C[i,j]| + u sum_j |C[i,j]|; column j when
    |sum_i C[i,j] - ((e^T A) B)_j - M bias_j| > tau sqrt(K) max_i |C[i,j]| +
    u sum_i |C[i,j]|, u = 2^-9 for bf16 outputs (2^-(p+1) for p significand
    bits: 2^-12 for fp16, 2^-25 for fp32).
    A mismatching row pairs with the unique mismatching column whose residual
    agrees within the two thresholds. Returns sorted (row, col) with -1 for an
    unpaired side.
    """
    a = np.asarray(a, np.float64)
    b = np.asarray(b_kn, np.float64)
    c = np.asarray(c, np.float64)
    m, k = a.shape
    tk = thr_k(thr_scale, k)
    bsum = 0.0 if bias is None else float(np.asarray(bias, np.float64).sum())
    bcol = np.zeros(c.shape[1]) if bias is None else m * np.asarray(bias, np.float64)
    rres = c.sum(axis=1) - (a @ b.sum(axis=1) + bsum)
    rthr = tk * np.abs(c).max(axis=1) + unit * np.abs(c).sum(axis=1)
    cres = c.sum(axis=0) - (a.sum(axis=0) @ b + bcol)
    cthr = tk * np.abs(c).max(axis=0) + unit * np.abs(c).sum(axis=0)
    rows = [int(i) for i in np.nonzero(np.abs(rres) > rthr)[0]]
    cols = [int(j) for j in np.nonzero(np.abs(cres) > cthr)[0]]
    used = set()
    out: List[Tuple[int, int]] = []
    for i in rows:
        cand = [j for j in cols if j not in used and abs(rres[i] - cres[j]) <= rthr[i] + cthr[j]]
        if len(cand) == 1:
            used.add(cand[0])
            out.append((i, cand[0]))
        else:
            out.append((i, -1))
    for j in cols:
        if j not in used:
            out.append((-1, j))
    return sorted(out)
