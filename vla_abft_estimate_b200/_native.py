"""ctypes binding of libabft_b200.so (declarations: include/abft_b200.h).

The C ABI takes plain pointers and sizes only; this module maps them to
ctypes and raises ``AbftError`` for every non-zero status. There is no
fallback: if the library is missing, every op fails loudly.
"""
from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass, field
from typing import List, Optional

from . import _build

# ---- constants mirrored from include/abft_b200.h ------------------------------
ABFT_OK = 0
MODE_OFF = 0
MODE_DETECT = 1
MODE_CORRECT = 2
MODE_REF = 4
MODE_REF_BF16 = 8

CHECK_LOCATE = 1
CHECK_NATIVE_SUMS = 2  # round sums to the operands' type (bf16 / fp16), as the python backend does
CHECK_BF16_SUMS = CHECK_NATIVE_SUMS

DTYPE_BF16 = 0
DTYPE_F16 = 1
DTYPE_F32 = 2

STATUS_FAULT = 1
STATUS_UNLOCATED = 2
STATUS_OVERFLOW = 4
STATUS_DEVICE_TIMEOUT = 8
STATUS_REF_FAIL = 16
STATUS_SUSPECT = 32
SUSPECT_ROWS = 16

REC_DETECTED = 1
REC_LOCATED = 2
REC_CORRECTED = 4
REC_SUPPRESSED = 8

MAX_INJECT = 64
REPORT_HEADER_BYTES = 64
RECORD_BYTES = 24
BATCH_COUNT_BYTES = 16  # uint32 {faults, located, corrected, 0} per batch after the records
LIB_VERSION = 5

EXPORTED_SYMBOLS = (
    "abft_version",
    "abft_status_string",
    "abft_report_bytes",
    "abft_report_bytes_batched",
    "abft_pick_tile_n",
    "abft_pick_tile_m",
    "abft_checksum_bytes",
    "abft_encode_weight",
    "abft_encode_weight_batched",
    "abft_checksum_bytes_typed",
    "abft_encode_weight_typed",
    "abft_gemm_workspace_bytes",
    "abft_gemm_plan",
    "abft_gemm_bf16",
    "abft_gemm",
    "abft_wait_selftest",
    "abft_check_workspace_bytes",
    "abft_check_only",
    "abft_check_only_noalloc",
)

NO_ALLOC_SCRATCH_BYTES = 4 << 20


class AbftError(RuntimeError):
    """A library call returned a non-zero abft_status."""

    def __init__(self, fn: str, code: int, text: str):
        super().__init__(f"{fn} failed with status {code}: {text}")
        self.fn = fn
        self.code = code


class GemmArgs(ctypes.Structure):
    """Mirror of ``abft_gemm_args``."""

    _fields_ = [
        ("A", ctypes.c_void_p),
        ("B", ctypes.c_void_p),
        ("C", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("M", ctypes.c_int64),
        ("N", ctypes.c_int64),
        ("K", ctypes.c_int64),
        ("lda", ctypes.c_int64),
        ("ldb", ctypes.c_int64),
        ("ldc", ctypes.c_int64),
        ("mode", ctypes.c_uint32),
        ("tile_n", ctypes.c_int32),
        ("thr_scale", ctypes.c_float),
        ("thr_abs", ctypes.c_float),
        ("tol_abs", ctypes.c_float),
        ("tol_rel", ctypes.c_float),
        ("checksums", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("inject_rows", ctypes.c_void_p),
        ("inject_cols", ctypes.c_void_p),
        ("inject_deltas", ctypes.c_void_p),
        ("n_inject", ctypes.c_int32),
        ("report", ctypes.c_void_p),
        ("report_capacity", ctypes.c_int32),
        ("num_sms", ctypes.c_int32),
        ("tile_m", ctypes.c_int32),
        ("swap_ab", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("b_kn", ctypes.c_int32),
        ("stride_a", ctypes.c_int64),
        ("stride_b", ctypes.c_int64),
        ("stride_c", ctypes.c_int64),
        ("dtype", ctypes.c_int32),
    ]


class PlanInfo(ctypes.Structure):
    """Mirror of ``abft_plan_info``."""

    _fields_ = [
        ("tile_n", ctypes.c_int32),
        ("tile_m", ctypes.c_int32),
        ("data_cols", ctypes.c_int32),
        ("tiles_n", ctypes.c_int32),
        ("last_cols", ctypes.c_int32),
        ("swapped", ctypes.c_int32),
        ("units", ctypes.c_int32),
        ("grid", ctypes.c_int32),
        ("dp_tiles", ctypes.c_int32),
        ("sk_units", ctypes.c_int32),
        ("tiles", ctypes.c_int64),
        ("workspace_bytes", ctypes.c_uint64),
    ]

    def as_dict(self) -> dict:
        return {name: int(getattr(self, name)) for name, _ in self._fields_}


class CheckArgs(ctypes.Structure):
    """Mirror of ``abft_check_args``."""

    _fields_ = [
        ("A", ctypes.c_void_p),
        ("B", ctypes.c_void_p),
        ("C", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("M", ctypes.c_int64),
        ("N", ctypes.c_int64),
        ("K", ctypes.c_int64),
        ("lda", ctypes.c_int64),
        ("ldb", ctypes.c_int64),
        ("ldc", ctypes.c_int64),
        ("b_kn", ctypes.c_int32),
        ("flags", ctypes.c_uint32),
        ("tol_abs", ctypes.c_float),
        ("tol_rel", ctypes.c_float),
        ("thr_scale", ctypes.c_float),
        ("report_capacity", ctypes.c_int32),
        ("report", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("dtype", ctypes.c_int32),
    ]


_LIB: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """Load the in-tree shared library (built by ``_build.build()``)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = _build.LIB_PATH
    if not path.exists():
        raise RuntimeError(
            f"{path} is missing: build it with `python -m vla_abft_estimate_b200._build` "
            "(or __graft_entry__.build()); there is no fallback path"
        )
    L = ctypes.CDLL(str(path))
    vp, i32, i64, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
    L.abft_version.restype = ctypes.c_int
    L.abft_version.argtypes = []
    if L.abft_version() != LIB_VERSION:
        raise RuntimeError(f"{path} has ABI version {L.abft_version()}, this binding needs {LIB_VERSION}: "
                           "rebuild it with `python -m vla_abft_estimate_b200._build`")
    L.abft_status_string.restype = ctypes.c_char_p
    L.abft_status_string.argtypes = [ctypes.c_int]
    L.abft_report_bytes.restype = sz
    L.abft_report_bytes.argtypes = [i32]
    L.abft_report_bytes_batched.restype = sz
    L.abft_report_bytes_batched.argtypes = [i32, i32]
    L.abft_pick_tile_n.restype = i32
    L.abft_pick_tile_n.argtypes = [i64, i64, i64, i32, ctypes.c_uint32]
    L.abft_pick_tile_m.restype = i32
    L.abft_pick_tile_m.argtypes = [i64, i64, i64, i32, ctypes.c_uint32, i32]
    L.abft_checksum_bytes.restype = sz
    L.abft_checksum_bytes.argtypes = [i64, i64, i32]
    L.abft_encode_weight.restype = ctypes.c_int
    L.abft_encode_weight.argtypes = [vp, i64, i64, i64, i32, vp, vp]
    L.abft_encode_weight_batched.restype = ctypes.c_int
    L.abft_encode_weight_batched.argtypes = [vp, i64, i64, i64, i64, i32, i32, vp, vp]
    L.abft_checksum_bytes_typed.restype = sz
    L.abft_checksum_bytes_typed.argtypes = [i64, i64, i32, i32]
    L.abft_encode_weight_typed.restype = ctypes.c_int
    L.abft_encode_weight_typed.argtypes = [vp, i64, i64, i64, i64, i32, i32, i32, vp, vp]
    L.abft_gemm_workspace_bytes.restype = sz
    L.abft_gemm_workspace_bytes.argtypes = [ctypes.POINTER(GemmArgs)]
    L.abft_gemm_plan.restype = ctypes.c_int
    L.abft_gemm_plan.argtypes = [ctypes.POINTER(GemmArgs), ctypes.POINTER(PlanInfo)]
    L.abft_gemm_bf16.restype = ctypes.c_int
    L.abft_gemm_bf16.argtypes = [ctypes.POINTER(GemmArgs), vp]
    L.abft_gemm.restype = ctypes.c_int
    L.abft_gemm.argtypes = [ctypes.POINTER(GemmArgs), vp]
    L.abft_wait_selftest.restype = ctypes.c_int
    L.abft_wait_selftest.argtypes = [vp, vp]
    L.abft_check_workspace_bytes.restype = sz
    L.abft_check_workspace_bytes.argtypes = [ctypes.POINTER(CheckArgs)]
    L.abft_check_only.restype = ctypes.c_int
    L.abft_check_only.argtypes = [ctypes.POINTER(CheckArgs), vp]
    L.abft_check_only_noalloc.restype = ctypes.c_int
    L.abft_check_only_noalloc.argtypes = [ctypes.POINTER(CheckArgs), vp]
    _LIB = L
    return L


def status_string(code: int) -> str:
    return lib().abft_status_string(int(code)).decode()


def check(fn: str, code: int) -> None:
    if code != ABFT_OK:
        raise AbftError(fn, code, status_string(code))


# ---- report parsing ----------------------------------------------------------------
@dataclass
class FaultRecord:
    row: int
    col: int
    residual: float
    residual_w: float
    threshold: float
    flags: int

    @property
    def located(self) -> bool:
        return bool(self.flags & REC_LOCATED)

    @property
    def corrected(self) -> bool:
        return bool(self.flags & REC_CORRECTED)

    @property
    def suppressed(self) -> bool:
        """Located, but left uncorrected: its slab mismatched in too many
        rows for single faults (stale checksums or a bad operand)."""
        return bool(self.flags & REC_SUPPRESSED)


@dataclass
class FaultReport:
    """Host copy of an ``abft_report``."""

    status: int = 0
    n_faults: int = 0
    n_located: int = 0
    n_corrected: int = 0
    overflow: int = 0
    capacity: int = 0
    tile_m: int = 0
    tile_n: int = 0
    corner: float = 0.0
    sum_c: float = 0.0
    abs_err: float = 0.0
    rel_err: float = 0.0
    ref_ok: int = -1
    records: List[FaultRecord] = field(default_factory=list)
    # batched calls: (faults, located, corrected) of each batch
    batch_counts: List[tuple] = field(default_factory=list)

    @property
    def fault_detected(self) -> bool:
        return bool(self.status & STATUS_FAULT)

    @property
    def device_timeout(self) -> bool:
        return bool(self.status & STATUS_DEVICE_TIMEOUT)

    @property
    def suspect(self) -> bool:
        """Some slab mismatched in so many rows that nothing in it was
        corrected: the checksums (e.g. a cached block of a weight changed
        behind the cache's back) or an operand are wrong."""
        return bool(self.status & STATUS_SUSPECT)

    def coords(self) -> List[tuple]:
        """Sorted (row, col) of every stored record."""
        return sorted((r.row, r.col) for r in self.records)

    @classmethod
    def from_bytes(cls, buf: bytes) -> "FaultReport":
        if len(buf) < REPORT_HEADER_BYTES:
            raise ValueError("report buffer shorter than its header")
        (status, n_faults, n_located, n_corrected, overflow, capacity, tile_m, tile_n, corner, sum_c, abs_err,
         rel_err, ref_ok) = struct.unpack_from("<8I4fi", buf, 0)
        (batch,) = struct.unpack_from("<I", buf, 52)
        rep = cls(status, n_faults, n_located, n_corrected, overflow, capacity, tile_m, tile_n, corner, sum_c,
                  abs_err, rel_err, ref_ok)
        n = min(n_faults, capacity, (len(buf) - REPORT_HEADER_BYTES) // RECORD_BYTES)
        for i in range(n):
            row, col, res, resw, thr, flags = struct.unpack_from("<iifffI", buf, REPORT_HEADER_BYTES + i * RECORD_BYTES)
            rep.records.append(FaultRecord(row, col, res, resw, thr, flags))
        base = REPORT_HEADER_BYTES + capacity * RECORD_BYTES
        if batch and len(buf) >= base + batch * BATCH_COUNT_BYTES:
            rep.batch_counts = [struct.unpack_from("<3I", buf, base + b * BATCH_COUNT_BYTES) for b in range(batch)]
        return rep

    def batch_view(self, b: int, rows: int) -> "FaultReport":
        """The part of a batched report that belongs to batch ``b`` (``rows``
        rows of C per batch): its counts, and its records with rows local to
        the batch. Without per-batch counters (a one-product call, or an
        empty launch whose header is zero) batch 0 has the header's counts."""
        if b < len(self.batch_counts):
            f, loc, cor = self.batch_counts[b]
        elif not self.batch_counts and b == 0:  # a one-product call: the header counts
            f, loc, cor = self.n_faults, self.n_located, self.n_corrected
        else:
            f, loc, cor = 0, 0, 0
        recs = [FaultRecord(r.row - b * rows, r.col, r.residual, r.residual_w, r.threshold, r.flags)
                for r in self.records if b * rows <= r.row < (b + 1) * rows]
        status = (STATUS_FAULT if f else 0) | (STATUS_UNLOCATED if f > loc else 0)
        status |= STATUS_OVERFLOW if len(recs) < f and (self.status & STATUS_OVERFLOW) else 0
        status |= self.status & STATUS_DEVICE_TIMEOUT
        if any(r.suppressed for r in recs) or (self.status & STATUS_SUSPECT and len(recs) < f):
            status |= STATUS_SUSPECT
        return FaultReport(status, f, loc, cor, max(f - len(recs), 0), self.capacity, self.tile_m, self.tile_n,
                           records=recs)
