"""Checker plugin interface of pytorch/abft/checkers.py on the B200 library.

``OpMeta``, ``AbftChecker``, ``CheapSumChecker`` and ``flatten_to_2d_for_mm``
keep the reference's names, signatures and results
(pytorch/abft/checkers.py:16-150). The reference computes its sums with
torch ops, a JIT CUDA extension or torch fp32 reductions depending on
``checker_backend`` and falls back to torch ops when the extension fails
(:79-92); here every backend name runs the native ``abft_check_only`` kernel
sequence and a failure raises -- there is no fallback path.

``RowColChecker`` is new: the same post-hoc check plus row and column
checksums of C that locate single faults. ``FusedB200Checker`` is the
scalar check with fp32 sums whatever ``checker_backend`` says, for checking
an existing C next to the fused path.
"""
from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from .. import _native as N
from .. import ops
from .config import AbftConfig
from .stats import CheckResult


@dataclass
class OpMeta:
    op_name: str
    phase: str
    shape_key: str


class UnsupportedOperand(ValueError):
    """An operand the library cannot take (dtype, device, alignment)."""


class AbftChecker(ABC):
    @abstractmethod
    def check(
        self,
        a_2d: torch.Tensor,
        b_2d: torch.Tensor,
        c_2d: torch.Tensor,
        meta: OpMeta,
        bias_1d: Optional[torch.Tensor] = None,
    ) -> CheckResult:
        raise NotImplementedError


def _as_lib_operands(
    a_2d: torch.Tensor, b_2d: torch.Tensor, c_2d: torch.Tensor, bias_1d: Optional[torch.Tensor]
) -> Tuple[torch.Tensor, torch.Tensor, str, torch.Tensor, Optional[torch.Tensor]]:
    """Validate and lay out (A, B, C, bias) for abft_check_only.

    B arrives as [K, N] (checkers.py:145-150). When it is the transposed view
    of an nn.Linear weight, the weight itself is passed ([N, K], no copy;
    the reference copies it, fused_backend.py:53-58).
    """
    for name, t in (("a", a_2d), ("b", b_2d), ("c", c_2d)):
        if not t.is_cuda:
            raise UnsupportedOperand(f"{name} is not a CUDA tensor; the library has no CPU path")
        if t.dtype not in ops.CHECK_DTYPES or t.dtype != a_2d.dtype:
            raise UnsupportedOperand(f"{name} is {t.dtype}; the library checks bfloat16, float16 or float32 "
                                     "operands of one type")
    k = a_2d.shape[1]
    n = b_2d.shape[1]
    if k % 8 or n % 8:
        return _padded_operands(a_2d, b_2d, c_2d, bias_1d)
    a = a_2d if a_2d.stride(1) == 1 and a_2d.stride(0) % 8 == 0 else a_2d.contiguous()
    c = c_2d if c_2d.stride(1) == 1 and c_2d.stride(0) % 8 == 0 else c_2d.contiguous()
    bt = b_2d.t()
    if bt.stride(1) == 1 and bt.stride(0) % 8 == 0:
        b, layout = bt, "nk"
    elif b_2d.stride(1) == 1 and b_2d.stride(0) % 8 == 0:
        b, layout = b_2d, "kn"
    else:
        b, layout = b_2d.contiguous(), "kn"
    bias = None
    if bias_1d is not None:
        if not bias_1d.is_cuda or bias_1d.dtype != a_2d.dtype:
            raise UnsupportedOperand(f"bias must be a CUDA {a_2d.dtype} tensor")
        bias = bias_1d.contiguous()
    return a, b, layout, c, bias


def _padded_operands(
    a_2d: torch.Tensor, b_2d: torch.Tensor, c_2d: torch.Tensor, bias_1d: Optional[torch.Tensor]
) -> Tuple[torch.Tensor, torch.Tensor, str, torch.Tensor, Optional[torch.Tensor]]:
    """(A, B, C, bias) zero-padded to K and N multiples of 8.

    The library reads rows in 16-byte pieces, so K and N must be multiples
    of 8; a VLA's action projections (K or N = 7) are not. Zero rows and
    columns add only +0 to the sums the check compares (column sums of A,
    row sums of B, the sums of C and of the bias), so the padded copies are
    checked for the same quantities as the original operands (up to fp32
    summation order, like any other call).
    """
    if bias_1d is not None and (not bias_1d.is_cuda or bias_1d.dtype != a_2d.dtype):
        raise UnsupportedOperand(f"bias must be a CUDA {a_2d.dtype} tensor")
    k = a_2d.shape[1]
    n = b_2d.shape[1]
    pk, pn = -k % 8, -n % 8
    a = F.pad(a_2d, (0, pk)) if pk else _rows_aligned(a_2d)
    b = F.pad(b_2d.t(), (0, pk, 0, pn))  # [N, K] padded, contiguous
    c = F.pad(c_2d, (0, pn)) if pn else _rows_aligned(c_2d)
    bias = None
    if bias_1d is not None:
        bias = F.pad(bias_1d, (0, pn)) if pn else bias_1d.contiguous()
    return a, b, "nk", c, bias


def _rows_aligned(t: torch.Tensor) -> torch.Tensor:
    """t itself when its rows are contiguous and 16-byte aligned, else a copy."""
    return t if t.stride(1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0 else t.contiguous()


class CheapSumChecker(AbftChecker):
    """Scalar full-checksum check (checkers.py:36-126) on libabft_b200.

    s_a = A.sum(0), s_b = B.sum(1), corner = dot(s_a, s_b) (+ M * sum(bias)),
    sum_c = C.sum(); ok = |corner - sum_c| <= tol_abs or
    |corner - sum_c| / max(|sum_c|, 1) <= tol_rel. Operands are bf16, fp16
    or fp32 (the reference's native checker dispatches on the same three,
    pytorch/abft/kernels/abft_fused.cu:116-118). Sums are fp32 unless
    ``cfg.bf16_sums`` (checker_backend "python" or force_fp32_check=False),
    which rounds them to the operands' type exactly as the reference's
    python backend does. The result is read back to the host, as in the
    reference (:103).
    """

    locate: bool = False

    def __init__(self, cfg: AbftConfig) -> None:
        self.cfg = cfg

    def check(
        self,
        a_2d: torch.Tensor,
        b_2d: torch.Tensor,
        c_2d: torch.Tensor,
        meta: OpMeta,
        bias_1d: Optional[torch.Tensor] = None,
    ) -> CheckResult:
        if not self.cfg.record_enable:
            # The reference computes and discards the sums here (:74-75);
            # the result it returns does not depend on them.
            return CheckResult(ok=True, abs_err=0.0, rel_err=0.0, abft_corner=0.0, sum_c=0.0)
        return self.result(self.launch(a_2d, b_2d, c_2d, bias_1d).read())

    def launch(
        self,
        a_2d: torch.Tensor,
        b_2d: torch.Tensor,
        c_2d: torch.Tensor,
        bias_1d: Optional[torch.Tensor] = None,
    ) -> ops.ReportBuffer:
        """Queue the check on the current stream; its report is read later
        (``result(report.read())``), so a caller can defer the host read."""
        a, b, layout, c, bias = _as_lib_operands(a_2d, b_2d, c_2d, bias_1d)
        return ops.check_only(a, b, c, bias, b_layout=layout, tol_abs=self.cfg.tol_abs, tol_rel=self.cfg.tol_rel,
                              locate=self.locate, bf16_sums=self.cfg.bf16_sums, thr_scale=self.cfg.thr_scale,
                              report=ops.ReportBuffer(self.cfg.report_capacity, a.device))

    def result(self, rep: N.FaultReport) -> CheckResult:
        """The CheckResult of a report written by ``launch``."""
        located = tuple((r.row, r.col) for r in rep.records if r.row >= 0 and r.col >= 0)
        ok = rep.ref_ok == 1 and (not self.locate or rep.n_faults == 0)
        return CheckResult(ok=ok, abs_err=float(rep.abs_err), rel_err=float(rep.rel_err),
                           abft_corner=float(rep.corner), sum_c=float(rep.sum_c), n_faults=int(rep.n_faults),
                           n_located=len(located), n_corrected=0, located=located)


class FusedB200Checker(CheapSumChecker):
    """The scalar check of an existing C (the fused kernel's reference mode,
    as a checker plugin): CheapSumChecker's rule with fp32 sums on the
    native kernels, whatever ``cfg.checker_backend`` and
    ``cfg.force_fp32_check`` select. The reference's fused and triton
    backends sum in fp32 too (abft_fused.cu:23-88, triton_backend.py:25-51);
    use CheapSumChecker with the "python" backend for its bf16-rounded sums.
    """

    def launch(
        self,
        a_2d: torch.Tensor,
        b_2d: torch.Tensor,
        c_2d: torch.Tensor,
        bias_1d: Optional[torch.Tensor] = None,
    ) -> ops.ReportBuffer:
        a, b, layout, c, bias = _as_lib_operands(a_2d, b_2d, c_2d, bias_1d)
        return ops.check_only(a, b, c, bias, b_layout=layout, tol_abs=self.cfg.tol_abs, tol_rel=self.cfg.tol_rel,
                              locate=self.locate, bf16_sums=False, thr_scale=self.cfg.thr_scale,
                              report=ops.ReportBuffer(self.cfg.report_capacity, a.device))


class RowColChecker(CheapSumChecker):
    """CheapSumChecker plus row and column checksums of C.

    Each row sum of C is compared with A (B e) and each column sum with
    (e^T A) B under tau sqrt(K) max|C| plus the bf16 rounding of the summed
    elements; a mismatching row and column with agreeing residuals locate a
    fault at their crossing. ``ok`` is False when the scalar rule fails or
    any row or column mismatches.
    """

    locate = True


def flatten_to_2d_for_mm(x: torch.Tensor, right_operand: bool = False) -> Optional[torch.Tensor]:
    """Left operand [..., m, k] -> [m*, k]; right operand [..., k, n] -> [k, n]
    only when the batch prefix is 1 (checkers.py:129-150)."""
    if x.dim() < 2:
        return None
    if not right_operand:
        k = x.shape[-1]
        return x.reshape(-1, k)
    k = x.shape[-2]
    n = x.shape[-1]
    if x.dim() == 2:
        return x
    prefix = 1
    for d in x.shape[:-2]:
        prefix *= int(d)
    if prefix != 1:
        return None
    return x.reshape(k, n)
