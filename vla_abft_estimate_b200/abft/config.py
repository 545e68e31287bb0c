"""AbftConfig: the flags of pytorch/abft/config.py:7-46, mapped 1:1.

Every field of the reference keeps its name, default and meaning; the B200
library adds the fields after ``dump_file``. The reference reads neither
``force_fp32_check`` nor ``detect_only``; here both act:
  * force_fp32_check (default True): checker sums in fp32. With False (or
    checker_backend "python") the scalar check rounds its intermediates to
    bf16, reproducing the reference's python backend bit for bit.
  * detect_only (default True): report faults only, like the reference.
    With False the fused linear also corrects every located fault before the
    bf16 store.
"""
from __future__ import annotations

from dataclasses import dataclass

CHECKER_BACKENDS = ("b200", "python", "fused", "triton")


@dataclass
class AbftConfig:
    enable: bool = False
    check_enable: bool = True
    record_enable: bool = True
    # b200 | python | fused | triton. All run on libabft_b200.so; "python"
    # keeps the reference python backend's bf16 arithmetic, the others use
    # fp32 sums. Only "b200" fuses the check into the linear's GEMM.
    checker_backend: str = "b200"
    enable_linear: bool = True
    enable_matmul: bool = True
    enable_bmm: bool = True
    phase: str = "all"  # all | prefill | decode
    sample_rate: float = 1.0
    tol_abs: float = 1e-2
    tol_rel: float = 1e-2
    seed: int = 2026
    force_fp32_check: bool = True
    detect_only: bool = True

    # fault injection (optional)
    inject_fault: bool = False
    inject_phase: str = "all"  # all | prefill | decode
    inject_probability: float = 0.0
    inject_magnitude: float = 1.0
    dump_shape_key: str = ""
    dump_phase: str = "all"  # all | prefill | decode
    dump_file: str = ""

    # ---- B200 library additions -------------------------------------------------
    fused_linear: bool = True  # b200 backend: one fused GEMM+check kernel per F.linear
    # b200 backend: torch.bmm (all batches) and torch.matmul with a 2-D right
    # operand run as one fused GEMM+check launch, per-batch results as the
    # reference's per-batch loop records them
    fused_matmul: bool = True
    # torch.matmul with a batched right operand (attention scores): the
    # reference leaves it unchecked (its b_2d is None); True checks every
    # batch through the fused kernel (b200 backend), recorded as "matmul"
    check_batched_matmul: bool = False
    thr_scale: float = 1e-3  # tau of the per-tile row-checksum bound tau*sqrt(K)*max|C|
    thr_abs: float = 0.0  # absolute floor added to that bound
    report_capacity: int = 64  # fault records kept per call
    # an NVTX range around every hooked F.linear / matmul / bmm call, named
    # "abft.<op> MxNxK" (profilers can select the checked GEMMs of a model
    # with it, e.g. ncu --nvtx --nvtx-include "regex:abft.*/"); read when the
    # injector is entered
    nvtx: bool = False

    def __post_init__(self) -> None:
        if self.checker_backend not in CHECKER_BACKENDS:
            raise ValueError(f"checker_backend must be one of {CHECKER_BACKENDS}, got {self.checker_backend!r}")

    def phase_enabled(self, current_phase: str) -> bool:
        if self.phase == "all":
            return True
        return self.phase == current_phase

    def inject_phase_enabled(self, current_phase: str) -> bool:
        if self.inject_phase == "all":
            return True
        return self.inject_phase == current_phase

    def dump_phase_enabled(self, current_phase: str) -> bool:
        if self.dump_phase == "all":
            return True
        return self.dump_phase == current_phase

    @property
    def bf16_sums(self) -> bool:
        """Whether the scalar check rounds its sums to the operands' type
        (bf16 or fp16), as the python backend's torch reductions do."""
        return self.checker_backend == "python" or not self.force_fp32_check
