"""CPU port of the reference's torch ABFT path -- TEST / BASELINE INFRASTRUCTURE.

Restates, with torch CPU ops, what the reference runs for one protected
GEMM on the host: the GEMM itself (``torch.matmul``, as F.linear /
torch.matmul dispatch it, pytorch/abft/injector.py:154/166) followed by
CheapSumChecker's python backend (pytorch/abft/checkers.py:112-126 sums,
:96-110 tolerance rule). Used only as bench.py's CPU baseline and reference
arm; never by the library.
"""
from __future__ import annotations

import time
from typing import Optional, Tuple

import torch


def reference_protected_matmul(a: torch.Tensor, b_kn: torch.Tensor, bias: Optional[torch.Tensor] = None,
                               tol_abs: float = 1e-2, tol_rel: float = 1e-2) -> Tuple[torch.Tensor, bool]:
    """C = A @ B (+ bias), then the scalar corner check on bf16 tensors."""
    c = torch.matmul(a, b_kn)
    if bias is not None:
        c = c + bias
    s_a = a.sum(dim=0)
    s_b = b_kn.sum(dim=1)
    corner = torch.dot(s_a, s_b)
    if bias is not None:
        corner = corner + float(a.shape[0]) * bias.sum()
    sum_c = c.sum()
    diff = torch.abs(corner - sum_c)
    rel = diff / torch.clamp(torch.abs(sum_c), min=1.0)
    ok = bool((diff <= tol_abs) or (rel <= tol_rel))
    return c, ok


def time_reference_sample(m: int, k: int, n: int, seed: int = 0, min_seconds: float = 0.0,
                          max_reps: int = 1) -> Tuple[float, int, float]:
    """Time the CPU path on an [m, k] x [k, n] bf16 sample.

    Returns (seconds per protected GEMM, repetitions, TFLOP/s).
    """
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(m, k, generator=g) * k ** -0.5).bfloat16()
    b = (torch.randn(k, n, generator=g) * k ** -0.5).bfloat16()
    reference_protected_matmul(a, b)  # first call pays one-time setup
    reps, t_total = 0, 0.0
    while reps < max_reps or t_total < min_seconds:
        t0 = time.perf_counter()
        reference_protected_matmul(a, b)
        t_total += time.perf_counter() - t0
        reps += 1
    per = t_total / reps
    return per, reps, 2.0 * m * n * k / per / 1e12
