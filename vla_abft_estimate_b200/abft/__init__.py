"""Drop-in counterpart of the reference package ``abft`` (pytorch/abft/__init__.py).

Same exported names; the checks run on libabft_b200.so.
"""
from .checkers import (AbftChecker, CheapSumChecker, FusedB200Checker, OpMeta, RowColChecker, UnsupportedOperand,
                       flatten_to_2d_for_mm)
from .config import AbftConfig
from .injector import AbftInjector, CapturedChecks, WeightChecksumCache, result_from_report
from .stats import AbftStatsCollector, CheckResult, percentile, summarize_ms

__all__ = [
    "AbftChecker",
    "AbftConfig",
    "AbftInjector",
    "AbftStatsCollector",
    "CheapSumChecker",
    # additions
    "CapturedChecks",
    "CheckResult",
    "FusedB200Checker",
    "OpMeta",
    "RowColChecker",
    "UnsupportedOperand",
    "WeightChecksumCache",
    "flatten_to_2d_for_mm",
    "percentile",
    "result_from_report",
    "summarize_ms",
]
