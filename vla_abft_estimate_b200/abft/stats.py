"""Check results and the statistics collector of pytorch/abft/stats.py.

``CheckResult``, ``percentile``, ``summarize_ms`` and ``AbftStatsCollector``
keep the reference's names and its ``export_summary`` JSON schema
(pytorch/abft/stats.py:175-220), so report scripts written against the
reference read this output unchanged. Added: per-result fault counts and
located coordinates, and an ``abft.faults`` section with located /
corrected / unlocated totals and checks skipped for unsupported shapes.
"""
from __future__ import annotations

import math
import statistics
from collections import Counter, defaultdict
from dataclasses import dataclass, field
from typing import Any, Dict, List, Tuple


@dataclass
class CheckResult:
    ok: bool
    abs_err: float
    rel_err: float
    abft_corner: float
    sum_c: float
    # B200 additions (defaults keep the reference's 5-field constructor valid)
    n_faults: int = 0
    n_located: int = 0
    n_corrected: int = 0
    located: Tuple[Tuple[int, int], ...] = field(default_factory=tuple)


def percentile(data: List[float], p: float) -> float:
    """Linear-interpolated percentile of sorted ``data`` (stats.py:19-29)."""
    if not data:
        return 0.0
    if len(data) == 1:
        return data[0]
    pos = (len(data) - 1) * p
    lo = int(math.floor(pos))
    hi = int(math.ceil(pos))
    if lo == hi:
        return data[lo]
    return data[lo] + (data[hi] - data[lo]) * (pos - lo)


def summarize_ms(samples: List[float]) -> Dict[str, float]:
    """count / mean / p50 / p90 / p99 of latency samples (stats.py:32-48)."""
    if not samples:
        return {"count": 0, "mean_ms": 0.0, "p50_ms": 0.0, "p90_ms": 0.0, "p99_ms": 0.0}
    xs = sorted(samples)
    return {
        "count": len(xs),
        "mean_ms": statistics.fmean(xs),
        "p50_ms": percentile(xs, 0.50),
        "p90_ms": percentile(xs, 0.90),
        "p99_ms": percentile(xs, 0.99),
    }


def _err_entry(phase: str, op_name: str, shape_key: str, result: CheckResult) -> Dict[str, Any]:
    return {
        "phase": phase,
        "op_name": op_name,
        "shape_key": shape_key,
        "abs_err": result.abs_err,
        "rel_err": result.rel_err,
        "abft_corner": result.abft_corner,
        "sum_c": result.sum_c,
    }


class AbftStatsCollector:
    """Per-phase / per-op / per-shape counters (stats.py:51-220)."""

    def __init__(self) -> None:
        self.current_phase: str = "prefill"
        self.total_checks: int = 0
        self.total_failures: int = 0
        self.total_injections: int = 0
        self.total_detected_injections: int = 0

        self.phase_checks: Counter = Counter()
        self.phase_failures: Counter = Counter()
        self.phase_injections: Counter = Counter()
        self.phase_detected_injections: Counter = Counter()

        self.op_checks: Counter = Counter()
        self.op_failures: Counter = Counter()
        self.shape_checks: Counter = Counter()
        self.shape_failures: Counter = Counter()
        self.max_abs_err: float = 0.0
        self.max_rel_err: float = 0.0
        self.max_abs_err_meta: Dict[str, Any] = {}
        self.max_rel_err_meta: Dict[str, Any] = {}
        self.top_abs_errs: List[Dict[str, Any]] = []
        self.shape_max_abs_err: Dict[str, Dict[str, Any]] = {}

        self.prefill_ms: List[float] = []
        self.decode_step_ms: List[float] = []
        self.e2e_request_ms: List[float] = []
        self.by_prompt_decode_ms: Dict[str, Dict[str, List[float]]] = defaultdict(
            lambda: {"prefill_ms": [], "decode_step_ms": [], "e2e_request_ms": []}
        )

        # B200 additions
        self.total_faults: int = 0
        self.total_located: int = 0
        self.total_corrected: int = 0
        self.total_unlocated: int = 0
        self.skipped_unsupported: int = 0
        self.located_coords: List[Dict[str, Any]] = []

    def set_phase(self, phase: str) -> None:
        self.current_phase = phase

    def record_check(self, op_name: str, shape_key: str, result: CheckResult, injected: bool = False) -> None:
        phase = self.current_phase
        self.total_checks += 1
        self.phase_checks[phase] += 1
        self.op_checks[op_name] += 1
        self.shape_checks[(phase, f"{op_name}:{shape_key}")] += 1

        if not result.ok:
            self.total_failures += 1
            self.phase_failures[phase] += 1
            self.op_failures[op_name] += 1
            self.shape_failures[(phase, f"{op_name}:{shape_key}")] += 1
            if injected:
                self.total_detected_injections += 1
                self.phase_detected_injections[phase] += 1
        self.max_abs_err = max(self.max_abs_err, result.abs_err)
        self.max_rel_err = max(self.max_rel_err, result.rel_err)
        if result.abs_err >= self.max_abs_err:
            self.max_abs_err_meta = _err_entry(phase, op_name, shape_key, result)
        if result.rel_err >= self.max_rel_err:
            self.max_rel_err_meta = _err_entry(phase, op_name, shape_key, result)
        self.top_abs_errs.append(_err_entry(phase, op_name, shape_key, result))
        if len(self.top_abs_errs) > 100:
            self.top_abs_errs = sorted(self.top_abs_errs, key=lambda x: -x["abs_err"])[:100]
        bucket = f"{phase}|{op_name}|{shape_key}"
        prev = self.shape_max_abs_err.get(bucket)
        if prev is None or result.abs_err > float(prev["abs_err"]):
            self.shape_max_abs_err[bucket] = _err_entry(phase, op_name, shape_key, result)

        self.total_faults += result.n_faults
        self.total_located += result.n_located
        self.total_corrected += result.n_corrected
        self.total_unlocated += max(result.n_faults - result.n_located, 0)
        for (r, c) in result.located[:8]:
            if len(self.located_coords) < 100:
                self.located_coords.append({"phase": phase, "op_name": op_name, "shape_key": shape_key,
                                            "row": int(r), "col": int(c)})

    def record_injection(self) -> None:
        self.total_injections += 1
        self.phase_injections[self.current_phase] += 1

    def record_skip_unsupported(self) -> None:
        self.skipped_unsupported += 1

    def record_prefill_latency(self, prompt_len: int, ms: float) -> None:
        self.prefill_ms.append(ms)
        self.by_prompt_decode_ms[str(prompt_len)]["prefill_ms"].append(ms)

    def record_decode_step_latency(self, prompt_len: int, ms: float) -> None:
        self.decode_step_ms.append(ms)
        self.by_prompt_decode_ms[str(prompt_len)]["decode_step_ms"].append(ms)

    def record_e2e_latency(self, prompt_len: int, ms: float) -> None:
        self.e2e_request_ms.append(ms)
        self.by_prompt_decode_ms[str(prompt_len)]["e2e_request_ms"].append(ms)

    def _top_items(self, counter: Counter, k: int = 20) -> List[Dict[str, Any]]:
        return [{"key": str(key), "count": int(v)} for key, v in counter.most_common(k)]

    def export_summary(self) -> Dict[str, Any]:
        detect_rate = (
            float(self.total_detected_injections) / float(self.total_injections) if self.total_injections > 0 else 0.0
        )
        return {
            "latency": {
                "prefill": summarize_ms(self.prefill_ms),
                "decode_step": summarize_ms(self.decode_step_ms),
                "e2e_request": summarize_ms(self.e2e_request_ms),
                "by_prompt_len": {
                    k: {
                        "prefill": summarize_ms(v["prefill_ms"]),
                        "decode_step": summarize_ms(v["decode_step_ms"]),
                        "e2e_request": summarize_ms(v["e2e_request_ms"]),
                    }
                    for k, v in self.by_prompt_decode_ms.items()
                },
            },
            "abft": {
                "checks_total": int(self.total_checks),
                "fail_total": int(self.total_failures),
                "max_abs_err": float(self.max_abs_err),
                "max_rel_err": float(self.max_rel_err),
                "max_abs_err_meta": self.max_abs_err_meta,
                "max_rel_err_meta": self.max_rel_err_meta,
                "top_abs_errs": sorted(self.top_abs_errs, key=lambda x: -x["abs_err"])[:10],
                "top_abs_errs_by_shape": sorted(self.shape_max_abs_err.values(), key=lambda x: -float(x["abs_err"]))[:10],
                "checks_by_phase": dict(self.phase_checks),
                "fails_by_phase": dict(self.phase_failures),
                "checks_by_op": dict(self.op_checks),
                "fails_by_op": dict(self.op_failures),
                "top_shapes_by_checks": self._top_items(self.shape_checks),
                "top_shapes_by_fails": self._top_items(self.shape_failures),
                "faults": {
                    "detected_total": int(self.total_faults),
                    "located_total": int(self.total_located),
                    "corrected_total": int(self.total_corrected),
                    "unlocated_total": int(self.total_unlocated),
                    "skipped_unsupported": int(self.skipped_unsupported),
                    "located": self.located_coords[:20],
                },
            },
            "fault_injection": {
                "injections_total": int(self.total_injections),
                "detected_injections_total": int(self.total_detected_injections),
                "injections_by_phase": dict(self.phase_injections),
                "detected_injections_by_phase": dict(self.phase_detected_injections),
                "detection_rate": detect_rate,
            },
        }
