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
from typing import Any, Dict, List, Optional, Tuple


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


# The error entries are kept as tuples (phase, op, shape key, abs_err,
# rel_err, corner, sum_c) and turned into the dicts above at export: a
# deferred flush records every check of a forward pass at once.
def _entry_dict(e: tuple) -> Dict[str, Any]:
    return {"phase": e[0], "op_name": e[1], "shape_key": e[2], "abs_err": e[3], "rel_err": e[4],
            "abft_corner": e[5], "sum_c": e[6]}


_TOP_KEEP = 100  # the reference keeps the 100 largest |err| entries (stats.py:137-139)


class CleanChecks:
    """A fixed sequence of checks, given as (phase, op name, shape key),
    whose results are all clean (no fault, zero error). Built once, it lets
    ``AbftStatsCollector.record_clean`` record the whole sequence again and
    again, as a replayed CUDA graph does, at the cost of its distinct keys
    rather than one ``record_check`` per check."""

    def __init__(self, calls: List[Tuple[str, str, str]]):
        self.n = len(calls)
        self.phase = Counter(p for p, _, _ in calls)
        self.op = Counter(o for _, o, _ in calls)
        self.shape = Counter((p, f"{o}:{k}") for p, o, k in calls)
        self.entries = [(p, o, k, 0.0, 0.0, 0.0, 0.0) for p, o, k in calls]
        self.first: Dict[str, tuple] = {}
        for e in self.entries:
            self.first.setdefault(f"{e[0]}|{e[1]}|{e[2]}", e)


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
        self._max_abs_meta: Optional[tuple] = None
        self._max_rel_meta: Optional[tuple] = None
        # Largest-|err| entries. The reference re-sorts and trims to 100 on
        # every check; trimming only when the list reaches 200 keeps exactly
        # the same 100 (a stable sort by -abs_err: ties keep insertion order).
        self._top: List[tuple] = []
        self._shape_max: Dict[str, tuple] = {}

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

    def record_clean(self, checks: CleanChecks) -> None:
        """``record_check`` of every check in ``checks`` with a clean result
        (ok, zero errors, no fault), in order: the same counters, maxima,
        kept entries and per-shape maxima, in bulk. (A zero error ties with
        a zero maximum, so the maxima's metadata moves to the last entry only
        while no error has been seen; the top list keeps the same entries
        because a stable top-k of a concatenation does not depend on where
        the list was trimmed in between.)"""
        if not checks.n:
            return
        self.total_checks += checks.n
        self.phase_checks.update(checks.phase)
        self.op_checks.update(checks.op)
        self.shape_checks.update(checks.shape)
        last = checks.entries[-1]
        if self.max_abs_err <= 0.0:
            self._max_abs_meta = last
        if self.max_rel_err <= 0.0:
            self._max_rel_meta = last
        self._top.extend(checks.entries)
        if len(self._top) >= 2 * _TOP_KEEP:
            self._trim_top()
        for bucket, e in checks.first.items():
            if bucket not in self._shape_max:
                self._shape_max[bucket] = e

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
        abs_err, rel_err = result.abs_err, result.rel_err
        entry = (phase, op_name, shape_key, abs_err, rel_err, result.abft_corner, result.sum_c)
        self.max_abs_err = max(self.max_abs_err, abs_err)
        self.max_rel_err = max(self.max_rel_err, rel_err)
        if abs_err >= self.max_abs_err:
            self._max_abs_meta = entry
        if rel_err >= self.max_rel_err:
            self._max_rel_meta = entry
        self._top.append(entry)
        if len(self._top) >= 2 * _TOP_KEEP:
            self._trim_top()
        bucket = f"{phase}|{op_name}|{shape_key}"
        prev = self._shape_max.get(bucket)
        if prev is None or abs_err > float(prev[3]):
            self._shape_max[bucket] = entry

        self.total_faults += result.n_faults
        self.total_located += result.n_located
        self.total_corrected += result.n_corrected
        self.total_unlocated += max(result.n_faults - result.n_located, 0)
        for (r, c) in result.located[:8]:
            if len(self.located_coords) < 100:
                self.located_coords.append({"phase": phase, "op_name": op_name, "shape_key": shape_key,
                                            "row": int(r), "col": int(c)})

    def _trim_top(self) -> None:
        self._top = sorted(self._top, key=lambda e: -e[3])[:_TOP_KEEP]

    @property
    def max_abs_err_meta(self) -> Dict[str, Any]:
        return _entry_dict(self._max_abs_meta) if self._max_abs_meta is not None else {}

    @property
    def max_rel_err_meta(self) -> Dict[str, Any]:
        return _entry_dict(self._max_rel_meta) if self._max_rel_meta is not None else {}

    @property
    def top_abs_errs(self) -> List[Dict[str, Any]]:
        """The (at most 100) largest-|err| entries, largest first."""
        self._trim_top()
        return [_entry_dict(e) for e in self._top]

    @property
    def shape_max_abs_err(self) -> Dict[str, Dict[str, Any]]:
        return {k: _entry_dict(e) for k, e in self._shape_max.items()}

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
