"""AbftStatsCollector keeps its error entries compactly and trims the
top-|err| list lazily; its export must equal the per-check bookkeeping of
pytorch/abft/stats.py:85-150 (restated below as the plain loop) on long
sequences with ties, failures and several phases, ops and shapes."""
import random

from vla_abft_estimate_b200.abft.stats import AbftStatsCollector, CheckResult


def _entry(phase, op, key, r):
    return {"phase": phase, "op_name": op, "shape_key": key, "abs_err": r.abs_err, "rel_err": r.rel_err,
            "abft_corner": r.abft_corner, "sum_c": r.sum_c}


class PlainErrors:
    """The error bookkeeping of the reference collector, check by check."""

    def __init__(self):
        self.max_abs_err = self.max_rel_err = 0.0
        self.max_abs_err_meta, self.max_rel_err_meta = {}, {}
        self.top, self.shape_max = [], {}

    def record(self, phase, op, key, r):
        self.max_abs_err = max(self.max_abs_err, r.abs_err)
        self.max_rel_err = max(self.max_rel_err, r.rel_err)
        if r.abs_err >= self.max_abs_err:
            self.max_abs_err_meta = _entry(phase, op, key, r)
        if r.rel_err >= self.max_rel_err:
            self.max_rel_err_meta = _entry(phase, op, key, r)
        self.top.append(_entry(phase, op, key, r))
        if len(self.top) > 100:
            self.top = sorted(self.top, key=lambda x: -x["abs_err"])[:100]
        bucket = f"{phase}|{op}|{key}"
        prev = self.shape_max.get(bucket)
        if prev is None or r.abs_err > float(prev["abs_err"]):
            self.shape_max[bucket] = _entry(phase, op, key, r)


def test_export_equals_plain_bookkeeping():
    rng = random.Random(5)
    for trial in range(6):
        st, plain = AbftStatsCollector(), PlainErrors()
        for i in range(rng.choice([50, 150, 399, 1200])):
            phase = rng.choice(["prefill", "decode"])
            st.set_phase(phase)
            op = rng.choice(["linear", "matmul", "bmm"])
            key = f"A{(rng.choice([8, 16]), 64)}_B{(64, 32)}"
            err = rng.choice([0.0, 0.0, 0.0, 1.0, 2.5, rng.random() * 10])  # many ties
            r = CheckResult(ok=err < 2.0, abs_err=err, rel_err=err / 7, abft_corner=float(i), sum_c=float(-i))
            st.record_check(op, key, r, injected=bool(i % 3 == 0))
            plain.record(phase, op, key, r)
        s = st.export_summary()["abft"]
        assert s["max_abs_err_meta"] == plain.max_abs_err_meta
        assert s["max_rel_err_meta"] == plain.max_rel_err_meta
        assert s["top_abs_errs"] == sorted(plain.top, key=lambda x: -x["abs_err"])[:10]
        assert s["top_abs_errs_by_shape"] == sorted(plain.shape_max.values(), key=lambda x: -float(x["abs_err"]))[:10]
        assert st.top_abs_errs == sorted(plain.top, key=lambda x: -x["abs_err"])[:100]
