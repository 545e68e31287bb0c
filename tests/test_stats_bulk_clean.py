"""``AbftStatsCollector.record_clean`` (a replayed graph's clean checks in
bulk) leaves the collector exactly as one ``record_check`` per check does:
the exported summary is identical, including maxima, their metadata, the
top-100 list and per-shape maxima, with non-clean checks interleaved and
across the top list's trims."""
import json

from vla_abft_estimate_b200.abft.stats import AbftStatsCollector, CheckResult, CleanChecks

CLEAN = CheckResult(ok=True, abs_err=0.0, rel_err=0.0, abft_corner=0.0, sum_c=0.0)


def _calls(n, tag):
    phases = ["prefill", "decode"]
    return [(phases[i % 2], "linear" if i % 3 else "bmm", f"A({i % 7}, 8)_B(8, {tag})_C({i % 7}, {tag})")
            for i in range(n)]


def _replay_per_check(st, calls):
    saved = st.current_phase
    for phase, op, key in calls:
        st.current_phase = phase
        st.record_check(op_name=op, shape_key=key, result=CLEAN)
    st.current_phase = saved


def _dump(st):
    return json.dumps(st.export_summary(), sort_keys=True, default=str)


def test_bulk_clean_matches_per_check_records():
    a, b = AbftStatsCollector(), AbftStatsCollector()
    small, big = _calls(9, 3), _calls(150, 5)
    cs, cb = CleanChecks(small), CleanChecks(big)
    for st, bulk in ((a, False), (b, True)):
        for step in range(6):
            for calls, cc in ((small, cs), (big, cb)):
                if bulk:
                    st.record_clean(cc)
                else:
                    _replay_per_check(st, calls)
            if step == 2:  # a failing check between replays moves the maxima
                st.current_phase = "decode"
                st.record_check(op_name="linear", shape_key="A(1, 8)_B(8, 3)_C(1, 3)",
                                result=CheckResult(ok=False, abs_err=0.5, rel_err=0.25, abft_corner=2.0, sum_c=1.5,
                                                   n_faults=1, n_located=1, n_corrected=1, located=[(0, 2)]),
                                injected=True)
        assert _dump(st) == _dump(a)
    assert a.total_checks == b.total_checks == 6 * 159 + 1


def test_bulk_clean_before_any_error_keeps_last_entry_as_max_meta():
    a, b = AbftStatsCollector(), AbftStatsCollector()
    calls = _calls(5, 11)
    _replay_per_check(a, calls)
    b.record_clean(CleanChecks(calls))
    assert a.max_abs_err_meta == b.max_abs_err_meta and b.max_abs_err_meta["shape_key"] == calls[-1][2]
    assert _dump(a) == _dump(b)
    b.record_clean(CleanChecks([]))
    assert _dump(a) == _dump(b)
