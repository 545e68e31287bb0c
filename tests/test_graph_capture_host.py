"""Host-side rules of ``AbftInjector.capture`` (no GPU needed).

A graph replay repeats the decisions made while it was captured, so
configurations that draw from the injector's random stream per call
(fault injection, sampling) or copy operands to the host (tensor dumps) are
refused before any capture starts. The refusal leaves the injector as it
was. ``CapturedChecks``' recording is checked against fake report arenas:
clean replays recorded in bulk, faults one check at a time (with the same
summary as per-check records), stale checksums warned about, and replays
recorded in order when synchronous and overlapped recording mix.
"""
import json

import pytest

from vla_abft_estimate_b200.abft import AbftConfig, AbftInjector, AbftStatsCollector, CheapSumChecker


def _injector(**kw):
    cfg = AbftConfig(enable=True, checker_backend="b200", **kw)
    return AbftInjector(cfg, CheapSumChecker(cfg), AbftStatsCollector(), defer_reports=False)


@pytest.mark.parametrize("kw,words", [
    (dict(inject_fault=True, inject_probability=0.5), "fault injection"),
    (dict(sample_rate=0.5), "sample_rate"),
    (dict(dump_file="x.pt", dump_shape_key="A(1, 2)_B(2, 3)_C(1, 3)"), "dump_file"),
])
def test_capture_refuses_per_call_draws(kw, words):
    inj = _injector(**kw)
    with pytest.raises(RuntimeError, match=words):
        with inj.capture(graph=None):
            pass
    assert inj.defer_reports is False and inj._graph_keep is None and inj._pending == []


def test_capture_allows_injection_at_probability_zero():
    inj = _injector(inject_fault=True, inject_probability=0.0)
    cap = inj.capture(graph=None)
    # the checks pass; entering would then start a CUDA capture, which needs a GPU
    assert cap.checks is not None and len(cap.checks) == 0


class _FakeArena:
    """Stands in for a device report arena: read() returns the next
    replay's results, and sets ``suspect`` when one of them is stale."""

    def __init__(self, replays):
        self.replays = list(replays)
        self.chunks = [None]
        self.suspect = False

    def read(self, host_chunks=None):
        results, stale = self.replays.pop(0)
        self.suspect |= stale
        return results


def _captured(inj, pending, arena):
    from vla_abft_estimate_b200.abft.injector import CapturedChecks

    checks = CapturedChecks(inj)
    checks._adopt(pending, {0: arena}, [])
    return checks


def test_captured_checks_record_clean_replays_in_bulk_and_faults_per_check():
    from vla_abft_estimate_b200.abft.injector import _CLEAN_RESULT
    from vla_abft_estimate_b200.abft.stats import CheckResult

    inj = _injector()
    pending = [(0, "linear", "decode", (1, 64, 128), False, None),
               (0, "linear", "decode", (1, 128, 64), False, None)]
    fault = CheckResult(ok=False, abs_err=3.0, rel_err=0.5, abft_corner=1.0, sum_c=4.0, n_faults=1, n_located=1,
                        n_corrected=1, located=((0, 5),))
    arena = _FakeArena([([_CLEAN_RESULT, _CLEAN_RESULT], False), ([_CLEAN_RESULT, fault], False),
                        ([_CLEAN_RESULT, _CLEAN_RESULT], False)])
    checks = _captured(inj, pending, arena)
    for _ in range(3):
        checks.record()
    summ = inj.stats.export_summary()
    assert checks.replays_recorded == 3 and summ["abft"]["checks_total"] == 6
    assert summ["abft"]["faults"]["detected_total"] == 1 and summ["abft"]["faults"]["corrected_total"] == 1
    assert summ["abft"]["max_abs_err"] == 3.0

    # the same replays recorded one check at a time give the same summary
    ref = _injector()
    for results in ([_CLEAN_RESULT] * 2, [_CLEAN_RESULT, fault], [_CLEAN_RESULT] * 2):
        ref._record_pending(pending, {0: iter(results)})
    assert json.dumps(summ, sort_keys=True, default=str) == json.dumps(ref.stats.export_summary(), sort_keys=True,
                                                                         default=str)


def test_captured_checks_warn_on_stale_checksums():
    from vla_abft_estimate_b200.abft.stats import CheckResult

    inj = _injector()
    stale = CheckResult(ok=False, abs_err=9.0, rel_err=1.0, abft_corner=0.0, sum_c=9.0, n_faults=40)
    checks = _captured(inj, [(0, "linear", "prefill", (256, 64, 64), False, None)], _FakeArena([([stale], True)]))
    with pytest.warns(RuntimeWarning, match="capture the graph again"):
        checks.record()
    assert checks.stale_checksums and checks.replays_recorded == 1


def test_captured_checks_sync_record_first_records_a_copy_in_flight():
    """A synchronous record() after overlapped ones records the copy still
    in flight first, so replays are recorded in order."""
    from vla_abft_estimate_b200.abft.injector import _CLEAN_RESULT

    inj = _injector()
    checks = _captured(inj, [(0, "linear", "decode", (1, 64, 64), False, None)],
                       _FakeArena([([_CLEAN_RESULT], False)]))
    order = []
    checks._in_flight = ("copy", None)
    checks._record_copy = lambda host, ev: order.append(host)
    checks.record()
    assert order == ["copy"] and checks._in_flight is None and checks.replays_recorded == 1
