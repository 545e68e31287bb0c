"""Host-side rules of ``AbftInjector.capture`` (no GPU needed).

A graph replay repeats the decisions made while it was captured, so
configurations that draw from the injector's random stream per call
(fault injection, sampling) or copy operands to the host (tensor dumps) are
refused before any capture starts. The refusal leaves the injector as it
was.
"""
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
