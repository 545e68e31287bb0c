"""NVTX ranges of the hooked calls (``AbftConfig(nvtx=True)``): one
balanced "abft.<op> MxNxK" range per F.linear / torch.matmul / torch.bmm,
closed even when the call raises, and none at all with the flag off. Run
on CPU tensors (the checks are then skipped as unsupported operands) with
a recording stand-in for ``torch.cuda.nvtx``."""
import pytest
import torch
import torch.nn.functional as F

from vla_abft_estimate_b200.abft import AbftConfig, AbftInjector, AbftStatsCollector, CheapSumChecker


@pytest.fixture
def ranges(monkeypatch):
    events = []
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda name: events.append(("push", name)))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: events.append(("pop", None)))
    return events


def _injector(nvtx):
    cfg = AbftConfig(enable=True, checker_backend="python", nvtx=nvtx)
    return AbftInjector(cfg, CheapSumChecker(cfg), AbftStatsCollector())


def test_each_hooked_call_is_one_named_range(ranges):
    x = torch.randn(2, 3, 8)
    w = torch.randn(16, 8)
    with _injector(True):
        F.linear(x, w)
        torch.matmul(torch.randn(5, 8), torch.randn(8, 4))
        torch.bmm(torch.randn(3, 5, 8), torch.randn(3, 8, 4))
    assert ranges == [("push", "abft.linear 6x16x8"), ("pop", None),
                      ("push", "abft.matmul 5x4x8"), ("pop", None),
                      ("push", "abft.bmm 15x4x8"), ("pop", None)]


def test_range_closes_when_the_call_raises(ranges):
    with _injector(True):
        with pytest.raises(RuntimeError):
            F.linear(torch.randn(2, 8), torch.randn(16, 9))
    assert [e[0] for e in ranges] == ["push", "pop"]


def test_no_ranges_when_off(ranges):
    with _injector(False):
        F.linear(torch.randn(2, 8), torch.randn(16, 8))
        torch.bmm(torch.randn(3, 5, 8), torch.randn(3, 8, 4))
    assert ranges == []
