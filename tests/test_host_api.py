"""Host-side mirror of the reference's pytorch/abft surface, on CPU.

The injector's reference flow runs F.linear on CPU tensors here; its checker
is a test double that evaluates the oracle's restatement of the reference
python backend, so the stream of injected faults, checks and detections can
be compared with the sequences the reference itself produced
(tests/golden/ref_injector_sequences.json).
"""
import dataclasses
import json
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import abft_oracle as O
from vla_abft_estimate_b200.abft import (AbftChecker, AbftConfig, AbftInjector, AbftStatsCollector, CheckResult,
                                         OpMeta, flatten_to_2d_for_mm, percentile, summarize_ms)

# Field names and defaults of pytorch/abft/config.py:7-31.
REFERENCE_CONFIG_DEFAULTS = {
    "enable": False, "check_enable": True, "record_enable": True, "checker_backend": "python",
    "enable_linear": True, "enable_matmul": True, "enable_bmm": True, "phase": "all", "sample_rate": 1.0,
    "tol_abs": 1e-2, "tol_rel": 1e-2, "seed": 2026, "force_fp32_check": True, "detect_only": True,
    "inject_fault": False, "inject_phase": "all", "inject_probability": 0.0, "inject_magnitude": 1.0,
    "dump_shape_key": "", "dump_phase": "all", "dump_file": "",
}


def test_config_keeps_reference_fields_and_defaults():
    cfg = AbftConfig()
    fields = {f.name for f in dataclasses.fields(cfg)}
    for name, default in REFERENCE_CONFIG_DEFAULTS.items():
        assert name in fields, name
        if name != "checker_backend":
            assert getattr(cfg, name) == default, name
    # the reference's backend names are accepted; only their arithmetic differs
    for backend in ("python", "fused", "triton", "b200"):
        AbftConfig(checker_backend=backend)
    with pytest.raises(ValueError):
        AbftConfig(checker_backend="cuda")
    assert AbftConfig(checker_backend="python").bf16_sums
    assert not AbftConfig(checker_backend="b200").bf16_sums
    assert AbftConfig(force_fp32_check=False).bf16_sums


def test_phase_helpers():
    cfg = AbftConfig(phase="prefill", inject_phase="decode", dump_phase="all")
    assert cfg.phase_enabled("prefill") and not cfg.phase_enabled("decode")
    assert cfg.inject_phase_enabled("decode") and not cfg.inject_phase_enabled("prefill")
    assert cfg.dump_phase_enabled("decode")


def test_percentile_and_summary():
    assert percentile([], 0.5) == 0.0
    assert percentile([3.0], 0.9) == 3.0
    assert percentile([1.0, 2.0, 3.0, 4.0], 0.5) == 2.5
    s = summarize_ms([4.0, 1.0, 3.0, 2.0])
    assert s["count"] == 4 and s["mean_ms"] == 2.5 and s["p50_ms"] == 2.5
    assert abs(s["p99_ms"] - 3.97) < 1e-12


class OracleChecker(AbftChecker):
    """Test double: the reference python backend, restated by the oracle."""

    def __init__(self, cfg):
        self.cfg = cfg
        self.calls = []

    def check(self, a_2d, b_2d, c_2d, meta, bias_1d=None):
        self.calls.append(meta)
        r = O.cheap_sum_check(a_2d.float().numpy(), b_2d.float().numpy(), c_2d.float().numpy(),
                              None if bias_1d is None else bias_1d.float().numpy(), self.cfg.tol_abs,
                              self.cfg.tol_rel, emulate_bf16=True)
        return CheckResult(ok=r.ok, abs_err=r.abs_err, rel_err=r.rel_err, abft_corner=r.abft_corner, sum_c=r.sum_c)


def _run_sequence(conf, shapes, gen_seed):
    cfg = AbftConfig(enable=True, inject_fault=True, inject_magnitude=1.0,
                     inject_probability=conf["inject_probability"], sample_rate=conf["sample_rate"],
                     seed=conf["seed"], enable_matmul=False, enable_bmm=False, checker_backend="python")
    stats = AbftStatsCollector()
    checker = OracleChecker(cfg)
    calls = []
    g = torch.Generator().manual_seed(gen_seed)
    with AbftInjector(cfg, checker, stats):
        for (m, k, n) in shapes:
            x = (torch.randn(m, k, generator=g) * 0.1).bfloat16()
            w = (torch.randn(n, k, generator=g) * 0.1).bfloat16()
            before = stats.total_checks
            y = F.linear(x, w)
            clean = torch.ops.aten.linear(x, w)
            diff = (y.float() - clean.float()).abs().view(-1)
            injected = bool(diff.max().item() > 0)
            calls.append({"shape": [m, k, n], "injected": injected,
                          "index": int(diff.argmax().item()) if injected else None,
                          "checked": stats.total_checks - before})
    return calls, stats


def test_injector_reproduces_reference_sequences(golden_dir):
    gold = json.load(open(os.path.join(golden_dir, "ref_injector_sequences.json")))
    for ci, conf in enumerate(gold["configs"]):
        shapes = [tuple(c["shape"]) for c in conf["calls"]]
        calls, stats = _run_sequence(conf, shapes, 100 + ci)
        assert calls == conf["calls"], conf["seed"]
        assert stats.total_injections == conf["total_injections"]
        assert stats.total_detected_injections == conf["detected_injections"]
        assert stats.total_checks == conf["total_checks"]
        assert stats.total_failures == conf["total_failures"]


def _key_paths(d, prefix=""):
    out = set()
    if isinstance(d, dict):
        for k, v in d.items():
            out.add(prefix + "/" + str(k))
            if k not in ("by_prompt_len",):
                out |= _key_paths(v, prefix + "/" + str(k))
    return out


def test_export_summary_schema_superset_of_reference(golden_dir):
    gold = json.load(open(os.path.join(golden_dir, "ref_injector_sequences.json")))
    conf = gold["configs"][0]
    _, stats = _run_sequence(conf, [tuple(c["shape"]) for c in conf["calls"]], 100)
    ours = stats.export_summary()
    ref = gold["summary_config0"]
    missing = _key_paths(ref) - _key_paths(ours)
    assert not missing, missing
    assert ours["fault_injection"] == ref["fault_injection"]
    assert ours["abft"]["checks_total"] == ref["abft"]["checks_total"]
    assert ours["abft"]["fail_total"] == ref["abft"]["fail_total"]
    assert ours["abft"]["checks_by_op"] == ref["abft"]["checks_by_op"]


def test_injector_restores_operators():
    lin, mm, bmm = F.linear, torch.matmul, torch.bmm
    cfg = AbftConfig(enable=True)
    with AbftInjector(cfg, OracleChecker(cfg), AbftStatsCollector()):
        assert F.linear is not lin and torch.matmul is not mm and torch.bmm is not bmm
    assert F.linear is lin and torch.matmul is mm and torch.bmm is bmm


def test_injector_matmul_and_bmm_flow():
    cfg = AbftConfig(enable=True, checker_backend="python")
    stats = AbftStatsCollector()
    checker = OracleChecker(cfg)
    g = torch.Generator().manual_seed(0)
    a = torch.randn(2, 3, 8, 16, generator=g).bfloat16()
    b = torch.randn(16, 8, generator=g).bfloat16()
    x = torch.randn(4, 8, 16, generator=g).bfloat16()
    y = torch.randn(4, 16, 8, generator=g).bfloat16()
    with AbftInjector(cfg, checker, stats):
        torch.matmul(a, b)  # checked: right operand is 2-D
        torch.matmul(a, b.expand(3, 16, 8))  # batched right operand: unchecked (checkers.py:145-149)
        torch.bmm(x, y)  # 4 per-batch checks
    assert stats.op_checks == {"matmul": 1, "bmm": 4}
    assert [m.op_name for m in checker.calls] == ["matmul"] + ["bmm"] * 4


def test_sampling_and_phase_gates():
    cfg = AbftConfig(enable=True, phase="decode", checker_backend="python")
    stats = AbftStatsCollector()
    with AbftInjector(cfg, OracleChecker(cfg), stats):
        F.linear(torch.randn(4, 8).bfloat16(), torch.randn(8, 8).bfloat16())
        stats.set_phase("decode")
        F.linear(torch.randn(4, 8).bfloat16(), torch.randn(8, 8).bfloat16())
    assert stats.total_checks == 1 and stats.phase_checks == {"decode": 1}


def test_dump_tensors(tmp_path):
    path = str(tmp_path / "dump.pt")
    cfg = AbftConfig(enable=True, checker_backend="python", dump_file=path,
                     dump_shape_key="A(4, 8)_B(8, 6)_C(4, 6)")
    with AbftInjector(cfg, OracleChecker(cfg), AbftStatsCollector()):
        F.linear(torch.randn(4, 8).bfloat16(), torch.randn(6, 8).bfloat16())
    payload = torch.load(path)
    assert payload["meta"]["op_name"] == "linear" and tuple(payload["c"].shape) == (4, 6)


def test_flatten_to_2d_for_mm():
    x = torch.zeros(2, 3, 5)
    assert tuple(flatten_to_2d_for_mm(x).shape) == (6, 5)
    assert flatten_to_2d_for_mm(torch.zeros(5)) is None
    assert tuple(flatten_to_2d_for_mm(torch.zeros(1, 4, 6), right_operand=True).shape) == (4, 6)
    assert flatten_to_2d_for_mm(torch.zeros(2, 4, 6), right_operand=True) is None


def test_cpu_operands_are_rejected_by_native_checker():
    from vla_abft_estimate_b200.abft import CheapSumChecker, UnsupportedOperand

    chk = CheapSumChecker(AbftConfig(enable=True))
    with pytest.raises(UnsupportedOperand):
        chk.check(torch.zeros(4, 8).bfloat16(), torch.zeros(8, 8).bfloat16(), torch.zeros(4, 8).bfloat16(),
                  OpMeta("linear", "prefill", "k"))


def test_unsupported_operands_are_counted_not_fatal():
    from vla_abft_estimate_b200.abft import CheapSumChecker

    cfg = AbftConfig(enable=True, checker_backend="fused")
    stats = AbftStatsCollector()
    with AbftInjector(cfg, CheapSumChecker(cfg), stats):
        F.linear(torch.randn(4, 8).bfloat16(), torch.randn(8, 8).bfloat16())
    assert stats.total_checks == 0 and stats.skipped_unsupported == 1


@pytest.mark.parametrize("m,k,n", [(5, 7, 3), (16, 7, 768), (16, 768, 7), (4, 8, 12)])
def test_narrow_operands_padded_with_zeros(m, k, n):
    """K or N not a multiple of 8: the checker's operands are zero-padded
    copies whose check sums (column sums of A times row sums of B, the sum
    of C) equal the originals'."""
    from vla_abft_estimate_b200.abft.checkers import _padded_operands

    torch.manual_seed(m + k + n)
    a = torch.randn(m, k).bfloat16()
    w = torch.randn(n, k).bfloat16()
    c = torch.randn(m, n).bfloat16()
    pa, pb, layout, pc, pbias = _padded_operands(a, w.t(), c, None)
    k8, n8 = -(-k // 8) * 8, -(-n // 8) * 8
    assert layout == "nk" and pbias is None
    assert tuple(pa.shape) == (m, k8) and tuple(pb.shape) == (n8, k8) and tuple(pc.shape) == (m, n8)
    assert torch.equal(pa[:, :k], a) and torch.equal(pb[:n, :k], w) and torch.equal(pc[:, :n], c)
    assert not pa[:, k:].any() and not pb[n:].any() and not pb[:, k:].any() and not pc[:, n:].any()
    corner = (a.double().sum(0) * w.double().sum(0)).sum()
    pcorner = (pa.double().sum(0) * pb.double().sum(0)).sum()
    assert corner.item() == pcorner.item() and c.double().sum().item() == pc.double().sum().item()


class DeferringOracleChecker(OracleChecker):
    """Test double with the launch / result split of the library checker:
    ``launch`` computes the oracle result at call time and returns a report
    stand-in that is only read at flush; ``result`` turns it into the
    CheckResult."""

    class _Report:
        def __init__(self, res):
            self.res = res
            self.reads = 0

        def read(self):
            self.reads += 1
            return self.res

    def __init__(self, cfg):
        super().__init__(cfg)
        self.reports = []

    def launch(self, a_2d, b_2d, c_2d, bias_1d=None):
        rep = self._Report(OracleChecker.check(self, a_2d, b_2d, c_2d, None, bias_1d))
        self.reports.append(rep)
        return rep

    def result(self, rep):
        return rep


def test_deferred_checker_reports_recorded_at_flush_in_call_order():
    """defer_reports with a checker that can launch: nothing is read during
    the forward, flush() records every check in call order with the phase
    of its call, and the statistics equal an immediate-mode run."""
    conf = dict(inject_probability=0.5, sample_rate=1.0, seed=11)
    shapes = [(4, 16, 8), (6, 8, 24), (3, 24, 16), (5, 16, 16)]
    summaries = []
    for defer in (False, True):
        cfg = AbftConfig(enable=True, inject_fault=True, inject_magnitude=1.0, seed=conf["seed"],
                         inject_probability=conf["inject_probability"], enable_matmul=False, enable_bmm=False,
                         checker_backend="python")
        stats = AbftStatsCollector()
        checker = DeferringOracleChecker(cfg)
        g = torch.Generator().manual_seed(3)
        with AbftInjector(cfg, checker, stats, defer_reports=defer) as inj:
            for i, (m, k, n) in enumerate(shapes):
                stats.set_phase("prefill" if i < 2 else "decode")
                F.linear((torch.randn(m, k, generator=g) * 0.1).bfloat16(),
                         (torch.randn(n, k, generator=g) * 0.1).bfloat16())
            if defer:
                assert stats.total_checks == 0 and all(r.reads == 0 for r in checker.reports)
                assert len(inj._pending) == len(shapes)
        if defer:
            assert all(r.reads == 1 for r in checker.reports) and len(checker.reports) == len(shapes)
        s = stats.export_summary()
        summaries.append((s["abft"]["checks_total"], s["abft"]["fail_total"], s["abft"]["checks_by_phase"],
                          s["abft"]["fails_by_phase"], s["fault_injection"]))
    assert summaries[0] == summaries[1]
    assert summaries[0][2] == {"prefill": 2, "decode": 2}
