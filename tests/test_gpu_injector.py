"""The injector's fused-linear path (checker_backend="b200") on a B200.

Every nn.Linear of a small model goes through abft_gemm_bf16. The reference's
random stream (oracle.InjectorRng, pinned on the reference's own sequences)
decides which calls get a fault and where; the kernel must report exactly
those coordinates, correct them, and leave the model output equal to the
clean one. Deferred reports (one device->host copy per flush) must give the
same statistics as reading every report at once.
"""
import pytest
import torch
import torch.nn as nn

from oracle import abft_oracle as O
from vla_abft_estimate_b200.abft import AbftConfig, AbftInjector, AbftStatsCollector, CheapSumChecker

pytestmark = pytest.mark.gpu

SHAPES = [(256, 512, True), (512, 384, False), (384, 1000, True), (1000, 248, False)]  # (in, out, bias)
TOKENS = 96


def make_model(device, seed=0):
    torch.manual_seed(seed)
    layers = []
    for k, n, bias in SHAPES:
        lin = nn.Linear(k, n, bias=bias)
        with torch.no_grad():
            lin.weight.normal_(0.0, k ** -0.5)
            if bias:
                lin.bias.normal_(0.0, 0.02)
        layers.append(lin)
    return nn.Sequential(*layers).to(device=device, dtype=torch.bfloat16).eval()


def run(model, x, cfg, defer):
    stats = AbftStatsCollector()
    inj = AbftInjector(cfg, CheapSumChecker(cfg), stats, defer_reports=defer)
    with torch.inference_mode(), inj:
        out = model(x)
    torch.cuda.synchronize()
    return out, stats, inj


def expected_faults(cfg):
    """(layer, row, col) the reference's random stream draws for SHAPES."""
    rng = O.InjectorRng(cfg.seed)
    out = []
    for li, (k, n, _) in enumerate(SHAPES):
        idx = rng.maybe_inject(TOKENS * n, cfg.inject_fault, cfg.inject_probability)
        if idx is not None:
            out.append((li, idx // n, idx % n))
    return out


def test_clean_model_has_no_detections(cuda_device):
    model = make_model(cuda_device)
    x = torch.randn(TOKENS, SHAPES[0][0], device=cuda_device).bfloat16()
    with torch.inference_mode():
        ref = model(x)
    for defer in (False, True):
        cfg = AbftConfig(enable=True, checker_backend="b200", detect_only=False)
        out, stats, _ = run(model, x, cfg, defer)
        s = stats.export_summary()
        assert s["abft"]["checks_total"] == len(SHAPES)
        assert s["abft"]["faults"]["detected_total"] == 0 and s["abft"]["fail_total"] == 0
        assert (out.float() - ref.float()).abs().max().item() <= 1e-2 * ref.float().abs().max().item()


@pytest.mark.parametrize("seed,prob", [(3, 1.0), (11, 0.5), (2026, 0.7)])
def test_injected_faults_located_corrected_with_reference_rng(cuda_device, seed, prob):
    model = make_model(cuda_device)
    x = torch.randn(TOKENS, SHAPES[0][0], device=cuda_device).bfloat16()
    with torch.inference_mode():
        clean = model(x)
    cfg = AbftConfig(enable=True, checker_backend="b200", detect_only=False, inject_fault=True,
                     inject_probability=prob, inject_magnitude=500.0, seed=seed)
    want = expected_faults(cfg)
    summaries = []
    for defer in (False, True):
        out, stats, _ = run(model, x, cfg, defer)
        s = stats.export_summary()
        located = sorted((p["row"], p["col"]) for p in s["abft"]["faults"]["located"])
        summaries.append((s["abft"]["faults"]["detected_total"], s["abft"]["faults"]["corrected_total"],
                          s["fault_injection"]["injections_total"], s["fault_injection"]["detected_injections_total"],
                          located))
        assert s["fault_injection"]["injections_total"] == len(want)
        assert s["fault_injection"]["detected_injections_total"] == len(want)
        assert s["abft"]["faults"]["corrected_total"] == len(want)
        # corrected faults leave the model output equal to the clean one
        assert (out.float() - clean.float()).abs().max().item() <= 1e-2 * clean.float().abs().max().item()
        assert located == sorted((r, c) for _, r, c in want)
    assert summaries[0] == summaries[1]


def test_detect_only_keeps_fault_in_output(cuda_device):
    model = make_model(cuda_device)
    x = torch.randn(TOKENS, SHAPES[0][0], device=cuda_device).bfloat16()
    cfg = AbftConfig(enable=True, checker_backend="b200", detect_only=True, inject_fault=True,
                     inject_probability=1.0, inject_magnitude=500.0, seed=5)
    _, stats, _ = run(model, x, cfg, True)
    s = stats.export_summary()
    assert s["abft"]["faults"]["detected_total"] == len(SHAPES)
    assert s["abft"]["faults"]["corrected_total"] == 0


def test_report_arena_spans_chunks(cuda_device):
    """More deferred calls than one arena chunk holds: all are recorded in order."""
    lin = nn.Linear(128, 256, bias=False).to(device=cuda_device, dtype=torch.bfloat16)
    x = torch.randn(64, 128, device=cuda_device).bfloat16()
    cfg = AbftConfig(enable=True, checker_backend="b200", detect_only=False, inject_fault=True,
                     inject_probability=0.3, inject_magnitude=500.0, seed=17)
    stats = AbftStatsCollector()
    inj = AbftInjector(cfg, CheapSumChecker(cfg), stats, defer_reports=True)
    calls = 600
    with torch.inference_mode(), inj:
        for _ in range(calls):
            lin(x)
    s = stats.export_summary()
    rng = O.InjectorRng(cfg.seed)
    n_inj = sum(rng.maybe_inject(64 * 256, True, 0.3) is not None for _ in range(calls))
    assert s["abft"]["checks_total"] == calls
    assert s["fault_injection"]["injections_total"] == n_inj
    assert s["fault_injection"]["detected_injections_total"] == n_inj
    assert s["abft"]["faults"]["corrected_total"] == n_inj
