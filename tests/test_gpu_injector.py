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
from vla_abft_estimate_b200.abft import AbftConfig, AbftInjector, AbftStatsCollector, CheapSumChecker, OpMeta

pytestmark = pytest.mark.gpu

SHAPES = [(256, 512, True), (512, 384, False), (384, 1000, True), (1000, 248, False)]  # (in, out, bias)
TOKENS = 96


def make_model(device, seed=0, dtype=torch.bfloat16):
    torch.manual_seed(seed)
    layers = []
    for k, n, bias in SHAPES:
        lin = nn.Linear(k, n, bias=bias)
        with torch.no_grad():
            lin.weight.normal_(0.0, k ** -0.5)
            if bias:
                lin.bias.normal_(0.0, 0.02)
        layers.append(lin)
    return nn.Sequential(*layers).to(device=device, dtype=dtype).eval()


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


@pytest.mark.parametrize("seed,prob,dtype", [(3, 1.0, torch.bfloat16), (11, 0.5, torch.bfloat16),
                                             (2026, 0.7, torch.bfloat16), (3, 1.0, torch.float16),
                                             (11, 0.5, torch.float16)])
def test_injected_faults_located_corrected_with_reference_rng(cuda_device, seed, prob, dtype):
    """Both fused element types: every fault the reference's random stream
    draws is located at its coordinates and corrected."""
    model = make_model(cuda_device, dtype=dtype)
    x = torch.randn(TOKENS, SHAPES[0][0], device=cuda_device).to(dtype)
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


# ------------------------------------------------------------ torch.bmm / matmul
# (batch, M, N, K, layout of mat2): row-major [B, K, N], or the transpose of a
# K-major [B, N, K] (attention scores, q @ k^T); M = 1 is decode-shaped.
BMM_CALLS = [(4, 96, 256, 128, "rowmajor"), (8, 1, 512, 128, "view"), (3, 64, 136, 72, "rowmajor"),
             (2, 200, 248, 256, "view")]


def bmm_operands(device, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = []
    for bsz, m, n, k, lay in BMM_CALLS:
        a = (torch.randn(bsz, m, k, generator=g) * k ** -0.5).bfloat16().to(device)
        w = (torch.randn(bsz, n, k, generator=g) * k ** -0.5).bfloat16().to(device)
        out.append((a, w.transpose(1, 2).contiguous() if lay == "rowmajor" else w.transpose(1, 2)))
    return out


def run_bmms(operands, cfg, defer):
    stats = AbftStatsCollector()
    inj = AbftInjector(cfg, CheapSumChecker(cfg), stats, defer_reports=defer)
    with torch.inference_mode(), inj:
        outs = [torch.bmm(a, b) for a, b in operands]
    torch.cuda.synchronize()
    return outs, stats.export_summary()


def expected_bmm(cfg):
    """(call, batch, row, col) of each drawn fault and the sample coin of
    every batch, in the reference's order: the injection draw over the
    whole output, then one check gate per batch (injector.py:176-187)."""
    rng = O.InjectorRng(cfg.seed)
    faults, gates = [], []
    for ci, (bsz, m, n, _, _) in enumerate(BMM_CALLS):
        idx = rng.maybe_inject(bsz * m * n, cfg.inject_fault, cfg.inject_probability)
        gates.append([rng.sample(cfg.sample_rate) for _ in range(bsz)])
        if idx is not None:
            faults.append((ci, idx // (m * n), (idx // n) % m, idx % n))
    return faults, gates


def test_bmm_clean_one_check_per_batch(cuda_device):
    operands = bmm_operands(cuda_device)
    for defer in (False, True):
        cfg = AbftConfig(enable=True, checker_backend="b200", detect_only=False)
        outs, s = run_bmms(operands, cfg, defer)
        assert s["abft"]["checks_total"] == sum(c[0] for c in BMM_CALLS)
        assert s["abft"]["checks_by_op"] == {"bmm": sum(c[0] for c in BMM_CALLS)}
        assert s["abft"]["fail_total"] == 0 and s["abft"]["faults"]["detected_total"] == 0
        for (a, b), o in zip(operands, outs):
            ref = torch.bmm(a.float(), b.float())
            assert (o.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()


@pytest.mark.parametrize("seed,prob", [(4, 1.0), (12, 0.6)])
def test_bmm_faults_located_corrected_with_reference_rng(cuda_device, seed, prob):
    operands = bmm_operands(cuda_device)
    with torch.inference_mode():
        clean = [torch.bmm(a, b) for a, b in operands]
    cfg = AbftConfig(enable=True, checker_backend="b200", detect_only=False, inject_fault=True,
                     inject_probability=prob, inject_magnitude=500.0, seed=seed)
    want, _ = expected_bmm(cfg)
    summaries = []
    for defer in (False, True):
        outs, s = run_bmms(operands, cfg, defer)
        f = s["abft"]["faults"]
        assert s["fault_injection"]["injections_total"] == len(want)
        # only the faulty batch's check fails; every batch's check carries the call's injected flag
        assert s["fault_injection"]["detected_injections_total"] == len(want)
        assert s["abft"]["fail_total"] == len(want) and f["corrected_total"] == len(want)
        assert sorted((p["row"], p["col"]) for p in f["located"]) == sorted((r, c) for _, _, r, c in want)
        for o, c in zip(outs, clean):
            assert (o.float() - c.float()).abs().max().item() <= 1e-2 * c.float().abs().max().item()
        summaries.append(s)
    assert summaries[0]["abft"] == summaries[1]["abft"]


def test_bmm_sampled_batches_only(cuda_device):
    """sample_rate < 1: each batch draws its own coin, as in the reference's
    loop; only sampled batches are checked (and corrected)."""
    operands = bmm_operands(cuda_device)
    cfg = AbftConfig(enable=True, checker_backend="b200", detect_only=False, inject_fault=True,
                     inject_probability=1.0, inject_magnitude=500.0, seed=8, sample_rate=0.5)
    want, gates = expected_bmm(cfg)
    outs, s = run_bmms(operands, cfg, True)
    assert s["abft"]["checks_total"] == sum(sum(g) for g in gates)
    caught = [(ci, b, r, c) for ci, b, r, c in want if gates[ci][b]]
    missed = [(ci, b, r, c) for ci, b, r, c in want if not gates[ci][b]]
    assert s["fault_injection"]["detected_injections_total"] == len(caught)
    assert sorted((p["row"], p["col"]) for p in s["abft"]["faults"]["located"]) == sorted((r, c) for _, _, r, c in caught)
    with torch.inference_mode():
        for ci, b, r, c in missed:  # an unchecked batch keeps its fault
            a, m2 = operands[ci]
            ref = torch.bmm(a[b:b + 1].float(), m2[b:b + 1].float())[0, r, c].item()
            assert abs(outs[ci][b, r, c].float().item() - ref) > 250.0


def test_matmul_two_d_fused_and_batched_rhs_follows_reference(cuda_device):
    """torch.matmul with a 2-D right operand: one fused check over the
    flattened rows. With a batched right operand the reference checks
    nothing but still draws its sample coin; check_batched_matmul checks
    every batch."""
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(2, 48, 128, generator=g) * 128 ** -0.5).bfloat16().to(cuda_device)
    w = (torch.randn(128, 256, generator=g) * 128 ** -0.5).bfloat16().to(cuda_device)
    q = (torch.randn(2, 4, 32, 64, generator=g) * 64 ** -0.5).bfloat16().to(cuda_device)
    kt = (torch.randn(2, 4, 64, 32, generator=g) * 64 ** -0.5).bfloat16().to(cuda_device)
    for check_batched in (False, True):
        cfg = AbftConfig(enable=True, checker_backend="b200", detect_only=False, inject_fault=True,
                         inject_probability=1.0, inject_magnitude=500.0, seed=21, sample_rate=0.99,
                         check_batched_matmul=check_batched)
        rng = O.InjectorRng(cfg.seed)
        i1 = rng.maybe_inject(96 * 256, True, 1.0)
        g1 = rng.sample(cfg.sample_rate)
        i2 = rng.maybe_inject(2 * 4 * 32 * 32, True, 1.0)
        g2 = rng.sample(cfg.sample_rate)
        stats = AbftStatsCollector()
        inj = AbftInjector(cfg, CheapSumChecker(cfg), stats, defer_reports=True)
        with torch.inference_mode(), inj:
            y = torch.matmul(x, w)
            sc = torch.matmul(q, kt)
        s = stats.export_summary()
        ref = torch.matmul(x.float(), w.float())
        assert tuple(y.shape) == (2, 48, 256)
        assert (y.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()
        n_checks = int(g1) + (8 * int(g2) if check_batched else 0)
        assert s["abft"]["checks_total"] == n_checks
        located = sorted((p["row"], p["col"]) for p in s["abft"]["faults"]["located"])
        want = ([(i1 // 256, i1 % 256)] if g1 else []) + ([((i2 // 32) % 32, i2 % 32)] if g2 and check_batched else [])
        assert located == sorted(want)
        flat = sc.reshape(-1)
        clean = torch.matmul(q.float(), kt.float()).reshape(-1)
        if not check_batched:  # unchecked: the drawn fault stays in the scores
            assert abs(flat[i2].float().item() - clean[i2].item()) > 250.0
        else:
            assert (flat.float() - clean).abs().max().item() <= 1e-2 * clean.abs().max().item()


@pytest.mark.parametrize("k,n,bias", [(7, 768, True), (768, 7, True), (5, 3, False), (12, 20, True)])
def test_narrow_linears_checked_on_padded_copies(cuda_device, k, n, bias):
    """K or N not a multiple of 8 (a VLA's 7-wide action projections): the
    injector checks the call on zero-padded copies instead of skipping it,
    the clean call passes, its corner and sum match the oracle on the
    original operands, and a perturbed output fails the check."""
    meta = OpMeta(op_name="linear", phase="prefill", shape_key="narrow")
    torch.manual_seed(k * 31 + n)
    x = torch.randn(16, k, device=cuda_device).bfloat16()
    w = (torch.randn(n, k, device=cuda_device) * k ** -0.5).bfloat16()
    b = (torch.randn(n, device=cuda_device) * 0.02).bfloat16() if bias else None
    cfg = AbftConfig(enable=True, checker_backend="fused")
    stats = AbftStatsCollector()
    with torch.inference_mode(), AbftInjector(cfg, CheapSumChecker(cfg), stats):
        y = torch.nn.functional.linear(x, w, b)
    torch.cuda.synchronize()
    assert stats.skipped_unsupported == 0 and stats.total_checks == 1 and stats.total_failures == 0

    chk = CheapSumChecker(cfg)
    res = chk.check(x, w.t(), y, meta, bias_1d=b)
    o = O.cheap_sum_check(x.float().cpu().numpy(), w.float().cpu().numpy().T, y.float().cpu().numpy(),
                          None if b is None else b.float().cpu().numpy())
    assert res.ok and o.ok
    assert abs(res.sum_c - o.sum_c) <= 1e-4 * max(1.0, abs(o.sum_c))
    assert abs(res.abft_corner - o.abft_corner) <= 1e-4 * max(1.0, abs(o.abft_corner))

    bad = y.clone()
    bad[3, n - 1] += 64.0
    assert not chk.check(x, w.t(), bad, meta, bias_1d=b).ok


@pytest.mark.parametrize("seed", [1, 4])
def test_narrow_linears_deferred_match_immediate(cuda_device, seed):
    """A model with 7-wide layers (checked on padded copies): deferring the
    checker's reports to flush() records the same checks, failures and
    errors as reading each report at its call."""
    torch.manual_seed(seed)
    model = nn.Sequential(nn.Linear(7, 768), nn.Linear(768, 768), nn.Linear(768, 7))
    model = model.to(device=cuda_device, dtype=torch.bfloat16).eval()
    x = torch.randn(16, 7, device=cuda_device).bfloat16()
    cfg = AbftConfig(enable=True, checker_backend="b200", inject_fault=True, inject_probability=0.5,
                     inject_magnitude=500.0, seed=seed)
    summaries = []
    for defer in (False, True):
        out, stats, _ = run(model, x, cfg, defer)
        s = stats.export_summary()["abft"]
        assert s["checks_total"] == 3 and s["faults"]["skipped_unsupported"] == 0
        summaries.append((s["checks_total"], s["fail_total"], s["faults"]["detected_total"],
                          stats.export_summary()["fault_injection"]))
    assert summaries[0] == summaries[1]


@pytest.mark.parametrize("layout", ["vector", "3d", "row_slice", "transposed"])
def test_fused_linear_input_layouts(cuda_device, layout):
    """The fused linear reads contiguous inputs of any rank in place and
    strided ones through a view or a copy: the output keeps the input's
    leading shape, matches torch, and a clean call records a passing check."""
    torch.manual_seed(7)
    k, n = 256, 384
    w = (torch.randn(n, k, device=cuda_device) * k ** -0.5).bfloat16()
    b = (torch.randn(n, device=cuda_device) * 0.02).bfloat16()
    if layout == "vector":
        x = torch.randn(k, device=cuda_device).bfloat16()
    elif layout == "3d":
        x = torch.randn(2, 5, k, device=cuda_device).bfloat16()
    elif layout == "row_slice":
        x = torch.randn(12, 2 * k, device=cuda_device).bfloat16()[:, :k]  # row stride 2k
    else:
        x = torch.randn(k, 12, device=cuda_device).bfloat16().t()  # column-major rows
    ref = torch.nn.functional.linear(x, w, b)
    cfg = AbftConfig(enable=True, checker_backend="b200")
    stats = AbftStatsCollector()
    with torch.inference_mode(), AbftInjector(cfg, CheapSumChecker(cfg), stats, defer_reports=True):
        y = torch.nn.functional.linear(x, w, b)
    torch.cuda.synchronize()
    assert y.shape == ref.shape
    assert (y.float() - ref.float()).abs().max().item() <= 1e-2 * ref.float().abs().max().item()
    s = stats.export_summary()["abft"]
    assert s["checks_total"] == 1 and s["fail_total"] == 0


@pytest.mark.parametrize("k,n,bias", [(7, 768, True), (768, 7, True), (5, 3, False), (12, 20, True)])
def test_b200_narrow_linears_fused_on_padded_copies(cuda_device, k, n, bias):
    """checker_backend "b200": a linear with K or N not a multiple of 8 runs
    the fused kernel on zero-padded copies. Clean: no detection and the
    F.linear result; with the reference's random fault (probability 1): the
    drawn (row, col) of the caller's output is located and corrected."""
    torch.manual_seed(k * 17 + n)
    x = torch.randn(16, k, device=cuda_device).bfloat16()
    w = (torch.randn(n, k, device=cuda_device) * k ** -0.5).bfloat16()
    b = (torch.randn(n, device=cuda_device) * 0.02).bfloat16() if bias else None
    ref = torch.nn.functional.linear(x.float(), w.float(), None if b is None else b.float())
    for inject in (False, True):
        cfg = AbftConfig(enable=True, checker_backend="b200", detect_only=False, inject_fault=inject,
                         inject_probability=1.0, inject_magnitude=64.0, seed=5)
        stats = AbftStatsCollector()
        with torch.inference_mode(), AbftInjector(cfg, CheapSumChecker(cfg), stats, defer_reports=True):
            y = torch.nn.functional.linear(x, w, b)
        torch.cuda.synchronize()
        s = stats.export_summary()["abft"]
        assert tuple(y.shape) == (16, n) and s["checks_total"] == 1 and stats.skipped_unsupported == 0
        assert (y.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 1e-3
        if not inject:
            assert s["faults"]["detected_total"] == 0
        else:
            idx = O.InjectorRng(5).maybe_inject(16 * n, True, 1.0)
            assert [(c["row"], c["col"]) for c in s["faults"]["located"]] == [(idx // n, idx % n)]
            assert s["faults"]["corrected_total"] == 1


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_f16_f32_linears_checked_not_skipped(cuda_device, dtype):
    """fp16 / fp32 linears (the reference's --dtype float16|float32) are
    checked, never counted as unsupported: fp16 under "b200" runs the fused
    kernel; fp32 (and every type under the other backends) takes the
    reference flow -- torch GEMM, then the native scalar check on operands of
    that type. A perturbed output fails the check."""
    torch.manual_seed(3)
    x = torch.randn(64, 256, device=cuda_device).to(dtype)
    w = (torch.randn(512, 256, device=cuda_device) * 256 ** -0.5).to(dtype)
    b = (torch.randn(512, device=cuda_device) * 0.02).to(dtype)
    for backend in ("b200", "fused", "python"):
        cfg = AbftConfig(enable=True, checker_backend=backend, inject_fault=True, inject_probability=1.0,
                         inject_magnitude=64.0, seed=3)
        stats = AbftStatsCollector()
        with torch.inference_mode(), AbftInjector(cfg, CheapSumChecker(cfg), stats):
            torch.nn.functional.linear(x, w, b)
        torch.cuda.synchronize()
        assert stats.skipped_unsupported == 0 and stats.total_checks == 1, backend
        assert stats.total_failures == 1 and stats.total_detected_injections == 1, backend
