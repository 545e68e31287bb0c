"""``ops.abft_linear`` (F.linear shapes through the fused kernel) and
``FusedB200Checker`` (the scalar check of an existing C with fp32 sums).

abft_linear: outputs within 1e-2 of F.linear in fp32 for [..., K] inputs
of bf16 and fp16, no record on clean inputs, injected faults located at
their (flattened row, col) and corrected, narrow K / N through zero-padded
copies. FusedB200Checker: the same result as the "b200" backend's scalar
check whatever backend string the config names, and the fault flagged.
"""
import pytest
import torch
import torch.nn.functional as F

from oracle import abft_oracle as O
from vla_abft_estimate_b200 import _native as N
from vla_abft_estimate_b200 import ops
from vla_abft_estimate_b200.abft import AbftConfig, CheapSumChecker, FusedB200Checker, OpMeta

pytestmark = pytest.mark.gpu

OUT_TOL = 1e-2


def rel_err(x, ref):
    return (x.float() - ref.float()).abs().max().item() / max(ref.float().abs().max().item(), 1e-30)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("lead,k,n", [((2, 48), 256, 512), ((3, 5, 40), 512, 1000), ((7,), 12, 20), ((16,), 768, 7)])
def test_abft_linear_matches_f_linear_and_corrects(cuda_device, dtype, lead, k, n):
    g = torch.Generator(device=cuda_device).manual_seed(k + n)
    x = torch.randn(*lead, k, device=cuda_device, generator=g).to(dtype)
    w = (torch.randn(n, k, device=cuda_device, generator=g) * k ** -0.5).to(dtype)
    b = (torch.randn(n, device=cuda_device, generator=g) * 0.02).to(dtype)
    ref = F.linear(x.float(), w.float(), b.float())
    y, rep = ops.abft_linear(x, w, b)
    assert y.shape == ref.shape and y.dtype == dtype
    assert rel_err(y, ref) <= OUT_TOL
    r = rep.read()
    assert r.status == 0 and r.n_faults == 0
    rows = ref.numel() // n
    (i, j), = O.seeded_fault_positions(rows, n, 1, k)
    delta = 256.0 * ref.abs().max().item()
    y2, rep2 = ops.abft_linear(x, w, b, inject=[(i, j, delta)])
    r2 = rep2.read()
    assert r2.coords() == [(i, j)] and r2.n_corrected == 1
    assert rel_err(y2, ref) <= OUT_TOL


def test_abft_linear_follows_the_config(cuda_device):
    x = torch.randn(64, 128, device=cuda_device).bfloat16()
    w = (torch.randn(256, 128, device=cuda_device) * 128 ** -0.5).bfloat16()
    ref = F.linear(x.float(), w.float())
    cfg = AbftConfig(detect_only=True, report_capacity=4)
    y, rep = ops.abft_linear(x, w, cfg=cfg, inject=[(3, 5, 100.0)])
    r = rep.read()
    assert rep.capacity == 4
    assert r.coords() == [(3, 5)] and r.n_corrected == 0  # detect only: the fault stays
    assert abs(y[3, 5].float().item() - (ref[3, 5].item() + 100.0)) <= 1.0
    y0, rep0 = ops.abft_linear(x, w, mode=N.MODE_OFF)
    assert rep0 is None and rel_err(y0, ref) <= OUT_TOL
    with pytest.raises(ValueError):
        ops.abft_linear(x, w.t())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_fused_b200_checker_sums_in_fp32_for_every_backend(cuda_device, dtype):
    g = torch.Generator(device=cuda_device).manual_seed(5)
    m, k, n = 256, 384, 512
    a = (torch.randn(m, k, device=cuda_device, generator=g) * k ** -0.5).to(dtype)
    w = (torch.randn(n, k, device=cuda_device, generator=g) * k ** -0.5).to(dtype)
    bias = (torch.randn(n, device=cuda_device, generator=g) * 0.02).to(dtype)
    c = F.linear(a, w, bias)
    meta = OpMeta("linear", "prefill", "k")
    want = CheapSumChecker(AbftConfig(checker_backend="b200")).check(a, w.t(), c, meta, bias)
    for backend in ("python", "fused", "triton", "b200"):
        got = FusedB200Checker(AbftConfig(checker_backend=backend)).check(a, w.t(), c, meta, bias)
        assert got == want, backend
    assert want.ok
    orc = O.cheap_sum_check(a.float().cpu().numpy(), w.float().t().cpu().numpy(), c.float().cpu().numpy(),
                            bias.float().cpu().numpy())
    assert abs(want.abft_corner - orc.abft_corner) <= 1e-4 * max(1.0, abs(orc.abft_corner))
    c_bad = c.clone()
    c_bad[7, 9] += 1000.0
    bad = FusedB200Checker(AbftConfig(checker_backend="python")).check(a, w.t(), c_bad, meta, bias)
    assert not bad.ok
