"""Parity at the BASELINE GEMM configurations, on a B200, through the C ABI.

* Config 1 (A[512 x 4096] . B[4096 x 4096], seeds 0-4, clean and one
  +2^8 max|C| fault): the reference's CheapSumChecker results were recorded
  by tests/golden/make_golden.py (ref_config1_cases.json) with SHA-256
  digests of the inputs. The inputs are regenerated and their digests
  asserted, then the library's bf16-sum check of the same (A, B, C) must
  give the reference's flags and values bit for bit, and the fused kernel's
  scalar reference rule (ABFT_MODE_REF | ABFT_MODE_REF_BF16) its flags.
* Config 2 (square M = N = K up to 16384, clean / 1 / 4 faults in distinct
  rows and columns): exact coordinates, corrections, and outputs within
  1e-2 of an fp32 GEMM on sampled rows.
* No false positives on data shaped like a real model's: outlier
  activation channels, weights with non-zero row means, SwiGLU products,
  bias, at the Qwen2-7B layer shapes including K = 18944, on bf16 and on
  fp16 operands.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import abft_oracle as O
from tests.golden import baseline_inputs as BI
from vla_abft_estimate_b200 import _native as N
from vla_abft_estimate_b200 import ops

pytestmark = pytest.mark.gpu

OUT_TOL = 1e-2
CHECKED = N.MODE_DETECT | N.MODE_CORRECT


def bits_to_dev(bits: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(dev)


def dev_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.fixture(scope="module")
def config1(golden_dir):
    return json.load(open(os.path.join(golden_dir, "ref_config1_cases.json")))


def config1_operands(seed, case_clean, dev):
    c1 = BI.CONFIG1
    a_bits, w_bits = BI.gemm_inputs(seed, c1["M"], c1["K"], c1["N"])
    assert BI.sha256_bits(a_bits) == case_clean["sha256_a"]
    assert BI.sha256_bits(w_bits) == case_clean["sha256_w"]
    a, w = bits_to_dev(a_bits, dev), bits_to_dev(w_bits, dev)
    # the float64 product rounded to float32, then bf16: the fixture's C
    c = (a.double() @ w.double().T).float().bfloat16()
    assert BI.sha256_bits(dev_bits(c)) == case_clean["sha256_c"]
    return a, w, c


SEEDS = [0, 1, 2, 3, 4]


@pytest.mark.parametrize("seed", SEEDS)
def test_config1_check_only_gives_reference_results(cuda_device, config1, seed):
    cases = [c for c in config1 if c["seed"] == seed]
    clean = next(c for c in cases if not c["fault"])
    a, w, c = config1_operands(seed, clean, cuda_device)
    for case in cases:
        cc = c
        if case["fault"]:
            cc = c.clone()
            cc.view(-1)[case["fault_index"]] += case["fault_magnitude"]
            assert BI.sha256_bits(dev_bits(cc)) == case["sha256_c"]
        for layout, bb in (("nk", w), ("kn", w.t().contiguous())):
            r = ops.check_only(a, bb, cc, b_layout=layout, bf16_sums=True).read()
            got = (r.ref_ok == 1, r.abs_err, r.rel_err, r.corner, r.sum_c)
            want = (case["ok"], case["abs_err"], case["rel_err"], case["abft_corner"], case["sum_c"])
            assert got == want, (seed, case["fault"], layout, got, want)


@pytest.mark.parametrize("seed", SEEDS)
def test_config1_fused_reference_rule_gives_reference_flags(cuda_device, config1, seed):
    """The fused kernel applies the reference's scalar rule to the output it
    stores: its flag equals the reference's, its corner is the reference's
    bit for bit (it depends on A and B only), and its sum_c equals the
    bf16-sum check run afterwards on the stored output."""
    cases = [c for c in config1 if c["seed"] == seed]
    clean = next(c for c in cases if not c["fault"])
    a, w, _ = config1_operands(seed, clean, cuda_device)
    n = clean["N"]
    for case in cases:
        inj = [(case["fault_index"] // n, case["fault_index"] % n, case["fault_magnitude"])] if case["fault"] else None
        for extra in (0, N.MODE_DETECT):  # detect without correcting keeps the fault in the stored output
            c, rep = ops.abft_gemm(a, w, mode=N.MODE_REF | N.MODE_REF_BF16 | extra, inject=inj)
            r = rep.read()
            assert (r.ref_ok == 1) == case["ok"], (seed, case["fault"], extra, r.rel_err, case["rel_err"])
            assert r.corner == case["abft_corner"]
            post = ops.check_only(a, w, c, b_layout="nk", bf16_sums=True).read()
            assert (r.sum_c, r.abs_err, r.rel_err, r.ref_ok) == (post.sum_c, post.abs_err, post.rel_err, post.ref_ok)
            if extra:
                want = [(inj[0][0], inj[0][1])] if inj else []
                assert r.coords() == want and r.n_corrected == 0


def sampled_rows_err(a, w, c, rows):
    ref = a[rows].float() @ w.float().T
    return (c[rows].float() - ref).abs().max().item() / max(ref.abs().max().item(), 1e-30)


@pytest.mark.parametrize("size", [1024, 2048, 4096, 8192, 16384])
def test_square_sweep_clean_one_and_four_faults(cuda_device, size):
    """M = N = K = size, N(0, 1/sqrt(K)) inputs, clean,
    then 1 and 4 faults of 2^8 max|C| at seeded distinct rows and columns."""
    m = n = k = size
    g = torch.Generator(device=cuda_device).manual_seed(size)
    a = (torch.randn(m, k, device=cuda_device, generator=g) * k ** -0.5).bfloat16()
    w = (torch.randn(n, k, device=cuda_device, generator=g) * k ** -0.5).bfloat16()
    c0, rep0 = ops.abft_gemm(a, w, mode=CHECKED)
    r0 = rep0.read()
    assert r0.status == 0 and r0.n_faults == 0 and r0.records == []
    delta = 256.0 * c0.float().abs().max().item()
    probe = torch.randperm(m, generator=torch.Generator().manual_seed(size))[:64].tolist()
    assert sampled_rows_err(a, w, c0, probe) <= OUT_TOL
    for count in (1, 4):
        faults = O.seeded_fault_positions(m, n, count, size + count)
        c, rep = ops.abft_gemm(a, w, mode=CHECKED, inject=[(i, j, delta) for i, j in faults])
        r = rep.read()
        assert r.coords() == sorted(faults)
        assert r.n_faults == r.n_located == r.n_corrected == count and r.status == N.STATUS_FAULT
        rows = probe + [i for i, _ in faults]
        assert sampled_rows_err(a, w, c, rows) <= OUT_TOL
        # the corrected elements themselves
        for i, j in faults:
            exact = (a[i].float() @ w[j].float()).item()
            assert abs(c[i, j].float().item() - exact) <= OUT_TOL * max(abs(exact), delta / 256.0)


def llm_like(kind, m, n, k, seed, dev, dtype=torch.bfloat16):
    """Activations and weights with the structure of a trained decoder's."""
    g = torch.Generator(device=dev).manual_seed(seed)
    if kind == "swiglu":  # the down projection's input: silu(gate) * up, heavy-tailed
        gate = torch.randn(m, k, device=dev, generator=g)
        up = torch.randn(m, k, device=dev, generator=g)
        x = torch.nn.functional.silu(gate) * up
    else:
        x = torch.randn(m, k, device=dev, generator=g)
        x += 0.5  # a non-zero mean in every channel
    out_ch = torch.randperm(k, generator=torch.Generator().manual_seed(seed))[:8].to(dev)
    x[:, out_ch] *= 100.0  # a few outlier channels, 100x the rest
    sigma = 0.02
    mu = torch.randn(n, 1, device=dev, generator=g) * (3 * sigma)  # non-zero row means
    w = mu + sigma * torch.randn(n, k, device=dev, generator=g)
    bias = torch.randn(n, device=dev, generator=g) * 0.1
    return x.to(dtype), w.to(dtype), bias.to(dtype)


@pytest.mark.parametrize("m,n,k,kind", [
    (512, 4608, 3584, "shifted"),    # Qwen2-7B fused QKV
    (512, 3584, 3584, "shifted"),    # O projection
    (512, 37888, 3584, "shifted"),   # fused gate + up
    (512, 3584, 18944, "swiglu"),    # down projection, K = 18944
    (4096, 4096, 4096, "swiglu"),
    (16, 3584, 18944, "swiglu"),     # decode-sized (swapped operands)
])
@pytest.mark.parametrize("seed,dtype", [(0, torch.bfloat16), (1, torch.bfloat16), (2, torch.bfloat16),
                                        (0, torch.float16), (1, torch.float16)])
def test_no_false_positive_on_llm_like_data(cuda_device, m, n, k, kind, seed, dtype):
    a, w, b = llm_like(kind, m, n, k, seed, cuda_device, dtype)
    c, rep = ops.abft_gemm(a, w, b, mode=CHECKED)
    r = rep.read()
    assert r.status == 0 and r.n_faults == 0, (r.status, r.records[:4])
    ref = a.float() @ w.float().T + b.float()
    err = (c.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err <= OUT_TOL
    # and a planted fault in the same data is still found and corrected
    i, j = O.seeded_fault_positions(m, n, 1, seed)[0]
    delta = 256.0 * ref.abs().max().item()
    c2, rep2 = ops.abft_gemm(a, w, b, mode=CHECKED, inject=[(i, j, delta)])
    r2 = rep2.read()
    assert r2.coords() == [(i, j)] and r2.n_corrected == 1
    assert (c2.float() - ref).abs().max().item() / ref.abs().max().item() <= OUT_TOL


def test_b200_and_reference_rules_disagree_exactly_where_predicted(cuda_device, config1):
    """The fused kernel's per-row rule (|residual| > tau sqrt(K) max|C_row
    segment|) and the reference's scalar rule (|corner - sum_c| > 1e-2 and
    relative > 1e-2, pytorch/abft/checkers.py:96-110) flag different faults:
    a fault small against the whole output's sum but large against its row
    is caught by the row rule only, and the scalar rule misses it. Faults at
    half and twice each rule's bound (config-1 inputs, seed 0) must give
    each rule's flag exactly as the oracle predicts, so the calls on which
    the two backends disagree are the predicted ones."""
    clean_case = next(c for c in config1 if c["seed"] == 0 and not c["fault"])
    a, w, c = config1_operands(0, clean_case, cuda_device)
    af, wf = a.float().cpu().numpy(), w.float().cpu().numpy()
    c_np = c.float().cpu().numpy()
    m, n, k = af.shape[0], wf.shape[0], af.shape[1]
    # the scalar rule's bound on the whole output; the row rule's bound of
    # the fault's 120-column row segment (128-wide tiles)
    ref_bound = 1e-2 * max(abs(float(c_np.astype(np.float64).sum())), 1.0)
    tk = float(np.float32(1e-3 * np.sqrt(k)))
    disagree = 0
    for (i, j) in [(7, 100), (300, 2000)]:
        s0 = (j // 120) * 120
        row_bound = tk * float(np.abs(c_np[i, s0:s0 + 120]).max())
        for delta in (0.5 * row_bound, 2.0 * row_bound, 0.5 * ref_bound, 2.0 * ref_bound):
            # predictions of the two oracles
            row = O.rowcheck_gemm(af[i:i + 1], wf, tile_n=120, inject=[(0, j, float(delta))])
            b200_pred = len(row.records) == 1
            cf = c_np.copy()
            cf[i, j] = O.bf16_round(np.array([cf[i, j] + np.float32(delta)], np.float32))[0]
            ref_pred = not O.cheap_sum_check(af, wf.T, cf, emulate_bf16=True).ok
            # the library: the fused kernel (fault on the accumulator) and the
            # bf16-sum post-hoc check of the reference rule (fault in C)
            _, rep = ops.abft_gemm(a, w, mode=CHECKED, tile_n=128, inject=[(i, j, float(delta))])
            b200_got = rep.read().coords() == [(i, j)]
            cc = c.clone()
            cc[i, j] += float(delta)
            ref_got = ops.check_only(a, w, cc, b_layout="nk", bf16_sums=True).read().ref_ok == 0
            assert (b200_got, ref_got) == (b200_pred, ref_pred), (delta, i, j)
            disagree += b200_got != ref_got
    assert disagree > 0  # the rules do differ on this data: between the two bounds
