"""Cached weight checksums on a B200: never stale, and harmless when they are.

The injector caches each weight's checksum block (the reference recomputes
``b_2d.sum(dim=1)`` per call, pytorch/abft/checkers.py:119). A block must
not be served for another tensor placed at a freed weight's address, and a
write the cache cannot see (``weight.data.copy_``) must not lead the
kernel to "correct" a right output: the slab mismatches in most rows, the
kernel reports STATUS_SUSPECT without changing anything, and the injector
drops its cache so that the next call is checked against fresh checksums.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import abft_oracle as O
from vla_abft_estimate_b200 import _native as N
from vla_abft_estimate_b200 import ops
from vla_abft_estimate_b200.abft import AbftConfig, AbftInjector, AbftStatsCollector, CheapSumChecker

pytestmark = pytest.mark.gpu

OUT_TOL = 1e-2


def rel_err(x: torch.Tensor, ref: torch.Tensor) -> float:
    return (x.float() - ref.float()).abs().max().item() / max(ref.float().abs().max().item(), 1e-30)


def injector(defer=False):
    cfg = AbftConfig(enable=True, checker_backend="b200", detect_only=False)
    stats = AbftStatsCollector()
    return AbftInjector(cfg, CheapSumChecker(cfg), stats, defer_reports=defer), stats


def summary(stats):
    s = stats.export_summary()["abft"]
    return s["checks_total"], s["faults"]["detected_total"], s["faults"].get("corrected_total", 0)


def test_new_tensor_at_a_freed_weights_address_is_encoded_afresh(cuda_device):
    m, n, k = 512, 1024, 768
    g = torch.Generator(device=cuda_device).manual_seed(0)
    x = (torch.randn(m, k, device=cuda_device, generator=g) * k ** -0.5).bfloat16()
    inj, stats = injector()
    w1 = (torch.randn(n, k, device=cuda_device, generator=g) * k ** -0.5).bfloat16()
    w2_values = (torch.randn(n, k, device=cuda_device, generator=g) * k ** -0.5).bfloat16()
    with torch.inference_mode(), inj:
        F.linear(x, w1)
    ptr = w1.data_ptr()
    del w1
    # the caching allocator hands the freed block to the next tensor of its size
    w2 = torch.empty(n, k, device=cuda_device, dtype=torch.bfloat16)
    assert w2.data_ptr() == ptr, "the allocator did not reuse the address; the test needs it"
    w2.copy_(w2_values)
    with torch.inference_mode(), inj:
        out = F.linear(x, w2)
    torch.cuda.synchronize()
    checks, detected, corrected = summary(stats)
    assert checks == 2 and detected == 0 and corrected == 0
    assert rel_err(out, x.float() @ w2.float().T) <= OUT_TOL


@pytest.mark.parametrize("defer", [False, True])
def test_untracked_weight_write_is_reported_not_corrected(cuda_device, defer):
    m, n, k = 384, 1000, 520
    g = torch.Generator(device=cuda_device).manual_seed(1)
    x = (torch.randn(m, k, device=cuda_device, generator=g) * k ** -0.5).bfloat16()
    w = torch.nn.Parameter((torch.randn(n, k, device=cuda_device, generator=g) * k ** -0.5).bfloat16(),
                           requires_grad=False)
    w_new = (torch.randn(n, k, device=cuda_device, generator=g) * k ** -0.5).bfloat16()
    inj, stats = injector(defer)
    with torch.inference_mode():
        with inj:
            F.linear(x, w)  # caches w's checksums
            w.data.copy_(w_new)  # behind the version counter: the cached block is stale
            stale_out = F.linear(x, w)
        torch.cuda.synchronize()
        checks, detected, corrected = summary(stats)
        assert checks == 2 and detected > 0 and corrected == 0
        # nothing was "corrected": the output is the plain product with the new weight
        assert rel_err(stale_out, x.float() @ w_new.float().T) <= OUT_TOL
        assert len(inj.checksums) == 0  # the suspect report cleared the cache
        with inj:
            fresh_out = F.linear(x, w)
        torch.cuda.synchronize()
    checks2, detected2, _ = summary(stats)
    assert checks2 == 3 and detected2 == detected  # re-encoded: the third call is clean
    assert rel_err(fresh_out, x.float() @ w_new.float().T) <= OUT_TOL


@pytest.mark.parametrize("tile_n,tile_m", [(128, 128), (256, 128), (256, 256)])
def test_stale_checksum_block_matches_oracle(cuda_device, tile_n, tile_m):
    """The kernel's records against the oracle run on the same stale block:
    every mismatching row found, none corrected, status SUSPECT."""
    m, n, k = 300, 704, 256
    rng = np.random.default_rng(7)
    a = O.bf16_round(rng.standard_normal((m, k)) * k ** -0.5)
    w_old = O.bf16_round(rng.standard_normal((n, k)) * k ** -0.5)
    w_new = O.bf16_round(rng.standard_normal((n, k)) * k ** -0.5)
    dev = cuda_device
    ad = torch.from_numpy(a).bfloat16().to(dev)
    wn = torch.from_numpy(w_new).bfloat16().to(dev)
    stale = ops.encode_weight(torch.from_numpy(w_old).bfloat16().to(dev), tile_n)
    c, rep = ops.abft_gemm(ad, wn, tile_n=tile_n, tile_m=tile_m, checksums=stale,
                           report=ops.ReportBuffer(4096, dev))
    r = rep.read()
    orc = O.rowcheck_gemm(a, w_new, tile_n=tile_n - 8, checksum_weight=w_old)
    assert r.status & N.STATUS_SUSPECT
    assert r.n_corrected == 0 and r.n_faults == len(orc.records) and r.overflow == 0
    assert sorted(x.row for x in r.records) == sorted(i for i, _, _ in orc.records)
    assert all(not x.corrected for x in r.records)
    assert rel_err(c.cpu(), torch.from_numpy(orc.out)) <= OUT_TOL


def test_weights_made_under_inference_mode_are_cached(cuda_device):
    """Inference tensors have no version counter; they are still cached
    (by storage identity) and checked."""
    m, n, k = 256, 512, 384
    inj, stats = injector()
    with torch.inference_mode():
        x = (torch.randn(m, k, device=cuda_device) * k ** -0.5).bfloat16()
        w = (torch.randn(n, k, device=cuda_device) * k ** -0.5).bfloat16()
        with inj:
            out1 = F.linear(x, w)
            out2 = F.linear(x, w)
    torch.cuda.synchronize()
    checks, detected, _ = summary(stats)
    assert checks == 2 and detected == 0 and len(inj.checksums) == 1
    assert torch.equal(out1, out2)
