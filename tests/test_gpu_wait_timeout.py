"""Failure detection on the GPU without a fault: the bounded device waits.

Every wait of the fused kernel (pipeline mbarriers, stream-K hand-off
flags, the report header) gives up after a limit instead of spinning on.
abft_wait_selftest makes two of them run out -- a flag that nothing sets
and an mbarrier phase that nothing completes -- and the report must say
so (ABFT_STATUS_DEVICE_TIMEOUT, two waits given up) after roughly the two
limits, with the context still usable for the next GEMM.
"""
import time

import pytest
import torch

from vla_abft_estimate_b200 import _native as N
from vla_abft_estimate_b200 import ops

pytestmark = pytest.mark.gpu


def test_bounded_waits_give_up_and_report(cuda_device):
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    r = ops.wait_selftest(cuda_device)
    elapsed = time.perf_counter() - t0
    assert r.status & N.STATUS_DEVICE_TIMEOUT and r.device_timeout
    assert r.n_faults == 2
    assert 3.5 <= elapsed <= 30.0  # two 2 s limits, then the kernel returns
    # the context is still usable: a checked GEMM runs clean
    a = (torch.randn(256, 512, device=cuda_device) * 512 ** -0.5).bfloat16()
    w = (torch.randn(512, 512, device=cuda_device) * 512 ** -0.5).bfloat16()
    c, rep = ops.abft_gemm(a, w)
    rr = rep.read()
    assert rr.status == 0 and rr.n_faults == 0 and not rr.device_timeout
    ref = a.float() @ w.float().T
    assert (c.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()
