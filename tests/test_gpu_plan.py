"""abft_gemm_plan: what a call will launch, without launching it.

Bars: the plan's tile shape is the one the launch records in its report
header; the schedule is self-consistent (data-parallel tiles in whole waves
of units, stream-K only over the rest, the last column's width); few-row
products report swapped operands; an empty product plans nothing.
"""
import pytest
import torch

from vla_abft_estimate_b200 import _native as N
from vla_abft_estimate_b200 import ops

pytestmark = pytest.mark.gpu

CHK = N.MODE_DETECT | N.MODE_CORRECT


@pytest.mark.parametrize("m,n,k,kw", [
    (512, 4096, 4096, {}),
    (512, 37888, 3584, {}),
    (8192, 8192, 8192, {}),
    (300, 1000, 520, {"tile_n": 128}),
    (2048, 4968, 512, {"tile_n": 256, "tile_m": 256}),
    (4096, 4096, 4096, {"mode": N.MODE_OFF}),
])
def test_plan_is_consistent(cuda_device, m, n, k, kw):
    p = ops.gemm_plan(m, n, k, device=cuda_device, **kw)
    check = kw.get("mode", CHK) != N.MODE_OFF
    assert p["tile_n"] in (128, 256) and p["tile_m"] in (128, 256)
    assert p["data_cols"] == p["tile_n"] - (8 if check else 0)
    assert p["tiles_n"] == -(-n // p["data_cols"])
    assert p["last_cols"] == n - (p["tiles_n"] - 1) * p["data_cols"]
    assert p["tiles"] == -(-m // p["tile_m"]) * p["tiles_n"]
    assert p["grid"] <= p["units"] * (2 if p["tile_m"] == 256 else 1)
    assert p["dp_tiles"] <= p["tiles"]
    if p["sk_units"]:
        assert p["dp_tiles"] % p["units"] == 0 and p["dp_tiles"] < p["tiles"]
        assert p["sk_units"] <= p["units"] and p["workspace_bytes"] > 0
    else:
        assert p["dp_tiles"] == p["tiles"]
    assert p["swapped"] == 0
    for key in ("tile_n", "tile_m"):
        if key in kw:
            assert p[key] == kw[key]


@pytest.mark.parametrize("m,n,k,kw", [(512, 4096, 4096, {}), (1024, 1024, 1024, {}), (200, 136, 72, {"tile_n": 128}),
                                      (8192, 8192, 2048, {})])
def test_plan_matches_report_header(cuda_device, m, n, k, kw):
    torch.manual_seed(m + n)
    a = (torch.randn(m, k, device=cuda_device) * k ** -0.5).bfloat16()
    w = (torch.randn(n, k, device=cuda_device) * k ** -0.5).bfloat16()
    p = ops.gemm_plan(m, n, k, device=cuda_device, cached_checksums=False, **kw)
    _, rep = ops.abft_gemm(a, w, **kw)
    r = rep.read()
    assert (r.tile_m, r.tile_n) == (p["tile_m"], p["data_cols"])
    assert r.status == 0 and r.n_faults == 0


def test_plan_few_rows_and_empty(cuda_device):
    p = ops.gemm_plan(1, 4096, 4096, device=cuda_device)
    assert p["swapped"] == 1 and p["tile_m"] == 128 and p["tile_n"] == 128
    assert ops.gemm_plan(1, 4096, 4096, swap_ab=1, device=cuda_device)["swapped"] == 0
    assert all(v == 0 for v in ops.gemm_plan(0, 4096, 4096, device=cuda_device).values())
    with pytest.raises(N.AbftError):
        ops.gemm_plan(64, 100, 64, device=cuda_device)  # N % 8


def test_plan_batched_and_n_major_right_operand(cuda_device):
    """Batched products count every batch's tiles, and an N-major right
    operand (torch.bmm's mat2) needs its K-major copy in the workspace: the
    plan's workspace is what abft_gemm_workspace_bytes asks for."""
    import ctypes

    one = ops.gemm_plan(1024, 1024, 128, tile_n=256, tile_m=256, device=cuda_device)
    four = ops.gemm_plan(1024, 1024, 128, batch=4, tile_n=256, tile_m=256, device=cuda_device)
    assert four["tiles"] == 4 * one["tiles"] and four["tile_n"] == one["tile_n"]
    L = N.lib()
    args = N.GemmArgs()
    fake = 1 << 20
    args.A = args.B = args.C = args.report = fake
    args.M, args.N, args.K = 1024, 1024, 128
    args.lda, args.ldb, args.ldc = 128, 1024, 1024
    args.mode, args.report_capacity, args.thr_scale = CHK, 16, 1e-3
    args.batch, args.b_kn = 4, 1
    args.tile_n, args.tile_m = 256, 256
    args.stride_a, args.stride_b, args.stride_c = 1024 * 128, 128 * 1024, 1024 * 1024
    info = N.PlanInfo()
    with torch.cuda.device(cuda_device):
        N.check("abft_gemm_plan", L.abft_gemm_plan(ctypes.byref(args), ctypes.byref(info)))
        ws = int(L.abft_gemm_workspace_bytes(ctypes.byref(args)))
    assert info.workspace_bytes == ws >= 4 * 1024 * 128 * 2  # the K-major copy of B at least
    assert info.tiles == four["tiles"]
