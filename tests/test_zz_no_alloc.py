"""abft_check_only_noalloc: the post-hoc check without a caller workspace.

Some callers cannot call cudaMalloc (a serving loop that may not take the
device synchronisation it implies, an engine whose pool already owns the
device memory, a binding from a runtime without a device allocator); this
entry point takes its scratch from a fixed device array inside the library.
The test calls it through the C ABI twice in a row and compares every
result with abft_check_only given a freshly allocated workspace. It lives in
a file collected last, so a run that stops at the first failure has run
everything else first; it also passes alone in a fresh process (its first
call performs the one-time set-up).
"""
import ctypes

import pytest
import torch

from vla_abft_estimate_b200 import _native as N
from vla_abft_estimate_b200 import ops

pytestmark = pytest.mark.gpu


def _args(a, b, c, bias, report, flags):
    """B is [N, K] (an nn.Linear weight) when it has a's K columns, else
    [K, N] (the reference checker's b_2d)."""
    args = N.CheckArgs()
    args.A, args.B, args.C = a.data_ptr(), b.data_ptr(), c.data_ptr()
    args.bias = None if bias is None else bias.data_ptr()
    kn = 0 if b.shape[1] == a.shape[1] else 1
    args.M, args.N, args.K = a.shape[0], c.shape[1], a.shape[1]
    args.lda, args.ldb, args.ldc = a.stride(0), b.stride(0), c.stride(0)
    args.b_kn = kn
    args.flags = flags
    args.tol_abs, args.tol_rel, args.thr_scale = 1e-2, 1e-2, 1e-3
    args.report, args.report_capacity = report.data_ptr(), report.capacity
    return args


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _with_workspace(a, w, c, bias, flags, dev):
    rep = ops.ReportBuffer(32, dev)
    args = _args(a, w, c, bias, rep, flags)
    L = N.lib()
    ws = torch.empty(int(L.abft_check_workspace_bytes(ctypes.byref(args))), dtype=torch.uint8, device=dev)
    args.workspace, args.workspace_bytes = ws.data_ptr(), ws.numel()
    N.check("abft_check_only", L.abft_check_only(ctypes.byref(args), _stream(dev)))
    return rep.read()


def _no_alloc(a, w, c, bias, flags, dev):
    rep = ops.ReportBuffer(32, dev)
    args = _args(a, w, c, bias, rep, flags)  # workspace left NULL: the entry point ignores it
    N.check("abft_check_only_noalloc", N.lib().abft_check_only_noalloc(ctypes.byref(args), _stream(dev)))
    return rep.read()


def _same(r1, r2):
    assert r1.ref_ok == r2.ref_ok
    assert r1.status == r2.status and r1.n_faults == r2.n_faults and r1.n_located == r2.n_located
    for key in ("corner", "sum_c", "abs_err", "rel_err"):
        x, y = getattr(r1, key), getattr(r2, key)
        assert abs(x - y) <= 1e-5 * max(1.0, abs(y)), (key, x, y)
    assert r1.coords() == r2.coords()


def test_noalloc_matches_workspace_entry_on_two_calls(cuda_device):
    dev = cuda_device
    g = torch.Generator().manual_seed(42)
    m, n, k = 384, 1000, 520
    a = (torch.randn(m, k, generator=g) * k ** -0.5).bfloat16().to(dev)
    w = (torch.randn(n, k, generator=g) * k ** -0.5).bfloat16().to(dev)
    bias = (torch.randn(n, generator=g) * 0.02).bfloat16().to(dev)
    clean = (a.float() @ w.float().T + bias.float()).bfloat16()
    faulty = clean.clone()
    faulty[17, 333] += 4.0
    flags = N.CHECK_LOCATE | N.CHECK_BF16_SUMS
    # two calls in a row; the second must not see anything the first left behind
    first = _no_alloc(a, w, clean, bias, flags, dev)
    second = _no_alloc(a, w, faulty, bias, flags, dev)
    _same(first, _with_workspace(a, w, clean, bias, flags, dev))
    _same(second, _with_workspace(a, w, faulty, bias, flags, dev))
    assert first.n_faults == 0 and first.ref_ok == 1
    assert second.coords() == [(17, 333)] and second.ref_ok == 0


@pytest.mark.parametrize("flags", [N.CHECK_LOCATE, N.CHECK_BF16_SUMS, 0])
def test_noalloc_kn_layout_matches_workspace_entry_on_two_calls(cuda_device, flags):
    """B given as [K, N] (b_kn = 1): its column sums go through the part of
    the array sized for the larger of the two partial-sum layouts."""
    dev = cuda_device
    g = torch.Generator().manual_seed(43)
    m, n, k = 256, 1528, 776
    a = (torch.randn(m, k, generator=g) * k ** -0.5).bfloat16().to(dev)
    b_kn = (torch.randn(k, n, generator=g) * k ** -0.5).bfloat16().to(dev)
    clean = (a.float() @ b_kn.float()).bfloat16()
    faulty = clean.clone()
    faulty[201, 1400] -= 6.0
    first = _no_alloc(a, b_kn, faulty, None, flags, dev)
    second = _no_alloc(a, b_kn, clean, None, flags, dev)
    _same(first, _with_workspace(a, b_kn, faulty, None, flags, dev))
    _same(second, _with_workspace(a, b_kn, clean, None, flags, dev))
    assert first.ref_ok == 0 and second.n_faults == 0
    if flags & N.CHECK_LOCATE:
        assert first.coords() == [(201, 1400)]
    else:
        assert first.n_faults == 0 and first.records == []


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda_device):
    args = N.CheckArgs()
    args.A, args.B, args.C, args.report = 0x10000, 0x20000, 0x30000, 0x40000
    args.M, args.N, args.K = 8192, 131072, 8192
    args.lda, args.ldb, args.ldc = 8192, 8192, 131072
    args.report_capacity = 0
    assert N.lib().abft_check_workspace_bytes(ctypes.byref(args)) > N.NO_ALLOC_SCRATCH_BYTES
    # rejected on the host before any device work touches the (unused) pointers
    assert N.lib().abft_check_only_noalloc(ctypes.byref(args), None) == -4
