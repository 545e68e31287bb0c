"""Parity of the sm_100a kernels with the oracle, through the C ABI.

Bars: bit-exact fault coordinates and flags (detect / locate / correct)
against the oracle; outputs within 1e-2 of max|C| of an fp32 GEMM of the
same bf16 inputs; no record at all on clean inputs.
"""
import numpy as np
import pytest
import torch

from oracle import abft_oracle as O
from vla_abft_estimate_b200 import _native as N
from vla_abft_estimate_b200 import ops

pytestmark = pytest.mark.gpu

OUT_TOL = 1e-2  # |C - C_ref| <= OUT_TOL * max|C_ref|


def seeded(m, n, k, seed, bias=False):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(m, k, generator=g) * k ** -0.5).bfloat16()
    w = (torch.randn(n, k, generator=g) * k ** -0.5).bfloat16()
    b = (torch.randn(n, generator=g) * 0.02).bfloat16() if bias else None
    return a, w, b


def f32(t):
    return t.float().cpu().numpy()


def max_rel_err(got, ref):
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


# ------------------------------------------------------------------ encode
@pytest.mark.parametrize("tile_n", [128, 256])
@pytest.mark.parametrize("n,k", [(300, 200), (1024, 512), (136, 72)])
def test_encode_weight_matches_oracle(cuda_device, tile_n, n, k):
    _, w, _ = seeded(8, n, k, 1)
    blk = f32(ops.encode_weight(w.to(cuda_device), tile_n)).astype(np.float64)
    v1, v2, v3 = O.encode_weight(f32(w), tile_n - 8)
    t = v1.shape[0]
    blk = blk.reshape(t, 8, k)
    tol = 1e-5 * max(1.0, np.abs(v2).max())
    assert np.abs(blk[:, 0] + blk[:, 1] + blk[:, 2] - v1).max() <= 1e-5
    assert np.abs(blk[:, 3] + blk[:, 4] + blk[:, 5] - v2).max() <= tol
    # two bf16 terms carry 16 significant bits
    assert np.abs(blk[:, 6] + blk[:, 7] - v3).max() <= 2.0 ** -15 * max(1.0, np.abs(v3).max())


# ------------------------------------------------------------ plain GEMM
@pytest.mark.parametrize("m,n,k,tile_n,bias", [
    (128, 256, 64, 256, False), (128, 128, 64, 128, False), (256, 512, 256, 0, True),
    (200, 136, 72, 256, True), (200, 136, 72, 128, True), (1, 8, 8, 0, False), (300, 1000, 520, 0, True),
    (1024, 1024, 1024, 0, False), (512, 4096, 4096, 0, True),
])
def test_plain_gemm_matches_fp32(cuda_device, m, n, k, tile_n, bias):
    a, w, b = seeded(m, n, k, 2, bias)
    ref = f32(a) @ f32(w).T + (f32(b) if b is not None else 0)
    c, rep = ops.abft_gemm(a.to(cuda_device), w.to(cuda_device), None if b is None else b.to(cuda_device),
                           mode=N.MODE_OFF, tile_n=tile_n)
    assert rep is None
    assert max_rel_err(f32(c), ref) <= OUT_TOL


# ---------------------------------------------------- checked GEMM parity
def run_checked(device, m, n, k, faults, *, tile_n=0, tile_m=0, bias=False, mode=N.MODE_DETECT | N.MODE_CORRECT,
                seed=3, magnitude=None):
    a, w, b = seeded(m, n, k, seed, bias)
    acc = f32(a).astype(np.float64) @ f32(w).astype(np.float64).T
    delta = 256.0 * np.abs(acc).max() if magnitude is None else magnitude
    inj = [(r, c, float(delta)) for (r, c) in faults]
    c, rep = ops.abft_gemm(a.to(device), w.to(device), None if b is None else b.to(device), mode=mode,
                           tile_n=tile_n, tile_m=tile_m, inject=inj or None)
    r = rep.read()
    orc = O.rowcheck_gemm(f32(a), f32(w), None if b is None else f32(b), tile_n=r.tile_n, inject=inj,
                          correct=bool(mode & N.MODE_CORRECT))
    return a, w, b, c, r, orc


@pytest.mark.parametrize("tile_n", [0, 128, 256])
@pytest.mark.parametrize("m,n,k,bias", [(256, 512, 256, False), (200, 136, 72, True), (512, 4096, 512, True),
                                        (384, 1000, 1024, False)])
def test_clean_inputs_have_no_records(cuda_device, tile_n, m, n, k, bias):
    a, w, b, c, r, orc = run_checked(cuda_device, m, n, k, [], tile_n=tile_n, bias=bias)
    assert r.status == 0 and r.n_faults == 0 and r.records == [] and orc.records == []
    ref = f32(a) @ f32(w).T + (f32(b) if b is not None else 0)
    assert max_rel_err(f32(c), ref) <= OUT_TOL
    assert r.tile_m in (128, 256) and r.tile_n in (120, 248)


@pytest.mark.parametrize("tile_n", [128, 256])
@pytest.mark.parametrize("count", [1, 4])
@pytest.mark.parametrize("m,n,k", [(256, 512, 256), (512, 4096, 1024), (1024, 1024, 1024), (300, 1000, 520)])
def test_faults_located_and_corrected_bit_exact(cuda_device, tile_n, count, m, n, k):
    faults = O.seeded_fault_positions(m, n, count, 11 * count + m)
    a, w, b, c, r, orc = run_checked(cuda_device, m, n, k, faults, tile_n=tile_n)
    got = sorted((x.row, x.col, x.flags) for x in r.records)
    assert got == orc.records
    assert sorted((i, j) for i, j, _ in got) == sorted(faults)
    assert r.n_faults == r.n_located == r.n_corrected == count
    assert r.status == N.STATUS_FAULT
    assert max_rel_err(f32(c), orc.out) <= OUT_TOL
    clean = f32(a) @ f32(w).T
    assert max_rel_err(f32(c), clean) <= OUT_TOL


@pytest.mark.parametrize("m,n,k", [
    (512, 4096, 4096),    # 68 tiles on 148 SMs: every tile split across ~2 CTAs
    (512, 3584, 18944),   # long K: 2-3 CTAs per tile
    (256, 1024, 8192),    # 10 tiles: ~15 CTAs per tile
    (512, 37888, 3584),   # 4 whole-tile waves, then a stream-K tail of 20 tiles
])
@pytest.mark.parametrize("mode", [N.MODE_OFF, N.MODE_DETECT | N.MODE_CORRECT])
def test_stream_k_schedules(cuda_device, m, n, k, mode):
    """Shapes whose schedule splits tiles across CTAs: same output as the
    fp32 GEMM, bit-identical across runs, faults found and corrected."""
    torch.manual_seed(m * 7 + n + k)
    a = (torch.randn(m, k, device=cuda_device) * k ** -0.5).bfloat16()
    w = (torch.randn(n, k, device=cuda_device) * k ** -0.5).bfloat16()
    ref = a.float() @ w.float().T
    c1, r1 = ops.abft_gemm(a, w, mode=mode)
    c2, _ = ops.abft_gemm(a, w, mode=mode)
    assert torch.equal(c1, c2)
    assert (c1.float() - ref).abs().max().item() <= OUT_TOL * ref.abs().max().item()
    if mode == N.MODE_OFF:
        return
    assert r1.read().n_faults == 0
    delta = 256.0 * ref.abs().max().item()
    faults = O.seeded_fault_positions(m, n, 4, m + k)
    c3, r3 = ops.abft_gemm(a, w, mode=mode, inject=[(i, j, delta) for i, j in faults])
    r3 = r3.read()
    assert r3.coords() == sorted(faults) and r3.n_corrected == 4
    assert (c3.float() - ref).abs().max().item() <= OUT_TOL * ref.abs().max().item()


def test_detect_only_keeps_the_fault(cuda_device):
    m, n, k = 256, 512, 256
    a, w, b, c, r, orc = run_checked(cuda_device, m, n, k, [(17, 300)], mode=N.MODE_DETECT, magnitude=5.0)
    assert [(x.row, x.col, x.flags) for x in r.records] == [(17, 300, N.REC_DETECTED | N.REC_LOCATED)]
    assert r.n_corrected == 0
    clean = f32(a) @ f32(w).T
    assert abs(f32(c)[17, 300] - (clean[17, 300] + 5.0)) < 0.05


def test_two_faults_in_one_row_segment_are_not_miscorrected(cuda_device):
    # (10, 201): mean column not an integer; (40, 42): integer mean 41, rejected
    # by the sign checksum (no three consecutive columns share a sign)
    for pair in ([(5, 10), (5, 201)], [(5, 40), (5, 42)], [(9, 0), (9, 2)]):
        a, w, b, c, r, orc = run_checked(cuda_device, 128, 248, 128, pair, tile_n=256, magnitude=3.0)
        row = pair[0][0]
        assert sorted((x.row, x.col, x.flags) for x in r.records) == orc.records == [(row, -1, N.REC_DETECTED)]
        assert r.status == N.STATUS_FAULT | N.STATUS_UNLOCATED
        assert r.n_corrected == 0


def test_ragged_edges_and_bias(cuda_device):
    a, w, b, c, r, orc = run_checked(cuda_device, 200, 136, 72, [(199, 135)], bias=True, tile_n=256)
    assert [(x.row, x.col) for x in r.records] == [(199, 135)]
    assert max_rel_err(f32(c), orc.out) <= OUT_TOL


def test_report_overflow(cuda_device):
    m, n, k = 256, 512, 128
    a, w, _ = seeded(m, n, k, 5)
    faults = [(i, (7 * i) % n, 50.0) for i in range(10)]
    c, rep = ops.abft_gemm(a.to(cuda_device), w.to(cuda_device), inject=faults,
                           report=ops.ReportBuffer(4, cuda_device))
    r = rep.read()
    assert r.n_faults == 10 and len(r.records) == 4 and r.overflow == 6
    assert r.status & N.STATUS_OVERFLOW


def test_cached_checksums_equal_inline_encode(cuda_device):
    m, n, k = 384, 1000, 512
    a, w, _ = seeded(m, n, k, 6)
    ad, wd = a.to(cuda_device), w.to(cuda_device)
    faults = [(3, 777, 9.0), (200, 5, -9.0)]
    c1, r1 = ops.abft_gemm(ad, wd, tile_n=256, inject=faults)
    v = ops.encode_weight(wd, 256)
    c2, r2 = ops.abft_gemm(ad, wd, tile_n=256, checksums=v, inject=faults)
    assert torch.equal(c1, c2)
    assert r1.read().coords() == r2.read().coords() == [(3, 777), (200, 5)]


def test_deterministic_bits(cuda_device):
    m, n, k = 1024, 2048, 1024
    a, w, b = seeded(m, n, k, 7, True)
    ad, wd, bd = a.to(cuda_device), w.to(cuda_device), b.to(cuda_device)
    outs = [ops.abft_gemm(ad, wd, bd, mode=N.MODE_DETECT | N.MODE_CORRECT | N.MODE_REF)[0] for _ in range(2)]
    assert torch.equal(outs[0], outs[1])


# ------------------------------------------------------- scalar (ref) mode
@pytest.mark.parametrize("fault", [None, 1.0])
def test_ref_mode_matches_oracle(cuda_device, fault):
    m, n, k = 256, 512, 256
    a, w, b = seeded(m, n, k, 4, True)
    inj = [(3, 4, fault)] if fault else None
    c, rep = ops.abft_gemm(a.to(cuda_device), w.to(cuda_device), b.to(cuda_device), mode=N.MODE_REF, inject=inj)
    r = rep.read()
    o = O.cheap_sum_check(f32(a), f32(w).T, f32(c), f32(b))
    assert (r.ref_ok == 1) == o.ok
    assert abs(r.corner - o.abft_corner) <= 1e-4 * max(1.0, abs(o.abft_corner))
    assert abs(r.sum_c - o.sum_c) <= 1e-4 * max(1.0, abs(o.sum_c))


def test_check_only_reproduces_reference_python_backend(cuda_device, golden_dir):
    """bf16-sum mode on the reference's own (A, B, C, bias): same flags as the
    reference's CheapSumChecker, values within one bf16 rounding."""
    import json
    import os

    meta = json.load(open(os.path.join(golden_dir, "ref_checker_cases.json")))
    arrays = np.load(os.path.join(golden_dir, "ref_checker_cases.npz"))

    def dev(name):
        return torch.from_numpy(arrays[name].view(np.int16)).view(torch.bfloat16).to(cuda_device)

    for case in meta:
        n = case["name"]
        a, w, c = dev(n + "_a"), dev(n + "_w"), dev(n + "_c")
        b = dev(n + "_bias") if case["bias"] else None
        for layout, bb in (("nk", w), ("kn", w.t().contiguous())):
            r = ops.check_only(a, bb, c, b, b_layout=layout, bf16_sums=True).read()
            assert (r.ref_ok == 1) == case["ok"], (n, layout)
            for key, ref in (("corner", "abft_corner"), ("sum_c", "sum_c")):
                got = getattr(r, key)
                assert abs(got - case[ref]) <= 2 ** -7 * max(abs(case[ref]), 1e-3), (n, key, got, case[ref])


def test_check_only_locates_post_hoc_fault(cuda_device):
    m, n, k = 300, 264, 136
    a, w, b = seeded(m, n, k, 6, True)
    c = (a.float() @ w.float().T + b.float()).bfloat16()
    c2 = c.clone()
    c2[17, 33] += 5.0
    for cc, want in ((c, []), (c2, [(17, 33)])):
        for layout, bb in (("nk", w), ("kn", w.t().contiguous())):
            r = ops.check_only(a.to(cuda_device), bb.to(cuda_device), cc.to(cuda_device), b.to(cuda_device),
                               b_layout=layout, locate=True).read()
            o = O.locate_post_hoc(f32(a), f32(w).T, f32(cc), f32(b))
            assert r.coords() == o == want
            ref = O.cheap_sum_check(f32(a), f32(w).T, f32(cc), f32(b))
            assert (r.ref_ok == 1) == ref.ok


# ------------------------------------------- full-size, size-independent checks
@pytest.mark.parametrize("m,n,k", [(512, 4096, 4096), (4096, 4096, 4096), (512, 37888, 3584)])
def test_full_size_seeded_faults(cuda_device, m, n, k):
    """No false positives on clean data; every seeded fault (2^8 max|C|) is
    found at its exact coordinate and the corrected output equals the clean
    one up to bf16 rounding."""
    torch.manual_seed(m + n + k)
    a = (torch.randn(m, k, device=cuda_device) * k ** -0.5).bfloat16()
    w = (torch.randn(n, k, device=cuda_device) * k ** -0.5).bfloat16()
    clean, r0 = ops.abft_gemm(a, w)
    r0 = r0.read()
    assert r0.n_faults == 0 and r0.status == 0
    delta = 256.0 * clean.float().abs().max().item()
    for count in (1, 4):
        faults = O.seeded_fault_positions(m, n, count, count)
        c, r = ops.abft_gemm(a, w, inject=[(i, j, delta) for i, j in faults])
        r = r.read()
        assert r.coords() == sorted(faults)
        assert r.n_corrected == count
        diff = (c.float() - clean.float()).abs().max().item()
        assert diff <= OUT_TOL * clean.float().abs().max().item()
    ref = (a.float() @ w.float().T)
    assert (clean.float() - ref).abs().max().item() <= OUT_TOL * ref.abs().max().item()


def test_no_device_timeouts_reported(cuda_device):
    a, w, _ = seeded(512, 1024, 512, 9)
    _, rep = ops.abft_gemm(a.to(cuda_device), w.to(cuda_device), mode=N.MODE_DETECT | N.MODE_REF)
    assert not rep.read().device_timeout


# ------------------------------------- 2-CTA pairs (256-row tiles, 256 or 128 wide)
PAIR_WIDTHS = [256, 128]


@pytest.mark.parametrize("tile_n", PAIR_WIDTHS)
@pytest.mark.parametrize("m,n,k,bias", [
    (256, 256, 64, False), (200, 136, 72, True), (300, 1000, 520, True), (1024, 1024, 1024, False),
    (1, 8, 8, False), (2048, 2048, 4096, True),
])
@pytest.mark.parametrize("mode", [N.MODE_OFF, N.MODE_DETECT | N.MODE_CORRECT])
def test_pair_tiles_match_fp32(cuda_device, m, n, k, bias, mode, tile_n):
    a, w, b = seeded(m, n, k, 12, bias)
    ref = f32(a) @ f32(w).T + (f32(b) if b is not None else 0)
    c, rep = ops.abft_gemm(a.to(cuda_device), w.to(cuda_device), None if b is None else b.to(cuda_device),
                           mode=mode, tile_n=tile_n, tile_m=256)
    assert max_rel_err(f32(c), ref) <= OUT_TOL
    if mode != N.MODE_OFF:
        r = rep.read()
        assert r.status == 0 and r.n_faults == 0 and r.tile_m == 256 and r.tile_n == tile_n - 8


@pytest.mark.parametrize("tile_n", PAIR_WIDTHS)
@pytest.mark.parametrize("count", [1, 4])
@pytest.mark.parametrize("m,n,k", [(256, 512, 256), (512, 4096, 1024), (1024, 1024, 1024), (300, 1000, 520)])
def test_pair_faults_located_and_corrected_bit_exact(cuda_device, count, m, n, k, tile_n):
    faults = O.seeded_fault_positions(m, n, count, 13 * count + m)
    a, w, b, c, r, orc = run_checked(cuda_device, m, n, k, faults, tile_n=tile_n, tile_m=256)
    got = sorted((x.row, x.col, x.flags) for x in r.records)
    assert got == orc.records
    assert r.n_faults == r.n_located == r.n_corrected == count
    assert max_rel_err(f32(c), orc.out) <= OUT_TOL
    assert max_rel_err(f32(c), f32(a) @ f32(w).T) <= OUT_TOL


@pytest.mark.parametrize("m,n,k", [
    (512, 4096, 4096),    # 34 pair tiles on 74 pairs: stream-K only
    (256, 1024, 8192),    # 5 tiles: many pairs per tile
    (512, 37888, 3584),   # 306 tiles: whole-tile waves, then a stream-K tail
    (4096, 4096, 4096),
])
@pytest.mark.parametrize("mode", [N.MODE_OFF, N.MODE_DETECT | N.MODE_CORRECT])
@pytest.mark.parametrize("tile_n", PAIR_WIDTHS)
def test_pair_stream_k_schedules(cuda_device, m, n, k, mode, tile_n):
    torch.manual_seed(m * 5 + n + k)
    a = (torch.randn(m, k, device=cuda_device) * k ** -0.5).bfloat16()
    w = (torch.randn(n, k, device=cuda_device) * k ** -0.5).bfloat16()
    ref = a.float() @ w.float().T
    c1, r1 = ops.abft_gemm(a, w, mode=mode, tile_n=tile_n, tile_m=256)
    c2, _ = ops.abft_gemm(a, w, mode=mode, tile_n=tile_n, tile_m=256)
    assert torch.equal(c1, c2)
    assert (c1.float() - ref).abs().max().item() <= OUT_TOL * ref.abs().max().item()
    if mode == N.MODE_OFF:
        return
    r1 = r1.read()
    assert r1.n_faults == 0 and not r1.device_timeout
    delta = 256.0 * ref.abs().max().item()
    faults = O.seeded_fault_positions(m, n, 4, m + k + 1)
    c3, r3 = ops.abft_gemm(a, w, mode=mode, tile_n=tile_n, tile_m=256, inject=[(i, j, delta) for i, j in faults])
    r3 = r3.read()
    assert r3.coords() == sorted(faults) and r3.n_corrected == 4
    assert (c3.float() - ref).abs().max().item() <= OUT_TOL * ref.abs().max().item()


@pytest.mark.parametrize("tile_n", PAIR_WIDTHS)
@pytest.mark.parametrize("fault", [None, 1.0])
def test_pair_ref_mode_matches_oracle(cuda_device, fault, tile_n):
    m, n, k = 384, 512, 256
    a, w, b = seeded(m, n, k, 14, True)
    inj = [(300, 4, fault)] if fault else None
    c, rep = ops.abft_gemm(a.to(cuda_device), w.to(cuda_device), b.to(cuda_device), mode=N.MODE_REF, inject=inj,
                           tile_n=tile_n, tile_m=256)
    r = rep.read()
    o = O.cheap_sum_check(f32(a), f32(w).T, f32(c), f32(b))
    assert (r.ref_ok == 1) == o.ok
    assert abs(r.sum_c - o.sum_c) <= 1e-4 * max(1.0, abs(o.sum_c))


def test_tile_shape_rejected(cuda_device):
    a, w, _ = seeded(256, 256, 64, 15)
    with pytest.raises(N.AbftError):
        ops.abft_gemm(a.to(cuda_device), w.to(cuda_device), tile_n=128, tile_m=192)


# --------------------------------------------- compact tail tiles (last column)
@pytest.mark.parametrize("tile_n,tile_m", [(256, 128), (256, 256), (128, 128), (128, 256)])
@pytest.mark.parametrize("n", [8, 16, 24, 40, 136, 248 + 8, 248 + 128, 248 + 232, 4096, 120 + 112])
@pytest.mark.parametrize("mode", [N.MODE_OFF, N.MODE_DETECT | N.MODE_CORRECT])
def test_tail_tile_widths(cuda_device, tile_n, tile_m, n, mode):
    """Every width of the last tile column: outputs match, and a fault in
    the tail's last data column is located and corrected."""
    m, k = 384, 320
    a, w, b = seeded(m, n, k, 16 + n, True)
    ad, wd, bd = a.to(cuda_device), w.to(cuda_device), b.to(cuda_device)
    ref = f32(a) @ f32(w).T + f32(b)
    c, rep = ops.abft_gemm(ad, wd, bd, mode=mode, tile_n=tile_n, tile_m=tile_m)
    assert max_rel_err(f32(c), ref) <= OUT_TOL
    if mode == N.MODE_OFF:
        return
    assert rep.read().n_faults == 0
    faults = [(m - 1, n - 1), (5, max(0, n - 9))]
    a2, w2, b2, c2, r, orc = run_checked(cuda_device, m, n, k, faults, tile_n=tile_n, tile_m=tile_m, bias=True,
                                          seed=16 + n)
    got = sorted((x.row, x.col, x.flags) for x in r.records)
    assert got == orc.records
    assert r.n_corrected == len(faults)
    assert max_rel_err(f32(c2), orc.out) <= OUT_TOL


# ------------------------------------- swapped operands (few rows: decode)
def run_swapped(device, m, n, k, faults, *, bias=True, mode=N.MODE_DETECT | N.MODE_CORRECT, swap_ab=0, seed=21):
    """The library computes out^T = W a^T; the oracle checks that transposed
    product (W rows against the tokens' checksums, 120 tokens per tile)."""
    a, w, b = seeded(m, n, k, seed, bias)
    acc = f32(a).astype(np.float64) @ f32(w).astype(np.float64).T
    delta = 256.0 * np.abs(acc).max()
    inj = [(r, c, float(delta)) for (r, c) in faults]
    c, rep = ops.abft_gemm(a.to(device), w.to(device), None if b is None else b.to(device), mode=mode,
                           inject=inj or None, swap_ab=swap_ab)
    r = rep.read() if rep is not None else None
    orc = O.rowcheck_gemm(f32(w), f32(a), None, tile_n=120, inject=[(cc, rr, d) for rr, cc, d in inj],
                          correct=bool(mode & N.MODE_CORRECT))
    return a, w, b, c, r, orc


@pytest.mark.parametrize("m", [1, 2, 8, 16, 31, 32, 64])
@pytest.mark.parametrize("n,k", [(256, 64), (1000, 520), (4608, 3584)])
def test_swapped_small_m_matches_fp32(cuda_device, m, n, k):
    for mode in (N.MODE_OFF, N.MODE_DETECT | N.MODE_CORRECT):
        a, w, b, c, r, orc = run_swapped(cuda_device, m, n, k, [], mode=mode)
        ref = f32(a) @ f32(w).T + f32(b)
        assert max_rel_err(f32(c), ref) <= OUT_TOL
        if r is not None:
            assert r.n_faults == 0 and r.status == 0 and orc.records == []


@pytest.mark.parametrize("m,n,k", [(1, 1000, 520), (8, 4608, 3584), (32, 3584, 18944 // 4), (64, 4096, 1024)])
def test_swapped_faults_located_in_output_coordinates(cuda_device, m, n, k):
    faults = O.seeded_fault_positions(m, n, min(m, 4), 31 + m)
    a, w, b, c, r, orc = run_swapped(cuda_device, m, n, k, faults)
    # oracle records are (feature, token): map to (token, feature)
    want = sorted((cc, rr, fl) if cc >= 0 else (-1, rr, fl) for rr, cc, fl in orc.records)
    got = sorted((x.row, x.col, x.flags) for x in r.records)
    assert got == want
    assert r.coords() == sorted(faults) and r.n_corrected == len(faults)
    clean = f32(a) @ f32(w).T + f32(b)
    assert max_rel_err(f32(c), clean) <= OUT_TOL


def test_swap_forced_and_refused(cuda_device):
    m, n, k = 200, 512, 256  # swapped by request: 2 token tiles
    faults = [(3, 7), (150, 400)]
    a, w, b, c, r, orc = run_swapped(cuda_device, m, n, k, faults, swap_ab=2)
    assert r.coords() == sorted(faults) and r.n_corrected == 2
    assert max_rel_err(f32(c), f32(a) @ f32(w).T + f32(b)) <= OUT_TOL
    # few rows, swap refused: the ordinary row checks
    a, w, b, c, r, orc = run_swapped(cuda_device, 8, 512, 256, [(2, 100)], swap_ab=1)
    assert r.coords() == [(2, 100)] and r.tile_n in (120, 248)


# ------------------------------------- stress: back-to-back stream-K launches
@pytest.mark.parametrize("m,n,k,tile_m", [(288, 12288, 4096, 256), (288, 4096, 11008, 128), (512, 4608, 3584, 0),
                                          (4096, 4096, 4096, 0), (24, 4096, 4096, 0)])
def test_back_to_back_stream_k_launches_stay_clean(cuda_device, m, n, k, tile_m):
    """Many launches queued without a host sync (each with its own report):
    no record on clean data, every output equal to the first. Stream-K
    partials must be fully visible before a contributor's flag is."""
    torch.manual_seed(m + n + k)
    a = (torch.randn(m, k, device=cuda_device) * k ** -0.5).bfloat16()
    w = (torch.randn(n, k, device=cuda_device) * k ** -0.5).bfloat16()
    tn = ops.pick_tile_n(m, n, k, cuda_device)
    cks = ops.encode_weight(w, tn)
    calls = 80
    arena = torch.zeros(calls * 2048, dtype=torch.uint8, device=cuda_device)
    outs = []
    for i in range(calls):
        rep = ops.ReportBuffer(64, cuda_device, tensor=arena[i * 2048:(i + 1) * 2048])
        outs.append(ops.abft_gemm(a, w, tile_n=tn, tile_m=tile_m, checksums=cks, report=rep)[0])
    torch.cuda.synchronize()
    host = arena.cpu().numpy().tobytes()
    for i in range(calls):
        r = N.FaultReport.from_bytes(host[i * 2048:(i + 1) * 2048])
        assert r.n_faults == 0 and r.status == 0, (i, r.records[:3])
        assert torch.equal(outs[i], outs[0]), i


# ------------------------------------------- post-hoc check on fp16 / fp32 operands
def _dtype_golden(golden_dir, device):
    import json
    import os

    meta = json.load(open(os.path.join(golden_dir, "ref_checker_cases_f16_f32.json")))
    arrays = np.load(os.path.join(golden_dir, "ref_checker_cases_f16_f32.npz"))
    for case in meta:
        dt = torch.float16 if case["dtype"] == "f16" else torch.float32

        def dev(name, dt=dt):
            return torch.from_numpy(arrays[name]).view(dt).to(device)

        n = case["name"]
        yield case, dev(n + "_a"), dev(n + "_w"), dev(n + "_c"), (dev(n + "_bias") if case["bias"] else None)


def test_check_only_f16_f32_reproduce_reference(cuda_device, golden_dir):
    """The reference's native checker dispatches on fp16, bf16 and fp32
    (pytorch/abft/kernels/abft_fused.cu:116-118): on its own fp16 / fp32
    (A, B, C, bias) the library gives its flags, with native-type sums for
    fp16 (as the python backend's fp16 tensors) and fp32 sums for fp32."""
    for case, a, w, c, b in _dtype_golden(golden_dir, cuda_device):
        native = case["dtype"] == "f16"
        tol = 2 ** -10 if native else 1e-5
        for layout, bb in (("nk", w), ("kn", w.t().contiguous())):
            r = ops.check_only(a, bb, c, b, b_layout=layout, bf16_sums=native).read()
            assert (r.ref_ok == 1) == case["ok"], (case["name"], layout)
            for key, ref in (("corner", "abft_corner"), ("sum_c", "sum_c")):
                got = getattr(r, key)
                assert abs(got - case[ref]) <= tol * max(abs(case[ref]), 1.0), (case["name"], key, got, case[ref])


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_check_only_f16_f32_locate_post_hoc_fault(cuda_device, dtype):
    m, n, k = 300, 264, 136
    g = torch.Generator().manual_seed(9)
    a = (torch.randn(m, k, generator=g) * k ** -0.5).to(dtype)
    w = (torch.randn(n, k, generator=g) * k ** -0.5).to(dtype)
    b = (torch.randn(n, generator=g) * 0.02).to(dtype)
    c = (a.double() @ w.double().T + b.double()).to(dtype)
    c2 = c.clone()
    c2[17, 33] += 5.0
    unit = 2.0 ** -12 if dtype == torch.float16 else 2.0 ** -25
    for cc, want in ((c, []), (c2, [(17, 33)])):
        for layout, bb in (("nk", w), ("kn", w.t().contiguous())):
            r = ops.check_only(a.to(cuda_device), bb.to(cuda_device), cc.to(cuda_device), b.to(cuda_device),
                               b_layout=layout, locate=True).read()
            f64 = [t.double().numpy() for t in (a, w, cc, b)]
            o = O.locate_post_hoc(f64[0], f64[1].T, f64[2], f64[3], unit=unit)
            assert r.coords() == o == want, (dtype, layout)


# ------------------------------------------------- output offsets and strides
def _strided_out(m, n, c_off, ld_pad, device, dtype=torch.bfloat16):
    """An [m, n] view whose rows start c_off elements into a 32-byte sector
    (0 or 8 bf16) with leading dimension n + ld_pad, inside a buffer filled
    with a sentinel (so that any write outside the view shows)."""
    ldc = n + ld_pad
    flat = torch.full((m * ldc + c_off + 64,), 7.0, dtype=dtype, device=device)
    assert flat.data_ptr() % 256 == 0
    return flat, torch.as_strided(flat, (m, n), (ldc, 1), c_off)


@pytest.mark.parametrize("mode", [N.MODE_OFF, N.MODE_DETECT | N.MODE_CORRECT])
@pytest.mark.parametrize("c_off,ld_pad", [(8, 0), (8, 16), (0, 8), (8, 8)])
@pytest.mark.parametrize("m,n,k,tile_n,tile_m", [
    (300, 1000, 136, 256, 0), (512, 4096, 512, 256, 256), (256, 744, 64, 128, 0), (200, 520, 72, 256, 128),
])
def test_output_sector_offsets_and_strides(cuda_device, mode, c_off, ld_pad, m, n, k, tile_n, tile_m):
    """C's rows starting 16 bytes into a 32-byte sector, or a leading
    dimension that is not a multiple of 16 elements: every element
    bit-identical to the call with a packed C, faults found as the oracle
    finds them, and nothing written outside C (the bulk stores' boxes and the
    plain stores of partial chunks both honour the view)."""
    a, w, b = seeded(m, n, k, 21, bias=True)
    ad, wd, bd = a.to(cuda_device), w.to(cuda_device), b.to(cuda_device)
    acc = f32(a).astype(np.float64) @ f32(w).astype(np.float64).T
    faults = [] if mode == N.MODE_OFF else O.seeded_fault_positions(m, n, 3, m + n)
    # one fault among the first columns of the second tile column
    if faults and tile_n:
        faults[0] = (faults[0][0], (tile_n - 8) + 5)
    delta = float(256.0 * np.abs(acc).max())
    inj = [(i, j, delta) for i, j in faults] or None
    ref_c, ref_rep = ops.abft_gemm(ad, wd, bd, mode=mode, tile_n=tile_n, tile_m=tile_m, inject=inj)
    flat, c = _strided_out(m, n, c_off, ld_pad, cuda_device)
    _, rep = ops.abft_gemm(ad, wd, bd, mode=mode, tile_n=tile_n, tile_m=tile_m, inject=inj, out=c)
    torch.cuda.synchronize()
    # nothing outside the view changed
    mask = torch.ones_like(flat, dtype=torch.bool)
    mask[c_off:c_off + m * (n + ld_pad)].view(m, n + ld_pad)[:, :n] = False
    assert bool((flat[mask] == 7.0).all())
    assert torch.equal(c, ref_c)
    ref = acc + f32(b)[None, :]
    assert max_rel_err(f32(c), ref) <= OUT_TOL
    if mode == N.MODE_OFF:
        assert rep is None
        return
    r = rep.read()
    orc = O.rowcheck_gemm(f32(a), f32(w), f32(b), tile_n=r.tile_n, inject=inj)
    assert sorted((x.row, x.col, x.flags) for x in r.records) == orc.records
    assert r.coords() == sorted(faults) and r.n_corrected == len(faults)
    assert sorted((x.row, x.col, x.flags) for x in ref_rep.read().records) == orc.records
