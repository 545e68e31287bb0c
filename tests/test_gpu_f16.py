"""The fused checksum GEMM on fp16 operands, against the oracle.

fp16 runs the same kind::f16 MMAs as bf16 (fp32 accumulation); what
differs is the checksum block: fp16's narrow exponent range makes the encode
scale each tile's checksums by a power of two (a table after the rows) that
the epilogue multiplies back. Bars, as for bf16: the encoded block
bit-identical to the oracle's restatement; fault coordinates and flags
bit-exact against the oracle; outputs within 1e-2 of max|C| of an fp32
product of the same fp16 inputs; no record on clean inputs -- including
weights near the top and the bottom of fp16's range.
"""
import numpy as np
import pytest
import torch

from oracle import abft_oracle as O
from vla_abft_estimate_b200 import _native as N
from vla_abft_estimate_b200 import ops

pytestmark = pytest.mark.gpu

OUT_TOL = 1e-2
CHECKED = N.MODE_DETECT | N.MODE_CORRECT


def seeded(m, n, k, seed, bias=False, w_scale=1.0, bsz=None):
    g = torch.Generator().manual_seed(seed)
    lead = () if bsz is None else (bsz,)
    a = (torch.randn(*lead, m, k, generator=g) * k ** -0.5).half()
    w = (torch.randn(*lead, n, k, generator=g) * (k ** -0.5 * w_scale)).half()
    b = (torch.randn(n, generator=g) * 0.02 * w_scale).half() if bias else None
    return a, w, b


def f32(t):
    return t.float().cpu().numpy()


def max_rel_err(got, ref):
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


# ------------------------------------------------------------------ encode
@pytest.mark.parametrize("tile_n", [128, 256])
@pytest.mark.parametrize("n,k,w_scale", [(300, 200, 1.0), (1024, 512, 1.0), (136, 72, 1.0), (496, 256, 3e4),
                                         (300, 64, 1e-3), (4096, 4104, 1.0)])  # the last: the many-CTA path
def test_encode_block_bit_identical_to_oracle(cuda_device, tile_n, n, k, w_scale):
    _, w, _ = seeded(8, n, k, 1, w_scale=w_scale)
    blk = ops.encode_weight(w.to(cuda_device), tile_n)
    assert blk.dtype == torch.uint8 and blk.numel() == ops.checksum_bytes(n, k, tile_n, torch.float16)
    want = np.frombuffer(O.encode_weight_f16_block(f32(w), tile_n - 8), dtype=np.uint8)
    got = blk.cpu().numpy()
    assert got.shape == want.shape
    assert np.array_equal(got, want)


@pytest.mark.parametrize("n", [1, 8, 32])
@pytest.mark.parametrize("k", [64, 3584, 18944, 32768, 32776])
def test_encode_few_rows_bit_identical_to_oracle(cuda_device, n, k):
    """Token tiles of a decode step (at most 32 rows: the column-parallel
    one-launch encode; K past 32768 takes the general cluster kernel)."""
    _, w, _ = seeded(8, n, k, 3 + n)
    blk = ops.encode_weight(w.to(cuda_device), 128).cpu().numpy()
    want = np.frombuffer(O.encode_weight_f16_block(f32(w), 120), dtype=np.uint8)
    assert np.array_equal(blk, want)


def test_encode_passes_over_nan_sums(cuda_device):
    """A NaN weight makes its k column's sums NaN; the tile's scales come
    from the other columns (as the oracle's restatement has it)."""
    n, k = 300, 136
    _, w, _ = seeded(8, n, k, 12)
    w[5, 70] = float("nan")
    blk = ops.encode_weight(w.to(cuda_device), 128).cpu().numpy()
    want = np.frombuffer(O.encode_weight_f16_block(f32(w), 120), dtype=np.uint8)
    tiles = -(-n // 120)
    rows_b = tiles * 8 * k * 2
    got_rows = blk[:rows_b].view(np.float16)
    want_rows = want[:rows_b].view(np.float16)
    assert np.array_equal(got_rows, want_rows, equal_nan=True)
    assert np.isnan(got_rows.reshape(tiles, 8, k)[0, :, 70]).all()
    assert np.array_equal(blk[rows_b:], want[rows_b:])


def test_encode_batched_blocks_and_cached_checksums(cuda_device):
    """abft_gemm with a caller's block gives the records of a call that
    encodes into its workspace."""
    m, n, k = 256, 1000, 520
    a, w, _ = seeded(m, n, k, 2)
    ad, wd = a.to(cuda_device), w.to(cuda_device)
    cks = ops.encode_weight(wd, 256)
    acc = f32(a).astype(np.float64) @ f32(w).astype(np.float64).T
    inj = [(5, 17, float(256 * np.abs(acc).max())), (200, 990, float(256 * np.abs(acc).max()))]
    c1, r1 = ops.abft_gemm(ad, wd, tile_n=256, checksums=cks, inject=inj)
    c2, r2 = ops.abft_gemm(ad, wd, tile_n=256, inject=inj)
    assert torch.equal(c1, c2)
    key = lambda x: (x.row, x.col)  # noqa: E731  (records land in atomic-slot order)
    assert sorted(r1.read().records, key=key) == sorted(r2.read().records, key=key)
    with pytest.raises(ValueError):
        ops.abft_gemm(ad, wd, tile_n=256, checksums=cks.view(torch.float16))


# ---------------------------------------------------------- clean and plain
@pytest.mark.parametrize("tile_n", [0, 128, 256])
@pytest.mark.parametrize("m,n,k,bias", [(256, 512, 256, False), (200, 136, 72, True), (512, 4096, 512, True),
                                        (384, 1000, 1024, False)])
def test_clean_inputs_have_no_records(cuda_device, tile_n, m, n, k, bias):
    a, w, b = seeded(m, n, k, 3, bias)
    ref = f32(a) @ f32(w).T + (f32(b) if b is not None else 0)
    for mode in (N.MODE_OFF, CHECKED):
        c, rep = ops.abft_gemm(a.to(cuda_device), w.to(cuda_device), None if b is None else b.to(cuda_device),
                               mode=mode, tile_n=tile_n)
        assert c.dtype == torch.float16
        assert max_rel_err(f32(c), ref) <= OUT_TOL
        if rep is not None:
            r = rep.read()
            assert r.status == 0 and r.n_faults == 0 and r.records == []


@pytest.mark.parametrize("w_scale", [200.0, 1e-3])
def test_weights_near_the_ends_of_fp16_range(cuda_device, w_scale):
    """Large weights (unscaled column-weighted checksums would overflow
    fp16) and tiny ones (many subnormal): clean calls record nothing,
    injected faults are located and corrected."""
    m, n, k = 512, 2048, 1024
    a, w, b = seeded(m, n, k, 4, True, w_scale=w_scale)
    ad, wd, bd = a.to(cuda_device), w.to(cuda_device), b.to(cuda_device)
    ref = f32(a).astype(np.float64) @ f32(w).astype(np.float64).T + f32(b)
    c, rep = ops.abft_gemm(ad, wd, bd)
    assert rep.read().n_faults == 0
    assert max_rel_err(f32(c), ref) <= OUT_TOL
    faults = O.seeded_fault_positions(m, n, 4, 77)
    delta = float(64 * np.abs(ref).max())
    c, rep = ops.abft_gemm(ad, wd, bd, inject=[(r, cc, delta) for r, cc in faults])
    r = rep.read()
    assert r.coords() == sorted(faults) and r.n_corrected == 4
    assert max_rel_err(f32(c), ref) <= OUT_TOL


# ------------------------------------------------------------ fault parity
@pytest.mark.parametrize("tile_n,tile_m", [(128, 128), (256, 128), (256, 256), (128, 256)])
@pytest.mark.parametrize("m,n,k,count", [(256, 512, 256, 1), (512, 4096, 1024, 4), (300, 1000, 520, 4),
                                         (512, 4096, 4096, 4)])
def test_faults_located_and_corrected_bit_exact(cuda_device, tile_n, tile_m, m, n, k, count):
    a, w, b = seeded(m, n, k, 5 + m, True)
    acc = f32(a).astype(np.float64) @ f32(w).astype(np.float64).T
    delta = float(256.0 * np.abs(acc).max())
    faults = O.seeded_fault_positions(m, n, count, 11 * count + m)
    inj = [(r, c, delta) for r, c in faults]
    c, rep = ops.abft_gemm(a.to(cuda_device), w.to(cuda_device), b.to(cuda_device), tile_n=tile_n, tile_m=tile_m,
                           inject=inj)
    r = rep.read()
    orc = O.rowcheck_gemm(f32(a), f32(w), f32(b), tile_n=r.tile_n, inject=inj, out_dtype="f16")
    assert sorted((x.row, x.col, x.flags) for x in r.records) == orc.records
    assert r.coords() == sorted(faults) and r.n_corrected == count
    assert max_rel_err(f32(c), orc.out) <= OUT_TOL
    assert max_rel_err(f32(c), acc + f32(b)) <= OUT_TOL


def test_detect_only_keeps_the_fault(cuda_device):
    m, n, k = 256, 512, 256
    a, w, _ = seeded(m, n, k, 6)
    c, rep = ops.abft_gemm(a.to(cuda_device), w.to(cuda_device), mode=N.MODE_DETECT, inject=[(17, 300, 5.0)])
    r = rep.read()
    orc = O.rowcheck_gemm(f32(a), f32(w), tile_n=r.tile_n, inject=[(17, 300, 5.0)], correct=False, out_dtype="f16")
    assert sorted((x.row, x.col, x.flags) for x in r.records) == orc.records
    assert r.n_corrected == 0
    # the fault stays in the output (fp32 accumulation order aside, as the oracle has it)
    assert max_rel_err(f32(c), orc.out) <= OUT_TOL
    assert abs(float(f32(c)[17, 300]) - orc.out[17, 300]) <= 1e-2 * abs(orc.out[17, 300])


# ------------------------------------------------ swapped operands (decode)
@pytest.mark.parametrize("m,n,k", [(1, 1000, 520), (8, 4608, 3584), (64, 4096, 1024)])
def test_swapped_few_rows(cuda_device, m, n, k):
    a, w, b = seeded(m, n, k, 21, True)
    acc = f32(a).astype(np.float64) @ f32(w).astype(np.float64).T
    clean = acc + f32(b)
    c, rep = ops.abft_gemm(a.to(cuda_device), w.to(cuda_device), b.to(cuda_device))
    assert rep.read().n_faults == 0 and max_rel_err(f32(c), clean) <= OUT_TOL
    faults = O.seeded_fault_positions(m, n, min(m, 4), 31 + m)
    delta = float(256.0 * np.abs(acc).max())
    inj = [(r, cc, delta) for r, cc in faults]
    c, rep = ops.abft_gemm(a.to(cuda_device), w.to(cuda_device), b.to(cuda_device), inject=inj)
    r = rep.read()
    orc = O.rowcheck_gemm(f32(w), f32(a), None, tile_n=120, inject=[(cc, rr, d) for rr, cc, d in inj])
    want = sorted((cc, rr, fl) if cc >= 0 else (-1, rr, fl) for rr, cc, fl in orc.records)
    assert sorted((x.row, x.col, x.flags) for x in r.records) == want
    assert r.coords() == sorted(faults) and r.n_corrected == len(faults)
    assert max_rel_err(f32(c), clean) <= OUT_TOL


# ----------------------------------------------------------------- batched
@pytest.mark.parametrize("layout", ["kn_rowmajor", "kn_view", "nk"])
@pytest.mark.parametrize("bsz,m,n,k", [(4, 256, 512, 256), (3, 300, 1000, 520), (6, 16, 256, 128),
                                      (3, 256, 4096, 2048)])  # the last encodes on the many-CTA path, batched
def test_bmm_faults_per_batch(cuda_device, layout, bsz, m, n, k):
    a, w, _ = seeded(m, n, k, 40 + bsz, bsz=bsz)
    acc = np.einsum("bmk,bnk->bmn", f32(a).astype(np.float64), f32(w).astype(np.float64))
    delta = float(256.0 * np.abs(acc).max())
    faults = []
    for i, bi in enumerate([0, bsz - 1]):
        (r, c), = O.seeded_fault_positions(m, n, 1, 50 + i)
        faults.append((bi, r, c))
    if layout == "kn_rowmajor":
        bmat, bl = w.transpose(1, 2).contiguous().to(cuda_device), "kn"
    elif layout == "kn_view":
        bmat, bl = w.to(cuda_device).transpose(1, 2), "kn"
    else:
        bmat, bl = w.to(cuda_device), "nk"
    c0, r0 = ops.abft_bmm(a.to(cuda_device), bmat, b_layout=bl)
    assert r0.read().n_faults == 0 and max_rel_err(f32(c0), acc) <= OUT_TOL
    c, rep = ops.abft_bmm(a.to(cuda_device), bmat, b_layout=bl, inject=[(bi * m + r, cc, delta) for bi, r, cc in faults])
    r = rep.read()
    assert c.dtype == torch.float16
    assert r.coords() == sorted((bi * m + rr, cc) for bi, rr, cc in faults)
    assert r.n_corrected == len(faults)
    assert max_rel_err(f32(c), acc) <= OUT_TOL


# --------------------------------------------------------- scalar (ref) mode
@pytest.mark.parametrize("fault", [None, 1.0])
def test_ref_mode_matches_oracle(cuda_device, fault):
    m, n, k = 256, 512, 256
    a, w, b = seeded(m, n, k, 8, True)
    inj = [(3, 4, fault)] if fault else None
    c, rep = ops.abft_gemm(a.to(cuda_device), w.to(cuda_device), b.to(cuda_device), mode=N.MODE_REF, inject=inj)
    r = rep.read()
    o = O.cheap_sum_check(f32(a), f32(w).T, f32(c), f32(b))
    assert (r.ref_ok == 1) == o.ok
    assert abs(r.corner - o.abft_corner) <= 1e-4 * max(1.0, abs(o.abft_corner))
    assert abs(r.sum_c - o.sum_c) <= 1e-4 * max(1.0, abs(o.sum_c))


def test_stream_k_bit_reproducible(cuda_device):
    m, n, k = 512, 3584, 18944
    torch.manual_seed(9)
    a = (torch.randn(m, k, device=cuda_device) * k ** -0.5).half()
    w = (torch.randn(n, k, device=cuda_device) * k ** -0.5).half()
    ref = a.float() @ w.float().T
    c1, r1 = ops.abft_gemm(a, w)
    c2, _ = ops.abft_gemm(a, w)
    assert torch.equal(c1, c2) and r1.read().n_faults == 0
    assert (c1.float() - ref).abs().max().item() <= OUT_TOL * ref.abs().max().item()


def test_mixed_types_rejected(cuda_device):
    a = torch.zeros(64, 64, device=cuda_device, dtype=torch.float16)
    w = torch.zeros(64, 64, device=cuda_device, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ops.abft_gemm(a, w)
    with pytest.raises(ValueError):
        ops.abft_gemm(a.float(), w.float())
