"""Batched products (torch.bmm) through the fused kernel, against the oracle.

One launch covers every product of the batch. Per batch the bars are those
of the single-product tests: fault coordinates and flags bit-exact against
the oracle (records carry rows flattened over the batch), per-batch counters
equal to the oracle's, outputs within 1e-2 of max|C| of an fp32 product of
the same bf16 inputs, no record on clean inputs. The right operand comes in
the three layouts a caller has: torch.bmm's row-major mat2 [B, K, N] (copied
K-major by the call), the transpose of a K-major tensor (k.transpose(1, 2),
read in place) and the weight layout [B, N, K].
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


def seeded(bsz, m, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(bsz, m, k, generator=g) * k ** -0.5).bfloat16()
    w = (torch.randn(bsz, n, k, generator=g) * k ** -0.5).bfloat16()  # [B, N, K]
    return a, w


def f32(t):
    return t.float().cpu().numpy()


def max_rel_err(got, ref):
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def right_operand(w, layout, device):
    """w [B, N, K] in the layout the test asks for; returns (b, b_layout)."""
    if layout == "kn_rowmajor":  # torch.bmm's mat2 as usually stored
        return w.transpose(1, 2).contiguous().to(device), "kn"
    if layout == "kn_view":  # k.transpose(1, 2) of a K-major tensor
        return w.to(device).transpose(1, 2), "kn"
    return w.to(device), "nk"


def batch_faults(bsz, m, n, batches, seed):
    """One fault per listed batch: [(batch, row, col)]."""
    out = []
    for i, b in enumerate(batches):
        (r, c), = O.seeded_fault_positions(m, n, 1, seed + 7 * i)
        out.append((b, r, c))
    return out


def run(device, bsz, m, n, k, faults, *, layout="kn_rowmajor", mode=CHECKED, tile_n=0, tile_m=0, swap_ab=0,
        seed=5):
    a, w = seeded(bsz, m, n, k, seed)
    acc = np.einsum("bmk,bnk->bmn", f32(a).astype(np.float64), f32(w).astype(np.float64))
    delta = float(256.0 * np.abs(acc).max())
    inj = [(b * m + r, c, delta) for (b, r, c) in faults]
    bmat, b_layout = right_operand(w, layout, device)
    c, rep = ops.abft_bmm(a.to(device), bmat, b_layout=b_layout, mode=mode, tile_n=tile_n, tile_m=tile_m,
                          swap_ab=swap_ab, inject=inj or None)
    return a, w, acc, delta, c, (rep.read() if rep is not None else None)


def oracle_batches(a, w, faults, delta, tile_n, swapped, correct=True):
    """Per-batch oracle runs; records as (flattened row, col, flags) in C's
    coordinates, and the per-batch (faults, located, corrected)."""
    bsz, m, _ = a.shape
    recs, counts, outs = [], [], []
    for b in range(bsz):
        fb = [(r, c, delta) for (bb, r, c) in faults if bb == b]
        if not swapped:
            o = O.rowcheck_gemm(f32(a[b]), f32(w[b]), tile_n=tile_n, inject=fb, correct=correct)
            recs += [(b * m + r, c, fl) for (r, c, fl) in o.records]
            outs.append(o.out)
        else:  # out^T = W a^T: the oracle's rows are C's columns
            o = O.rowcheck_gemm(f32(w[b]), f32(a[b]), tile_n=120, inject=[(c, r, d) for (r, c, d) in fb],
                                correct=correct)
            recs += [(b * m + cc, rr, fl) for (rr, cc, fl) in o.records]
            outs.append(o.out.T)
        fl = [x[2] for x in o.records]
        counts.append((len(fl), sum(1 for x in fl if x & N.REC_LOCATED), sum(1 for x in fl if x & N.REC_CORRECTED)))
    return sorted(recs), counts, np.stack(outs)


# ------------------------------------------------------------ plain and clean
@pytest.mark.parametrize("layout", ["kn_rowmajor", "kn_view", "nk"])
@pytest.mark.parametrize("bsz,m,n,k", [(4, 128, 256, 64), (3, 200, 136, 72), (8, 256, 512, 256), (2, 1, 8, 8),
                                       (16, 64, 128, 128), (5, 300, 1000, 520)])
def test_bmm_matches_fp32_and_clean_has_no_records(cuda_device, layout, bsz, m, n, k):
    for mode in (N.MODE_OFF, CHECKED):
        a, w, acc, _, c, r = run(cuda_device, bsz, m, n, k, [], layout=layout, mode=mode)
        assert tuple(c.shape) == (bsz, m, n)
        assert max_rel_err(f32(c), acc) <= OUT_TOL
        if r is not None:
            assert r.status == 0 and r.n_faults == 0 and r.records == []
            assert r.batch_counts == ([(0, 0, 0)] * bsz if bsz > 1 else [])


def test_bmm_equals_torch_bmm(cuda_device):
    """Through the public torch entry: the same numbers as torch.bmm."""
    torch.manual_seed(0)
    a = (torch.randn(12, 256, 128, device=cuda_device) * 128 ** -0.5).bfloat16()
    b = (torch.randn(12, 128, 512, device=cuda_device) * 128 ** -0.5).bfloat16()
    c, rep = ops.abft_bmm(a, b)
    ref = torch.bmm(a.float(), b.float())
    assert (c.float() - ref).abs().max().item() <= OUT_TOL * ref.abs().max().item()
    assert rep.read().n_faults == 0


# -------------------------------------------------------- faults, per batch
@pytest.mark.parametrize("layout", ["kn_rowmajor", "kn_view", "nk"])
@pytest.mark.parametrize("tile_n", [128, 256])
@pytest.mark.parametrize("bsz,m,n,k", [(4, 256, 512, 256), (6, 300, 1000, 520), (3, 512, 4096, 1024)])
def test_bmm_faults_located_per_batch_bit_exact(cuda_device, layout, tile_n, bsz, m, n, k):
    faults = batch_faults(bsz, m, n, [0, bsz // 2, bsz - 1], 40 + m + bsz)
    a, w, acc, delta, c, r = run(cuda_device, bsz, m, n, k, faults, layout=layout, tile_n=tile_n)
    want, counts, out = oracle_batches(a, w, faults, delta, r.tile_n, swapped=False)
    got = sorted((x.row, x.col, x.flags) for x in r.records)
    assert got == want
    assert sorted((x.row, x.col) for x in r.records) == sorted((b * m + rr, cc) for b, rr, cc in faults)
    assert r.batch_counts == counts
    assert r.n_faults == r.n_corrected == len(set(faults))
    for b in range(bsz):
        view = r.batch_view(b, m)
        assert sorted((x.row, x.col) for x in view.records) == sorted((rr, cc) for bb, rr, cc in faults if bb == b)
    assert max_rel_err(f32(c), out) <= OUT_TOL
    assert max_rel_err(f32(c), acc) <= OUT_TOL  # corrected back to the clean product


def test_bmm_detect_only_keeps_faults(cuda_device):
    bsz, m, n, k = 4, 256, 512, 256
    faults = batch_faults(bsz, m, n, [1, 3], 77)
    a, w, acc, delta, c, r = run(cuda_device, bsz, m, n, k, faults, mode=N.MODE_DETECT)
    want, counts, _ = oracle_batches(a, w, faults, delta, r.tile_n, swapped=False, correct=False)
    assert sorted((x.row, x.col, x.flags) for x in r.records) == want
    assert r.n_corrected == 0 and r.batch_counts == counts
    for b, rr, cc in faults:
        assert abs(float(c[b, rr, cc]) - acc[b, rr, cc]) > 0.5 * delta


# ------------------------------------------------- pairs, stream-K, swapped
@pytest.mark.parametrize("tile_n", [256, 128])
def test_bmm_cta_pairs(cuda_device, tile_n):
    bsz, m, n, k = 3, 512, 1000, 512
    faults = batch_faults(bsz, m, n, [0, 1, 2], 91)
    a, w, acc, delta, c, r = run(cuda_device, bsz, m, n, k, faults, tile_n=tile_n, tile_m=256)
    assert r.tile_m == 256
    want, counts, out = oracle_batches(a, w, faults, delta, r.tile_n, swapped=False)
    assert sorted((x.row, x.col, x.flags) for x in r.records) == want and r.batch_counts == counts
    assert max_rel_err(f32(c), acc) <= OUT_TOL


@pytest.mark.parametrize("mode", [N.MODE_OFF, CHECKED])
def test_bmm_stream_k_across_batches_is_deterministic(cuda_device, mode):
    """50 tiles of 32 k-blocks on 148 SMs: tiles split across CTAs, pieces of
    different batches meet in the partials; results repeat bit for bit."""
    bsz, m, n, k = 5, 256, 1024, 2048
    a, w = seeded(bsz, m, n, k, 13)
    ad, wd = a.to(cuda_device), w.to(cuda_device)
    outs = [ops.abft_bmm(ad, wd, b_layout="nk", mode=mode, tile_n=256)[0] for _ in range(3)]
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    acc = np.einsum("bmk,bnk->bmn", f32(a).astype(np.float64), f32(w).astype(np.float64))
    assert max_rel_err(f32(outs[0]), acc) <= OUT_TOL


@pytest.mark.parametrize("layout", ["kn_view", "kn_rowmajor"])
@pytest.mark.parametrize("bsz,m,n,k", [(8, 1, 512, 128), (4, 16, 1024, 256), (32, 1, 2048, 128), (3, 64, 1000, 520)])
def test_bmm_swapped_few_rows(cuda_device, layout, bsz, m, n, k):
    """Decode-shaped batches (one query row per head against a long key
    block): the library computes out^T per batch with token checksums."""
    faults = batch_faults(bsz, m, n, sorted({0, bsz - 1}), 60 + m)
    a, w, acc, delta, c, r = run(cuda_device, bsz, m, n, k, faults, layout=layout)
    want, counts, out = oracle_batches(a, w, faults, delta, 128, swapped=True)
    assert sorted((x.row, x.col, x.flags) for x in r.records) == want
    assert r.batch_counts == counts
    assert max_rel_err(f32(c), acc) <= OUT_TOL


# ------------------------------------------------------------ strided views
def test_bmm_strided_operands_read_in_place(cuda_device):
    """Operands that are views with padded rows and batches (leading
    dimension and batch stride larger than the extents) are read in place."""
    bsz, m, n, k = 4, 128, 256, 128
    big_a = (torch.randn(bsz, m + 8, k + 64, device=cuda_device) * k ** -0.5).bfloat16()
    big_b = (torch.randn(bsz + 1, n, k + 32, device=cuda_device) * k ** -0.5).bfloat16()
    a = big_a[:, :m, :k]
    w = big_b[1:, :, 16:16 + k]
    assert ops._mat_layout(a) is not None and ops._mat_layout(w) is not None
    c, rep = ops.abft_bmm(a, w, b_layout="nk", inject=[(2 * m + 5, 100, 50.0)])
    ref = torch.einsum("bmk,bnk->bmn", a.float(), w.float())
    assert (c.float() - ref).abs().max().item() <= OUT_TOL * ref.abs().max().item()
    r = rep.read()
    assert r.coords() == [(2 * m + 5, 100)] and r.batch_counts[2] == (1, 1, 1)


def test_bmm_heads_interleaved_along_rows(cuda_device):
    """Per-head views of a [S, H, D] tensor (batch stride D, row stride
    H * D): read in place when the tensor-map encoder accepts the strides,
    else on packed copies; the result is the same either way."""
    s_len, heads, d = 256, 4, 64
    x = (torch.randn(s_len, heads, d, device=cuda_device) * d ** -0.5).bfloat16()
    y = (torch.randn(s_len, heads, d, device=cuda_device) * d ** -0.5).bfloat16()
    q = x.transpose(0, 1)  # [H, S, D], strides (D, H*D, 1)
    kt = y.transpose(0, 1).transpose(1, 2)  # [H, D, S]: K-major view of y
    c, rep = ops.abft_bmm(q, kt, inject=[(3 * s_len + 17, 200, 64.0)])
    ref = torch.bmm(q.float(), kt.float())
    assert (c.float() - ref).abs().max().item() <= OUT_TOL * ref.abs().max().item()
    r = rep.read()
    assert r.coords() == [(3 * s_len + 17, 200)] and r.batch_counts[3] == (1, 1, 1)


@pytest.mark.parametrize("bsz,m,n,k", [(4, 256, 512, 256), (3, 16, 1000, 520), (5, 300, 136, 72)])
def test_bmm_with_bias_faults_per_batch(cuda_device, bsz, m, n, k):
    """A bias (one per output column, shared by the batch) is added after the
    checks, in the normal and the swapped frame (m = 16: out^T per batch)."""
    a, w = seeded(bsz, m, n, k, 31)
    g = torch.Generator().manual_seed(32)
    bias = (torch.randn(n, generator=g) * 0.02).bfloat16()
    acc = np.einsum("bmk,bnk->bmn", f32(a).astype(np.float64), f32(w).astype(np.float64))
    delta = float(256.0 * np.abs(acc).max())
    faults = batch_faults(bsz, m, n, sorted({0, bsz - 1}), 90 + m)
    inj = [(b * m + r, c, delta) for (b, r, c) in faults]
    c, rep = ops.abft_bmm(a.to(cuda_device), w.transpose(1, 2).contiguous().to(cuda_device), bias.to(cuda_device),
                          inject=inj)
    r = rep.read()
    swapped = m <= 64 and n >= 2 * m
    want, counts, _ = oracle_batches(a, w, faults, delta, r.tile_n, swapped=swapped)
    assert sorted((x.row, x.col, x.flags) for x in r.records) == want
    assert r.batch_counts == counts
    ref = acc + f32(bias)[None, None, :]
    assert max_rel_err(f32(c), ref) <= OUT_TOL
