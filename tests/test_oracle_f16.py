"""The oracle's fp16 checksum block (CPU).

fp16 keeps 5 exponent bits (largest finite 65504), so the checksum rows of
an fp16 weight are scaled per tile and per checksum by a power of two before
they are split into fp16 terms. These tests pin the restatement on the
CPU: the terms times the table's factor give back the sums, the scaled
terms stay inside fp16's range for weights near both ends of it, and the
exponent rule handles zero, subnormal and non-finite maxima.
"""
import numpy as np
import pytest

from oracle import abft_oracle as O


def _block(w, bd):
    raw = O.encode_weight_f16_block(w, bd)
    n, k = w.shape
    tiles = -(-n // bd)
    rows = np.frombuffer(raw[:tiles * 8 * k * 2], dtype=np.float16).reshape(tiles, 8, k)
    table = np.frombuffer(raw[tiles * 8 * k * 2:], dtype=np.float32).reshape(tiles, 8)
    assert len(raw) == tiles * 8 * k * 2 + tiles * 32
    return rows, table


def _f16(x):
    with np.errstate(over="ignore"):
        return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


@pytest.mark.parametrize("scale", [1.0, 3000.0, 1e-6])
@pytest.mark.parametrize("n,k,bd", [(300, 200, 248), (136, 72, 120), (1024, 64, 248)])
def test_scaled_terms_give_back_the_sums(scale, n, k, bd):
    rng = np.random.default_rng(n + k)
    w = _f16(rng.standard_normal((n, k)) * scale)
    rows, table = _block(w, bd)
    assert np.all(np.isfinite(rows.astype(np.float32)))
    v = O.encode_weight(w, bd)
    r = rows.astype(np.float64)
    sums = [r[:, 0] + r[:, 1] + r[:, 2], r[:, 3] + r[:, 4] + r[:, 5], r[:, 6] + r[:, 7]]
    for q in range(3):
        got = sums[q] * table[:, 4 + q:5 + q]
        ref = v[q]
        # fp32 sums of the encode pass in their fixed order, then the terms
        assert np.abs(got - ref).max() <= 1e-6 * np.abs(ref).max()
        hi = np.abs(r[:, 3 * q] if q < 2 else r[:, 6]).max(axis=1)
        assert np.all(hi <= 2.0 ** 15)  # rounding may reach 2^15 itself
        assert np.all(hi >= 2.0 ** 14)
        assert np.array_equal(table[:, q], np.abs(O.encode_weight_f32_order(w, bd)[q]).max(axis=1))
    assert np.all(table[:, 3] == 0) and np.all(table[:, 7] == 0)


def test_unscaled_fp16_terms_would_overflow():
    """The reason for the scale: column-weighted sums of large fp16 weights
    exceed 65504 (v2 grows with the square of the tile width)."""
    w = np.full((248, 8), 600.0, dtype=np.float32)
    v2 = O.encode_weight(w, 248)[1]
    assert np.all(np.isinf(_f16(v2)))
    rows, table = _block(w, 248)
    assert np.all(np.isfinite(rows.astype(np.float32)))
    assert table[0, 5] == 2.0 ** O.f16_checksum_exponent(float(np.abs(v2).max()))


def test_zero_tile_has_unit_scale():
    w = np.zeros((130, 16), dtype=np.float32)
    w[:120] = 1.0
    rows, table = _block(w, 120)  # second tile (rows 120..129) all zero
    assert np.all(rows[1] == 0)
    assert list(table[1]) == [0, 0, 0, 0, 1, 1, 1, 0]


def test_exponent_rule():
    e = O.f16_checksum_exponent
    assert e(0.0) == 0 and e(float("inf")) == 0 and e(float("nan")) == 0
    assert e(1e-40) == 0  # subnormal float32
    assert e(1.0) == -14 and e(2.0 ** 14) == 0 and e(2.0 ** 15 - 1) == 0 and e(2.0 ** 15) == 1
    assert e(3e38) == 100 and e(1e-30) == -100
    for m in [1e-3, 0.7, 5.0, 65504.0, 1e9]:
        s = np.float32(m) * np.float32(2.0 ** -e(m))
        assert 2.0 ** 14 <= s < 2.0 ** 15
