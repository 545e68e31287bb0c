"""Weight-checksum cache identity and the stale-checksum guard, on the CPU.

The cache replaces the reference's per-call ``b_2d.sum(dim=1)``
(pytorch/abft/checkers.py:119). A cached block must never outlive the
memory it describes: these tests drive ``WeightChecksumCache`` with a
counting stand-in for the encoder (no GPU needed) and check the oracle's
rule that a slab mismatching in most rows is reported, not "corrected".
"""
import gc
import re

import numpy as np
import pytest
import torch

from oracle import abft_oracle as O
from vla_abft_estimate_b200 import _build
from vla_abft_estimate_b200 import _native as N
from vla_abft_estimate_b200.abft import injector as inj_mod


@pytest.fixture
def counting_encoder(monkeypatch):
    calls = []

    def fake_encode(weight, tile_n):
        calls.append((weight.data_ptr(), tile_n))
        return torch.full((8,), float(len(calls)))

    monkeypatch.setattr(inj_mod.ops, "encode_weight", fake_encode)
    return calls


def test_cache_hits_for_the_same_weight_and_its_views(counting_encoder):
    cache = inj_mod.WeightChecksumCache()
    w = torch.randn(64, 32)
    v1 = cache.get(w, 256)
    assert cache.get(w, 256) is v1
    assert cache.get(w.view(64, 32), 256) is v1  # a view shares storage and version
    assert len(counting_encoder) == 1
    cache.get(w, 128)  # another tile width is another block
    assert len(counting_encoder) == 2


def test_cache_reencodes_after_a_tracked_in_place_update(counting_encoder):
    cache = inj_mod.WeightChecksumCache()
    w = torch.randn(64, 32)
    v1 = cache.get(w, 256)
    with torch.no_grad():
        w.mul_(2.0)  # bumps the version counter
    assert cache.get(w, 256) is not v1
    assert len(counting_encoder) == 2


def test_cache_drops_entries_of_freed_weights(counting_encoder):
    cache = inj_mod.WeightChecksumCache()
    w = torch.randn(64, 32)
    cache.get(w, 256)
    assert len(cache) == 1
    del w
    gc.collect()
    assert len(cache) == 0  # the storage's weak reference dropped the entry


def test_cache_never_serves_a_new_tensor_at_a_reused_address(counting_encoder):
    """A different tensor at the same address and shape is encoded afresh,
    even while the old entry is still held (modelled by keeping the key)."""
    cache = inj_mod.WeightChecksumCache()
    w = torch.randn(64, 32)
    v1 = cache.get(w, 256)
    key = cache._key(w, 256)
    stale_entry = cache._d[key]
    other = torch.randn(64, 32)
    # plant the old entry under the new tensor's key: same address, shape,
    # strides and version, but another storage object
    cache._d[cache._key(other, 256)] = stale_entry
    assert cache.get(other, 256) is not v1
    assert len(counting_encoder) == 2


def test_cache_invalidate_after_an_untracked_write(counting_encoder):
    cache = inj_mod.WeightChecksumCache()
    w = torch.nn.Parameter(torch.randn(64, 32))
    v1 = cache.get(w, 256)
    w.data.copy_(torch.randn(64, 32))  # .data writes bypass the version counter
    assert cache.get(w, 256) is v1  # the cache cannot see it ...
    cache.invalidate(w)  # ... so the caller says so
    assert cache.get(w, 256) is not v1
    assert len(counting_encoder) == 2


def test_oracle_leaves_stale_checksum_slabs_uncorrected():
    rng = np.random.default_rng(3)
    m, n, k = 200, 300, 96
    a = O.bf16_round(rng.standard_normal((m, k)) * k ** -0.5)
    w_old = O.bf16_round(rng.standard_normal((n, k)) * k ** -0.5)
    w_new = O.bf16_round(rng.standard_normal((n, k)) * k ** -0.5)
    r = O.rowcheck_gemm(a, w_new, tile_n=120, checksum_weight=w_old)
    clean = O.rowcheck_gemm(a, w_new, tile_n=120)
    assert clean.records == []
    assert len(r.records) > 0.9 * m * 3  # nearly every row of every tile segment mismatches
    assert all(not (f & O.REC_CORRECTED) for _, _, f in r.records)
    assert any(f & O.REC_SUPPRESSED for _, _, f in r.records)
    assert np.array_equal(r.out, clean.out)  # the plain product: nothing was changed


def test_oracle_still_corrects_a_few_faults_per_slab():
    rng = np.random.default_rng(4)
    m, n, k = 128, 120, 64
    a = O.bf16_round(rng.standard_normal((m, k)) * k ** -0.5)
    w = O.bf16_round(rng.standard_normal((n, k)) * k ** -0.5)
    faults = [(i, (37 * i) % n, 8.0) for i in range(0, 128, 8)]  # 16 rows of one slab
    r = O.rowcheck_gemm(a, w, tile_n=120, inject=faults)
    assert len(r.records) == 16 == O.SUSPECT_ROWS
    assert all(f == O.REC_DETECTED | O.REC_LOCATED | O.REC_CORRECTED for _, _, f in r.records)
    more = faults + [(3, 5, 8.0)]
    r2 = O.rowcheck_gemm(a, w, tile_n=120, inject=more)
    assert all(f == O.REC_DETECTED | O.REC_LOCATED | O.REC_SUPPRESSED for _, _, f in r2.records)


def _header_defines():
    text = (_build.INCLUDE_DIR / "abft_b200.h").read_text()
    return {k: int(v) for k, v in re.findall(r"#define\s+(ABFT_\w+)\s+\(?(\d+)u?", text)}


@pytest.mark.parametrize("name,value", [
    ("ABFT_MODE_DETECT", N.MODE_DETECT), ("ABFT_MODE_CORRECT", N.MODE_CORRECT), ("ABFT_MODE_REF", N.MODE_REF),
    ("ABFT_MODE_REF_BF16", N.MODE_REF_BF16), ("ABFT_STATUS_FAULT", N.STATUS_FAULT),
    ("ABFT_STATUS_UNLOCATED", N.STATUS_UNLOCATED), ("ABFT_STATUS_OVERFLOW", N.STATUS_OVERFLOW),
    ("ABFT_STATUS_DEVICE_TIMEOUT", N.STATUS_DEVICE_TIMEOUT), ("ABFT_STATUS_REF_FAIL", N.STATUS_REF_FAIL),
    ("ABFT_STATUS_SUSPECT", N.STATUS_SUSPECT), ("ABFT_SUSPECT_ROWS", N.SUSPECT_ROWS),
    ("ABFT_REC_DETECTED", N.REC_DETECTED), ("ABFT_REC_LOCATED", N.REC_LOCATED),
    ("ABFT_REC_CORRECTED", N.REC_CORRECTED), ("ABFT_REC_SUPPRESSED", N.REC_SUPPRESSED),
    ("ABFT_CHECK_LOCATE", N.CHECK_LOCATE), ("ABFT_CHECK_NATIVE_SUMS", N.CHECK_NATIVE_SUMS),
    ("ABFT_MAX_INJECT", N.MAX_INJECT), ("ABFT_DTYPE_BF16", N.DTYPE_BF16), ("ABFT_DTYPE_F16", N.DTYPE_F16),
    ("ABFT_DTYPE_F32", N.DTYPE_F32), ("ABFT_B200_VERSION", N.LIB_VERSION),
])
def test_binding_constants_match_the_header(name, value):
    assert _header_defines()[name] == value


def test_bf16_sums_flag_is_the_native_sums_bit():
    text = (_build.INCLUDE_DIR / "abft_b200.h").read_text()
    assert re.search(r"#define\s+ABFT_CHECK_BF16_SUMS\s+ABFT_CHECK_NATIVE_SUMS", text)
    assert N.CHECK_BF16_SUMS == N.CHECK_NATIVE_SUMS


def test_oracle_suspect_rule_matches_the_header():
    assert O.SUSPECT_ROWS == _header_defines()["ABFT_SUSPECT_ROWS"]
    assert O.REC_SUPPRESSED == N.REC_SUPPRESSED


def test_cache_takes_inference_tensors(counting_encoder):
    cache = inj_mod.WeightChecksumCache()
    with torch.inference_mode():
        w = torch.randn(64, 32)
        v1 = cache.get(w, 256)
        assert cache.get(w, 256) is v1
    assert len(counting_encoder) == 1
