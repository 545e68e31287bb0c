"""The CPU oracle against outputs of the reference itself (tests/golden/).

The fixtures were written by tests/golden/make_golden.py, which ran the
reference's CheapSumChecker (pytorch/abft/checkers.py:55-126) and
AbftInjector (pytorch/abft/injector.py) on seeded CPU bf16 inputs.
"""
import json
import os
import random

import numpy as np
import pytest

from oracle import abft_oracle as O


@pytest.fixture(scope="module")
def cases(golden_dir):
    meta = json.load(open(os.path.join(golden_dir, "ref_checker_cases.json")))
    arrays = np.load(os.path.join(golden_dir, "ref_checker_cases.npz"))
    out = []
    for c in meta:
        n = c["name"]
        a = O.bf16_bits_to_f32(arrays[n + "_a"])
        w = O.bf16_bits_to_f32(arrays[n + "_w"])
        cc = O.bf16_bits_to_f32(arrays[n + "_c"])
        b = O.bf16_bits_to_f32(arrays[n + "_bias"]) if c["bias"] else None
        out.append((c, a, w, cc, b))
    return out


def test_bf16_round_trip():
    x = np.array([0.0, 1.0, -2.5, 3.140625, 1e-3, 65504.0, -1e30], dtype=np.float32)
    bits = O.f32_to_bf16_bits(x)
    back = O.bf16_bits_to_f32(bits)
    assert np.all(O.f32_to_bf16_bits(back) == bits)
    # round to nearest even on the dropped 16 bits
    assert O.f32_to_bf16_bits(np.array([1.0 + 2 ** -8], np.float32))[0] == 0x3F80
    assert O.f32_to_bf16_bits(np.array([1.0 + 3 * 2 ** -9], np.float32))[0] == 0x3F81
    assert O.f32_to_bf16_bits(np.array([1.0 + 3 * 2 ** -8], np.float32))[0] == 0x3F82


def test_cheap_sum_bf16_emulation_matches_reference(cases):
    """Bit-exact flags and values of the reference python backend."""
    for c, a, w, cc, b in cases:
        r = O.cheap_sum_check(a, w.T, cc, b, emulate_bf16=True)
        assert r.ok == c["ok"], c["name"]
        assert r.abs_err == c["abs_err"], c["name"]
        assert r.rel_err == c["rel_err"], c["name"]
        assert r.abft_corner == c["abft_corner"], c["name"]
        assert r.sum_c == c["sum_c"], c["name"]


def test_cheap_sum_fp32_flags(cases):
    """fp32/fp64 sums agree with the reference except where its bf16 rounding
    alone trips the 1e-2 rule on a clean or sub-tolerance output."""
    bf16_false_positive = {"mid_clean", "mid_fault_tiny"}
    for c, a, w, cc, b in cases:
        r = O.cheap_sum_check(a, w.T, cc, b, emulate_bf16=False)
        if c["name"] in bf16_false_positive:
            assert c["ok"] is False and r.ok is True, c["name"]
        else:
            assert r.ok == c["ok"], c["name"]
            assert abs(r.abft_corner - c["abft_corner"]) <= 2 ** -7 * max(1.0, abs(c["abft_corner"])) * 2


def test_fault_positions_follow_reference_rng(cases):
    for c, a, w, cc, b in cases:
        if c["fault_index"] is None:
            continue
        idx = random.Random(c["seed"]).randrange(c["M"] * c["N"])
        assert idx == c["fault_index"]
        assert (idx // c["N"], idx % c["N"]) == (c["fault_row"], c["fault_col"])


def test_injector_rng_replays_reference_sequences(golden_dir):
    seqs = json.load(open(os.path.join(golden_dir, "ref_injector_sequences.json")))["configs"]
    for conf in seqs:
        rng = O.InjectorRng(conf["seed"])
        for call in conf["calls"]:
            m, k, n = call["shape"]
            idx = rng.maybe_inject(m * n, True, conf["inject_probability"])
            checked = rng.sample(conf["sample_rate"])
            assert (idx is not None) == call["injected"], conf
            if idx is not None:
                assert idx == call["index"]
            assert int(checked) == call["checked"]


def test_seeded_fault_positions_distinct():
    pos = O.seeded_fault_positions(512, 4096, 4, 1)
    assert len({r for r, _ in pos}) == 4 and len({c for _, c in pos}) == 4
    assert pos == O.seeded_fault_positions(512, 4096, 4, 1)


# ------------------------------------------------------------ row-check oracle
def _inputs(m, n, k, seed, bias=False):
    rng = np.random.default_rng(seed)
    a = O.bf16_round(rng.standard_normal((m, k)).astype(np.float32) / np.sqrt(k))
    w = O.bf16_round(rng.standard_normal((n, k)).astype(np.float32) / np.sqrt(k))
    b = O.bf16_round(0.02 * rng.standard_normal(n).astype(np.float32)) if bias else None
    return a, w, b


@pytest.mark.parametrize("tile_n", [248, 120])
def test_rowcheck_clean_has_no_records(tile_n):
    a, w, b = _inputs(200, 520, 136, 0, bias=True)
    r = O.rowcheck_gemm(a, w, b, tile_n=tile_n)
    assert r.records == []
    ref = O.bf16_round((a.astype(np.float64) @ w.T.astype(np.float64) + b).astype(np.float32))
    assert np.abs(r.out - ref).max() <= 2 ** -7 * np.abs(ref).max()


@pytest.mark.parametrize("tile_n", [248, 120])
def test_rowcheck_locates_and_corrects_distinct_faults(tile_n):
    m, n, k = 256, 512, 256
    a, w, _ = _inputs(m, n, k, 1)
    clean = a.astype(np.float64) @ w.T.astype(np.float64)
    delta = 256.0 * np.abs(clean).max()
    for count in (1, 4):
        pos = O.seeded_fault_positions(m, n, count, 7 + count)
        r = O.rowcheck_gemm(a, w, tile_n=tile_n, inject=[(i, j, delta) for i, j in pos])
        assert [(i, j) for i, j, _ in r.records] == sorted(pos)
        assert all(f == O.REC_DETECTED | O.REC_LOCATED | O.REC_CORRECTED for _, _, f in r.records)
        assert np.abs(r.out - O.bf16_round(clean.astype(np.float32))).max() <= 2 ** -7 * np.abs(clean).max()


def test_rowcheck_detect_only_keeps_fault():
    a, w, _ = _inputs(128, 248, 64, 2)
    clean = a.astype(np.float64) @ w.T.astype(np.float64)
    r = O.rowcheck_gemm(a, w, tile_n=248, inject=[(3, 40, 5.0)], correct=False)
    assert r.records == [(3, 40, O.REC_DETECTED | O.REC_LOCATED)]
    assert abs(r.out[3, 40] - (clean[3, 40] + 5.0)) < 0.05


def test_rowcheck_two_faults_in_one_row_are_unlocated():
    a, w, _ = _inputs(128, 248, 64, 3)
    r = O.rowcheck_gemm(a, w, tile_n=248, inject=[(5, 10, 3.0), (5, 201, 3.0)])
    assert r.records == [(5, -1, O.REC_DETECTED)]


def test_sign_checksum_rejects_integer_mean_double_faults():
    a, w, _ = _inputs(64, 248, 64, 8)
    # adjacent-pair means (c, c+2) are always rejected: no three consecutive
    # Thue-Morse signs are equal
    for c in range(0, 240, 7):
        r = O.rowcheck_gemm(a, w, tile_n=248, inject=[(3, c, 2.0), (3, c + 2, 2.0)])
        assert r.records == [(3, -1, O.REC_DETECTED)], c
    # over all equal-magnitude pairs with an integer mean, at most 1/3 slip through
    slipped = total = 0
    for c1 in range(0, 64, 3):
        for c2 in range(c1 + 2, 64, 2):
            r = O.rowcheck_gemm(a, w, tile_n=248, inject=[(3, c1, 2.0), (3, c2, 2.0)])
            total += 1
            slipped += r.records[0][1] >= 0
    assert slipped <= total // 3


def test_col_signs_thue_morse():
    s = O.col_signs(16)
    assert list(s) == [1, -1, -1, 1, -1, 1, 1, -1, -1, 1, 1, -1, 1, -1, -1, 1]


def test_rowcheck_ragged_last_tile():
    m, n, k = 200, 136, 72
    a, w, b = _inputs(m, n, k, 4, bias=True)
    r = O.rowcheck_gemm(a, w, b, tile_n=120, inject=[(199, 135, 10.0)])
    assert [(i, j) for i, j, _ in r.records] == [(199, 135)]


def test_split3_reconstructs_24_bits():
    rng = np.random.default_rng(0)
    v = (rng.standard_normal(1000) * 100).astype(np.float32)
    s = O.split3_bf16(v).astype(np.float64).sum(axis=0)
    assert np.all(np.abs(s - v) <= np.abs(v) * 2.0 ** -23)


def test_locate_post_hoc_single_fault():
    m, n, k = 96, 64, 80
    a, w, b = _inputs(m, n, k, 5, bias=True)
    c = O.bf16_round((a.astype(np.float64) @ w.T + b).astype(np.float32))
    assert O.locate_post_hoc(a, w.T, c, b) == []
    c2 = c.copy()
    c2[17, 33] += 5.0
    assert O.locate_post_hoc(a, w.T, c2, b) == [(17, 33)]


# ------------------------------------------------ BASELINE config 1 (512x4096x4096)
@pytest.fixture(scope="module")
def config1_cases(golden_dir):
    return json.load(open(os.path.join(golden_dir, "ref_config1_cases.json")))


def _config1_tensors(seed):
    from tests.golden import baseline_inputs as BI

    c1 = BI.CONFIG1
    a_bits, w_bits = BI.gemm_inputs(seed, c1["M"], c1["K"], c1["N"])
    c_bits = BI.product_bits(a_bits, w_bits)
    return BI, a_bits, w_bits, c_bits


def test_config1_inputs_regenerate_bit_exact(config1_cases):
    """The seeded inputs of the fixtures are reproduced here (digests)."""
    for seed in sorted({c["seed"] for c in config1_cases})[:2]:
        BI, a_bits, w_bits, c_bits = _config1_tensors(seed)
        case = next(c for c in config1_cases if c["seed"] == seed and not c["fault"])
        assert BI.sha256_bits(a_bits) == case["sha256_a"]
        assert BI.sha256_bits(w_bits) == case["sha256_w"]
        assert BI.sha256_bits(c_bits) == case["sha256_c"]


def test_config1_cheap_sum_bf16_emulation_matches_reference(config1_cases):
    """The oracle's bf16 emulation reproduces the reference's CheapSumChecker
    (pytorch/abft/checkers.py:96-126) bit for bit at the config-1 size, clean
    and with the seeded +2^8 max|C| fault -- including the seed whose clean
    rel_err lands exactly on the bf16-rounded 1e-2 tolerance."""
    for seed in sorted({c["seed"] for c in config1_cases}):
        BI, a_bits, w_bits, c_bits = _config1_tensors(seed)
        a = O.bf16_bits_to_f32(a_bits)
        w = O.bf16_bits_to_f32(w_bits)
        for case in (c for c in config1_cases if c["seed"] == seed):
            cc = O.bf16_bits_to_f32(c_bits).copy()
            if case["fault"]:
                idx, mag = BI.fault_for(seed, c_bits)
                assert (idx, mag) == (case["fault_index"], case["fault_magnitude"])
                flat = cc.reshape(-1)
                flat[idx] = O.bf16_round(np.array([flat[idx] + np.float32(mag)], np.float32))[0]
                assert BI.sha256_bits(O.f32_to_bf16_bits(cc)) == case["sha256_c"]
            r = O.cheap_sum_check(a, w.T, cc, emulate_bf16=True)
            got = (r.ok, r.abs_err, r.rel_err, r.abft_corner, r.sum_c)
            want = (case["ok"], case["abs_err"], case["rel_err"], case["abft_corner"], case["sum_c"])
            assert got == want, (seed, case["fault"], got, want)


# ------------------------------------------------ fp16 and fp32 operands
def _dtype_cases(golden_dir):
    meta = json.load(open(os.path.join(golden_dir, "ref_checker_cases_f16_f32.json")))
    arrays = np.load(os.path.join(golden_dir, "ref_checker_cases_f16_f32.npz"))

    def val(key, tag):
        raw = arrays[key]
        return raw.view(np.float16).astype(np.float32) if tag == "f16" else raw.view(np.float32)

    for c in meta:
        n, tag = c["name"], c["dtype"]
        yield (c, val(n + "_a", tag), val(n + "_w", tag), val(n + "_c", tag),
               val(n + "_bias", tag) if c["bias"] else None)


def test_cheap_sum_f16_emulation_matches_reference(golden_dir):
    """fp16 operands: the python backend's sums are fp16 tensors; the oracle's
    fp16 rounding of every intermediate reproduces its results bit for bit."""
    n = 0
    for c, a, w, cc, b in _dtype_cases(golden_dir):
        if c["dtype"] != "f16":
            continue
        r = O.cheap_sum_check(a, w.T, cc, b, emulate_f16=True)
        assert (r.ok, r.abs_err, r.rel_err, r.abft_corner, r.sum_c) == \
            (c["ok"], c["abs_err"], c["rel_err"], c["abft_corner"], c["sum_c"]), c["name"]
        n += 1
    assert n == 6


def test_cheap_sum_f32_matches_reference(golden_dir):
    """fp32 operands: fp32 sums in the reference, float64 here -- same flags,
    values within fp32 rounding."""
    n = 0
    for c, a, w, cc, b in _dtype_cases(golden_dir):
        if c["dtype"] != "f32":
            continue
        r = O.cheap_sum_check(a, w.T, cc, b)
        assert r.ok == c["ok"], c["name"]
        for got, want in ((r.abft_corner, c["abft_corner"]), (r.sum_c, c["sum_c"])):
            assert abs(got - want) <= 1e-5 * max(1.0, abs(want)), c["name"]
        n += 1
    assert n == 6
