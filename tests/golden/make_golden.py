"""Write the golden fixtures of the reference's own ABFT path.

Run where a checkout of the reference is available (read-only is enough),
giving its root directory:

    python tests/golden/make_golden.py --reference <reference checkout>

(or set ABFT_REFERENCE_ROOT). It imports the reference package ``abft``
(pytorch/abft) and records, on seeded CPU bf16 inputs:

  ref_checker_cases.npz / .json
      CheapSumChecker.check results (python backend,
      pytorch/abft/checkers.py:55-126) on clean and fault-injected outputs,
      with and without bias, including a ragged shape.
  ref_injector_sequences.json
      the fault indices, injection flags and check counts AbftInjector
      (pytorch/abft/injector.py:19-189) produces for several seeds,
      probabilities and sample rates, plus one export_summary()
      (pytorch/abft/stats.py:175-220).
  ref_checker_cases_f16_f32.npz / .json
      the same check on fp16 and fp32 operands (its sums then have the
      operands' type), including a ragged shape and a bias.
  ref_config1_cases.json
      CheapSumChecker.check results at the BASELINE config-1 size
      (A[512 x 4096] . B[4096 x 4096], seeds 0-4, clean and with one
      +2^8 max|C| fault), with SHA-256 digests of the regenerated inputs
      (tests/golden/baseline_inputs.py) instead of the tensors.

Nothing under tests/ reads the reference at test time: only these fixtures.
"""
from __future__ import annotations

import argparse
import json
import os
import random
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def seeded(m: int, n: int, k: int, seed: int, with_bias: bool):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(m, k, generator=g) * k ** -0.5).bfloat16()
    w = (torch.randn(n, k, generator=g) * k ** -0.5).bfloat16()
    b = (torch.randn(n, generator=g) * 0.02).bfloat16() if with_bias else None
    return a, w, b


CASES = [
    # name, M, K, N, bias, seed, fault magnitude (None = clean; "max" = 2^8 * max|C|)
    ("small_clean", 64, 128, 96, False, 0, None),
    ("small_fault_1", 64, 128, 96, False, 0, 1.0),
    ("ragged_bias_clean", 200, 136, 72, True, 1, None),
    ("ragged_bias_fault_max", 200, 136, 72, True, 1, "max"),
    ("mid_bias_fault_1", 128, 384, 256, True, 2, 1.0),
    ("mid_clean", 256, 256, 128, False, 3, None),
    ("mid_fault_tiny", 256, 256, 128, False, 3, 1e-3),
    ("wide_fault_max", 96, 512, 384, False, 4, "max"),
]


def run_cases(abft):
    from abft.checkers import OpMeta

    cfg = abft.AbftConfig(enable=True)
    checker = abft.CheapSumChecker(cfg)
    arrays = {}
    meta = []
    for name, m, k, n, with_bias, seed, fault in CASES:
        a, w, b = seeded(m, n, k, seed, with_bias)
        c = F.linear(a, w, b)
        idx = None
        mag = None
        if fault is not None:
            rng = random.Random(seed)
            idx = rng.randrange(c.numel())
            mag = float(2.0 ** 8 * c.float().abs().max().item()) if fault == "max" else float(fault)
            c = c.clone()
            c.view(-1)[idx] += mag
        b2 = w.t()
        res = checker.check(a, b2, c, OpMeta("linear", "prefill", "golden"), bias_1d=b)
        arrays[f"{name}_a"] = bits(a)
        arrays[f"{name}_w"] = bits(w)
        arrays[f"{name}_c"] = bits(c)
        if b is not None:
            arrays[f"{name}_bias"] = bits(b)
        meta.append({
            "name": name, "M": m, "K": k, "N": n, "bias": with_bias, "seed": seed,
            "fault_index": idx, "fault_row": None if idx is None else idx // n,
            "fault_col": None if idx is None else idx % n, "fault_magnitude": mag,
            "ok": bool(res.ok), "abs_err": res.abs_err, "rel_err": res.rel_err,
            "abft_corner": res.abft_corner, "sum_c": res.sum_c,
        })
    return arrays, meta


INJ_CONFIGS = [
    {"seed": 2026, "inject_probability": 1.0, "sample_rate": 1.0},
    {"seed": 7, "inject_probability": 0.5, "sample_rate": 1.0},
    {"seed": 11, "inject_probability": 0.5, "sample_rate": 0.5},
    {"seed": 3, "inject_probability": 0.0, "sample_rate": 0.5},
]
INJ_SHAPES = [(4, 16, 8), (3, 16, 8), (8, 32, 24), (1, 16, 8), (5, 8, 40), (4, 16, 8), (2, 64, 16), (6, 16, 8),
              (7, 24, 8), (4, 16, 32), (9, 8, 8), (4, 16, 8)]


def run_injector(abft):
    out = []
    summary = None
    for ci, conf in enumerate(INJ_CONFIGS):
        cfg = abft.AbftConfig(enable=True, inject_fault=True, inject_magnitude=1.0,
                              inject_probability=conf["inject_probability"], sample_rate=conf["sample_rate"],
                              seed=conf["seed"], enable_matmul=False, enable_bmm=False)
        stats = abft.AbftStatsCollector()
        checker = abft.CheapSumChecker(cfg)
        calls = []
        g = torch.Generator().manual_seed(100 + ci)
        with abft.AbftInjector(cfg, checker, stats):
            for (m, k, n) in INJ_SHAPES:
                x = (torch.randn(m, k, generator=g) * 0.1).bfloat16()
                w = (torch.randn(n, k, generator=g) * 0.1).bfloat16()
                before = stats.total_checks
                y = F.linear(x, w)
                clean = torch.ops.aten.linear(x, w)
                diff = (y.float() - clean.float()).abs().view(-1)
                injected = bool(diff.max().item() > 0)
                calls.append({"shape": [m, k, n], "injected": injected,
                              "index": int(diff.argmax().item()) if injected else None,
                              "checked": stats.total_checks - before})
        entry = dict(conf)
        entry["calls"] = calls
        entry["total_injections"] = stats.total_injections
        entry["detected_injections"] = stats.total_detected_injections
        entry["total_checks"] = stats.total_checks
        entry["total_failures"] = stats.total_failures
        out.append(entry)
        if ci == 0:
            summary = stats.export_summary()
    return out, summary


DTYPE_CASES = [
    # name, M, K, N, bias, seed, fault magnitude (as CASES)
    ("clean", 64, 128, 96, False, 0, None),
    ("fault_1", 64, 128, 96, False, 0, 1.0),
    ("ragged_bias_clean", 200, 136, 72, True, 1, None),
    ("bias_fault_max", 200, 136, 72, True, 1, "max"),
    ("mid_clean", 256, 256, 128, False, 3, None),
    ("mid_fault_small", 256, 256, 128, False, 3, 0.05),
]


def run_dtype_cases(abft):
    """CheapSumChecker.check on fp16 and fp32 CPU tensors (the python
    backend's sums then have the operands' type)."""
    from abft.checkers import OpMeta

    checker = abft.CheapSumChecker(abft.AbftConfig(enable=True))
    arrays, meta = {}, []
    for dt, tag in ((torch.float16, "f16"), (torch.float32, "f32")):
        for name, m, k, n, with_bias, seed, fault in DTYPE_CASES:
            g = torch.Generator().manual_seed(seed)
            a = (torch.randn(m, k, generator=g) * k ** -0.5).to(dt)
            w = (torch.randn(n, k, generator=g) * k ** -0.5).to(dt)
            b = (torch.randn(n, generator=g) * 0.02).to(dt) if with_bias else None
            c = F.linear(a, w, b)
            idx, mag = None, None
            if fault is not None:
                idx = random.Random(seed).randrange(c.numel())
                mag = float(2.0 ** 8 * c.float().abs().max().item()) if fault == "max" else float(fault)
                c = c.clone()
                c.view(-1)[idx] += mag
            res = checker.check(a, w.t(), c, OpMeta("linear", "prefill", "golden"), bias_1d=b)
            key = f"{tag}_{name}"
            view = torch.int16 if dt == torch.float16 else torch.int32
            for suffix, t in (("a", a), ("w", w), ("c", c), ("bias", b)):
                if t is not None:
                    arrays[f"{key}_{suffix}"] = t.contiguous().view(view).numpy().copy()
            meta.append({"name": key, "dtype": tag, "M": m, "K": k, "N": n, "bias": with_bias, "seed": seed,
                         "fault_index": idx, "fault_row": None if idx is None else idx // n,
                         "fault_col": None if idx is None else idx % n, "fault_magnitude": mag,
                         "ok": bool(res.ok), "abs_err": res.abs_err, "rel_err": res.rel_err,
                         "abft_corner": res.abft_corner, "sum_c": res.sum_c})
    return arrays, meta


CONFIG1_SEEDS = [0, 1, 2, 3, 4]


def run_config1(abft):
    """The reference's check at config 1, clean and with one seeded fault."""
    import baseline_inputs as BI
    from abft.checkers import OpMeta

    checker = abft.CheapSumChecker(abft.AbftConfig(enable=True))
    m, k, n = BI.CONFIG1["M"], BI.CONFIG1["K"], BI.CONFIG1["N"]
    out = []
    for seed in CONFIG1_SEEDS:
        a_bits, w_bits = BI.gemm_inputs(seed, m, k, n)
        c_bits = BI.product_bits(a_bits, w_bits)
        idx, mag = BI.fault_for(seed, c_bits)

        def t(bits):
            return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)

        a, w, c = t(a_bits), t(w_bits), t(c_bits)
        cf = c.clone()
        cf.view(-1)[idx] += mag  # the reference injector's update (injector.py:72-73)
        for fault, cc in ((False, c), (True, cf)):
            res = checker.check(a, w.t(), cc, OpMeta("linear", "prefill", "config1"))
            out.append({
                "seed": seed, "M": m, "K": k, "N": n, "fault": fault,
                "fault_index": idx if fault else None, "fault_row": idx // n if fault else None,
                "fault_col": idx % n if fault else None, "fault_magnitude": mag if fault else None,
                "sha256_a": BI.sha256_bits(a_bits), "sha256_w": BI.sha256_bits(w_bits),
                "sha256_c": BI.sha256_bits(bits(cc)),
                "ok": bool(res.ok), "abs_err": res.abs_err, "rel_err": res.rel_err,
                "abft_corner": res.abft_corner, "sum_c": res.sum_c,
            })
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ABFT_REFERENCE_ROOT"),
                    help="root of a reference checkout (or set ABFT_REFERENCE_ROOT)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <reference checkout> or set ABFT_REFERENCE_ROOT")
    sys.path.insert(0, str(Path(args.reference) / "pytorch"))
    sys.path.insert(0, str(HERE))
    sys.path.insert(0, str(HERE.parent.parent))  # the oracle's package root
    import abft  # the reference package

    torch.set_num_threads(1)
    arrays, meta = run_cases(abft)
    np.savez_compressed(HERE / "ref_checker_cases.npz", **arrays)
    (HERE / "ref_checker_cases.json").write_text(json.dumps(meta, indent=1))
    inj, summary = run_injector(abft)
    (HERE / "ref_injector_sequences.json").write_text(json.dumps({"configs": inj, "summary_config0": summary},
                                                                 indent=1))
    d_arrays, d_meta = run_dtype_cases(abft)
    np.savez_compressed(HERE / "ref_checker_cases_f16_f32.npz", **d_arrays)
    (HERE / "ref_checker_cases_f16_f32.json").write_text(json.dumps(d_meta, indent=1))
    cfg1 = run_config1(abft)
    (HERE / "ref_config1_cases.json").write_text(json.dumps(cfg1, indent=1))
    print(f"wrote {len(meta)} checker cases, {len(inj)} injector sequences and {len(cfg1)} config-1 cases to {HERE}")


if __name__ == "__main__":
    main()
